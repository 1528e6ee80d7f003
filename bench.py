#!/usr/bin/env python
"""Benchmark: Voxtral backbone decode frames/s on B200 (BASELINE.json metric, config C2).

Workload (configs[1] of BASELINE.json): the full 26-layer Ministral-3B-shaped backbone,
f16 synthetic weights (seed 0, N(0,0.02)), prompt of 512 text ids + 100 voice rows
(617 positions, prefilled once before the timed region), then one STEP = a 500-frame
batch-1 decode (frame 0 is the AUDIO kick, frames 1..499 embed the previous frame's
37 codes) from the post-prefill checkpoint.  value = frames/s of the whole job.

  N = 1   : one utterance on one GPU.
  N > 1   : launched by torchrun, one process per GPU; data-parallel replicas (each
            rank decodes its own utterance, no collective in the data path), weak
            scaling, device time = max over ranks.

`--impl reference` times the reference's algorithm on the host cores instead: the CPU
restatement in oracle/ (the reference itself is TypeScript + WGSL and cannot run here).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import re
import signal
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

N_TEXT, N_VOICE = 512, 100
WORKLOAD = ("C2: 26-layer Voxtral backbone (d=3072, 32q/8kv heads x 128, SwiGLU 9216), synthetic f16 weights; "
            "prompt 512 text ids + 100 voice rows (617 positions, prefilled before timing); one step = 500-frame "
            "batch-1 decode, KV f16 paged; maxSeqLen 4096")
BYTES_PER_LAYER = 232_796_160          # f16 weight bytes of one backbone layer
KV_BYTES_PER_POS = 106_496             # f16 K+V bytes per position, all 26 layers
METRIC = "backbone decode frames/s (batch 1)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--frames", type=int, default=500)
    ap.add_argument("--layers", type=int, default=26)
    ap.add_argument("--text", type=int, default=N_TEXT, help="text ids in the prompt (C2: 512)")
    ap.add_argument("--voice", type=int, default=N_VOICE, help="voice rows in the prompt (C2: 100)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes of the weight-streaming GEMV from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "k_gemv_c2.md")
    if not os.path.exists(p):
        return None
    m = re.search(r"dram_bytes_per_step:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    def __init__(self, gpu: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.send_signal(signal.SIGTERM)
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def cpu_sample(n_layers: int, seconds: float, n_frames_min: int = 2):
    """The CPU restatement (oracle/) on the host cores: decode frames at the C2 context length."""
    import oracle
    o = oracle.Oracle(n_layers=n_layers, max_seq=4096, with_fm=False)
    o.fill_kv(N_TEXT + N_VOICE + 5, seed=11)
    rng = np.random.default_rng(0)
    emb = rng.standard_normal(3072).astype(np.float32) * 0.1
    o.backbone_step(0, embed=emb)                 # warm-up step
    n, t0 = 0, time.perf_counter()
    while n < n_frames_min or time.perf_counter() - t0 < seconds:
        o.backbone_step(0, embed=emb)
        n += 1
    dt = time.perf_counter() - t0
    cores = oracle.num_threads()
    o.close()
    return n / dt, n, dt, cores


def run_reference(args):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return 0
    import oracle
    o = oracle.Oracle(n_layers=args.layers, max_seq=4096, with_fm=False)
    o.fill_kv(N_TEXT + N_VOICE + 5, seed=11)
    emb = (np.random.default_rng(0).standard_normal(3072) * 0.1).astype(np.float32)
    frames_per_step = 2
    start = o.position

    def step():
        o.position = start
        for _ in range(frames_per_step):
            o.backbone_step(0, embed=emb)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = frames_per_step * args.steps / dt
    cores = oracle.num_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 weights, f32 math, f32 KV", "data": "synthetic",
        "config": {"workload": WORKLOAD, "parallelism": "host cores", "sample": "per step: 2 backbone frames at "
                   f"position {start} (KV prefilled with synthetic values) of the {args.layers}-layer model"},
        "cpu_baseline": {"value": value, "unit": "frames/s", "cores": cores, "kind": "port",
                         "sample": f"{frames_per_step} frames x {args.steps} steps at position {start}"},
        "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    o.close()
    return 0


def run_b200(args):
    import torch

    vx = importlib.import_module("webgpu-voxtral_b200")
    synth = importlib.import_module("webgpu-voxtral_b200.synth")
    vdist = importlib.import_module("webgpu-voxtral_b200.dist")
    rank, local, world = vdist.env_rank()
    torch.cuda.set_device(local)
    vdist.init(timeout_s=300)
    F = args.frames
    eng = vx.VoxtralEngine({"config": {"backbone": {"n_layers": args.layers}}, "maxSeqLen": 4096,
                            "maxFrames": max(1024, F + 8), "enableFM": False, "device": local})
    eng.init()
    eng.loadRandomWeights(0)
    # A dedicated stream: the engine's kernels and the timing events share it (the
    # legacy default stream would not order with the engine's work).
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)
    utt = rank
    toks, a0, na = synth.prompt(utt, args.text, args.voice)
    voice = synth.voice_rows(utt, args.voice)
    eng.set_streams(3, 4, utt)
    eng.reset()
    eng.prefill(toks, a0, na, voice)
    eng.checkpoint()
    p0 = eng.position()

    def step():
        eng.rewind()
        eng.decode(F, with_fm=False)

    for _ in range(args.warmup):
        step()
    eng.synchronize()

    # ------------------------------------------------------------------ timed region
    vdist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local)
    time.sleep(0.3)
    l0 = eng.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_enqueue_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    e1.record(stream)
    torch.cuda.synchronize()
    vdist.barrier()
    clocks = clk.stop()
    launches = eng.launch_count() - l0
    ms = e0.elapsed_time(e1)
    ms_max = vdist.max_over_ranks(ms)
    frames_total = F * args.steps * world
    value = frames_total / (ms_max / 1e3)
    ms_per_step = ms_max / args.steps

    # ------------------------------------------------------------------ roofline of the GEMV kernel
    eng.rewind()
    eng.decode(F // 2, with_fm=False)           # profile at the middle of the decode window
    prof = eng.profile_step(reps=16)
    peak, peak_kind = measured_peaks()
    achieved = prof["gemv_bytes"] / (prof["gemv_ms"] / 1e3) / 1e9
    traffic = ncu_traffic()
    avg_pos = p0 + F / 2
    step_bytes = args.layers * BYTES_PER_LAYER + 6144 + avg_pos * KV_BYTES_PER_POS * args.layers / 26
    step_gbs = step_bytes * (F * args.steps) / (ms / 1e3) / 1e9

    # ------------------------------------------------------------------ end to end through the C ABI
    e2e_vals, h2d, d2h = [], 0, 0
    for i in range(2):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record(stream)
        eng.reset()
        eng.prefill(toks, a0, na, voice)                    # host tokens + voice rows -> device
        eng.decode(F, with_fm=False)
        codes = eng.read_codes(0, F)                        # device -> host
        normed = eng.read_normed(0, F)
        t1.record(stream)
        torch.cuda.synchronize()
        if i > 0:
            e2e_vals.append(F / (t0.elapsed_time(t1) / 1e3))
        h2d = toks.nbytes + voice.nbytes
        d2h = codes.nbytes + normed.nbytes
    e2e = vdist.sum_over_ranks(min(e2e_vals)) if world > 1 else e2e_vals[0]

    # ------------------------------------------------------------------ CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fps, n, dt, cores = cpu_sample(args.layers, args.cpu_seconds)
        cpu = {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
               "sample": f"{n} backbone frames of the {args.layers}-layer model at position {N_TEXT + N_VOICE + 5} "
                         f"(KV prefilled synthetically), {dt:.1f} s, oracle/oracle.cpp with OpenMP"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 weights, f32 math, f16 KV", "data": "synthetic",
            "config": {"workload": WORKLOAD, "frames_per_step": F, "prompt_positions": int(p0),
                       "layers": args.layers, "global_batch": world, "parallelism": f"dp{world}",
                       "l2": "inputs larger than L2: 6.05 GB of weights streamed per frame"},
            "roofline": {"bound": "hbm", "kernel": "k_gemv: the 104 weight-streaming GEMV launches of one "
                                                    "step, graph-launched as a chain, CUDA events",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "bytes_per_step": prof["gemv_bytes"], "gemv_ms_per_step": prof["gemv_ms"],
                         "attn_ms_per_step": prof["attn_ms"], "full_step_ms": prof["step_ms"],
                         "step_gbs": step_gbs, "step_frac": step_gbs / peak},
            "host_enqueue_ms_per_step": host_enqueue_ms,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": "frames/s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "includes": "prefill of 617 positions + 500-frame decode + readback of codes and hidden states"},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    eng.destroy()
    vdist.shutdown()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
