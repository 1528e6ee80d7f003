#!/usr/bin/env python
"""Benchmark: Voxtral backbone decode frames/s on B200 (BASELINE.json metric, config C2).

Workload (configs[1] of BASELINE.json): the full 26-layer Ministral-3B-shaped backbone,
f16 synthetic weights (seed 0, N(0,0.02)), prompt of 512 text ids + 100 voice rows
(617 positions, prefilled once before the timed region), then one STEP = a 500-frame
batch-1 decode (frame 0 is the AUDIO kick, frames 1..499 embed the previous frame's
37 codes) from the post-prefill checkpoint.  value = frames/s of the whole job.

  N = 1   : one utterance on one GPU.
  N > 1   : launched by torchrun, one process per GPU.  The headline is the batch-1
            latency path: ONE utterance decoded tensor-parallel over the N GPUs (heads and
            FFN columns sharded, two all-reduces per layer inside the persistent kernel
            over NVLink peer memory), strong scaling, device time = max over ranks.
            `--mode dp` instead runs N independent replicas (weak scaling).  The batched
            throughput leg (C4) is always data-parallel: every rank decodes its own 64
            utterances, and its frames/s is summed over ranks (time = max over ranks).

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
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="length of the cpu_baseline sample of the GPU arm (the reference arm times --steps steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", default="tp", choices=["dp", "tp"],
                    help="N > 1: tp = one utterance over N GPUs (strong scaling, default); dp = one utterance "
                         "per GPU (weak scaling)")
    ap.add_argument("--c3-frames", type=int, default=40, help="frames of the backbone+FM (C3) sample; 0 = skip")
    ap.add_argument("--c4-slots", type=int, default=64, help="utterances decoded in lockstep per GPU (C4)")
    ap.add_argument("--c4-frames", type=int, default=1500, help="frames of the batched (C4) run; 0 = skip")
    ap.add_argument("--c5-slots", type=int, default=16, help="utterances of the long-context (C5) run")
    ap.add_argument("--c5-context", type=int, default=32768, help="synthetic K/V positions per utterance (C5)")
    ap.add_argument("--c5-frames", type=int, default=256, help="frames of the long-context (C5) run; 0 = skip")
    ap.add_argument("--codec-frames", type=int, default=500, help="frames of the codec-decoder run; 0 = skip")
    ap.add_argument("--trace", action="store_true",
                    help="instead of the bench line: per-phase time breakdown of the persistent decode kernel "
                         "(vx_trace) on the C2 shape at the step's mean position, one JSON line")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    """DRAM bytes per decoded frame per layer of the persistent kernel (committed ncu summary)."""
    p = os.path.join(ROOT, "profiles", "k_decode_steps_c2.md")
    if not os.path.exists(p):
        return None
    m = re.search(r"dram_bytes_per_frame_per_layer:\s*([0-9.eE+]+)", open(p).read())
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


def nccl_lib_path():
    try:
        import nvidia.nccl
        p = os.path.join(list(nvidia.nccl.__path__)[0], "lib", "libnccl.so.2")
        return p if os.path.exists(p) else None
    except Exception:  # noqa: BLE001
        return None


def mean_position(args) -> int:
    """Mean KV position of a decode step: the prompt (text + voice + 5 control tokens)
    plus half the step's frames.  The CPU legs sample frames there, so the per-frame KV
    work matches the average frame of the GPU arm."""
    return args.text + args.voice + 5 + (args.frames - 1) // 2


def cpu_sample(args, seconds: float, n_frames_min: int = 2):
    """The CPU restatement (oracle/) on the host cores: decode frames at the step's mean position."""
    import oracle
    o = oracle.Oracle(n_layers=args.layers, max_seq=4096, with_fm=False)
    o.fill_kv(mean_position(args), seed=11)
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
    o.fill_kv(mean_position(args), seed=11)
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
                   f"position {start} (the mean position of a {args.frames}-frame step after a "
                   f"{args.text + args.voice + 5}-position prompt; KV prefilled with synthetic values) of the "
                   f"{args.layers}-layer model"},
        "cpu_baseline": {"value": value, "unit": "frames/s", "cores": cores, "kind": "port",
                         "sample": f"{frames_per_step} frames x {args.steps} steps at position {start}"},
        "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    o.close()
    return 0


def run_c4(args, vx, synth, local, stream, vdist, rank, world):
    """C4: S utterances per GPU (prompt 256 text ids + 100 voice rows each),
    decoded in lockstep for F frames with vx_decode_batch (tensor-core GEMMs over the
    slots, paged f16 KV).  Times the whole F-frame run with CUDA events (inputs resident)."""
    import torch
    S, F4 = args.c4_slots, args.c4_frames
    eng = vx.VoxtralEngine({"config": {"backbone": {"n_layers": args.layers}}, "maxSeqLen": 2048,
                            "maxFrames": F4 + 8, "enableFM": False, "device": local, "maxSlots": S})
    eng.init()
    eng.loadRandomWeights(0)
    eng.set_stream(stream.cuda_stream)
    p0 = None
    ub = 1000 + S * rank                      # every rank decodes its own utterances
    for u in range(S):
        toks, a0, na = synth.prompt(ub + u, 256, 100)
        eng.reset(slot=u)
        eng.set_streams(3, 4, ub + u, slot=u)
        eng.prefill(toks, a0, na, synth.voice_rows(ub + u, 100), slot=u)
        p0 = len(toks)
    eng.synchronize()
    for u in range(S):
        eng.checkpoint(slot=u)
    eng.decode_batch(4, S)                    # warm-up: graph capture
    for u in range(S):
        eng.rewind(slot=u)
    torch.cuda.synchronize()
    vdist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = eng.launch_count()
    e0.record(stream)
    eng.decode_batch(F4, S)
    e1.record(stream)
    torch.cuda.synchronize()
    vdist.barrier()
    ms = vdist.max_over_ranks(e0.elapsed_time(e1))
    launches = eng.launch_count() - l0
    eng.destroy()
    step_ms = ms / F4
    avg_pos = p0 + (F4 - 1) / 2
    step_bytes = args.layers * BYTES_PER_LAYER + 6144 + S * (37 * 3072 * 2 + (avg_pos + 1) * KV_BYTES_PER_POS * args.layers / 26)
    flops = 2.0 * S * args.layers * (BYTES_PER_LAYER / 2)
    peak, kind = measured_peaks()
    return {"workload": f"C4: {S} utterances per GPU in lockstep (prompt 256 text ids + 100 voice rows = {p0} positions "
                        f"each), {F4} frames, paged f16 KV, maxSeqLen 2048; weights streamed once per step for all slots; "
                        f"data-parallel over {world} GPU(s), frames/s summed over ranks, time = max over ranks",
            "frames_per_s": world * S * F4 / (ms / 1e3), "frames_per_s_per_gpu": S * F4 / (ms / 1e3),
            "parallelism": f"dp{world}", "ms_per_step": step_ms, "slots": S, "frames": F4,
            "avg_position": avg_pos, "gpu_launches": launches,
            "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": step_bytes,
                         "achieved": step_bytes / (step_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": step_bytes / (step_ms / 1e3) / 1e9 / peak, "peak_kind": kind},
            "tensor": {"gemm_tflops_per_step": flops / (step_ms / 1e3) / 1e12,
                       "note": "2 flops per weight per slot; the tensor cores run twice that (activations as f16 hi + lo)"}}


def run_c5(args, vx, local, stream, vdist, rank, tp):
    """C5: S utterances whose K/V cache holds P synthetic positions (f16
    N(0,1), vx_fill_kv), decoded F frames in lockstep (vx_decode_batch, split-KV
    attention).  The KV stream dominates: S * P * 106,496 bytes per step.  With tp > 1
    the utterances are decoded tensor-parallel over the ranks: each GPU holds 8/tp KV
    heads of every utterance (1 at TP-8) and 1/tp of the weights, with an NCCL
    all-reduce after o_proj and after down in every layer."""
    import torch
    S, P, F5 = args.c5_slots, args.c5_context, args.c5_frames
    eng = vx.VoxtralEngine({"config": {"backbone": {"n_layers": args.layers}}, "maxSeqLen": P + F5 + 8,
                            "maxFrames": F5 + 8, "enableFM": False, "enableCodec": False, "device": local,
                            "maxSlots": S, "maxVoiceRows": 1, "tpSize": tp, "tpRank": rank if tp > 1 else 0})
    eng.init()
    if tp > 1:
        lib = nccl_lib_path()
        uid = vdist.broadcast_bytes(vx.nccl_unique_id(lib) if rank == 0 else None)
        vx.tp_init(eng, uid, lib, p2p=False)
    eng.loadRandomWeights(0)
    eng.set_stream(stream.cuda_stream)
    for u in range(S):
        eng.reset(slot=u)
        eng.set_streams(3, 4, 2000 + u, slot=u)
        eng.fill_kv(P, seed=5000 + u, slot=u)
        eng.checkpoint(slot=u)
    eng.decode_batch(2, S)                    # warm-up: graph capture
    for u in range(S):
        eng.rewind(slot=u)
    torch.cuda.synchronize()
    vdist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    eng.decode_batch(F5, S)
    e1.record(stream)
    torch.cuda.synchronize()
    vdist.barrier()
    ms = vdist.max_over_ranks(e0.elapsed_time(e1))
    eng.destroy()
    step_ms = ms / F5
    avg_pos = P + (F5 - 1) / 2
    kv = S * (avg_pos + 1) * KV_BYTES_PER_POS * args.layers / 26 / tp
    step_bytes = (args.layers * BYTES_PER_LAYER + 6144) / tp + S * 37 * 3072 * 2 + kv
    peak, kind = measured_peaks()
    where = "one GPU" if tp == 1 else f"TP-{tp} (1/{tp} of the KV heads and weights per GPU, NCCL all-reduce x2 per layer)"
    return {"workload": f"C5 on {where}: {S} utterances with {P} synthetic f16 K/V positions each (vx_fill_kv), "
                        f"{F5} frames in lockstep, split-KV flash-decode over the paged cache",
            "frames_per_s": S * F5 / (ms / 1e3), "ms_per_step": step_ms, "slots": S, "frames": F5,
            "parallelism": f"tp{tp}" if tp > 1 else "single GPU",
            "avg_position": avg_pos, "kv_bytes_per_step_per_gpu": kv,
            "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": step_bytes,
                         "achieved": step_bytes / (step_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": step_bytes / (step_ms / 1e3) / 1e9 / peak, "peak_kind": kind}}


# Codec decoder FLOPs per frame (2 per weight per token): input conv 1024 x 292 x 3, 8
# layers over 30 token-layers per frame (stage s has 2^s tokens per frame, 2 layers)
# of 16.8 M weights, transposed convs (14 outputs per frame x 2 taps x 1024 x 1024),
# output conv (8 outputs per frame x 240 x 7168).
CODEC_FLOP_PER_FRAME = 2 * (1024 * 876 + 30 * 16777216 + 14 * 2 * 1024 * 1024 + 8 * 240 * 7168)


def measured_tflops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def run_codec(args, vx, local, stream):
    """codecDecode of one utterance of T frames (T * 1920 samples at 24 kHz), codes
    copied in and the waveform copied out inside the timed region."""
    import torch
    T = args.codec_frames
    eng = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 1}}, "maxSeqLen": 64, "maxFrames": 8,
                            "enableFM": False, "device": local, "maxVoiceRows": 1})
    eng.init()
    eng.loadRandomWeights(0)
    eng.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(7)
    sem = rng.integers(2, 8194, T).astype(np.uint32)
    ac = rng.integers(2, 23, (T, 36)).astype(np.uint32)
    for _ in range(3):
        eng.codecDecode(sem, ac)
    ts = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        audio = eng.codecDecode(sem, ac)
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    eng.destroy()
    ms = float(np.median(ts))
    flop = CODEC_FLOP_PER_FRAME * T
    peak, kind = measured_tflops()
    return {"workload": f"codec decoder: {T} frames -> {audio.size} samples ({audio.size / 24000:.1f} s at 24 kHz), "
                        "every projection and convolution a tcgen05 GEMM with hi/lo f16 activations",
            "ms": ms, "frames_per_s": T / (ms / 1e3), "realtime_factor": (audio.size / 24000) / (ms / 1e3),
            "roofline": {"bound": "tensor", "algorithmic_flop": flop, "achieved": flop / (ms / 1e3) / 1e12,
                         "peak": peak, "unit": "TFLOP/s", "frac": flop / (ms / 1e3) / 1e12 / peak, "peak_kind": kind,
                         "note": "two MMAs per K step (hi/lo activation halves), so the tensor pipe does 2x the "
                                 "algorithmic FLOPs"}}


def run_b200(args):
    import torch

    vx = importlib.import_module("webgpu-voxtral_b200")
    synth = importlib.import_module("webgpu-voxtral_b200.synth")
    vdist = importlib.import_module("webgpu-voxtral_b200.dist")
    rank, local, world = vdist.env_rank()
    torch.cuda.set_device(local)
    vdist.init(timeout_s=300)
    F = args.frames
    tp = world if (args.mode == "tp" and world > 1) else 1
    eng = vx.VoxtralEngine({"config": {"backbone": {"n_layers": args.layers}}, "maxSeqLen": 4096,
                            "maxFrames": max(1024, F + 8), "enableFM": args.c3_frames > 0, "device": local,
                            "tpSize": tp, "tpRank": rank if tp > 1 else 0})
    eng.init()
    if tp > 1:
        lib = nccl_lib_path()
        uid = vdist.broadcast_bytes(vx.nccl_unique_id(lib) if rank == 0 else None)
        vx.tp_init(eng, uid, lib)
    eng.loadRandomWeights(0)
    # A dedicated stream: the engine's kernels and the timing events share it (the
    # legacy default stream would not order with the engine's work).
    stream = torch.cuda.Stream(device=local)
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)
    utt = rank if tp == 1 else 0
    toks, a0, na = synth.prompt(utt, args.text, args.voice)
    voice = synth.voice_rows(utt, args.voice)
    eng.set_streams(3, 4, utt)
    eng.reset()
    eng.prefill(toks, a0, na, voice)
    eng.checkpoint()
    p0 = eng.position()

    # time-to-first-frame: the batched prefill of the prompt (tensor-core GEMMs)
    pf_ms = []
    for _ in range(3):
        eng.reset()
        torch.cuda.synchronize()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q0.record(stream)
        eng.prefill(toks, a0, na, voice)
        q1.record(stream)
        torch.cuda.synchronize()
        pf_ms.append(q0.elapsed_time(q1))
    eng.checkpoint()
    prefill = {"positions": int(p0), "ms": min(pf_ms),
               "gemm_tflops": 2.0 * p0 * args.layers * (BYTES_PER_LAYER / 2) / (min(pf_ms) / 1e3) / 1e12,
               "note": "batched prefill: every projection one tcgen05 GEMM over <=512 positions, "
                       "activations as an f16 hi/lo pair (2 MMAs per K step; TFLOP/s counts 2 flops per weight "
                       "per position once)"}

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
    frames_total = F * args.steps * (world if tp == 1 else 1)
    value = frames_total / (ms_max / 1e3)
    ms_per_step = ms_max / args.steps

    # ------------------------------------------------------------------ roofline of the decode kernel
    # One step is one launch of the persistent decode kernel (k_decode_steps) over F frames.
    # Algorithmic bytes per launch: every frame streams all f16 weights once, reads the f16 KV
    # of its position and the 37 embedding rows.
    peak, peak_kind = measured_peaks()
    avg_pos = p0 + (F - 1) / 2
    frame_bytes = (args.layers * BYTES_PER_LAYER + 6144 + 37 * 3072 * 2
                   + (avg_pos + 1) * KV_BYTES_PER_POS * args.layers / 26) / tp
    launch_bytes = F * frame_bytes
    achieved = launch_bytes / (ms_per_step / 1e3) / 1e9
    # ncu traffic of the weight stream per frame-layer (small-case capture), scaled to this
    # launch, plus the algorithmic KV bytes (they grow with the position, not the units).
    per_layer = ncu_traffic()
    kv_bytes = F * (avg_pos + 1) * KV_BYTES_PER_POS * args.layers / 26 / tp
    traffic = per_layer * args.layers * F / tp + kv_bytes if per_layer else None
    prof = None
    if tp == 1:
        eng.rewind()
        eng.decode(F // 2, with_fm=False)
        prof = eng.profile_step(reps=8)       # the per-op kernel path, for comparison

    # ------------------------------------------------------------------ C3 sample: backbone + FM per frame
    c3 = None
    if args.c3_frames > 0:
        eng.rewind()
        eng.set_sampling("top_p", 0.9, 0.8, seed=1)   # generate()'s sampleTopP(semLogits, 0.9, 0.8)
        eng.backboneStep(24)                       # AUDIO kick: frame 0's hidden state
        eng.decode(2, with_fm=True)                # warm-up (captures the FM graph)
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        eng.decode(args.c3_frames, with_fm=True)
        c1.record(stream)
        torch.cuda.synchronize()
        c3_ms = vdist.max_over_ranks(c0.elapsed_time(c1)) / args.c3_frames
        eng.set_sampling("argmax")
        c3 = {"frames_per_s": 1e3 / c3_ms, "ms_per_frame": c3_ms, "frames": args.c3_frames,
              "workload": "C3: one backbone step + FM (7 Euler steps, CFG as batch 2, M=6 skinny GEMMs) + "
                          "semantic code by the reference's top-p sampler (p 0.9, temperature 0.8, seeded draws) "
                          f"per frame, device-resident; {'one GPU' if tp == 1 else f'tensor-parallel over {tp} GPUs'}",
              "fm_bytes_per_frame": 4961851392,
              "frame_gbs": (frame_bytes + 4961851392) / (c3_ms / 1e3) / 1e9}

    # ------------------------------------------------------------------ C4: batched lockstep decode
    c4 = None
    if args.c4_frames > 0:
        c4 = run_c4(args, vx, synth, local, stream, vdist, rank, world)

    codec = None
    if args.codec_frames > 0 and tp == 1 and rank == 0:
        codec = run_codec(args, vx, local, stream)

    c5 = None
    if args.c5_frames > 0:
        c5 = run_c5(args, vx, local, stream, vdist, rank, tp)

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
    # frames/s of the whole job: the slowest rank's time (TP: one utterance; DP: one per rank)
    e2e = (world if tp == 1 else 1) * vdist.min_over_ranks(min(e2e_vals))

    # ------------------------------------------------------------------ CPU baseline (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        fps, n, dt, cores = cpu_sample(args, args.cpu_seconds)
        cpu = {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
               "sample": f"{n} backbone frames of the {args.layers}-layer model at position {mean_position(args)} "
                         f"(the step's mean position; KV prefilled synthetically), {dt:.1f} s, oracle/oracle.cpp "
                         "with OpenMP"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak" if tp == 1 else "strong",
            "vs_baseline": None, "dtype": "f16 weights, f32 math, f16 KV", "data": "synthetic",
            "config": {"workload": WORKLOAD, "frames_per_step": F, "prompt_positions": int(p0),
                       "layers": args.layers, "global_batch": world if tp == 1 else 1,
                       "parallelism": f"dp{world}" if tp == 1 else f"tp{tp}",
                       "l2": "inputs larger than L2: 6.05 GB of weights streamed per frame"},
            "roofline": {"bound": "hbm", "kernel": "k_decode_steps (persistent decode kernel, one launch per step)"
                                                    if tp == 1 else
                                                    f"k_decode_steps<{tp}> (persistent decode kernel per rank, "
                                                    "all-reduces over peer memory inside the kernel)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "traffic": traffic, "algorithmic_bytes_per_launch": launch_bytes,
                         "launch_ms": ms_per_step,
                         "per_op_path": None if prof is None else {
                             "gemv_chain_gbs": prof["gemv_bytes"] / (prof["gemv_ms"] / 1e3) / 1e9,
                             "gemv_ms_per_frame": prof["gemv_ms"], "attn_ms_per_frame": prof["attn_ms"],
                             "full_ms_per_frame": prof["step_ms"]}},
            "c3_backbone_plus_fm": c3,
            "prefill": prefill,
            "c4_batched": c4,
            "c5_long_context": c5,
            "codec": codec,
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


def run_trace(args):
    """Phase breakdown of k_decode_steps (one GPU): frames/s at the step's mean position, then
    the per-phase spans, hand-off gaps and consumer waits of the second traced step."""
    import torch
    vx = importlib.import_module("webgpu-voxtral_b200")
    vdist = importlib.import_module("webgpu-voxtral_b200.dist")
    rank, local, world = vdist.env_rank()
    torch.cuda.set_device(local)
    vdist.init(timeout_s=300)
    if world > 4:   # the persistent kernel serves tensor-parallel degrees up to 4
        if rank == 0:
            print(json.dumps({"trace": "k_decode_steps phase breakdown", "tp": world,
                              "unavailable": "the persistent decode kernel is not used at this degree"}), flush=True)
        vdist.shutdown()
        return 0
    L = args.layers
    pos = mean_position(args)
    eng = vx.VoxtralEngine({"config": {"backbone": {"n_layers": L}}, "maxSeqLen": 4096, "maxFrames": 1024,
                            "enableFM": False, "enableCodec": False, "device": local, "tpSize": world,
                            "tpRank": rank})
    eng.init()
    if world > 1:
        lib = nccl_lib_path()
        uid = vdist.broadcast_bytes(vx.nccl_unique_id(lib) if rank == 0 else None)
        vx.tp_init(eng, uid, lib)
    eng.loadRandomWeights(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    eng.set_stream(stream.cuda_stream)
    eng.set_streams(3, 4, 0)
    eng.fill_kv(pos, seed=5)
    eng.checkpoint()
    ms = []
    for i in range(4):
        eng.rewind()
        torch.cuda.synchronize()
        vdist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        eng.decode(100, with_fm=False)
        b.record(stream)
        torch.cuda.synchronize()
        if i:
            ms.append(vdist.max_over_ranks(a.elapsed_time(b) / 100))
    eng.rewind()
    eng.trace_arm()
    eng.decode(4, with_fm=False)
    eng.synchronize()
    tr = eng.trace_read().astype(np.int64)[:, 1]   # [cta, phase, slot] of the second step
    eng.destroy()
    vdist.barrier()
    vdist.shutdown()
    if rank != 0:
        return 0
    t0 = tr[:, 0, 0].min()
    rel, done, arr, pro = (tr[:, :, i] - t0 for i in range(4))
    names = ["qkv", "attention", "o_proj", "gate_up", "down"]
    mhz = float(os.environ.get("SM_MHZ", "1965"))
    phases = {}
    for j, nm in enumerate(names):
        ks = [1 + 5 * l + j for l in range(L)]
        span = np.mean([np.median(rel[:, k + 1]) - np.median(rel[:, k]) for k in ks]) / 1e3
        d = {"span_us": span,
             "consumers_median_us": np.mean([np.median(done[:, k] - rel[:, k]) for k in ks]) / 1e3,
             "consumers_max_us": np.mean([np.max(done[:, k] - rel[:, k]) for k in ks]) / 1e3}
        if nm == "attention":
            # CTAs holding an attention item: stamps of its K/V pair landing, split partial
            # stored, merge ticket taken, relative to the phase's release
            for slot, key in ((4, "kv_pair_in_smem_us"), (5, "partial_stored_us"), (6, "ticket_taken_us")):
                v = [np.median(tr[tr[:, k, slot] > 0, k, slot] - rel[tr[:, k, slot] > 0, k] - t0) for k in ks
                     if (tr[:, k, slot] > 0).any()]
                if v:
                    d[key] = float(np.mean(v)) / 1e3
        else:
            d["prologue_us"] = np.mean([np.median(pro[:, k] - rel[:, k]) for k in ks]) / 1e3
            d["epilogue_lag_us"] = np.mean([arr[:, k].max() - done[:, k].max() for k in ks]) / 1e3
            d["stage_wait_us"] = np.mean([np.median(tr[:, k, 4]) for k in ks]) / mhz
            d["reduction_slot_wait_us"] = np.mean([np.median(tr[:, k, 5]) for k in ks]) / mhz
        phases[nm] = {k: round(float(v), 3) for k, v in d.items()}
    step_us = (np.median(rel[:, -1]) - np.median(rel[:, 0])) / 1e3
    print(json.dumps({"trace": "k_decode_steps phase breakdown", "layers": L, "position": pos, "tp": world,
                      "ms_per_frame": min(ms), "traced_step_us": float(step_us), "us_per_layer": float(step_us / L),
                      "phases": phases, "note": "spans: median release to the next phase's median release; "
                      "waits converted from SM cycles at SM_MHZ (default 1965)"}), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.trace:
        return run_trace(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
