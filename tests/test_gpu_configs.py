"""Parity on the benchmark's own configurations (BASELINE.json configs[1..4]), not only the
2-layer shape: the CUDA path through the C ABI against the CPU oracle, at full depth and
width.  Tolerance (north_star): per-tensor max|a-b| / max|b| <= 2e-2; semantic codes
identical on >= 99 % of frames; acoustic codes identical on >= 99 % of elements.

* C2 depth: 26 layers, the 617-position C2 prompt through the batched prefill, then 16
  frames of the persistent decode kernel, against tests/golden/c2_depth.npz (the oracle
  is too slow to prefill 617 positions at 26 layers inside a test).
* Per-layer state of the benchmarked kernel at 26 layers: vx_decode_record and
  debugBackboneLayerByLayer (both the persistent decode kernel) against the oracle's
  per-layer tensors (src/engine.ts:2106-2287), on a synthetic 900-position context.
* C3 depth: 26 layers + the acoustic transformer, 32 frames, masked argmax; the oracle is
  teacher-forced with the engine's codes so that both sides see the same history.
* C4 width: 64 slots decoded in lockstep by vx_decode_batch; 4 slots against the oracle.
* C5 context: 32,768 synthetic K/V positions (f16 in the engine, f32 in the oracle),
  through the batched path and the persistent kernel.
"""
import os

import numpy as np
import pytest

import oracle
from conftest import ROOT, max_abs_rel

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _print(msg):
    print(msg, flush=True)


@pytest.fixture(scope="module")
def orc26():
    o = oracle.Oracle(n_layers=26, max_seq=1100, with_fm=True)
    yield o
    o.close()


def test_c2_depth_matches_golden(vx, synth):
    g = np.load(os.path.join(ROOT, "tests", "golden", "c2_depth.npz"))
    utt, n_frames = int(g["utt"]), g["normed"].shape[0]
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": int(g["n_layers"])}}, "maxSeqLen": 1024,
                          "maxFrames": 64, "enableFM": False, "enableCodec": False})
    e.init()
    try:
        e.loadRandomWeights(0)
        toks, a0, na = synth.prompt(utt, int(g["n_text"]), int(g["n_voice"]))
        e.set_streams(noise_seed=3, codes_seed=4, utt=utt)
        e.prefill(toks, a0, na, synth.voice_rows(utt, int(g["n_voice"])))
        assert e.position() == int(g["positions"]) == 617
        e.decode(n_frames, with_fm=False)
        got = e.read_normed(0, n_frames)
        assert np.array_equal(e.read_codes(0, n_frames - 1), synth.feedback_codes(utt, 0, n_frames - 1))
        errs = [max_abs_rel(got[f], g["normed"][f]) for f in range(n_frames)]
        _print(f"C2 depth: max-abs-rel per frame max {max(errs):.3e} (frame 0 {errs[0]:.3e})")
        assert max(errs) < TOL, errs
    finally:
        e.destroy()


def test_per_layer_record_26_layers(vx, synth, orc26):
    """The persistent kernel's per-layer tensors at full depth, inside a multi-frame decode
    (vx_decode_record) and as debugBackboneLayerByLayer."""
    npos, utt, n, rec = 900, 12, 6, 4
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 26}}, "maxSeqLen": 1024, "maxFrames": 64,
                          "enableFM": False, "enableCodec": False})
    e.init()
    try:
        e.loadRandomWeights(0)
        e.set_streams(noise_seed=3, codes_seed=4, utt=utt)
        e.fill_kv(npos, seed=77)
        got = e.decode_record(n, rec)
        normed = e.read_normed(0, n)
        codes = synth.feedback_codes(utt, 0, n)
        orc26.fill_kv(npos, seed=77)
        ref = orc26.backbone_step(24, debug=(rec == 0))
        worst_norm = max_abs_rel(normed[0], ref["normed"])
        for f in range(1, n):
            emb = orc26.multi_codebook_embed(int(codes[f - 1][0]), codes[f - 1][1:])
            ref = orc26.backbone_step(embed=emb, debug=(f == rec))
            worst_norm = max(worst_norm, max_abs_rel(normed[f], ref["normed"]))
            if f == rec:
                dbg = ref["debug"]
        errs = [max_abs_rel(got[i], dbg[i]) for i in range(dbg.shape[0])]
        _print(f"26-layer record (frame {rec} of {n}): worst row {int(np.argmax(errs))} {max(errs):.3e}; "
               f"normed {worst_norm:.3e}")
        assert max(errs) < TOL, (int(np.argmax(errs)), max(errs))
        assert worst_norm < TOL
        # debugBackboneLayerByLayer on the same kernel, next position
        d = e.debugBackboneLayerByLayer(24)["raw"]
        ref = orc26.backbone_step(24, debug=True)["debug"]
        errs = [max_abs_rel(d[i], ref[i]) for i in range(ref.shape[0])]
        _print(f"26-layer debugBackboneLayerByLayer: worst {max(errs):.3e}")
        assert max(errs) < TOL, (int(np.argmax(errs)), max(errs))
    finally:
        e.destroy()


def test_c3_depth_teacher_forced(vx, synth, orc26):
    """26 layers + FM, 32 frames, masked argmax.  Frame f of the oracle runs on the codes
    the engine chose for frame f-1, so every frame compares the same computation."""
    npos, utt, n = 617, 13, 32
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 26}}, "maxSeqLen": 1024, "maxFrames": 64,
                          "enableFM": True, "enableCodec": False})
    e.init()
    try:
        e.loadRandomWeights(0)
        e.set_streams(noise_seed=3, codes_seed=4, utt=utt)
        e.fill_kv(npos, seed=91)
        e.backboneStep(24)
        e.decode(n, with_fm=True)
        codes = e.read_codes(0, n)
        normed = e.read_normed(1, n - 1)
    finally:
        e.destroy()
    noise = synth.fm_noise(utt, 0, n)
    orc26.fill_kv(npos, seed=91)
    orc26.backbone_step(24)
    sem_ok, ac_ok, worst = 0, 0, 0.0
    for f in range(n):
        if f > 0:
            emb = orc26.multi_codebook_embed(int(codes[f - 1][0]), codes[f - 1][1:])
            st = orc26.backbone_step(embed=emb)
            worst = max(worst, max_abs_rel(normed[f - 1], st["normed"]))
        r = orc26.fm_forward(noise[f])
        sem_ok += int(r["semantic_code"] == codes[f][0])
        ac_ok += int(np.sum(r["acoustic_codes"] == codes[f][1:]))
    _print(f"C3 depth: semantic {sem_ok}/{n}, acoustic {ac_ok}/{36 * n}, normed max-abs-rel {worst:.3e}")
    assert worst < TOL
    assert sem_ok >= 0.99 * n
    assert ac_ok >= 0.99 * 36 * n


def test_c4_width_64_slots(vx, synth):
    """64 slots in lockstep (C4's width), 2 layers; slots 0, 21, 42, 63 against the oracle."""
    S, frames = 64, 6
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 256, "maxFrames": 16,
                          "enableFM": False, "enableCodec": False, "maxSlots": S, "maxVoiceRows": 32})
    e.init()
    try:
        e.loadRandomWeights(0)
        prompts = {}
        for s in range(S):
            u = 300 + s
            toks, a0, na = synth.prompt(u, 40 + (s % 7) * 5, 8 + s % 5)
            prompts[s] = (toks, a0, na, synth.voice_rows(u, na))
            e.reset(slot=s)
            e.set_streams(noise_seed=3, codes_seed=4, utt=u, slot=s)
            e.prefill(*prompts[s], slot=s)
        e.decode_batch(frames, S)
        o = oracle.Oracle(n_layers=2, max_seq=256, with_fm=False)
        worst = 0.0
        for s in (0, 21, 42, 63):
            toks, a0, na, voice = prompts[s]
            ref = o.generate(toks, a0, na, voice, frames, codes_in=synth.feedback_codes(300 + s, 0, frames),
                             want_normed=True)
            got = e.read_normed(0, frames, slot=s)
            worst = max(worst, max(max_abs_rel(got[f], ref["normed"][f]) for f in range(frames)))
        o.close()
        _print(f"C4 width (64 slots): worst max-abs-rel {worst:.3e}")
        assert worst < TOL
    finally:
        e.destroy()


@pytest.mark.parametrize("path", ["batched", "persistent"])
def test_c5_32k_context(vx, synth, path):
    """32,768 synthetic f16 K/V positions (the C5 context) against the oracle's f32 cache."""
    npos, frames = 32768, 3
    S = 2 if path == "batched" else 1
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": npos + 64, "maxFrames": 16,
                          "enableFM": False, "enableCodec": False, "maxSlots": S, "maxVoiceRows": 1})
    e.init()
    try:
        e.loadRandomWeights(0)
        for s in range(S):
            e.reset(slot=s)
            e.set_streams(noise_seed=3, codes_seed=4, utt=500 + s, slot=s)
            e.fill_kv(npos, seed=900 + s, slot=s)
        if path == "batched":
            e.decode_batch(frames, S)
        else:
            e.decode(frames, with_fm=False)
        s = S - 1
        got = e.read_normed(0, frames, slot=s)
    finally:
        e.destroy()
    o = oracle.Oracle(n_layers=2, max_seq=npos + 64, with_fm=False)
    o.fill_kv(npos, seed=900 + s)
    codes = synth.feedback_codes(500 + s, 0, frames)
    errs = [max_abs_rel(got[0], o.backbone_step(24)["normed"])]
    for f in range(1, frames):
        emb = o.multi_codebook_embed(int(codes[f - 1][0]), codes[f - 1][1:])
        errs.append(max_abs_rel(got[f], o.backbone_step(embed=emb)["normed"]))
    o.close()
    _print(f"C5 32k context ({path}): max-abs-rel per frame {', '.join(f'{x:.3e}' for x in errs)}")
    assert max(errs) < TOL
