"""Tensor-core (tcgen05 / TMEM) token-batch path: the GEMM itself, and the batched
prefill that replaces the reference's token-by-token prefill loop
(src/engine.ts:2457-2472) against the token-by-token path and the CPU oracle."""
import numpy as np
import pytest

import oracle
from conftest import max_abs_rel

pytestmark = pytest.mark.gpu
TOL = 2e-2           # reference tolerance (per-tensor max-abs-rel) against the oracle
TOL_PATHS = 1e-3     # batched vs token-by-token prefill: same f32 arithmetic up to summation order
TOL_GEMM = 2e-5      # tensor-core GEMM (f16 W x hi/lo f16 X, f32 accumulate) vs f32 CUDA-core product


@pytest.fixture(scope="module")
def eng(vx):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 1024, "maxFrames": 64,
                          "enableFM": False})
    e.init()
    e.loadRandomWeights(0)
    yield e
    e.destroy()


@pytest.mark.parametrize("M,N,K,bn,splits", [
    (128, 1, 64, 128, 1),          # one tile, one K chunk, one token
    (384, 100, 3072, 128, 1),      # ragged token tile
    (6144, 512, 3072, 128, 8),     # QKV of a 512-token batch
    (3072, 77, 9216, 128, 8),      # down projection, split-K
    (256, 64, 4096, 64, 4),        # narrow tile, split-K
    (512, 300, 1024, 256, 2),      # wide tile, two token tiles (second ragged)
    (6144, 6, 3072, 16, 3),        # the acoustic transformer's 6 rows, QKV shape
    (3072, 6, 9216, 16, 8),        # its down projection, split-K
    (384, 40, 1024, 16, 1),        # 16-row tiles over a ragged 40-row batch
])
def test_tc_gemm_selftest(eng, M, N, K, bn, splits):
    e_store, e_acc = eng.selftest_gemm(M, N, K, bn=bn, max_splits=splits, seed=M + N + K)
    assert e_store < TOL_GEMM, e_store
    assert e_acc < TOL_GEMM, e_acc


def _kick_layers(vx, synth, utt, T, R, batched):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 1024, "maxFrames": 16,
                          "enableFM": False})
    e.init()
    try:
        e.set_option("batched_prefill", 1 if batched else 0)
        e.loadRandomWeights(0)
        toks, a0, na = synth.prompt(utt, T, R)
        e.prefill(toks, a0, na, synth.voice_rows(utt, R))
        pos = e.position()
        raw = e.debugBackboneLayerByLayer(24)["raw"]
        return pos, raw
    finally:
        e.destroy()


def test_batched_prefill_matches_token_by_token(vx, synth):
    """600 prompt positions = two token batches (512 + 88): every per-layer tensor of
    the step after prefill agrees with the token-by-token prefill."""
    pa, a = _kick_layers(vx, synth, 7, 560, 35, batched=True)
    pb, b = _kick_layers(vx, synth, 7, 560, 35, batched=False)
    assert pa == pb == 600
    for i in range(a.shape[0]):
        assert max_abs_rel(a[i], b[i]) < TOL_PATHS, i


def test_batched_prefill_then_decode_matches_oracle(eng, synth):
    """Batched prefill of 545 positions, then backbone-only decode, against the oracle."""
    toks, a0, na = synth.prompt(8, 500, 40)
    voice = synth.voice_rows(8, 40)
    n = 6
    codes_in = synth.feedback_codes(9, 0, n)
    o = oracle.Oracle(n_layers=2, max_seq=1024, with_fm=False)
    ref = o.generate(toks, a0, na, voice, n, codes_in=codes_in, want_normed=True)
    o.close()
    eng.reset()
    eng.set_streams(noise_seed=3, codes_seed=4, utt=9)
    eng.prefill(toks, a0, na, voice)
    assert eng.position() == len(toks)
    eng.decode(n, with_fm=False)
    got = eng.read_normed(0, n)
    for f in range(n):
        assert max_abs_rel(got[f], ref["normed"][f]) < TOL, f


def _prefill_slots(e, synth, n, base_utt=20):
    """Slots 0..n-1 hold different prompts (different lengths, so different positions)."""
    for s in range(n):
        u = base_utt + s
        toks, a0, na = synth.prompt(u, 40 + 13 * s, 6 + s)
        e.reset(slot=s)
        e.set_streams(noise_seed=3, codes_seed=4, utt=u, slot=s)
        e.prefill(toks, a0, na, synth.voice_rows(u, 6 + s), slot=s)


def test_batched_decode_matches_per_slot_decode(vx, synth):
    """vx_decode_batch over 8 slots (tensor-core GEMMs, one row per slot) reproduces the
    batch-1 decode of each slot: same feedback codes, same normed states."""
    n, frames = 8, 10
    cfg = {"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 1024, "maxFrames": 64, "enableFM": False,
           "maxSlots": n}
    a = vx.VoxtralEngine(cfg)
    a.init()
    a.loadRandomWeights(0)
    try:
        _prefill_slots(a, synth, n)
        a.decode_batch(frames, n)
        got = [a.read_normed(0, frames, slot=s) for s in range(n)]
        got_codes = [a.read_codes(0, frames - 1, slot=s) for s in range(n)]
        pos = [a.position(s) for s in range(n)]
        _prefill_slots(a, synth, n)
        for s in range(n):
            a.decode(frames, with_fm=False, slot=s)
        for s in range(n):
            ref = a.read_normed(0, frames, slot=s)
            assert np.array_equal(got_codes[s], a.read_codes(0, frames - 1, slot=s)), s
            assert pos[s] == a.position(s), s
            for f in range(frames):
                assert max_abs_rel(got[s][f], ref[f]) < TOL_PATHS, (s, f)
    finally:
        a.destroy()


def test_batched_decode_matches_oracle(vx, synth):
    """One slot of a batched decode against the CPU oracle (reference tolerance)."""
    n, frames = 4, 6
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 1024, "maxFrames": 64,
                          "enableFM": False, "maxSlots": n})
    e.init()
    e.loadRandomWeights(0)
    try:
        _prefill_slots(e, synth, n, base_utt=30)
        e.decode_batch(frames, n)
        s = 2
        u = 30 + s
        toks, a0, na = synth.prompt(u, 40 + 13 * s, 6 + s)
        o = oracle.Oracle(n_layers=2, max_seq=1024, with_fm=False)
        ref = o.generate(toks, a0, na, synth.voice_rows(u, 6 + s), frames,
                         codes_in=synth.feedback_codes(u, 0, frames), want_normed=True)
        o.close()
        got = e.read_normed(0, frames, slot=s)
        for f in range(frames):
            assert max_abs_rel(got[f], ref["normed"][f]) < TOL, f
    finally:
        e.destroy()


def test_long_context_fill_and_batched_decode_matches_oracle(vx, synth):
    """Long-context form (C5): a synthetic 3000-position K/V context per slot
    (vx_fill_kv), then batched decode with split-KV attention, against the oracle
    filled with the same generator (f32 there, f16 in the engine's cache)."""
    n, frames, npos = 3, 4, 3000
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 3072, "maxFrames": 16,
                          "enableFM": False, "maxSlots": n})
    e.init()
    e.loadRandomWeights(0)
    try:
        for s in range(n):
            e.reset(slot=s)
            e.set_streams(noise_seed=3, codes_seed=4, utt=40 + s, slot=s)
            e.fill_kv(npos, seed=100 + s, slot=s)
        assert e.position(1) == npos
        e.decode_batch(frames, n)
        s = 1
        o = oracle.Oracle(n_layers=2, max_seq=3072, with_fm=False)
        o.fill_kv(npos, seed=100 + s)
        codes = synth.feedback_codes(40 + s, 0, frames)
        ref = [o.backbone_step(24)["normed"]]
        for f in range(1, frames):
            emb = o.multi_codebook_embed(int(codes[f - 1][0]), codes[f - 1][1:])
            ref.append(o.backbone_step(embed=emb)["normed"])
        o.close()
        got = e.read_normed(0, frames, slot=s)
        assert np.array_equal(e.read_codes(0, frames - 1, slot=s), codes[: frames - 1])
        for f in range(frames):
            assert max_abs_rel(got[f], ref[f]) < TOL, f
    finally:
        e.destroy()
