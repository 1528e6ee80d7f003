"""Device top-p sampler (k_fm_sample / k_top_p_test through the C ABI) against the oracle's
restatement of sampleTopP (src/engine.ts:247-289).  The result is an index, so the bar
is equality.  The device adds the probabilities in a tree, the reference in sequence;
the two orders can disagree only when a running sum lies within ~1e-12 of its
threshold, so every draw is also required to clear that margin in the oracle (a draw
that did not would make the comparison meaningless rather than fail it)."""
import numpy as np
import pytest

from oracle import sampling

pytestmark = pytest.mark.gpu
MARGIN = 1e-10


@pytest.fixture(scope="module")
def eng(vx):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 512, "maxFrames": 64})
    e.init()
    e.loadRandomWeights(0)
    yield e
    e.destroy()


def _draws(rng, k):
    return np.concatenate([[0.0, 1.0 - 2.0 ** -53, 0.5], rng.random(k - 3)])


def _rows(rng):
    n = 8320
    flat = rng.normal(size=n).astype(np.float32)                   # random weights: thousands in the nucleus
    peaked = (rng.normal(size=n) * 6).astype(np.float32)           # a handful in the nucleus
    ties = np.round(rng.normal(size=n) * 2).astype(np.float32)     # many equal probabilities
    one = np.full(n, -30.0, np.float32)
    one[4000] = 10.0
    equal = np.zeros(n, np.float32)   # one run of 8193 equal probabilities: every running sum is exact
                                      # on both sides, so draws may land exactly on one
    return [("flat", flat, 0.9, 0.8), ("peaked", peaked, 0.9, 0.8), ("ties", ties, 0.9, 0.8), ("equal", equal, 0.9, 0.8),
            ("one", one, 0.9, 0.8), ("over_1", flat, 1.5, 0.8), ("top_p_0", ties, 0.0, 0.8),
            ("hot", flat, 0.5, 3.0), ("cold", flat, 0.95, 0.1)]


def test_top_p_selftest_matches_oracle(eng):
    rng = np.random.default_rng(11)
    for name, lg, top_p, temp in _rows(rng):
        u = _draws(rng, 48)
        got = eng.selftest_top_p(lg, u, top_p, temp, valid_lo=1, valid_hi=8194)
        masked = sampling.mask_semantic(lg)
        for k, uk in enumerate(u):
            want, margin = sampling.sample_top_p(masked, top_p, temp, uk, return_margin=True)
            assert margin > MARGIN or name == "equal", (name, k)
            assert got[k] == want, (name, k, got[k], want)


@pytest.mark.parametrize("n", [1, 2, 37, 1024, 1025, 16384])
def test_top_p_selftest_sizes(eng, n):
    rng = np.random.default_rng(n)
    lg = (rng.normal(size=n) * 2).astype(np.float32)
    u = _draws(rng, 16)
    got = eng.selftest_top_p(lg, u, 0.9, 0.8)
    for k, uk in enumerate(u):
        want, margin = sampling.sample_top_p(lg, 0.9, 0.8, uk, return_margin=True)
        assert margin > MARGIN
        assert got[k] == want, (k, got[k], want)


def test_fm_graph_samples_like_the_reference(eng, synth):
    """Inside the FM graph: each frame's code is sampleTopP(masked logits, 0.9, 0.8) with
    the frame's draw from the seeded stream, on the engine's own logits."""
    toks, a0, na = synth.prompt(8, 12, 4)
    eng.reset()
    eng.set_streams(noise_seed=3, codes_seed=4, utt=8)
    eng.set_sampling("top_p", 0.9, 0.8, seed=21)
    eng.prefill(toks, a0, na, synth.voice_rows(8, 4))
    eng.backboneStep(24)
    key = synth.sample_key(21)
    codes = []
    for f in range(6):
        r = eng.debugFMStep()
        u = float(synth.uniform01(key, np.array([f], np.uint64))[0])
        want, margin = sampling.sample_top_p(sampling.mask_semantic(r["semantic_logits"]), 0.9, 0.8, u,
                                             return_margin=True)
        assert margin > MARGIN
        assert r["semantic_code"] == want, f
        codes.append(want)
        if want > 1:
            eng.backboneStepCodes(want, r["acoustic_codes"])
    assert len(set(codes)) > 1
    eng.set_sampling("argmax")


def test_decode_top_p_zero_is_argmax(eng, synth):
    """top_p 0 at temperature 1 keeps only the most probable code: the free-running decode
    must then reproduce the masked-argmax decode frame for frame."""
    toks, a0, na = synth.prompt(9, 10, 2)
    eng.reset()
    eng.set_streams(noise_seed=3, codes_seed=4, utt=9)
    eng.set_sampling("argmax")
    eng.prefill(toks, a0, na, synth.voice_rows(9, 2))
    eng.backboneStep(24)
    eng.checkpoint()
    eng.decode(8, with_fm=True)
    a = eng.read_codes(0, 8)
    eng.rewind()
    eng.set_sampling("top_p", 0.0, 1.0, seed=5)
    eng.decode(8, with_fm=True)
    b = eng.read_codes(0, 8)
    eng.set_sampling("argmax")
    assert np.array_equal(a, b)


def test_decode_sampling_is_seeded(eng, synth):
    toks, a0, na = synth.prompt(10, 10, 2)
    eng.reset()
    eng.set_streams(noise_seed=3, codes_seed=4, utt=10)
    eng.prefill(toks, a0, na, synth.voice_rows(10, 2))
    eng.backboneStep(24)
    eng.checkpoint()
    runs = []
    for seed in (1, 1, 2):
        eng.rewind()
        eng.set_sampling("top_p", 0.9, 0.8, seed=seed)
        eng.decode(8, with_fm=True)
        runs.append(eng.read_codes(0, 8))
    eng.set_sampling("argmax")
    assert np.array_equal(runs[0], runs[1])
    assert not np.array_equal(runs[0][:, 0], runs[2][:, 0])
    assert np.all((runs[0][:, 0] >= 1) & (runs[0][:, 0] < 8194))


def test_generate_top_p(vx, synth):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 256, "maxFrames": 32,
                          "sampling": "top_p", "samplingSeed": 4})
    e.init()
    e.loadRandomWeights(0)
    toks, a0, na = synth.prompt(4, 8, 2)
    a = e.generate(toks, a0, na, synth.voice_rows(4, 2), maxFrames=6, eos=False)
    b = e.generate(toks, a0, na, synth.voice_rows(4, 2), maxFrames=6, eos=False)
    e.destroy()
    assert a.semanticCodes == b.semanticCodes and len(a.semanticCodes) == 6
    assert all(1 <= c < 8194 for c in a.semanticCodes)


def test_sampling_arguments_checked(eng, vx):
    with pytest.raises(vx.VoxtralError):
        eng.set_sampling("top_p", 0.9, 0.0)
    with pytest.raises(vx.VoxtralError):
        eng.set_sampling("top_p", float("nan"), 0.8)
    with pytest.raises(ValueError):
        eng.set_sampling("greedy")
