"""Host-side logic of the VoxtralEngine mirror and the sampler oracle (no GPU)."""
import math
import struct

import numpy as np
import pytest

from oracle import sampling


def test_sampler_oracle_restricts_to_nucleus():
    logits = np.full(100, -10.0, np.float32)
    logits[[3, 7]] = [5.0, 4.9]
    seen = {sampling.sample_top_p(logits, 0.9, 0.8, u) for u in np.linspace(0, 1, 200, endpoint=False)}
    assert seen == {3, 7}


def test_sampler_oracle_masked_never_chosen():
    rng = np.random.default_rng(1)
    logits = sampling.mask_semantic(rng.normal(size=8320).astype(np.float32))
    for u in rng.random(100):
        c = sampling.sample_top_p(logits, 0.9, 0.8, u)
        assert 1 <= c < 8194


# (logits, top_p, temperature, u, index), each worked out by hand from sampleTopP
SAMPLER_CASES = [
    ([0, 0, 0, 0], 0.6, 1.0, 0.5, 1),      # p = 1/4 each; sums .25 .5 .75: cutoff 3; r = .375 -> position 1
    ([0, 0, 0, 0], 0.6, 1.0, 0.0, 0),      # r = 0: first position
    ([0, 0, 0, 0], 0.6, 1.0, 0.999, 2),    # r = .749: the cutoff excludes index 3
    ([0, 0, 0, 0], 1.0, 1.0, 0.999, 3),    # top_p 1: all four kept
    ([1, 3, 3, 1], 0.5, 1.0, 0.3, 1),      # ties keep index order: sorted 1, 2, 0, 3; sums .44 .88: cutoff 2
    ([1, 3, 3, 1], 0.5, 1.0, 0.6, 2),      # r = .528 -> second sorted position
    ([2, 0], 0.9, 0.5, 0.99, 0),           # scaled 4, 0: p0 = .982 >= .9 -> cutoff 1
    ([0, 0.5], 0.0, 1.0, 0.7, 1),          # top_p 0: the most probable index only
]


@pytest.mark.parametrize("logits,top_p,temp,u,want", SAMPLER_CASES)
def test_sampler_oracle_hand_cases(logits, top_p, temp, u, want):
    assert sampling.sample_top_p(np.array(logits, np.float32), top_p, temp, u) == want


def _f32(x):
    return struct.unpack("<f", struct.pack("<f", x))[0]


def _loop_sampler(logits, top_p, temperature, u):
    """Plain-loop restatement (Python floats are doubles; _f32 is a Float32Array store)."""
    n = len(logits)
    scaled = [_f32(float(v) / temperature) for v in logits]
    mx = max(scaled)
    s = 0.0
    for i in range(n):
        scaled[i] = _f32(math.exp(scaled[i] - mx))
        s += scaled[i]
    p = [_f32(v / s) for v in scaled]
    order = sorted(range(n), key=lambda i: -p[i])    # sorted() is stable
    cum, cutoff = 0.0, n
    for i in range(n):
        cum += p[order[i]]
        if cum >= top_p:
            cutoff = i + 1
            break
    re_sum = 0.0
    for i in range(cutoff):
        re_sum += p[order[i]]
    r = u * re_sum
    acc = 0.0
    for i in range(cutoff):
        acc += p[order[i]]
        if acc >= r:
            return order[i]
    return order[0]


def test_sampler_oracle_matches_plain_loop():
    rng = np.random.default_rng(3)
    for trial in range(12):
        n = int(rng.integers(2, 600))
        logits = (rng.normal(size=n) * rng.choice([0.1, 1.0, 4.0])).astype(np.float32)
        if trial % 3 == 0:
            logits[rng.integers(0, n, n // 3)] = logits[0]     # ties
        top_p = float(rng.choice([0.0, 0.5, 0.9, 1.0]))
        temp = float(rng.choice([0.8, 1.0, 1.7]))
        for u in rng.random(8):
            assert sampling.sample_top_p(logits, top_p, temp, u) == _loop_sampler(logits, top_p, temp, u)


def test_uniform_draw_mirror(synth):
    """uniform01 = top 53 bits of the counter's 64 bits / 2^53, in [0, 1)."""
    key = synth.sample_key(7)
    b = synth.bits(key, np.arange(4, dtype=np.uint64))
    u = synth.uniform01(key, np.arange(4, dtype=np.uint64))
    assert np.array_equal(u, np.array([int(x) >> 11 for x in b], np.float64) / 2.0 ** 53)
    assert np.all((u >= 0) & (u < 1))
    assert synth.sample_key(7) == synth.stream_key(7, 0x73616D706C65)


def test_options_map_to_config(vx):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}, "fm": {"nfe": 8}}, "maxSeqLen": 1024,
                          "maxSlots": 3})
    assert e.config.n_layers == 2 and e.config.max_seq_len == 1024 and e.config.max_slots == 3
    assert e.config.fm_nfe == 8
    assert not e.isReady


def test_tts_result_shape(vx):
    r = vx.TTSResult(semanticCodes=[5], acousticCodes=[[2] * 36], audio=np.zeros(0, np.float32),
                     stats={"framesGenerated": 1})
    assert r.stats["framesGenerated"] == 1 and r.audio.size == 0
