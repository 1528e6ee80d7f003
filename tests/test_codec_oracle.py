"""The codec decoder's CPU oracle (oracle.cpp, orc_codec_*), pinned without a GPU:
against an independent float64 restatement, by causality, and by hand-worked input
rows (VQ lookup, FSQ dequantisation, codebook normalisation)."""
import numpy as np
import pytest

import oracle
from oracle import numpy_codec
from conftest import max_abs_rel


@pytest.fixture(scope="module")
def codec():
    c = oracle.Codec()
    yield c
    c.close()


def _codes(seed, T):
    rng = np.random.default_rng(seed)
    return rng.integers(2, 8194, T).astype(np.uint32), rng.integers(2, 23, (T, 36)).astype(np.uint32)


def test_oracle_matches_float64_restatement(codec):
    sem, ac = _codes(1, 3)
    got = codec.decode(sem, ac)
    want = numpy_codec.decode(codec.tensor, sem, ac)
    for name in oracle.CODEC_ORDER:
        assert max_abs_rel(got[name[0]], want[name[0]]) < 1e-4, name[0]


def test_oracle_is_causal(codec):
    """Frame t's output depends on frames <= t only: a prefix decodes to a prefix."""
    sem, ac = _codes(2, 6)
    full = codec.decode(sem, ac)
    part = codec.decode(sem[:3], ac[:3])
    for name, s, _ in oracle.CODEC_ORDER:
        rows = part[name].shape[0]
        assert np.array_equal(part[name], full[name][:rows]), name


def test_input_rows_by_hand(codec):
    """FSQ: code c -> (c - 2) * 2 / 20 - 1 in f32; VQ: codebook row `code` (= embedding_sum / 2 with
    the synthetic usage 2.0); codes 8192 and 8193 give a zero row."""
    sem = np.array([2, 8191, 8192, 8193], np.uint32)
    ac = np.tile(np.arange(2, 23, dtype=np.uint32)[:18], 2).reshape(1, 36).repeat(4, axis=0)
    d = codec.decode(sem, ac)
    fsq = d["concat"][:, 256:]
    f32 = np.float32   # the shader's f32 steps: ((c - 2) * 2) / 20 - 1
    want = np.array([(f32(c - 2) * f32(2)) / f32(20) - f32(1) for c in ac[0]], np.float32)
    assert np.array_equal(fsq[0], want)
    assert fsq[0, 0] == -1.0 and fsq[0, 10] == 0.0
    total = codec.tensor("audio_tokenizer.quantizer.semantic_codebook.embedding_sum", 8192 * 256).reshape(8192, 256)
    for i, code in enumerate(sem[:2]):
        row = (total[code].view(np.float16).astype(np.float32) / np.float32(2.0)).astype(np.float16)
        assert np.array_equal(d["concat"][i, :256], row.astype(np.float32))
    assert not d["concat"][2:, :256].any()


def test_codebook_normalisation_uses_usage():
    c = oracle.Codec()
    try:
        rng = np.random.default_rng(3)
        name = "audio_tokenizer.quantizer.semantic_codebook.cluster_usage"
        usage = rng.uniform(0.5, 40.0, 8192).astype(np.float16)
        usage[7] = 0.0                                     # max(usage, 1e-5) guards the division
        c.set_tensor(name, usage.view(np.uint16))
        sem = np.array([5, 7, 100], np.uint32)
        d = c.decode(sem, np.full((3, 36), 12, np.uint32))
        total = c.tensor("audio_tokenizer.quantizer.semantic_codebook.embedding_sum", 8192 * 256).reshape(8192, 256)
        for i, code in enumerate(sem):
            u = max(np.float32(usage[code]), np.float32(1e-5))
            row = (total[code].view(np.float16).astype(np.float32) / u).astype(np.float16).astype(np.float32)
            assert np.array_equal(d["concat"][i, :256], row)
    finally:
        c.close()


def test_debug_layout_matches_engine(vx):
    """The engine's vx_codec_debug buffer and the oracle's use the same layout."""
    eng_mod = __import__("importlib").import_module("webgpu-voxtral_b200.engine")
    assert [n for n, _, _ in eng_mod.CODEC_DEBUG_ORDER] == [n for n, _, _ in oracle.CODEC_ORDER]
    T = 3
    n = vx.load_library().vx_codec_debug_size(T)
    assert n == oracle.lib().orc_codec_debug_size(T)
    parts = eng_mod.split_codec_debug(np.zeros(n, np.float32), T)
    assert parts["audio"].shape == (8 * T, 240) and parts["after_stage2_conv_up"].shape == (8 * T, 1024)
