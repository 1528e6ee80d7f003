"""The synthetic-input generator is bit-identical between numpy (synth.py), the C oracle
and (on the GPU, test_gpu_parity.py) the CUDA engine."""
import numpy as np
import pytest

import oracle


@pytest.fixture(scope="module")
def orc():
    o = oracle.Oracle(n_layers=1, max_seq=8, with_fm=False)
    yield o
    o.close()


@pytest.mark.parametrize("name", ["layers.0.attention.wq.weight", "layers.0.feed_forward.w2.weight",
                                  "mm_audio_embeddings.audio_codebook_embeddings.embeddings.weight"])
def test_oracle_weights_equal_numpy(orc, synth, name):
    n = 200_000
    a = orc.tensor(name, n)
    b = synth.tensor_values(name, 0, n)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


def test_normal_moments(synth):
    z = synth.normal(synth.stream_key(9, 1), np.arange(400_000))
    assert abs(float(z.mean())) < 5e-3
    assert abs(float(z.std()) - 1.0) < 5e-3
    assert float(np.abs(z).max()) <= 6.0


def test_f16_rounding_is_rne(synth):
    # 0.02 * z rounded by the oracle's software RNE == numpy's RNE for every value
    z = synth.normal(synth.stream_key(0, synth.fnv1a("layers.0.attention.wq.weight")), np.arange(200_000))
    want = (z * np.float32(0.02)).astype(np.float16)
    got = synth.tensor_values("layers.0.attention.wq.weight", 0, 200_000)
    assert np.array_equal(want.view(np.uint16), got.view(np.uint16))


def test_prompt_layout(synth):
    toks, a0, na = synth.prompt(3, 5, 4)
    assert toks[:2].tolist() == [1, 25] and a0 == 2 and na == 4
    assert toks[2:6].tolist() == [24] * 4 and toks[6] == 36
    assert toks[-2:].tolist() == [35, 25]
    assert len(toks) == 5 + 4 + 5
    assert np.all((toks[7:12] >= 1000) & (toks[7:12] < 131072))


def test_feedback_codes_range(synth):
    c = synth.feedback_codes(0, 0, 50)
    assert np.all((c[:, 0] >= 2) & (c[:, 0] < 8194))
    assert np.all((c[:, 1:] >= 2) & (c[:, 1:] <= 22))
