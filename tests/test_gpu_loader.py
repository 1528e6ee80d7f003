"""Checkpoint loading through the C ABI (vx_load_tensor_typed via
VoxtralEngine.loadWeightsFromSafetensors): BF16 / F32 / F16 tensors of a safetensors file
are converted on the GPU with the reference loader's bit rules; read back, they must equal
the oracle's restatement of those rules bit for bit, for every class of input (normals,
values beyond F16 range, values below it, zeros, BF16 subnormals, Inf, NaN)."""
import os

import numpy as np
import pytest

from oracle import convert

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng(vx):
    e = vx.VoxtralEngine({"config": {"backbone": {"n_layers": 2}}, "maxSeqLen": 256, "maxFrames": 16,
                          "enableFM": False})
    e.init()
    e.loadRandomWeights(0)
    yield e
    e.destroy()


def test_partial_safetensors_load_matches_reference_rules(eng, tmp_path):
    st = __import__("importlib").import_module("webgpu-voxtral_b200.safetensors")
    rng = np.random.default_rng(5)
    shapes = {"layers.0.attention.wk.weight": (1024, 3072), "layers.1.feed_forward.w2.weight": (3072, 9216),
              "norm.weight": (3072,), "layers.1.attention_norm.weight": (3072,)}
    bf = rng.integers(0, 1 << 16, size=shapes["layers.0.attention.wk.weight"], dtype=np.uint16)
    bf[0, :16] = [0x3F80, 0x3800, 0x3400, 0x4780, 0x0001, 0x7FC0, 0xFF80, 0x3880, 0, 0x8000, 0x477F, 0x3300,
                  0x8001, 0xFF81, 0x3FC0, 0x7F80]
    bf2 = (rng.standard_normal(shapes["layers.1.feed_forward.w2.weight"]).astype(np.float32) * 0.02
           ).view(np.uint32) >> 16   # realistic weights, BF16-truncated
    f32 = rng.integers(0, 1 << 32, size=shapes["norm.weight"], dtype=np.uint32)
    f16 = rng.standard_normal(shapes["layers.1.attention_norm.weight"]).astype(np.float16).view(np.uint16)
    p = os.path.join(tmp_path, "ckpt.safetensors")
    st.write(p, {"layers.0.attention.wk.weight": (bf, "BF16"),
                 "layers.1.feed_forward.w2.weight": (bf2.astype(np.uint16), "BF16"),
                 "norm.weight": (f32, "F32"), "layers.1.attention_norm.weight": (f16, "F16"),
                 "codec.unused": (np.zeros(4, np.uint16), "BF16")})
    untouched = eng.readTensor("layers.0.attention.wq.weight").copy()
    loaded = eng.loadWeightsFromSafetensors(p, required=False)
    assert sorted(loaded) == sorted(shapes)
    got = {n: eng.readTensor(n).view(np.uint16) for n in shapes}
    assert np.array_equal(got["layers.0.attention.wk.weight"], convert.bf16_to_f16_bits(bf).ravel())
    assert np.array_equal(got["layers.1.feed_forward.w2.weight"],
                          convert.bf16_to_f16_bits(bf2.astype(np.uint16)).ravel())
    assert np.array_equal(got["norm.weight"], convert.f32_to_f16_bits(f32))
    assert np.array_equal(got["layers.1.attention_norm.weight"], f16)
    assert np.array_equal(eng.readTensor("layers.0.attention.wq.weight"), untouched)


def test_missing_tensors_are_reported(eng, vx, tmp_path):
    st = __import__("importlib").import_module("webgpu-voxtral_b200.safetensors")
    p = os.path.join(tmp_path, "partial.safetensors")
    st.write(p, {"norm.weight": (np.zeros(3072, np.uint16), "BF16")})
    names = eng.tensorNames()
    assert "norm.weight" in names and "layers.1.feed_forward.w2.weight" in names
    with pytest.raises(vx.VoxtralError, match="Missing weight"):
        eng.loadWeightsFromSafetensors(p, required=True)
    eng.loadRandomWeights(0)   # leave the shared engine ready
