"""Checkpoint loading on the host: the safetensors reader and the oracle's restatement of
the reference's F16 conversion rules (src/weights.ts:94-138, :222-232), pinned by cases
worked out by hand from those rules."""
import importlib
import os

import numpy as np
import pytest

from oracle import convert

st = importlib.import_module("webgpu-voxtral_b200.safetensors")


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.integers(0, 1 << 16, size=(3, 5), dtype=np.uint16)
    b = rng.integers(0, 1 << 32, size=(7,), dtype=np.uint32)
    c = rng.standard_normal((2, 2)).astype(np.float16).view(np.uint16)
    p = os.path.join(tmp_path, "t.safetensors")
    st.write(p, {"x.weight": (a, "BF16"), "y": (b, "F32"), "z": (c, "F16")}, metadata={"format": "pt"})
    f = st.SafetensorsFile(p)
    assert sorted(f.names()) == ["x.weight", "y", "z"]
    assert f.metadata == {"format": "pt"}
    for name, ref, dt in [("x.weight", a, "BF16"), ("y", b, "F32"), ("z", c, "F16")]:
        raw, d = f.raw(name)
        assert d == dt
        assert np.array_equal(raw, ref.ravel())
    f.close()


def test_safetensors_rejects_bad_offsets(tmp_path):
    p = os.path.join(tmp_path, "bad.safetensors")
    st.write(p, {"x": (np.zeros(4, np.uint16), "BF16")})
    raw = bytearray(open(p, "rb").read())
    raw = raw.replace(b"[0, 8]", b"[0, 6]")
    open(p, "wb").write(bytes(raw))
    with pytest.raises(ValueError):
        st.SafetensorsFile(p)


# (BF16 bits, F16 bits), each worked out by hand from convertBF16toF16
BF16_CASES = [
    (0x3F80, 0x3C00),   # 1.0
    (0xBF80, 0xBC00),   # -1.0
    (0x3FC0, 0x3E00),   # 1.5: mantissa 0x40 << 3
    (0x4700, 0x7800),   # 32768: exponent 15, largest in range
    (0x477F, 0x7BF8),   # 65280
    (0x4780, 0x7C00),   # 65536: overflow -> Inf
    (0x3880, 0x0400),   # 2^-14: smallest F16 normal
    (0x3800, 0x0020),   # 2^-15: the rule's subnormal (shift 1, then 1 more)
    (0x3400, 0x0000),   # 2^-23: shift 9 leaves no bit
    (0x3300, 0x0000),   # 2^-25: shift 11 > 10 -> zero
    (0x0001, 0x0000),   # BF16 subnormal -> zero
    (0x8001, 0x8000),   # negative BF16 subnormal -> -0
    (0x7F80, 0x7C00),   # +Inf
    (0xFF80, 0xFC00),   # -Inf
    (0x7FC0, 0x7E00),   # NaN -> quiet NaN
    (0xFF81, 0xFE00),   # negative NaN
]
# (F32 bits, F16 bits), each worked out by hand from float32ToFloat16
F32_CASES = [
    (0x3F800000, 0x3C00),   # 1.0
    (0x477FE000, 0x7BFF),   # 65504
    (0x477FF000, 0x7BFF),   # 65520: truncated, not rounded up
    (0x47800000, 0x7C00),   # 65536 -> Inf
    (0x38800000, 0x0400),   # 2^-14
    (0x38000000, 0x0000),   # 2^-15: no F16 subnormals
    (0xC0000000, 0xC000),   # -2.0
    (0x7FC00000, 0x7C00),   # NaN -> Inf
    (0x3F802000, 0x3C01),   # 1 + 2^-10
    (0x3F801000, 0x3C00),   # 1 + 2^-11: truncated
    (0x80000000, 0x8000),   # -0
]


@pytest.mark.parametrize("src,want", BF16_CASES)
def test_bf16_rule(src, want):
    assert int(convert.bf16_to_f16_bits([src])[0]) == want


@pytest.mark.parametrize("src,want", F32_CASES)
def test_f32_rule(src, want):
    assert int(convert.f32_to_f16_bits([src])[0]) == want


def test_bf16_rule_is_exact_in_the_normal_range():
    """Every BF16 value whose F16 image is normal is exactly representable in F16, so the
    rule must agree with numpy's value conversion there."""
    b = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    exp = (b.astype(np.int64) >> 7) & 0xFF
    normal = (exp >= 127 - 14) & (exp <= 127 + 15)
    vals = (b.astype(np.uint32) << 16).view(np.float32)
    want = vals[normal].astype(np.float16).view(np.uint16)
    assert np.array_equal(convert.bf16_to_f16_bits(b[normal]), want)
