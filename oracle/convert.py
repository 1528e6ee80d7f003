"""Test infrastructure (the checker, not the product): numpy restatement of the
reference loader's conversions to F16 bit patterns, used to check the engine's
on-GPU conversion (vx_load_tensor_typed) bit for bit.

- bf16_to_f16_bits: convertBF16toF16, src/weights.ts:94-138.  Kept exactly, including
  its treatment of results below the F16 normal range: the 8-bit significand is shifted
  right by (-14 - exponent) and then once more, so such values come out 16x smaller
  than their true value (e.g. BF16 2^-15 -> F16 bits 0x0020).  Parity requires the
  same bits.
- f32_to_f16_bits: float32ToFloat16, src/weights.ts:222-232 (truncating; no F16
  subnormals; overflow and NaN become Inf).
"""
import numpy as np


def bf16_to_f16_bits(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16).astype(np.int64)
    sign = b & 0x8000
    exp = (b >> 7) & 0xFF
    mant = b & 0x7F
    unb = exp - 127
    out = np.empty_like(b)
    # normal range (src/weights.ts:127-131)
    out[:] = sign | ((unb + 15) << 10) | ((mant << 3) & 0x3FF)
    # below the F16 normal range (:117-126)
    shift = -14 - unb
    low = unb < -14
    sub = ((((0x80 | (mant << 1)) >> np.clip(shift, 0, 31)) >> 1) & 0x3FF) | sign
    out = np.where(low, np.where(shift > 10, sign, sub), out)
    out = np.where(unb > 15, sign | 0x7C00, out)                              # overflow (:114-116)
    out = np.where(exp == 0, sign, out)                                        # zero / subnormal (:106-108)
    out = np.where(exp == 0xFF, sign | 0x7C00 | np.where(mant != 0, 0x200, 0), out)   # Inf / NaN (:103-105)
    return out.astype(np.uint16)


def f32_to_f16_bits(bits) -> np.ndarray:
    b = np.asarray(bits, dtype=np.uint32).astype(np.int64)
    sign = (b >> 16) & 0x8000
    exp = ((b >> 23) & 0xFF) - 127 + 15
    frac = (b >> 13) & 0x3FF
    out = sign | (np.clip(exp, 0, 31) << 10) | frac
    out = np.where(exp <= 0, sign, out)
    out = np.where(exp >= 31, sign | 0x7C00, out)
    return out.astype(np.uint16)
