"""Synthetic workload of the benchmark configurations (numpy mirror of csrc/vx_rng.h).

The reference streams real weights and uses an unseeded Math.random for the FM
noise and for sampling (src/engine.ts:1265-1274, :247-289), so nothing it computes
is reproducible.  Every synthetic input here comes from the counter-based
generator of csrc/vx_rng.h, restated in numpy with bit-identical results:

* weights   : key = stream_key(0, fnv1a(tensor name)); value i = f16(normal(key, i) * 0.02f);
              norm gains are 1.0
* prompt    : [BOS=1, BEGIN_AUDIO=25, AUDIO=24 x R, TEXT_TO_AUDIO=36, text x T,
              AUDIO_TO_TEXT=35, BEGIN_AUDIO=25] (src/tokenizer.ts:127-165), text ids
              uniform in [1000, 131072) from stream_key(1, utt)
* voice rows: f32 normal, stream_key(2, utt), [R, 3072]
* FM noise  : f32 normal, stream_key(3, utt), index frame*36 + i
* codes     : backbone-only configs feed frame f with codes from stream_key(4, utt):
              semantic 2 + u % 8192 at counter 37f, acoustic 2 + u % 21 at 37f+1+k
"""
from __future__ import annotations

import numpy as np

MASK64 = (1 << 64) - 1
SEED_WEIGHTS, SEED_PROMPT, SEED_VOICE, SEED_FM_NOISE, SEED_CODES = 0, 1, 2, 3, 4
WEIGHT_SIGMA = np.float32(0.02)

BOS, AUDIO, BEGIN_AUDIO, AUDIO_TO_TEXT, TEXT_TO_AUDIO = 1, 24, 25, 35, 36
DIM = 3072


def splitmix64_int(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & MASK64
    return x ^ (x >> 31)


def stream_key(seed: int, stream: int) -> int:
    return splitmix64_int(splitmix64_int(seed) ^ ((stream * 0xD1B54A32D192ED03) & MASK64))


def fnv1a(name: str) -> int:
    h = 0xCBF29CE484222325
    for b in name.encode():
        h = ((h ^ b) * 0x100000001B3) & MASK64
    return h


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return x ^ (x >> np.uint64(31))


def bits(key: int, idx: np.ndarray) -> np.ndarray:
    idx = np.asarray(idx, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _splitmix64(np.uint64(key) ^ (idx * np.uint64(0x9FB21C651E98DF25)))


def uniform01(key: int, idx) -> np.ndarray:
    """Uniform double in [0, 1) from the top 53 bits, bit-identical to vx_uniform01()."""
    return (bits(key, idx) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


SAMPLE_STREAM = 0x73616D706C65   # stream id of the device sampler's draws ("sample")


def sample_key(seed: int) -> int:
    """Key of vx_set_sampling(seed): the draw of frame f is uniform01(sample_key(seed), f)."""
    return stream_key(seed, SAMPLE_STREAM)


def normal(key: int, idx: np.ndarray) -> np.ndarray:
    """Irwin-Hall-12 approximate N(0,1) in f32, bit-identical to vx_normal()."""
    idx = np.asarray(idx, dtype=np.uint64)
    s = np.zeros(idx.shape, dtype=np.int64)
    m16 = np.uint64(0xFFFF)
    for t in range(3):
        with np.errstate(over="ignore"):
            h = bits(key, np.uint64(3) * idx + np.uint64(t))
        for sh in (0, 16, 32, 48):
            s += ((h >> np.uint64(sh)) & m16).astype(np.int64)
    c = 2 * s - 12 * 65535
    return c.astype(np.float32) * np.float32(1.0 / 131072.0)


def tensor_values(name: str, start: int, count: int, is_norm: bool = False) -> np.ndarray:
    """Elements [start, start+count) of a synthetic f16 tensor (row-major)."""
    if is_norm:
        return np.ones(count, dtype=np.float16)
    key = stream_key(SEED_WEIGHTS, fnv1a(name))
    z = normal(key, np.arange(start, start + count, dtype=np.uint64))
    return (z * WEIGHT_SIGMA).astype(np.float16)


def tensor_rows(name: str, rows, ncols: int) -> np.ndarray:
    rows = np.asarray(rows, dtype=np.int64)
    out = np.empty((len(rows), ncols), dtype=np.float16)
    for i, r in enumerate(rows):
        out[i] = tensor_values(name, int(r) * ncols, ncols)
    return out


def prompt(utt: int, n_text: int, n_voice: int):
    """Token ids and voice-row span of one synthetic utterance."""
    key = stream_key(SEED_PROMPT, utt)
    text = (1000 + (bits(key, np.arange(n_text)) % np.uint64(131072 - 1000))).astype(np.int32)
    toks = [BOS, BEGIN_AUDIO] + [AUDIO] * n_voice + [TEXT_TO_AUDIO] + text.tolist() + [AUDIO_TO_TEXT, BEGIN_AUDIO]
    return np.asarray(toks, dtype=np.int32), 2, n_voice


def voice_rows(utt: int, n_voice: int, dim: int = DIM) -> np.ndarray:
    key = stream_key(SEED_VOICE, utt)
    return normal(key, np.arange(n_voice * dim, dtype=np.uint64)).reshape(n_voice, dim)


def fm_noise(utt: int, frame0: int, n_frames: int) -> np.ndarray:
    key = stream_key(SEED_FM_NOISE, utt)
    idx = np.arange(frame0 * 36, (frame0 + n_frames) * 36, dtype=np.uint64)
    return normal(key, idx).reshape(n_frames, 36)


def feedback_codes(utt: int, frame0: int, n_frames: int) -> np.ndarray:
    """[n_frames, 37] codes (semantic, 36 acoustic) fed to frames frame0+1.."""
    key = stream_key(SEED_CODES, utt)
    out = np.empty((n_frames, 37), dtype=np.uint32)
    for f in range(n_frames):
        base = (frame0 + f) * 37
        b = bits(key, np.arange(base, base + 37, dtype=np.uint64))
        out[f, 0] = 2 + int(b[0] % np.uint64(8192))
        out[f, 1:] = (2 + (b[1:] % np.uint64(21))).astype(np.uint32)
    return out
