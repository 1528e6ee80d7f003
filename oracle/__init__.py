"""ctypes binding of the CPU oracle (oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs, never by the product.  PARITY UNPINNED: the reference
(TypeScript + WGSL) cannot run here and ships no golden vectors, so this restatement is
cross-checked against an independent float64 numpy restatement (oracle/numpy_ref.py)
and pinned by tests/golden/.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
DIM = 3072

_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u16p = ctypes.POINTER(ctypes.c_uint16)


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_create.restype = ctypes.c_void_p
        L.orc_create.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_destroy.argtypes = [ctypes.c_void_p]
        L.orc_reset.argtypes = [ctypes.c_void_p]
        L.orc_position.argtypes = [ctypes.c_void_p]
        L.orc_set_position.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.orc_tensor_f16.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _u16p, ctypes.c_size_t]
        L.orc_backbone_step.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p, _f32p,
                                        ctypes.c_int, _u32p]
        L.orc_multi_codebook_embed.argtypes = [ctypes.c_void_p, ctypes.c_uint32, _u32p, _f32p]
        L.orc_fm_forward.argtypes = [ctypes.c_void_p, _f32p, _f32p, _f32p, _u32p, _f32p, _u32p]
        L.orc_masked_argmax.restype = ctypes.c_uint32
        L.orc_masked_argmax.argtypes = [_f32p, ctypes.c_int, ctypes.c_int]
        L.orc_argmax_shader.restype = ctypes.c_uint32
        L.orc_argmax_shader.argtypes = [_f32p, ctypes.c_int]
        L.orc_fill_kv.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64]
        L.orc_generate.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p,
                                   ctypes.c_int, _f32p, _u32p, ctypes.c_int, _u32p, _u32p, _f32p]
        L.orc_num_threads.restype = ctypes.c_int
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_codec_create.restype = ctypes.c_void_p
        L.orc_codec_create.argtypes = []
        L.orc_codec_destroy.argtypes = [ctypes.c_void_p]
        L.orc_codec_set_tensor.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _u16p, ctypes.c_size_t]
        L.orc_codec_get_tensor.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _u16p, ctypes.c_size_t]
        L.orc_codec_debug_size.restype = ctypes.c_size_t
        L.orc_codec_debug_size.argtypes = [ctypes.c_int]
        L.orc_codec_decode.argtypes = [ctypes.c_void_p, _u32p, _u32p, ctypes.c_int, _f32p, ctypes.c_size_t]
        _lib = L
    return _lib


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


class Oracle:
    """One CPU model instance with the reference's shapes and synthetic weights."""

    def __init__(self, n_layers: int = 2, max_seq: int = 4096, with_fm: bool = True):
        self.n_layers = n_layers
        self.h = lib().orc_create(n_layers, max_seq, int(with_fm))

    def close(self):
        if self.h:
            lib().orc_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def position(self) -> int:
        return lib().orc_position(self.h)

    @position.setter
    def position(self, p: int):
        lib().orc_set_position(self.h, p)

    def reset(self):
        lib().orc_reset(self.h)

    def tensor(self, name: str, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.uint16)
        k = lib().orc_tensor_f16(self.h, name.encode(), _p(out, _u16p), n)
        if k < 0:
            raise KeyError(name)
        return out[:k].view(np.float16)

    def backbone_step(self, token: int = 0, use_audio: bool = False, embed=None, debug: bool = False,
                      lm_head: bool = False):
        normed = np.empty(DIM, np.float32)
        hidden = np.empty(DIM, np.float32)
        dbg = np.empty((4 * self.n_layers + 3, DIM), np.float32) if debug else None
        am = np.zeros(1, np.uint32)
        e = None if embed is None else np.ascontiguousarray(embed, dtype=np.float32)
        rc = lib().orc_backbone_step(self.h, int(token), int(use_audio), _p(e, _f32p), _p(normed, _f32p),
                                     _p(hidden, _f32p), _p(dbg, _f32p), int(lm_head), _p(am, _u32p))
        if rc:
            raise RuntimeError(f"oracle backbone_step failed ({rc})")
        return {"normed": normed, "hidden": hidden, "debug": dbg, "argmax": int(am[0]) if lm_head else None}

    def multi_codebook_embed(self, sem: int, ac) -> np.ndarray:
        out = np.empty(DIM, np.float32)
        a = np.ascontiguousarray(ac, dtype=np.uint32)
        if lib().orc_multi_codebook_embed(self.h, int(sem), _p(a, _u32p), _p(out, _f32p)):
            raise ValueError("code out of range")
        return out

    def fm_forward(self, noise, normed=None):
        lg = np.empty(8320, np.float32)
        ac = np.empty(36, np.uint32)
        xf = np.empty(36, np.float32)
        sem = np.zeros(1, np.uint32)
        nz = np.ascontiguousarray(noise, dtype=np.float32)
        n = None if normed is None else np.ascontiguousarray(normed, dtype=np.float32)
        if lib().orc_fm_forward(self.h, _p(n, _f32p), _p(nz, _f32p), _p(lg, _f32p), _p(ac, _u32p), _p(xf, _f32p),
                                _p(sem, _u32p)):
            raise RuntimeError("oracle has no FM")
        return {"semantic_logits": lg, "acoustic_codes": ac, "x_final": xf, "semantic_code": int(sem[0])}

    def fill_kv(self, npos: int, seed: int = 7):
        lib().orc_fill_kv(self.h, npos, seed)

    def generate(self, tokens, audio_start, audio_count, voice, n_frames, noise=None, codes_in=None, eos=False,
                 want_normed=False):
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        v = None if voice is None else np.ascontiguousarray(voice, dtype=np.float32)
        nz = None if noise is None else np.ascontiguousarray(noise, dtype=np.float32)
        ci = None if codes_in is None else np.ascontiguousarray(codes_in, dtype=np.uint32)
        sem = np.zeros(n_frames, np.uint32)
        ac = np.zeros((n_frames, 36), np.uint32)
        nr = np.zeros((n_frames, DIM), np.float32) if want_normed else None
        n = lib().orc_generate(self.h, _p(toks, _i32p), len(toks), audio_start, audio_count, _p(v, _f32p), n_frames,
                               _p(nz, _f32p), _p(ci, _u32p), int(eos), _p(sem, _u32p), _p(ac, _u32p), _p(nr, _f32p))
        if n < 0:
            raise RuntimeError(f"oracle generate failed ({n})")
        return {"frames": n, "semantic_codes": sem[:n], "acoustic_codes": ac[:n], "normed": nr}


def num_threads() -> int:
    return lib().orc_num_threads()


def set_threads(n: int):
    lib().orc_set_threads(n)


def masked_argmax(x, valid=8194) -> int:
    a = np.ascontiguousarray(x, dtype=np.float32)
    return int(lib().orc_masked_argmax(_p(a, _f32p), len(a), valid))


def argmax_shader(x) -> int:
    a = np.ascontiguousarray(x, dtype=np.float32)
    return int(lib().orc_argmax_shader(_p(a, _f32p), len(a)))


# Order and widths of the codec intermediates (debugCodecDecode, src/engine.ts:1719-1975);
# rows = T * 2^stage.
CODEC_ORDER = [("concat", 0, 292), ("after_input_conv", 0, 1024)] + [
    item for s in range(4) for item in
    [(f"after_stage{s}_transformer", s, 1024)] + ([(f"after_stage{s}_conv_up", s + 1, 1024)] if s < 3 else [])
] + [("audio", 3, 240)]


class Codec:
    """CPU restatement of the codec decoder (oracle.cpp, orc_codec_*), synthetic weights."""

    def __init__(self):
        self._h = lib().orc_codec_create()

    def close(self):
        if self._h:
            lib().orc_codec_destroy(self._h)
            self._h = None

    def set_tensor(self, name: str, f16_bits: np.ndarray):
        a = np.ascontiguousarray(f16_bits, dtype=np.uint16).ravel()
        rc = lib().orc_codec_set_tensor(self._h, name.encode(), a.ctypes.data_as(_u16p), a.size)
        if rc:
            raise KeyError(f"{name}: {rc}")

    def tensor(self, name: str, n: int) -> np.ndarray:
        out = np.empty(n, np.uint16)
        rc = lib().orc_codec_get_tensor(self._h, name.encode(), out.ctypes.data_as(_u16p), n)
        if rc:
            raise KeyError(f"{name}: {rc}")
        return out

    def decode(self, sem, ac) -> dict:
        sem = np.ascontiguousarray(sem, dtype=np.uint32).ravel()
        ac = np.ascontiguousarray(ac, dtype=np.uint32).ravel()
        T = sem.size
        n = lib().orc_codec_debug_size(T)
        buf = np.empty(n, np.float32)
        rc = lib().orc_codec_decode(self._h, sem.ctypes.data_as(_u32p), ac.ctypes.data_as(_u32p), T,
                                    buf.ctypes.data_as(_f32p), n)
        if rc:
            raise RuntimeError(f"orc_codec_decode: {rc}")
        out, off = {}, 0
        for name, s, w in CODEC_ORDER:
            rows = (T << s) if name != "audio" else 8 * T
            out[name] = buf[off: off + rows * w].reshape(rows, w)
            off += rows * w
        return out
