"""Host-side mirror of the reference's VoxtralEngine over the C ABI (include/voxtral_b200.h).

Method names, argument meaning and error behaviour follow the reference's TypeScript
class (svenflow/webgpu-voxtral src/engine.ts:291-2633) so that code written against
it reads the same here:

    eng = VoxtralEngine({"maxSeqLen": 4096})
    eng.init()
    eng.loadRandomWeights(0)          # stands in for loadWeightsFromHF() (:569)
    res = eng.generate(tokens, audioTokenStart, audioTokenCount, voice, maxFrames=500)

Everything runs in libvoxtral_b200.so (CUDA, sm_100a).  There is no CPU fallback:
constructing an engine without the library or without a B200 raises.
"""
from __future__ import annotations

import ctypes
import os
import time
from dataclasses import dataclass, field
from typing import Callable, Optional

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libvoxtral_b200.so")
HEADER = os.path.join(os.path.dirname(_PKG), "include", "voxtral_b200.h")

VX_OK = 0
_ERRORS = {-1: "VX_E_INVALID", -2: "VX_E_CUDA", -3: "VX_E_STATE", -4: "VX_E_RANGE", -5: "VX_E_NOMEM",
           -6: "VX_E_NCCL", -7: "VX_E_DEVICE"}
AUDIO_TOKEN = 24   # TOKENS.AUDIO (src/tokenizer.ts:20)


class VxConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("dim", "n_layers", "head_dim", "hidden_dim", "n_heads", "n_kv_heads",
                                                "vocab_size")] + \
               [("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float),
                ("fm_n_layers", ctypes.c_int32), ("fm_nfe", ctypes.c_int32), ("fm_cfg_alpha", ctypes.c_float)] + \
               [(n, ctypes.c_int32) for n in ("fm_n_acoustic", "fm_semantic_vocab", "acoustic_levels", "audio_vocab",
                                               "max_seq_len", "max_slots", "max_frames", "max_voice_rows",
                                               "enable_fm", "device", "tp_size", "tp_rank", "enable_codec")]


class VoxtralError(RuntimeError):
    """Raised for every non-zero status of the C ABI (the reference throws Error)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{message} [{_ERRORS.get(code, code)}]")
        self.code = code


_lib = None
_f32p = ctypes.POINTER(ctypes.c_float)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)


def library_path() -> str:
    return LIB_PATH


def load_library():
    """Load libvoxtral_b200.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python webgpu-voxtral_b200/build.py` "
                          "(the decode path has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    H = ctypes.c_void_p
    sig = {
        "vx_default_config": (None, [ctypes.POINTER(VxConfig)]),
        "vx_create": (ctypes.c_int, [ctypes.POINTER(VxConfig), ctypes.POINTER(H)]),
        "vx_destroy": (None, [H]),
        "vx_last_error": (ctypes.c_char_p, [H]),
        "vx_init_random_weights": (ctypes.c_int, [H, ctypes.c_uint64]),
        "vx_load_tensor": (ctypes.c_int, [H, ctypes.c_char_p, _u16p, ctypes.c_size_t]),
        "vx_load_tensor_typed": (ctypes.c_int, [H, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t]),
        "vx_tensor_names": (ctypes.c_size_t, [H, ctypes.c_char_p, ctypes.c_size_t]),
        "vx_tensor_numel": (ctypes.c_size_t, [H, ctypes.c_char_p]),
        "vx_read_tensor": (ctypes.c_int, [H, ctypes.c_char_p, _u16p, ctypes.c_size_t]),
        "vx_mark_weights_loaded": (ctypes.c_int, [H]),
        "vx_reset": (ctypes.c_int, [H, ctypes.c_int32]),
        "vx_get_position": (ctypes.c_int, [H, ctypes.c_int32, _i32p]),
        "vx_prefill": (ctypes.c_int, [H, ctypes.c_int32, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                      _f32p]),
        "vx_backbone_step": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _f32p, _f32p, _i32p]),
        "vx_backbone_step_codes": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_uint32, _u32p, _f32p]),
        "vx_fm_step": (ctypes.c_int, [H, ctypes.c_int32, _f32p, _f32p, _u32p, _u32p, _f32p]),
        "vx_codec_decode": (ctypes.c_int, [H, _u32p, _u32p, ctypes.c_int32, _f32p]),
        "vx_codec_debug_size": (ctypes.c_size_t, [ctypes.c_int32]),
        "vx_codec_debug": (ctypes.c_int, [H, _u32p, _u32p, ctypes.c_int32, _f32p, ctypes.c_size_t]),
        "vx_debug_layers": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, _f32p]),
        "vx_decode": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
        "vx_decode_batch": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
        "vx_fill_kv": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_uint64]),
        "vx_set_streams": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int32]),
        "vx_read_codes": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _u32p]),
        "vx_read_normed": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _f32p]),
        "vx_checkpoint": (ctypes.c_int, [H, ctypes.c_int32]),
        "vx_rewind": (ctypes.c_int, [H, ctypes.c_int32]),
        "vx_set_stream": (ctypes.c_int, [H, ctypes.c_void_p]),
        "vx_synchronize": (ctypes.c_int, [H]),
        "vx_launch_count": (ctypes.c_int64, [H]),
        "vx_profile_step": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, _f32p,
                                           ctypes.POINTER(ctypes.c_double)]),
        "vx_trace": (ctypes.c_int, [H, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t, _i32p]),
        "vx_set_sampling": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_double, ctypes.c_double,
                                           ctypes.c_uint64]),
        "vx_selftest_top_p": (ctypes.c_int, [H, _f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_double,
                                             ctypes.c_double, ctypes.POINTER(ctypes.c_double), ctypes.c_int32,
                                             ctypes.POINTER(ctypes.c_int32)]),
        "vx_selftest_gemm": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_uint64, ctypes.POINTER(ctypes.c_double)]),
        "vx_nccl_unique_id": (ctypes.c_int, [ctypes.c_char_p, _u8p]),
        "vx_tp_init": (ctypes.c_int, [H, ctypes.c_char_p, _u8p]),
        "vx_tp_p2p_handle": (ctypes.c_int, [H, _u8p]),
        "vx_tp_p2p_open": (ctypes.c_int, [H, _u8p]),
        "vx_set_option": (ctypes.c_int, [H, ctypes.c_char_p, ctypes.c_int64]),
        "vx_decode_record": (ctypes.c_int, [H, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _f32p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


def default_config() -> VxConfig:
    c = VxConfig()
    load_library().vx_default_config(ctypes.byref(c))
    return c


@dataclass
class TTSResult:
    """TTSResult (src/engine.ts:222-237).  `audio` stays empty: the codec decoder
    that turns codes into 24 kHz samples is outside this decode path."""
    semanticCodes: list
    acousticCodes: list
    audio: np.ndarray
    stats: dict = field(default_factory=dict)


class VoxtralEngine:
    """B200 counterpart of the reference's VoxtralEngine (src/engine.ts:291)."""

    def __init__(self, options: Optional[dict] = None):
        o = dict(options or {})
        self._cfg = default_config()
        cfg = o.get("config") or {}
        bb, fm = cfg.get("backbone", {}), cfg.get("fm", {})
        for k_ts, k_c in (("dim", "dim"), ("n_layers", "n_layers"), ("head_dim", "head_dim"),
                          ("hidden_dim", "hidden_dim"), ("n_heads", "n_heads"), ("n_kv_heads", "n_kv_heads"),
                          ("vocab_size", "vocab_size"), ("rope_theta", "rope_theta"), ("norm_eps", "norm_eps")):
            if k_ts in bb:
                setattr(self._cfg, k_c, bb[k_ts])
        for k_ts, k_c in (("n_layers", "fm_n_layers"), ("nfe", "fm_nfe"), ("cfg_alpha", "fm_cfg_alpha"),
                          ("n_acoustic_out", "fm_n_acoustic"), ("semantic_vocab", "fm_semantic_vocab")):
            if k_ts in fm:
                setattr(self._cfg, k_c, fm[k_ts])
        self._cfg.max_seq_len = int(o.get("maxSeqLen", 4096))
        self._cfg.max_slots = int(o.get("maxSlots", 1))
        self._cfg.max_frames = int(o.get("maxFrames", 2048))
        self._cfg.max_voice_rows = int(o.get("maxVoiceRows", 256))
        self._cfg.enable_fm = int(bool(o.get("enableFM", True)))
        self._cfg.enable_codec = int(bool(o.get("enableCodec", True)))
        self._cfg.device = int(o.get("device", 0))
        self._cfg.tp_size = int(o.get("tpSize", 1))
        self._cfg.tp_rank = int(o.get("tpRank", 0))
        self._h = None
        self._ready = False
        self._sampling = o.get("sampling", "argmax")
        if self._sampling not in ("argmax", "top_p"):
            raise ValueError(f"sampling {self._sampling!r}: 'argmax' or 'top_p'")
        self._sampling_seed = int(o.get("samplingSeed", 0))

    # ------------------------------------------------------------------ lifecycle
    def _check(self, rc: int):
        if rc != VX_OK:
            msg = load_library().vx_last_error(self._h).decode() if self._h else "engine not created"
            raise VoxtralError(rc, msg)

    def init(self):
        """init() (src/engine.ts:313): device, buffers, KV cache."""
        L = load_library()
        h = ctypes.c_void_p()
        rc = L.vx_create(ctypes.byref(self._cfg), ctypes.byref(h))
        self._h = h
        self._check(rc)
        return self

    @property
    def handle(self):
        return self._h

    @property
    def config(self) -> VxConfig:
        return self._cfg

    @property
    def isReady(self) -> bool:
        return self._h is not None and self._ready

    def loadRandomWeights(self, seed: int = 0):
        """Synthetic weights (vx_rng.h): the benchmark's stand-in for loadWeightsFromHF."""
        self._check(load_library().vx_init_random_weights(self._h, seed))
        self._ready = True

    def loadWeights(self, tensors: dict):
        """loadWeights() (src/engine.ts:539) from a {checkpoint name: f16 array} mapping."""
        L = load_library()
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, dtype=np.float16).view(np.uint16).ravel()
            self._check(L.vx_load_tensor(self._h, name.encode(), _p(a, _u16p), a.size))
        self._check(L.vx_mark_weights_loaded(self._h))
        self._ready = True

    def tensorNames(self) -> list:
        """Checkpoint tensor names this engine holds (sorted)."""
        L = load_library()
        n = L.vx_tensor_names(self._h, None, 0)
        buf = ctypes.create_string_buffer(n)
        L.vx_tensor_names(self._h, buf, n)
        return [x for x in buf.value.decode().split("\n") if x]

    def loadWeightsFromSafetensors(self, path: str, required: bool = True) -> list:
        """loadWeightsFromHF / loadFromSafetensors (src/engine.ts:569, src/weights.ts:491-669)
        from a local safetensors file: every tensor the engine has a slot for is copied in its
        stored dtype and converted to F16 on the GPU (BF16 and F32 with the reference's bit
        rules).  Tensors the engine has no slot for (tokenizer extras, the codec when it is
        disabled) are skipped.  With
        `required`, a slot the file does not provide raises, as the reference throws
        "Missing weight".  Returns the loaded names."""
        from .safetensors import DTYPES, SafetensorsFile
        L = load_library()
        st = SafetensorsFile(path)
        loaded = []
        try:
            for name in st.names():
                n = L.vx_tensor_numel(self._h, name.encode())
                if n == 0:
                    continue
                raw, dt = st.raw(name)
                code = DTYPES[dt][1]
                if code is None:
                    raise VoxtralError(-1, f"{name}: dtype {dt} cannot be loaded as a weight")
                self._check(L.vx_load_tensor_typed(self._h, name.encode(), raw.ctypes.data_as(ctypes.c_void_p),
                                                   code, raw.size))
                loaded.append(name)
                del raw
        finally:
            st.close()
        if required:
            missing = [m for m in self.tensorNames() if m not in set(loaded)]
            if missing:
                raise VoxtralError(-1, f"Missing weight: {missing[0]} (and {len(missing) - 1} more)")
        self._check(L.vx_mark_weights_loaded(self._h))
        self._ready = True
        return loaded

    def readTensor(self, name: str) -> np.ndarray:
        L = load_library()
        n = L.vx_tensor_numel(self._h, name.encode())
        if n == 0:
            raise KeyError(name)
        out = np.empty(n, dtype=np.uint16)
        self._check(L.vx_read_tensor(self._h, name.encode(), _p(out, _u16p), n))
        return out.view(np.float16)

    def destroy(self):
        """destroy() (src/engine.ts:2621)."""
        if self._h:
            load_library().vx_destroy(self._h)
        self._h = None
        self._ready = False

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass

    def _require_ready(self):
        if not self.isReady:
            raise VoxtralError(-3, "Engine not initialized. Call init() and loadWeights() first.")

    # ------------------------------------------------------------------ state
    def reset(self, slot: int = 0):
        """reset() (src/engine.ts:2323)."""
        self._check(load_library().vx_reset(self._h, slot))

    def position(self, slot: int = 0) -> int:
        v = ctypes.c_int32()
        self._check(load_library().vx_get_position(self._h, slot, ctypes.byref(v)))
        return v.value

    def set_streams(self, noise_seed: int = 3, codes_seed: int = 4, utt: int = 0, slot: int = 0):
        self._check(load_library().vx_set_streams(self._h, slot, noise_seed, codes_seed, utt))

    def set_sampling(self, mode: str = "top_p", top_p: float = 0.9, temperature: float = 0.8, seed: int = 0,
                     slot: int = 0):
        """Semantic selection of the slot's FM frames on the device: 'argmax' (masked argmax)
        or 'top_p' (sampleTopP, src/engine.ts:247-289, with the draw of frame f taken from
        the seeded stream instead of Math.random)."""
        if mode not in ("argmax", "top_p"):
            raise ValueError(f"sampling mode {mode!r}")
        self._check(load_library().vx_set_sampling(self._h, slot, int(mode == "top_p"), float(top_p),
                                                   float(temperature), int(seed)))

    def set_stream(self, stream_ptr: Optional[int]):
        self._check(load_library().vx_set_stream(self._h, ctypes.c_void_p(stream_ptr or 0)))

    def synchronize(self):
        self._check(load_library().vx_synchronize(self._h))

    def set_option(self, name: str, value: int):
        """Engine option of vx_set_option (persistent_decode, batched_prefill, l2_prefetch_tiles,
        wait_limit, tp_loopback)."""
        self._check(load_library().vx_set_option(self.handle, name.encode(), int(value)))

    def launch_count(self) -> int:
        return int(load_library().vx_launch_count(self._h))

    def checkpoint(self, slot: int = 0):
        self._check(load_library().vx_checkpoint(self._h, slot))

    def rewind(self, slot: int = 0):
        self._check(load_library().vx_rewind(self._h, slot))

    def profile_step(self, reps: int = 8, slot: int = 0) -> dict:
        """ms per backbone step of the full graph, its GEMV chain and its attention chain."""
        ms = np.zeros(3, np.float32)
        by = ctypes.c_double()
        self._check(load_library().vx_profile_step(self._h, slot, reps, _p(ms, _f32p), ctypes.byref(by)))
        return {"step_ms": float(ms[0]), "gemv_ms": float(ms[1]), "attn_ms": float(ms[2]),
                "gemv_bytes": float(by.value)}

    def selftest_gemm(self, M: int, N: int, K: int, bn: int = 128, max_splits: int = 8, seed: int = 0):
        """Tensor-core GEMM vs an f32 CUDA-core product: (rel err of Y = XW^T, rel err of Y += XW^T)."""
        err = (ctypes.c_double * 2)()
        self._check(load_library().vx_selftest_gemm(self._h, M, N, K, bn, max_splits, seed, err))
        return float(err[0]), float(err[1])

    def selftest_top_p(self, logits, u, top_p: float = 0.9, temperature: float = 0.8, valid_lo: int = 0,
                       valid_hi: Optional[int] = None) -> np.ndarray:
        """Device top-p sampler on a logit row, one index per uniform draw in u."""
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        uu = np.ascontiguousarray(u, dtype=np.float64).ravel()
        out = np.empty(uu.size, np.int32)
        hi = lg.size if valid_hi is None else valid_hi
        self._check(load_library().vx_selftest_top_p(
            self._h, _p(lg, _f32p), lg.size, valid_lo, hi, float(top_p), float(temperature),
            uu.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), uu.size,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return out

    def trace_arm(self):
        """Record phase timestamps of the next persistent-kernel launch (first 2 steps)."""
        self._check(load_library().vx_trace(self._h, 1, None, 0, None))

    def trace_read(self) -> np.ndarray:
        """[cta, step, phase, 8]: {released, consumers done, epilogue arrival, prologue done} in ns, then
        SM cycles waiting {consumer warp 0 on stages, on reduction slots, epilogue on results} (0 = not recorded)."""
        L = load_library()
        dims = np.zeros(4, np.int32)
        self._check(L.vx_trace(self._h, 2, None, 0, _p(dims, _i32p)))
        n = int(np.prod(dims))
        out = np.zeros(n, np.uint64)
        self._check(L.vx_trace(self._h, 0, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), n, _p(dims, _i32p)))
        return out.reshape(tuple(int(d) for d in dims))

    # ------------------------------------------------------------------ steps
    def prefill(self, tokens, audioTokenStart: int = 0, audioTokenCount: int = 0, voiceEmbeddings=None, slot: int = 0):
        self._require_ready()
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        v = None if voiceEmbeddings is None else np.ascontiguousarray(voiceEmbeddings, dtype=np.float32)
        n_voice = audioTokenCount if v is not None else 0
        self._check(load_library().vx_prefill(self._h, slot, _p(t, _i32p), t.size, audioTokenStart, n_voice,
                                              _p(v, _f32p)))

    def backboneStep(self, tokenId: int = 0, useAudioEmbedding: bool = False, embed=None, lmHead: bool = False,
                     slot: int = 0):
        self._require_ready()
        normed = np.empty(self._cfg.dim, np.float32)
        am = np.zeros(1, np.int32)
        e = None if embed is None else np.ascontiguousarray(embed, dtype=np.float32)
        self._check(load_library().vx_backbone_step(self._h, slot, int(tokenId), int(useAudioEmbedding),
                                                    _p(e, _f32p), _p(normed, _f32p), _p(am, _i32p) if lmHead else None))
        return normed, (int(am[0]) if lmHead else None)

    def backboneStepAndRead(self, tokenId: int, useAudioEmbedding: bool = False, slot: int = 0) -> int:
        """backboneStepAndRead (src/engine.ts:2333): LM-head argmax of the step."""
        return self.backboneStep(tokenId, useAudioEmbedding, lmHead=True, slot=slot)[1]

    def debugBackboneStepFull(self, tokenId: int, useAudioEmbedding: bool = False, slot: int = 0) -> np.ndarray:
        """debugBackboneStepFull (src/engine.ts:2348): the final-norm output."""
        return self.backboneStep(tokenId, useAudioEmbedding, slot=slot)[0]

    def backboneStepCodes(self, semanticCode: int, acousticCodes, slot: int = 0) -> np.ndarray:
        self._require_ready()
        normed = np.empty(self._cfg.dim, np.float32)
        ac = np.ascontiguousarray(acousticCodes, dtype=np.uint32)
        self._check(load_library().vx_backbone_step_codes(self._h, slot, int(semanticCode), _p(ac, _u32p),
                                                          _p(normed, _f32p)))
        return normed

    def debugFMStep(self, debugNoise=None, slot: int = 0) -> dict:
        """debugFMStep(noise) (src/engine.ts:2363) plus the semantic code the slot selects
        (masked argmax, or top-p after set_sampling('top_p'))."""
        self._require_ready()
        lg = np.empty(self._cfg.fm_semantic_vocab, np.float32)
        sem = np.zeros(1, np.uint32)
        ac = np.empty(36, np.uint32)
        xf = np.empty(36, np.float32)
        nz = None if debugNoise is None else np.ascontiguousarray(debugNoise, dtype=np.float32)
        self._check(load_library().vx_fm_step(self._h, slot, _p(nz, _f32p), _p(lg, _f32p), _p(sem, _u32p),
                                              _p(ac, _u32p), _p(xf, _f32p)))
        return {"semantic_logits": lg, "acoustic_codes": ac, "x_final": xf, "semantic_code": int(sem[0])}

    # ------------------------------------------------------------------ codec decoder
    @staticmethod
    def _codes(semanticCodes, acousticCodes):
        sem = np.ascontiguousarray(semanticCodes, dtype=np.uint32).ravel()
        ac = np.ascontiguousarray(acousticCodes, dtype=np.uint32).ravel()
        if sem.size == 0 or ac.size != sem.size * 36:
            raise ValueError(f"{sem.size} semantic codes need {sem.size * 36} acoustic codes, got {ac.size}")
        return sem, ac

    def codecDecode(self, semanticCodes, acousticCodes) -> np.ndarray:
        """codecDecode (src/engine.ts:1402-1713): [T] semantic + [T, 36] acoustic codes ->
        T * 1920 samples at 24 kHz (f32)."""
        self._require_ready()
        sem, ac = self._codes(semanticCodes, acousticCodes)
        out = np.empty(sem.size * 1920, np.float32)
        self._check(load_library().vx_codec_decode(self._h, _p(sem, _u32p), _p(ac, _u32p), sem.size, _p(out, _f32p)))
        return out

    def debugCodecDecode(self, semanticCodes, acousticCodes) -> dict:
        """debugCodecDecode (src/engine.ts:1719-1975): the intermediates by the reference's names."""
        self._require_ready()
        sem, ac = self._codes(semanticCodes, acousticCodes)
        T = sem.size
        n = load_library().vx_codec_debug_size(T)
        buf = np.empty(n, np.float32)
        self._check(load_library().vx_codec_debug(self._h, _p(sem, _u32p), _p(ac, _u32p), T, _p(buf, _f32p), n))
        return split_codec_debug(buf, T)

    def fmStepAndRead(self, slot: int = 0) -> np.ndarray:
        """fmStepAndRead (src/engine.ts:2386): the 36 acoustic codes."""
        return self.debugFMStep(None, slot)["acoustic_codes"]

    def debugBackboneLayerByLayer(self, tokenId: int, slot: int = 0) -> dict:
        """debugBackboneLayerByLayer (src/engine.ts:2106)."""
        self._require_ready()
        L = self._cfg.n_layers
        out = np.empty((4 * L + 3, self._cfg.dim), np.float32)
        self._check(load_library().vx_debug_layers(self._h, slot, int(tokenId), _p(out, _f32p)))
        layers = [{"attn_norm": out[1 + 4 * l], "attn_out": out[2 + 4 * l], "ffn_norm": out[3 + 4 * l],
                   "ffn_out": out[4 + 4 * l]} for l in range(L)]
        return {"embed": out[0], "layers": layers, "final_norm": out[1 + 4 * L], "hidden": out[2 + 4 * L],
                "raw": out}

    # ------------------------------------------------------------------ decode loop
    def decode(self, n_frames: int, with_fm: bool = True, slot: int = 0):
        """Enqueue n_frames device-resident frames (no host round trip); asynchronous."""
        self._require_ready()
        self._check(load_library().vx_decode(self._h, slot, n_frames, int(with_fm)))

    def decode_record(self, n_frames: int, record_frame: int, slot: int = 0) -> np.ndarray:
        """Backbone-only decode of n_frames frames (as decode(n, with_fm=False)) that returns the
        per-layer tensors of frame record_frame, rows as in debugBackboneLayerByLayer's "raw"."""
        self._require_ready()
        out = np.empty((4 * self._cfg.n_layers + 3, self._cfg.dim), np.float32)
        self._check(load_library().vx_decode_record(self._h, slot, n_frames, record_frame, _p(out, _f32p)))
        return out

    def decode_batch(self, n_frames: int, n_slots: int, slot0: int = 0):
        """Backbone-only decode of n_frames frames for slots [slot0, slot0+n_slots) in lockstep
        (tensor-core GEMMs over the slots); asynchronous."""
        self._require_ready()
        self._check(load_library().vx_decode_batch(self._h, slot0, n_slots, n_frames))

    def fill_kv(self, n_positions: int, seed: int, slot: int = 0):
        """Synthetic context: f16 N(0,1) K/V for positions [0, n_positions) of every layer."""
        self._require_ready()
        self._check(load_library().vx_fill_kv(self._h, slot, n_positions, seed))

    def read_codes(self, frame0: int, n: int, slot: int = 0) -> np.ndarray:
        out = np.empty((n, 37), np.uint32)
        self._check(load_library().vx_read_codes(self._h, slot, frame0, n, _p(out, _u32p)))
        return out

    def read_normed(self, frame0: int, n: int, slot: int = 0) -> np.ndarray:
        out = np.empty((n, self._cfg.dim), np.float32)
        self._check(load_library().vx_read_normed(self._h, slot, frame0, n, _p(out, _f32p)))
        return out

    def generate(self, tokens, audioTokenStart: int, audioTokenCount: int, voiceEmbeddings=None,
                 maxFrames: int = 500, onFrame: Optional[Callable] = None, onStage: Optional[Callable] = None,
                 eos: bool = True, slot: int = 0, chunk: int = 16) -> TTSResult:
        """generate() (src/engine.ts:2416-2616).

        Prefill (voice rows replace the [AUDIO] embeddings), the AUDIO kick, then
        maxFrames frames on the device.  Semantic selection runs inside the FM graph:
        the masked argmax (sampling='argmax', the parity mode) or the reference's
        sampleTopP(0.9, 0.8) (sampling='top_p'; the draw of frame f comes from the
        seeded stream samplingSeed, so a run is reproducible).  EOS (semantic code <= 1)
        stops the loop as in the reference; frames are run in chunks and anything after
        EOS is discarded."""
        self._require_ready()
        t0 = time.perf_counter()
        self.reset(slot)
        self.set_sampling(self._sampling, 0.9, 0.8, self._sampling_seed, slot)
        if onStage:
            onStage("backbone")
        self.prefill(tokens, audioTokenStart, audioTokenCount, voiceEmbeddings, slot)
        self.backboneStep(AUDIO_TOKEN, slot=slot)
        t_prefill = time.perf_counter()
        if onStage:
            onStage("backbone", (t_prefill - t0) * 1e3)
            onStage("fm")
        sem_codes, ac_codes = [], []
        f = 0
        done = False
        while f < maxFrames and not done:
            n = min(chunk, maxFrames - f)
            self.decode(n, with_fm=True, slot=slot)
            codes = self.read_codes(f, n, slot)
            for i in range(n):
                code = int(codes[i, 0])
                if eos and code <= 1:
                    done = True
                    break
                sem_codes.append(code)
                ac_codes.append(codes[i, 1:].astype(np.int64))
                if onFrame:
                    onFrame(f + i, code, codes[i, 1:])
            f += n
        t_gen = time.perf_counter()
        if onStage:
            onStage("fm", (t_gen - t_prefill) * 1e3)
            onStage("codec")
        # Phase 3: codec decode of all frames (src/engine.ts:2590-2601)
        audio = np.zeros(0, np.float32)
        if sem_codes and self._cfg.enable_codec:
            audio = self.codecDecode(np.asarray(sem_codes, np.uint32), np.stack(ac_codes).astype(np.uint32))
        t_codec = time.perf_counter()
        if onStage:
            onStage("codec", (t_codec - t_gen) * 1e3)
        return TTSResult(
            semanticCodes=sem_codes, acousticCodes=[a.tolist() for a in ac_codes], audio=audio,
            stats={"backboneMs": (t_prefill - t0) * 1e3, "fmMs": (t_gen - t_prefill) * 1e3,
                   "codecMs": (t_codec - t_gen) * 1e3, "totalMs": (t_codec - t0) * 1e3,
                   "framesGenerated": len(sem_codes)})


CODEC_DEBUG_ORDER = [("concat", 0, 292), ("after_input_conv", 0, 1024)] + [
    item for s in range(4) for item in
    [(f"after_stage{s}_transformer", s, 1024)] + ([(f"after_stage{s}_conv_up", s + 1, 1024)] if s < 3 else [])
] + [("audio", 3, 240)]


def split_codec_debug(buf: np.ndarray, T: int) -> dict:
    """The concatenated intermediates of vx_codec_debug (and of the oracle) by name, each
    [rows, channels] with rows = T * 2^stage; vq_embed / fsq_dequant are the two parts of
    concat, after_output_conv the audio rows."""
    out, off = {}, 0
    for name, s, w in CODEC_DEBUG_ORDER:
        rows = (T << s) if name != "audio" else 8 * T
        out[name] = buf[off: off + rows * w].reshape(rows, w)
        off += rows * w
    assert off == buf.size, (off, buf.size)
    out["vq_embed"] = out["concat"][:, :256]
    out["fsq_dequant"] = out["concat"][:, 256:]
    out["after_output_conv"] = out["audio"]
    return out


def header_symbols() -> list:
    """Function names declared in include/voxtral_b200.h."""
    import re
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vx_[a-z_0-9]+)\s*\(", src)))


def nccl_unique_id(nccl_lib: Optional[str] = None) -> bytes:
    buf = (ctypes.c_uint8 * 128)()
    rc = load_library().vx_nccl_unique_id(nccl_lib.encode() if nccl_lib else None, buf)
    if rc != VX_OK:
        raise VoxtralError(rc, "ncclGetUniqueId failed")
    return bytes(buf)


def tp_init(engine: VoxtralEngine, uid: bytes, nccl_lib: Optional[str] = None, p2p: bool = True):
    """Tensor-parallel set-up of one rank: NCCL (per-op path) and, with p2p, the peer-memory
    all-reduce of the persistent decode kernel (IPC handles exchanged with torch.distributed;
    ends with a barrier so no rank starts decoding before every rank's buffers are open)."""
    buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
    L = load_library()
    engine._check(L.vx_tp_init(engine.handle, nccl_lib.encode() if nccl_lib else None, buf))
    if p2p:
        from . import dist as vdist
        mine = (ctypes.c_uint8 * 64)()
        engine._check(L.vx_tp_p2p_handle(engine.handle, mine))
        allh = b"".join(vdist.all_gather_bytes(bytes(mine)))
        engine._check(L.vx_tp_p2p_open(engine.handle, (ctypes.c_uint8 * len(allh)).from_buffer_copy(allh)))
        vdist.barrier()
