"""Independent float64 numpy restatement of the reference's decode path.

TEST INFRASTRUCTURE ONLY (used by tests/golden/make_golden.py).  It shares no code
with oracle.cpp except the synthetic-input generator, and computes in float64 with
plain formulas (no mimicry of the WGSL reduction orders), so agreement between the
two restatements checks the f32 oracle's arithmetic, not just its plumbing.
PARITY UNPINNED: both restate src/shaders.ts and src/engine.ts of the reference,
which cannot run here.

Formulas (reference file:line):
  RMSNorm            x / sqrt(mean(x^2) + 1e-5) * w          src/shaders.ts:137-183
  RoPE (interleaved) freq_i = theta^(-2i/128), angle = pos*freq src/shaders.ts:224-256
  GQA attention      softmax(q.K^T / sqrt(128)) V, kv = h // 4 src/shaders.ts:306-447
  SwiGLU             silu(w1 x) * (w3 x)                      src/shaders.ts:483-501
  block              h += Wo attn(norm(h)); h += W2 ffn(norm(h)) src/engine.ts:859-1007
  FM                 3-token bidirectional pass, no RoPE      src/engine.ts:1057-1225
  Euler/CFG/FSQ      v = 1.2 vc - 0.2 vu; x += v/7; codes      src/shaders.ts:611-673
"""
from __future__ import annotations

import importlib
import os
import sys

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)
synth = importlib.import_module("webgpu-voxtral_b200.synth")

D, HD, NH, NKV, F = 3072, 128, 32, 8, 9216
Q, KV = NH * HD, NKV * HD


def _mat(name: str, rows: int, cols: int) -> np.ndarray:
    out = np.empty((rows, cols), dtype=np.float64)
    step = max(1, (1 << 24) // cols)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        out[r0:r1] = synth.tensor_values(name, r0 * cols, (r1 - r0) * cols).astype(np.float64).reshape(r1 - r0, cols)
    return out


def _layer(prefix: str):
    return {
        "wq": _mat(prefix + "attention.wq.weight", Q, D),
        "wk": _mat(prefix + "attention.wk.weight", KV, D),
        "wv": _mat(prefix + "attention.wv.weight", KV, D),
        "wo": _mat(prefix + "attention.wo.weight", D, Q),
        "w1": _mat(prefix + "feed_forward.w1.weight", F, D),
        "w2": _mat(prefix + "feed_forward.w2.weight", D, F),
        "w3": _mat(prefix + "feed_forward.w3.weight", F, D),
    }


def rmsnorm(x, eps=1e-5):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)  # gains are 1.0


def rope(v, pos, theta):
    nh = v.shape[0] // HD
    vv = v.reshape(nh, HD // 2, 2)
    freq = theta ** (-(2.0 * np.arange(HD // 2)) / HD)
    c, s = np.cos(pos * freq), np.sin(pos * freq)
    x0, x1 = vv[..., 0], vv[..., 1]
    return np.stack([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1).reshape(-1)


def silu(g):
    return g / (1.0 + np.exp(-g))


class RefModel:
    def __init__(self, n_layers: int = 2, with_fm: bool = True, lm_head: bool = False):
        self.layers = [_layer(f"layers.{i}.") for i in range(n_layers)]
        self.audio_name = "mm_audio_embeddings.audio_codebook_embeddings.embeddings.weight"
        self.tok_name = "mm_audio_embeddings.tok_embeddings.weight"
        self.tok = _mat(self.tok_name, 131072, D) if lm_head else None
        self.K = [[] for _ in range(n_layers)]
        self.V = [[] for _ in range(n_layers)]
        self.pos = 0
        if with_fm:
            p = "acoustic_transformer."
            self.fm_layers = [_layer(f"{p}layers.{i}.") for i in range(3)]
            self.fm_in = _mat(p + "input_projection.weight", D, 36)
            self.fm_llm = _mat(p + "llm_projection.weight", D, D)
            self.fm_time = _mat(p + "time_projection.weight", D, D)
            self.fm_sem = _mat(p + "semantic_codebook_output.weight", 8320, D)
            self.fm_ac = _mat(p + "acoustic_codebook_output.weight", 36, D)

    def tok_row(self, t):
        return synth.tensor_values(self.tok_name, t * D, D).astype(np.float64)

    def audio_row(self, t):
        return synth.tensor_values(self.audio_name, t * D, D).astype(np.float64)

    def multi_codebook_embed(self, sem, ac):
        h = self.audio_row(sem)
        for k in range(36):
            h = h + self.audio_row(8194 + 23 * k + int(ac[k]))
        return h

    def step(self, token=0, embed=None, debug=False):
        h = np.asarray(embed, np.float64) if embed is not None else self.tok_row(token)
        dbg = [h.copy()]
        pos = self.pos
        for l, L in enumerate(self.layers):
            x = rmsnorm(h)
            q = rope(L["wq"] @ x, pos, 1e6)
            k = rope(L["wk"] @ x, pos, 1e6)
            v = L["wv"] @ x
            self.K[l].append(k)
            self.V[l].append(v)
            Km = np.stack(self.K[l]).reshape(-1, NKV, HD)
            Vm = np.stack(self.V[l]).reshape(-1, NKV, HD)
            att = np.empty(Q)
            for hh in range(NH):
                kv = hh // (NH // NKV)
                s = Km[:, kv, :] @ q[hh * HD:(hh + 1) * HD] / np.sqrt(HD)
                p = np.exp(s - s.max())
                p /= p.sum()
                att[hh * HD:(hh + 1) * HD] = p @ Vm[:, kv, :]
            h = h + L["wo"] @ att
            dbg += [x, h.copy()]
            x2 = rmsnorm(h)
            h = h + L["w2"] @ (silu(L["w1"] @ x2) * (L["w3"] @ x2))
            dbg += [x2, h.copy()]
        normed = rmsnorm(h)
        self.pos += 1
        # reorder debug into [embed, (attn_norm, attn_out, ffn_norm, ffn_out) * L, final_norm, hidden]
        out = {"normed": normed, "hidden": h}
        if debug:
            out["debug"] = np.stack(dbg + [normed, h])
        if self.tok is not None:
            out["argmax"] = int(np.argmax(self.tok @ normed))
        return out

    def fm_pass(self, seq):
        """seq: [nseq, 3, D] -> velocity [nseq, 36]."""
        seq = seq.copy()
        for L in self.fm_layers:
            x = rmsnorm(seq)
            q = (x @ L["wq"].T).reshape(seq.shape[0], 3, NH, HD)
            k = (x @ L["wk"].T).reshape(seq.shape[0], 3, NKV, HD)
            v = (x @ L["wv"].T).reshape(seq.shape[0], 3, NKV, HD)
            kr = np.repeat(k, NH // NKV, axis=2)
            vr = np.repeat(v, NH // NKV, axis=2)
            s = np.einsum("bqhd,bkhd->bhqk", q, kr) / np.sqrt(HD)
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            att = np.einsum("bhqk,bkhd->bqhd", p, vr).reshape(seq.shape[0], 3, Q)
            seq = seq + att @ L["wo"].T
            x2 = rmsnorm(seq)
            seq = seq + (silu(x2 @ L["w1"].T) * (x2 @ L["w3"].T)) @ L["w2"].T
        return rmsnorm(seq[:, 0, :]) @ self.fm_ac.T

    def fm_forward(self, normed, noise):
        sem_logits = self.fm_sem @ normed
        llm = self.fm_llm @ normed
        x = np.asarray(noise, np.float64).copy()
        half = D // 2
        freq = np.exp(-np.log(1e4) * np.arange(half) / half)
        for s in range(7):
            t = s / 7.0
            te = np.concatenate([np.cos(t * freq), np.sin(t * freq)])
            tp = self.fm_time @ te
            xp = self.fm_in @ x
            seq = np.stack([np.stack([xp, tp, llm]), np.stack([xp, tp, np.zeros(D)])])
            vel = self.fm_pass(seq)
            x = x + (1.2 * vel[0] - 0.2 * vel[1]) / 7.0
        codes = np.rint((np.clip(x, -1, 1) + 1) * 0.5 * 20).clip(0, 20).astype(np.uint32) + 2
        masked = sem_logits.copy()
        masked[0] = -np.inf
        masked[8194:] = -np.inf
        return {"semantic_logits": sem_logits, "x_final": x, "acoustic_codes": codes,
                "semantic_code": int(np.argmax(masked))}
