"""Independent float64 numpy restatement of the codec decoder.

TEST INFRASTRUCTURE ONLY (tests/test_codec_oracle.py).  It takes its weights from
the C++ oracle (so both use the same synthetic tensors) but shares none of its
arithmetic: plain float64 formulas, no mimicry of the WGSL reduction orders, so its
agreement with oracle.cpp checks that restatement's arithmetic.  PARITY UNPINNED:
both restate src/shaders.ts and src/engine.ts of the reference, which cannot run here.

Formulas (reference file:line):
  codebook          f16(embedding_sum / max(usage, 1e-5))            src/shaders.ts:856-888
  VQ / FSQ / concat [codebook[sem], (ac - 2) * 2/20 - 1]               src/shaders.ts:817-917, 1840-1867
  causal conv       y[t] = sum_k W_k x[t - K + 1 + k],  W = g v / |v|  src/shaders.ts:919-979
                    (|v| over (c_in, k) per output channel)
  layer             x += s_a * Wo attn(norm(x)); x += s_f * W2 swiglu(norm(x))   src/engine.ts:1501-1646
                    norm eps 0.01; per-head q/k RMSNorm eps 1e-6
  attention         softmax(q.k / sqrt(128) - 2^-(h+1) (qi - ki)) over ki in (qi - W, qi]
                    with W = 2, 4, 8, 16 per stage                      src/shaders.ts:1432-1575
  transposed conv   y[t] = sum_{k: t-k even} W_k^T x[(t-k)/2],  W = v g[ci] / |v[ci]|   src/shaders.ts:1004-1104
  output conv       7 taps, 1024 -> 240, flattened to the waveform       src/engine.ts:1690-1702
"""
from __future__ import annotations

import numpy as np

DIM, HID, NH, HD = 1024, 4096, 8, 128
P = "audio_tokenizer."


def _f(a) -> np.ndarray:
    return np.asarray(a, dtype=np.uint16).view(np.float16).astype(np.float64)


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def _conv(x, v, g, c_out, c_in, K):
    W = _f(v).reshape(c_out, c_in, K)
    W = W * (_f(g)[:, None, None] / np.sqrt(np.sum(W * W, axis=(1, 2), keepdims=True) + 1e-12))
    T = x.shape[0]
    y = np.zeros((T, c_out))
    for k in range(K):
        sh = K - 1 - k
        if sh < T:
            y[sh:] += x[: T - sh] @ W[:, :, k].T
    return y


def _conv_t(x, v, g):
    W = _f(v).reshape(DIM, DIM, 4)
    W = W * (_f(g)[:, None, None] / np.sqrt(np.sum(W * W, axis=(1, 2), keepdims=True) + 1e-12))
    T = x.shape[0]
    y = np.zeros((2 * T, DIM))
    for k in range(4):
        for t in range(2 * T):
            if t - k >= 0 and (t - k) % 2 == 0:
                y[t] += x[(t - k) // 2] @ W[:, :, k]
    return y


def _layer(get, pre, x, W):
    N = x.shape[0]
    n = _rms(x, _f(get(pre + "attention_norm.weight", DIM)), 0.01)
    q = n @ _f(get(pre + "attention.wq.weight", DIM * DIM)).reshape(DIM, DIM).T
    k = n @ _f(get(pre + "attention.wk.weight", DIM * DIM)).reshape(DIM, DIM).T
    v = n @ _f(get(pre + "attention.wv.weight", DIM * DIM)).reshape(DIM, DIM).T
    q = _rms(q.reshape(N, NH, HD), _f(get(pre + "attention.q_norm.weight", DIM)).reshape(NH, HD), 1e-6)
    k = _rms(k.reshape(N, NH, HD), _f(get(pre + "attention.k_norm.weight", DIM)).reshape(NH, HD), 1e-6)
    v = v.reshape(N, NH, HD)
    att = np.zeros((N, NH, HD))
    for h in range(NH):
        for qi in range(N):
            ks = np.arange(max(0, qi - W + 1), qi + 1)
            s = k[ks, h] @ q[qi, h] / np.sqrt(HD) - 2.0 ** -(h + 1) * (qi - ks)
            p = np.exp(s - s.max())
            att[qi, h] = (p / p.sum()) @ v[ks, h]
    wo = _f(get(pre + "attention.wo.weight", DIM * DIM)).reshape(DIM, DIM)
    x = x + (att.reshape(N, DIM) @ wo.T) * _f(get(pre + "attention_scale", DIM))
    n = _rms(x, _f(get(pre + "ffn_norm.weight", DIM)), 0.01)
    g = n @ _f(get(pre + "feed_forward.w1.weight", HID * DIM)).reshape(HID, DIM).T
    u = n @ _f(get(pre + "feed_forward.w3.weight", HID * DIM)).reshape(HID, DIM).T
    a = g / (1.0 + np.exp(-g)) * u
    x = x + (a @ _f(get(pre + "feed_forward.w2.weight", DIM * HID)).reshape(DIM, HID).T) * _f(get(pre + "ffn_scale", DIM))
    return x


def decode(get, sem, ac) -> dict:
    """get(name, numel) -> f16 bits of a codec tensor.  Returns the debugCodecDecode
    intermediates (float64)."""
    sem = np.asarray(sem, dtype=np.uint32)
    ac = np.asarray(ac, dtype=np.uint32).reshape(-1, 36)
    total = _f(get(P + "quantizer.semantic_codebook.embedding_sum", 8192 * 256)).reshape(8192, 256)
    usage = _f(get(P + "quantizer.semantic_codebook.cluster_usage", 8192))
    cb = (total.astype(np.float32) / np.maximum(usage.astype(np.float32), np.float32(1e-5))[:, None]).astype(np.float16)
    vq = np.zeros((sem.size, 256))
    ok = sem < 8192
    vq[ok] = cb[sem[ok]].astype(np.float64)
    fsq = (ac - np.uint32(2)).astype(np.float64) * 2.0 / 20.0 - 1.0
    out = {"concat": np.concatenate([vq, fsq], axis=1)}
    blk = P + "decoder_blocks."
    x = _conv(out["concat"], get(blk + "0.conv.parametrizations.weight.original1", DIM * 292 * 3),
              get(blk + "0.conv.parametrizations.weight.original0", DIM), DIM, 292, 3)
    out["after_input_conv"] = x
    for s in range(4):
        for l in range(2):
            x = _layer(get, f"{blk}{1 + 2 * s}.layers.{l}.", x, 2 << s)
        out[f"after_stage{s}_transformer"] = x
        if s < 3:
            c = f"{blk}{2 + 2 * s}.conv.parametrizations.weight."
            x = _conv_t(x, get(c + "original1", DIM * DIM * 4), get(c + "original0", DIM))
            out[f"after_stage{s}_conv_up"] = x
    out["audio"] = _conv(x, get(P + "output_proj.conv.parametrizations.weight.original1", 240 * DIM * 7),
                         get(P + "output_proj.conv.parametrizations.weight.original0", 240), 240, DIM, 7)
    return out
