// oracle.cpp — CPU restatement of the reference's per-frame decode path.
//
// TEST INFRASTRUCTURE ONLY.  Nothing in the product imports, links or runs this
// file: tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and
// `bench.py --impl reference`) use it as the checker / CPU baseline.
//
// PARITY UNPINNED.  The reference (svenflow/webgpu-voxtral) is TypeScript that
// drives WGSL shaders through a browser WebGPU implementation.  It has no CPU
// code path and no golden vectors (its fixtures are git-ignored:
// .gitignore:5-10), and no WebGPU implementation can run on this machine, so
// this restatement cannot be checked against outputs of the reference itself.
// It is cross-checked against an independent float64 numpy restatement
// (oracle/numpy_ref.py) and pinned by the fixtures in tests/golden/.
//
// Each function follows one reference shader or engine routine, cited as
// file:line of the reference tree, with the same f32 operation order where the
// order is observable (strided 256-lane partial sums + tree reductions, the
// (x*rms)*w norm product, sequential attention dot products).  Weights are f16
// bits, activations f32, the KV cache f32 — as in the reference
// (src/engine.ts:510-530).  Build with -ffp-contract=off so that no FMA
// contraction changes the rounding.
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#if defined(__F16C__) && defined(__AVX2__)
#include <immintrin.h>
#define ORC_F16C 1
#endif
#include <omp.h>

#include "../webgpu-voxtral_b200/csrc/vx_rng.h"

namespace {

// VoxtralConfig (src/types.ts:70-122); n_layers / max_seq are overridable.
struct Dims {
  int dim = 3072, n_layers = 26, head_dim = 128, hidden = 9216, n_heads = 32, n_kv = 8;
  int vocab = 131072;
  float rope_theta = 1.0e6f, eps = 1e-5f;
  int fm_layers = 3, nfe = 8, n_ac = 36, sem_vocab = 8320, ac_levels = 21;
  float cfg_alpha = 1.2f;
  int audio_rows = 9088;
};

float g_f16_lut[65536];
void init_lut() {
  static bool done = false;
  if (done) return;
  for (int i = 0; i < 65536; ++i) g_f16_lut[i] = vx_f16_bits_to_f32((uint16_t)i);
  done = true;
}

struct Layer {
  std::vector<uint16_t> wq, wk, wv, wo, w1, w2, w3, attn_norm, ffn_norm;
};

struct Model {
  Dims d;
  int max_seq = 4096;
  bool with_fm = true;
  std::vector<uint16_t> tok_emb, audio_emb, final_norm;
  std::vector<Layer> layers;
  // FM (acoustic transformer)
  std::vector<uint16_t> fm_in, fm_llm, fm_time, fm_norm, fm_sem, fm_ac;
  std::vector<Layer> fm_layers;
  // state
  std::vector<float> kc, vc;  // [L][max_seq][1024] f32 (src/engine.ts:510-530)
  int position = 0;
  std::vector<float> hidden, normed;
};

// ---------------------------------------------------------------------------
// Synthetic weights: the reference's tensor names and shapes (organizeWeights,
// src/engine.ts:659-743), values from vx_rng.h.
void gen_tensor(std::vector<uint16_t>& t, const std::string& name, size_t n, bool is_norm) {
  t.resize(n);
  if (is_norm) {
    std::fill(t.begin(), t.end(), (uint16_t)0x3C00);  // gain 1.0
    return;
  }
  const uint64_t key = vx_stream_key(VX_SEED_WEIGHTS, vx_fnv1a(name.c_str()));
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < (long long)n; ++i)
    t[i] = vx_f32_to_f16_bits(vx_normal(key, (uint64_t)i) * VX_WEIGHT_SIGMA);
}

void gen_layer(Layer& L, const std::string& p, const Dims& d) {
  const size_t D = d.dim, Q = (size_t)d.n_heads * d.head_dim, KV = (size_t)d.n_kv * d.head_dim,
               F = d.hidden;
  gen_tensor(L.wq, p + "attention.wq.weight", Q * D, false);
  gen_tensor(L.wk, p + "attention.wk.weight", KV * D, false);
  gen_tensor(L.wv, p + "attention.wv.weight", KV * D, false);
  gen_tensor(L.wo, p + "attention.wo.weight", D * Q, false);
  gen_tensor(L.w1, p + "feed_forward.w1.weight", F * D, false);
  gen_tensor(L.w2, p + "feed_forward.w2.weight", D * F, false);
  gen_tensor(L.w3, p + "feed_forward.w3.weight", F * D, false);
  gen_tensor(L.attn_norm, p + "attention_norm.weight", D, true);
  gen_tensor(L.ffn_norm, p + "ffn_norm.weight", D, true);
}

// ---------------------------------------------------------------------------
// matvecF16 (src/shaders.ts:21-71): one 256-lane workgroup per output row; lane
// t sums pairs pk = t, t+256, ... as sum += (w0*x0 + w1*x1); then a tree
// reduction sdata[t] += sdata[t+s] for s = 128..1.  `nvec` input vectors share
// each weight row (the FM runs the same matrix on several positions, each as
// its own dispatch of this shader: src/engine.ts:1096-1105).
void matvec_f16(const uint16_t* A, int M, int K, int nvec, const float* const* xs, float* const* ys) {
  init_lut();
  const int K2 = K / 2;
  std::vector<std::vector<float>> xe(nvec, std::vector<float>(K2)), xo(nvec, std::vector<float>(K2));
  for (int v = 0; v < nvec; ++v)
    for (int k = 0; k < K2; ++k) { xe[v][k] = xs[v][2 * k]; xo[v][k] = xs[v][2 * k + 1]; }
#pragma omp parallel
  {
    std::vector<float> we(K2 + 16), wo(K2 + 16);
    float s[256];
#pragma omp for schedule(static)
    for (int row = 0; row < M; ++row) {
      const uint16_t* w = A + (size_t)row * K;
      int k = 0;
#ifdef ORC_F16C
      for (; k + 8 <= K2; k += 8) {
        __m256 a = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(w + 2 * k)));
        __m256 b = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(w + 2 * k + 8)));
        __m256 e = _mm256_shuffle_ps(a, b, 0x88);
        __m256 o = _mm256_shuffle_ps(a, b, 0xDD);
        e = _mm256_castpd_ps(_mm256_permute4x64_pd(_mm256_castps_pd(e), 0xD8));
        o = _mm256_castpd_ps(_mm256_permute4x64_pd(_mm256_castps_pd(o), 0xD8));
        _mm256_storeu_ps(&we[k], e);
        _mm256_storeu_ps(&wo[k], o);
      }
#endif
      for (; k < K2; ++k) { we[k] = g_f16_lut[w[2 * k]]; wo[k] = g_f16_lut[w[2 * k + 1]]; }
      for (int v = 0; v < nvec; ++v) {
        const float* e = xe[v].data();
        const float* o = xo[v].data();
        for (int t = 0; t < 256; ++t) s[t] = 0.f;
        for (int base = 0; base < K2; base += 256) {
          const int n = std::min(256, K2 - base);
          for (int t = 0; t < n; ++t)
            s[t] = s[t] + (we[base + t] * e[base + t] + wo[base + t] * o[base + t]);
        }
        for (int st = 128; st > 0; st >>= 1)
          for (int t = 0; t < st; ++t) s[t] += s[t + st];
        ys[v][row] = s[0];
      }
    }
  }
}

void matvec1(const uint16_t* A, int M, int K, const float* x, float* y) {
  const float* xs[1] = {x};
  float* ys[1] = {y};
  matvec_f16(A, M, K, 1, xs, ys);
}

// rmsNorm (src/shaders.ts:137-183): strided 256-lane sum of squares, tree
// reduction, rms = 1/sqrt(ss/dim + eps), y = (x*rms)*w.
void rms_norm(const float* x, const uint16_t* w, int dim, float eps, float* y) {
  init_lut();
  float s[256];
  for (int t = 0; t < 256; ++t) {
    float ss = 0.f;
    for (int i = t; i < dim; i += 256) ss += x[i] * x[i];
    s[t] = ss;
  }
  for (int st = 128; st > 0; st >>= 1)
    for (int t = 0; t < st; ++t) s[t] += s[t + st];
  const float rms = 1.0f / sqrtf(s[0] / (float)dim + eps);
  for (int i = 0; i < dim; ++i) y[i] = x[i] * rms * g_f16_lut[w[i]];
}

// rope (src/shaders.ts:224-256): interleaved pairs (2i, 2i+1) of each head,
// freq_i = 1/theta^(2i/head_dim), angle = f32(pos)*freq_i.  The frequency table
// is formed in double and rounded to f32 once (the shader's f32 pow() carries
// an implementation-defined error of its own).
void rope(float* qk, int n_heads, int hd, int pos, float theta) {
  for (int h = 0; h < n_heads; ++h)
    for (int i = 0; i < hd / 2; ++i) {
      const float freq = (float)(1.0 / pow((double)theta, (double)(2 * i) / (double)hd));
      const float ang = (float)pos * freq;
      const float c = cosf(ang), s = sinf(ang);
      float* p = qk + h * hd + 2 * i;
      const float x0 = p[0], x1 = p[1];
      p[0] = x0 * c - x1 * s;
      p[1] = x0 * s + x1 * c;
    }
}

// softmax (src/shaders.ts:348-409) over n values: strided max (init -1e30),
// tree max, exp(s-max) with strided sums + tree, then s /= sum.
void softmax_256(float* sc, int n) {
  float s[256];
  for (int t = 0; t < 256; ++t) {
    float m = -1e30f;
    for (int i = t; i < n; i += 256) m = std::max(m, sc[i]);
    s[t] = m;
  }
  for (int st = 128; st > 0; st >>= 1)
    for (int t = 0; t < st; ++t) s[t] = std::max(s[t], s[t + st]);
  const float gmax = s[0];
  for (int t = 0; t < 256; ++t) {
    float acc = 0.f;
    for (int i = t; i < n; i += 256) {
      const float e = expf(sc[i] - gmax);
      sc[i] = e;
      acc += e;
    }
    s[t] = acc;
  }
  for (int st = 128; st > 0; st >>= 1)
    for (int t = 0; t < st; ++t) s[t] += s[t + st];
  const float tot = s[0];
  for (int i = 0; i < n; ++i) sc[i] /= tot;
}

// swiGLU (src/shaders.ts:483-501): g = (g / (1 + exp(-g))) * u.
inline float swiglu(float g, float u) {
  const float silu = g / (1.0f + expf(-g));
  return silu * u;
}

// argmax (src/shaders.ts:1154-1211): lane t keeps the first strict maximum of
// its stride (init -1e30, index 0); the tree keeps the lower lane on ties.
uint32_t argmax_shader(const float* x, int n) {
  float bv[256];
  uint32_t bi[256];
  for (int t = 0; t < 256; ++t) {
    float v = -1e30f;
    uint32_t idx = 0;
    for (int i = t; i < n; i += 256)
      if (x[i] > v) { v = x[i]; idx = (uint32_t)i; }
    bv[t] = v;
    bi[t] = idx;
  }
  for (int st = 128; st > 0; st >>= 1)
    for (int t = 0; t < st; ++t)
      if (bv[t + st] > bv[t]) { bv[t] = bv[t + st]; bi[t] = bi[t + st]; }
  return bi[0];
}

// Masked semantic selection used for parity in place of the host's
// sampleTopP (src/engine.ts:2551-2565): index 0 and indices >= 8194 masked,
// maximum over the rest, ties to the lowest index.
uint32_t masked_argmax(const float* x, int n, int valid) {
  uint32_t best = 1;
  float bv = x[1];
  for (int i = 2; i < std::min(n, valid); ++i)
    if (x[i] > bv) { bv = x[i]; best = (uint32_t)i; }
  return best;
}

// ---------------------------------------------------------------------------
// backboneStep (src/engine.ts:814-1042).  `embed` overrides the row lookup
// (voice rows and multi-codebook sums REPLACE the embedding: :843-854).
// debug (nullable) receives the tensors of debugBackboneLayerByLayer
// (src/engine.ts:2106-2287): embed, per layer {attn_norm, attn_out (hidden after
// the attention residual), ffn_norm, ffn_out}, then final_norm and hidden.
int backbone_step(Model& m, int token, bool use_audio, const float* embed, float* debug,
                  bool lm_head, uint32_t* argmax_out) {
  const Dims& d = m.d;
  const int D = d.dim, hd = d.head_dim, Q = d.n_heads * hd, KV = d.n_kv * hd, F = d.hidden;
  const int pos = m.position;
  if (pos >= m.max_seq) return -1;
  std::vector<float>& h = m.hidden;
  std::vector<float> res(D), x(D), q(Q), k(KV), v(KV), att(Q), gate(F), up(F), tmp(D);
  // embeddingLookup (src/shaders.ts:193-213) / copyBuffer of the override.
  if (embed) {
    memcpy(h.data(), embed, sizeof(float) * D);
  } else {
    const std::vector<uint16_t>& tab = use_audio ? m.audio_emb : m.tok_emb;
    const int rows = use_audio ? d.audio_rows : d.vocab;
    if (token < 0 || token >= rows) return -2;
    for (int i = 0; i < D; ++i) h[i] = g_f16_lut[tab[(size_t)token * D + i]];
  }
  if (debug) memcpy(debug, h.data(), sizeof(float) * D);
  const float scale = 1.0f / sqrtf((float)hd);
  const int seq = pos + 1, rep = d.n_heads / d.n_kv;
  std::vector<float> sc((size_t)d.n_heads * seq);
  for (int l = 0; l < d.n_layers; ++l) {
    const Layer& L = m.layers[l];
    res = h;
    rms_norm(h.data(), L.attn_norm.data(), D, d.eps, x.data());
    if (debug) memcpy(debug + (size_t)(1 + 4 * l) * D, x.data(), sizeof(float) * D);
    matvec1(L.wq.data(), Q, D, x.data(), q.data());
    matvec1(L.wk.data(), KV, D, x.data(), k.data());
    matvec1(L.wv.data(), KV, D, x.data(), v.data());
    rope(q.data(), d.n_heads, hd, pos, d.rope_theta);
    rope(k.data(), d.n_kv, hd, pos, d.rope_theta);
    // kvCacheWrite (src/shaders.ts:452-473)
    float* Kc = m.kc.data() + (size_t)l * m.max_seq * KV;
    float* Vc = m.vc.data() + (size_t)l * m.max_seq * KV;
    memcpy(Kc + (size_t)pos * KV, k.data(), sizeof(float) * KV);
    memcpy(Vc + (size_t)pos * KV, v.data(), sizeof(float) * KV);
    // attnScore (src/shaders.ts:306-342): sequential dot over d, times scale.
#pragma omp parallel for schedule(static)
    for (int hp = 0; hp < d.n_heads * seq; ++hp) {
      const int hh = hp / seq, p = hp % seq, kvh = hh / rep;
      const float* qq = q.data() + hh * hd;
      const float* kk = Kc + (size_t)p * KV + kvh * hd;
      float dot = 0.f;
      for (int e = 0; e < hd; ++e) dot += qq[e] * kk[e];
      sc[(size_t)hh * seq + p] = dot * scale;
    }
    for (int hh = 0; hh < d.n_heads; ++hh) softmax_256(sc.data() + (size_t)hh * seq, seq);
    // attnValue (src/shaders.ts:414-447): out[h,d] = sum_p s[h,p]*V[p,kvh,d].
#pragma omp parallel for schedule(static)
    for (int idx = 0; idx < Q; ++idx) {
      const int hh = idx / hd, e = idx % hd, kvh = hh / rep;
      float s = 0.f;
      for (int p = 0; p < seq; ++p) s += sc[(size_t)hh * seq + p] * Vc[(size_t)p * KV + kvh * hd + e];
      att[idx] = s;
    }
    // o_proj, then addInPlace with the residual (src/engine.ts:950-961).
    matvec1(L.wo.data(), D, Q, att.data(), h.data());
    for (int i = 0; i < D; ++i) h[i] = h[i] + res[i];
    if (debug) memcpy(debug + (size_t)(2 + 4 * l) * D, h.data(), sizeof(float) * D);
    res = h;
    rms_norm(h.data(), L.ffn_norm.data(), D, d.eps, x.data());
    if (debug) memcpy(debug + (size_t)(3 + 4 * l) * D, x.data(), sizeof(float) * D);
    matvec1(L.w1.data(), F, D, x.data(), gate.data());
    matvec1(L.w3.data(), F, D, x.data(), up.data());
    for (int i = 0; i < F; ++i) gate[i] = swiglu(gate[i], up[i]);
    matvec1(L.w2.data(), D, F, gate.data(), h.data());
    for (int i = 0; i < D; ++i) h[i] = h[i] + res[i];
    if (debug) memcpy(debug + (size_t)(4 + 4 * l) * D, h.data(), sizeof(float) * D);
  }
  rms_norm(h.data(), m.final_norm.data(), D, d.eps, m.normed.data());
  if (debug) {
    memcpy(debug + (size_t)(1 + 4 * d.n_layers) * D, m.normed.data(), sizeof(float) * D);
    memcpy(debug + (size_t)(2 + 4 * d.n_layers) * D, h.data(), sizeof(float) * D);
  }
  if (lm_head) {  // tied LM head + argmax (src/engine.ts:1017-1041)
    std::vector<float> logits(d.vocab);
    matvec1(m.tok_emb.data(), d.vocab, D, m.normed.data(), logits.data());
    if (argmax_out) *argmax_out = argmax_shader(logits.data(), d.vocab);
  }
  m.position++;
  return 0;
}

// multiCodebookEmbed (src/shaders.ts:1878-1917): row `sem` plus rows
// 8194 + 23k + ac[k] for the 36 acoustic codebooks, summed in that order.
int multi_codebook_embed(const Model& m, uint32_t sem, const uint32_t* ac, float* out) {
  const int D = m.d.dim;
  if ((int)sem >= m.d.audio_rows) return -2;
  for (int k = 0; k < 36; ++k)
    if (8194 + 23 * k + (int)ac[k] >= m.d.audio_rows) return -2;
  for (int i = 0; i < D; ++i) {
    float s = 0.f;
    s += g_f16_lut[m.audio_emb[(size_t)sem * D + i]];
    for (int k = 0; k < 36; ++k) s += g_f16_lut[m.audio_emb[(size_t)(8194 + 23 * k + ac[k]) * D + i]];
    out[i] = s;
  }
  return 0;
}

// fmTransformerPass (src/engine.ts:1057-1225) for `nseq` independent 3-token
// sequences (cond / uncond).  seq: [nseq][3][D], updated in place; vel: [nseq][36].
void fm_pass(const Model& m, int nseq, float* seq, float* vel) {
  const Dims& d = m.d;
  const int D = d.dim, hd = d.head_dim, Q = d.n_heads * hd, KV = d.n_kv * hd, F = d.hidden;
  const int P = 3 * nseq, rep = d.n_heads / d.n_kv;
  const float scale = 1.0f / sqrtf((float)hd);
  std::vector<float> down((size_t)P * D), nrm((size_t)P * D), q((size_t)P * Q), k((size_t)P * KV),
      v((size_t)P * KV), att((size_t)P * Q), g((size_t)P * F), u((size_t)P * F), o((size_t)P * D);
  std::vector<const float*> xs(P);
  std::vector<float*> ys(P);
  auto run = [&](const std::vector<uint16_t>& W, int M, int K, const float* X, int xstride, float* Y,
                 int ystride) {
    for (int p = 0; p < P; ++p) { xs[p] = X + (size_t)p * xstride; ys[p] = Y + (size_t)p * ystride; }
    matvec_f16(W.data(), M, K, P, xs.data(), ys.data());
  };
  for (int l = 0; l < d.fm_layers; ++l) {
    const Layer& L = m.fm_layers[l];
    memcpy(down.data(), seq, sizeof(float) * P * D);
    for (int p = 0; p < P; ++p) rms_norm(seq + (size_t)p * D, L.attn_norm.data(), D, 1e-5f, &nrm[(size_t)p * D]);
    run(L.wq, Q, D, nrm.data(), D, q.data(), Q);
    run(L.wk, KV, D, nrm.data(), D, k.data(), KV);
    run(L.wv, KV, D, nrm.data(), D, v.data(), KV);
    // biAttnScore / biSoftmax / biAttnValue (src/shaders.ts:684-807), no RoPE
    // (src/engine.ts:1108-1109), within each 3-token sequence.
    for (int s = 0; s < nseq; ++s)
      for (int hh = 0; hh < d.n_heads; ++hh) {
        const int kvh = hh / rep;
        float sc[3][3];
        for (int qi = 0; qi < 3; ++qi)
          for (int ki = 0; ki < 3; ++ki) {
            const float* qq = &q[(size_t)(3 * s + qi) * Q + hh * hd];
            const float* kk = &k[(size_t)(3 * s + ki) * KV + kvh * hd];
            float dot = 0.f;
            for (int e = 0; e < hd; ++e) dot += qq[e] * kk[e];
            sc[qi][ki] = dot * scale;
          }
        for (int qi = 0; qi < 3; ++qi) {
          float mx = -1e30f;
          for (int j = 0; j < 3; ++j) mx = std::max(mx, sc[qi][j]);
          float sum = 0.f;
          for (int j = 0; j < 3; ++j) { const float e = expf(sc[qi][j] - mx); sc[qi][j] = e; sum += e; }
          for (int j = 0; j < 3; ++j) sc[qi][j] /= sum;
        }
        for (int qi = 0; qi < 3; ++qi)
          for (int e = 0; e < hd; ++e) {
            float acc = 0.f;
            for (int ki = 0; ki < 3; ++ki) acc += sc[qi][ki] * v[(size_t)(3 * s + ki) * KV + kvh * hd + e];
            att[(size_t)(3 * s + qi) * Q + hh * hd + e] = acc;
          }
      }
    run(L.wo, D, Q, att.data(), Q, o.data(), D);
    for (size_t i = 0; i < (size_t)P * D; ++i) seq[i] = o[i] + down[i];
    memcpy(down.data(), seq, sizeof(float) * P * D);
    for (int p = 0; p < P; ++p) rms_norm(seq + (size_t)p * D, L.ffn_norm.data(), D, 1e-5f, &nrm[(size_t)p * D]);
    run(L.w1, F, D, nrm.data(), D, g.data(), F);
    run(L.w3, F, D, nrm.data(), D, u.data(), F);
    for (size_t i = 0; i < (size_t)P * F; ++i) g[i] = swiglu(g[i], u[i]);
    run(L.w2, D, F, g.data(), F, o.data(), D);
    for (size_t i = 0; i < (size_t)P * D; ++i) seq[i] = o[i] + down[i];
  }
  // Final norm of position 0 and acoustic_codebook_output (src/engine.ts:1211-1223).
  std::vector<float> n0((size_t)nseq * D);
  for (int s = 0; s < nseq; ++s) rms_norm(seq + (size_t)(3 * s) * D, m.fm_norm.data(), D, 1e-5f, &n0[(size_t)s * D]);
  for (int s = 0; s < nseq; ++s) matvec1(m.fm_ac.data(), d.n_ac, D, &n0[(size_t)s * D], vel + (size_t)s * d.n_ac);
}

// timeEmbedding (src/shaders.ts:579-602): freq_i = exp(-ln(1e4)*i/half) in f32,
// out = [cos(t*freq) | sin(t*freq)].
void time_embedding(float t, int dim, float* out) {
  const int half = dim / 2;
  const float c = -9.210340371976184f;
  for (int i = 0; i < half; ++i) {
    const float freq = expf(c * (float)i / (float)half);
    const float ang = t * freq;
    out[i] = cosf(ang);
    out[half + i] = sinf(ang);
  }
}

// fmForward (src/engine.ts:1240-1380) with caller-supplied noise (the
// debugNoise hook, :1265-1274).  Outputs: semantic logits [8320], acoustic
// codes [36], x_final [36].
void fm_forward(const Model& m, const float* normed, const float* noise, float* sem_logits, uint32_t* ac_codes,
                float* x_final) {
  const Dims& d = m.d;
  const int D = d.dim, A = d.n_ac;
  matvec1(m.fm_sem.data(), d.sem_vocab, D, normed, sem_logits);
  std::vector<float> llm(D), te(D), tp(D), xp(D), seq((size_t)6 * D), vel(2 * A);
  matvec1(m.fm_llm.data(), D, D, normed, llm.data());
  std::vector<float> x(noise, noise + A);
  const int steps = d.nfe - 1;
  const float dt = (float)(1.0 / steps);
  const float alpha = d.cfg_alpha;
  for (int s = 0; s < steps; ++s) {
    const float t = (float)((double)s / steps);
    time_embedding(t, D, te.data());
    matvec1(m.fm_time.data(), D, D, te.data(), tp.data());
    matvec1(m.fm_in.data(), D, A, x.data(), xp.data());
    // cond = [x_proj, t_proj, llm]; uncond = [x_proj, t_proj, 0] (:1317-1352)
    memcpy(&seq[0], xp.data(), sizeof(float) * D);
    memcpy(&seq[D], tp.data(), sizeof(float) * D);
    memcpy(&seq[2 * D], llm.data(), sizeof(float) * D);
    memcpy(&seq[3 * D], xp.data(), sizeof(float) * D);
    memcpy(&seq[4 * D], tp.data(), sizeof(float) * D);
    memset(&seq[5 * D], 0, sizeof(float) * D);
    fm_pass(m, 2, seq.data(), vel.data());
    // cfgCombine + eulerStep (src/shaders.ts:611-648)
    for (int i = 0; i < A; ++i) {
      const float vv = alpha * vel[i] + (1.0f - alpha) * vel[A + i];
      x[i] = x[i] + vv * dt;
    }
  }
  // fsqQuantize (src/shaders.ts:653-673); WGSL round() is half-to-even.
  for (int i = 0; i < A; ++i) {
    const float c = std::min(std::max(x[i], -1.0f), 1.0f);
    const float sc = nearbyintf((c + 1.0f) * 0.5f * (float)(d.ac_levels - 1));
    ac_codes[i] = (uint32_t)std::min(std::max(sc, 0.0f), (float)(d.ac_levels - 1)) + 2u;
    if (x_final) x_final[i] = x[i];
  }
}

}  // namespace

// ===========================================================================
// C API (ctypes)
// ===========================================================================
extern "C" {

struct orc_handle {
  Model m;
};

int orc_num_threads(void) { return omp_get_max_threads(); }
void orc_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }

// Build a model with the reference's shapes and synthetic weights (seed 0).
orc_handle* orc_create(int n_layers, int max_seq, int with_fm) {
  init_lut();
  orc_handle* h = new orc_handle();
  Model& m = h->m;
  m.d.n_layers = n_layers;
  m.max_seq = max_seq;
  m.with_fm = with_fm != 0;
  const Dims& d = m.d;
  const size_t D = d.dim;
  gen_tensor(m.tok_emb, "mm_audio_embeddings.tok_embeddings.weight", (size_t)d.vocab * D, false);
  gen_tensor(m.audio_emb, "mm_audio_embeddings.audio_codebook_embeddings.embeddings.weight",
             (size_t)d.audio_rows * D, false);
  gen_tensor(m.final_norm, "norm.weight", D, true);
  m.layers.resize(n_layers);
  for (int l = 0; l < n_layers; ++l) gen_layer(m.layers[l], "layers." + std::to_string(l) + ".", d);
  if (m.with_fm) {
    const std::string p = "acoustic_transformer.";
    gen_tensor(m.fm_in, p + "input_projection.weight", D * d.n_ac, false);
    gen_tensor(m.fm_llm, p + "llm_projection.weight", D * D, false);
    gen_tensor(m.fm_time, p + "time_projection.weight", D * D, false);
    gen_tensor(m.fm_norm, p + "norm.weight", D, true);
    gen_tensor(m.fm_sem, p + "semantic_codebook_output.weight", (size_t)d.sem_vocab * D, false);
    gen_tensor(m.fm_ac, p + "acoustic_codebook_output.weight", (size_t)d.n_ac * D, false);
    m.fm_layers.resize(d.fm_layers);
    for (int l = 0; l < d.fm_layers; ++l) gen_layer(m.fm_layers[l], p + "layers." + std::to_string(l) + ".", d);
  }
  const size_t kv = (size_t)n_layers * max_seq * d.n_kv * d.head_dim;
  m.kc.assign(kv, 0.f);
  m.vc.assign(kv, 0.f);
  m.hidden.assign(D, 0.f);
  m.normed.assign(D, 0.f);
  return h;
}

void orc_destroy(orc_handle* h) { delete h; }
void orc_reset(orc_handle* h) { h->m.position = 0; }  // reset() (src/engine.ts:2323-2327)
int orc_position(orc_handle* h) { return h->m.position; }
void orc_set_position(orc_handle* h, int pos) { h->m.position = pos; }

// Copy a synthetic tensor out (for bit-exactness tests against the GPU).
int orc_tensor_f16(orc_handle* h, const char* name, uint16_t* out, size_t n) {
  Model& m = h->m;
  const std::vector<uint16_t>* t = nullptr;
  std::string s(name);
  if (s == "mm_audio_embeddings.tok_embeddings.weight") t = &m.tok_emb;
  else if (s == "mm_audio_embeddings.audio_codebook_embeddings.embeddings.weight") t = &m.audio_emb;
  else if (s == "acoustic_transformer.semantic_codebook_output.weight") t = &m.fm_sem;
  else if (s == "acoustic_transformer.input_projection.weight") t = &m.fm_in;
  else if (s.rfind("layers.", 0) == 0) {
    int l = atoi(s.c_str() + 7);
    if (l < 0 || l >= (int)m.layers.size()) return -1;
    std::string rest = s.substr(s.find('.', 7) + 1);
    Layer& L = m.layers[l];
    if (rest == "attention.wq.weight") t = &L.wq;
    else if (rest == "attention.wk.weight") t = &L.wk;
    else if (rest == "attention.wv.weight") t = &L.wv;
    else if (rest == "attention.wo.weight") t = &L.wo;
    else if (rest == "feed_forward.w1.weight") t = &L.w1;
    else if (rest == "feed_forward.w2.weight") t = &L.w2;
    else if (rest == "feed_forward.w3.weight") t = &L.w3;
  }
  if (!t) return -1;
  const size_t k = std::min(n, t->size());
  memcpy(out, t->data(), k * 2);
  return (int)k;
}

int orc_backbone_step(orc_handle* h, int token, int use_audio, const float* embed, float* normed_out,
                      float* hidden_out, float* debug, int lm_head, uint32_t* argmax_out) {
  int rc = backbone_step(h->m, token, use_audio != 0, embed, debug, lm_head != 0, argmax_out);
  if (rc) return rc;
  if (normed_out) memcpy(normed_out, h->m.normed.data(), sizeof(float) * h->m.d.dim);
  if (hidden_out) memcpy(hidden_out, h->m.hidden.data(), sizeof(float) * h->m.d.dim);
  return 0;
}

int orc_multi_codebook_embed(orc_handle* h, uint32_t sem, const uint32_t* ac, float* out) {
  return multi_codebook_embed(h->m, sem, ac, out);
}

// fmForward on the current normed hidden state (or on `normed` if given).
int orc_fm_forward(orc_handle* h, const float* normed, const float* noise, float* sem_logits, uint32_t* ac_codes,
                   float* x_final, uint32_t* sem_code_masked) {
  if (!h->m.with_fm) return -3;
  std::vector<float> logits(h->m.d.sem_vocab);
  float* lg = sem_logits ? sem_logits : logits.data();
  fm_forward(h->m, normed ? normed : h->m.normed.data(), noise, lg, ac_codes, x_final);
  if (sem_code_masked) *sem_code_masked = masked_argmax(lg, h->m.d.sem_vocab, 8194);
  return 0;
}

uint32_t orc_masked_argmax(const float* x, int n, int valid) { return masked_argmax(x, n, valid); }
uint32_t orc_argmax_shader(const float* x, int n) { return argmax_shader(x, n); }

// Fill the first `npos` KV positions of every layer with synthetic values and
// set the position (used to time decode steps at a realistic context length
// without running the whole token-by-token prefill).
void orc_fill_kv(orc_handle* h, int npos, uint64_t seed) {
  Model& m = h->m;
  const int KV = m.d.n_kv * m.d.head_dim;
  for (int l = 0; l < m.d.n_layers; ++l) {
    const uint64_t kk = vx_stream_key(seed, 2 * l), vk = vx_stream_key(seed, 2 * l + 1);
    float* K = m.kc.data() + (size_t)l * m.max_seq * KV;
    float* V = m.vc.data() + (size_t)l * m.max_seq * KV;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)npos * KV; ++i) {
      K[i] = vx_normal(kk, (uint64_t)i);
      V[i] = vx_normal(vk, (uint64_t)i);
    }
  }
  m.position = npos;
}

// generate() (src/engine.ts:2416-2585) with masked argmax in place of the
// host's top-p sampler.  Prefill token by token (voice rows replace the
// embeddings of positions [audio_start, audio_start+audio_count)), the AUDIO
// kick (token 24 through the text embedding), then per frame:
// multi-codebook embed of the previous codes -> backbone step -> fmForward with
// noise[frame] -> masked argmax.  With fm disabled (backbone-only configs),
// feedback codes come from `codes_in` [n_frames][37] instead.
// Outputs: sem_out [n_frames], ac_out [n_frames][36], normed_out
// [n_frames][3072] (nullable).  Returns the number of frames produced.
int orc_generate(orc_handle* h, const int32_t* tokens, int n_tokens, int audio_start, int audio_count,
                 const float* voice, int n_frames, const float* noise, const uint32_t* codes_in, int eos,
                 uint32_t* sem_out, uint32_t* ac_out, float* normed_out) {
  Model& m = h->m;
  const int D = m.d.dim;
  m.position = 0;
  for (int i = 0; i < n_tokens; ++i) {
    const bool is_voice = voice && i >= audio_start && i < audio_start + audio_count;
    int rc = backbone_step(m, tokens[i], false, is_voice ? voice + (size_t)(i - audio_start) * D : nullptr,
                           nullptr, false, nullptr);
    if (rc) return rc;
  }
  int rc = backbone_step(m, 24, false, nullptr, nullptr, false, nullptr);
  if (rc) return rc;
  std::vector<float> emb(D), logits(m.d.sem_vocab);
  uint32_t sem = 0;
  uint32_t ac[36] = {0};
  int f = 0;
  for (; f < n_frames; ++f) {
    if (f > 0) {
      if (m.with_fm) multi_codebook_embed(m, sem, ac, emb.data());
      else multi_codebook_embed(m, codes_in[(size_t)(f - 1) * 37], codes_in + (size_t)(f - 1) * 37 + 1, emb.data());
      rc = backbone_step(m, 0, false, emb.data(), nullptr, false, nullptr);
      if (rc) return rc;
    }
    if (normed_out) memcpy(normed_out + (size_t)f * D, m.normed.data(), sizeof(float) * D);
    if (m.with_fm) {
      fm_forward(m, m.normed.data(), noise + (size_t)f * 36, logits.data(), ac, nullptr);
      sem = masked_argmax(logits.data(), m.d.sem_vocab, 8194);
      if (eos && sem <= 1) break;
      sem_out[f] = sem;
      memcpy(ac_out + (size_t)f * 36, ac, sizeof(ac));
    }
  }
  return f;
}

}  // extern "C"

// ===========================================================================
// Codec decoder: codecDecode (src/engine.ts:1402-1713) with the intermediates of
// debugCodecDecode (:1719-1975).  Same conventions as above: f16 weight bits, f32
// activations, the shaders' operation order.
namespace {

constexpr int kCDim = 1024, kCHidden = 4096, kCHeads = 8, kCHd = 128;

struct CodecLayerW {
  std::vector<uint16_t> wq, wk, wv, wo, w1, w2, w3, attn_norm, ffn_norm, q_norm, k_norm, attn_scale, ffn_scale;
};

struct CodecW {
  std::vector<uint16_t> sem_sum, usage, in_v, in_g, out_v, out_g, up_v[3], up_g[3];
  CodecLayerW L[8];
  std::vector<uint16_t> cb;   // normalised codebook (f16)
  std::vector<std::pair<std::string, std::vector<uint16_t>*>> named;
};

// Synthetic codec tensors: N(0, 0.02) matrices, or a constant for gains (1.0), the
// layer scales (0.1) and the codebook usage counts (2.0) — the values the engine's
// vx_init_random_weights writes.
void gen_fill(CodecW& c, std::vector<uint16_t>& t, const std::string& name, size_t n, float fill) {
  c.named.push_back({name, &t});
  if (fill != 0.f) {
    t.assign(n, vx_f32_to_f16_bits(fill));
    return;
  }
  gen_tensor(t, name, n, false);
}

// normalizeCodebook (src/shaders.ts:856-888): f16(sum / max(usage, 1e-5)).
void codec_normalize(CodecW& c) {
  init_lut();
  c.cb.resize(c.sem_sum.size());
  for (size_t i = 0; i < c.sem_sum.size(); ++i) {
    const float u = std::max(g_f16_lut[c.usage[i / 256]], 1e-5f);
    c.cb[i] = vx_f32_to_f16_bits(g_f16_lut[c.sem_sum[i]] / u);
  }
}

// causalConv1d (src/shaders.ts:919-979), [T, c] time-major, weight norm per output
// channel: wNorm = 1/sqrt(sum over consecutive pairs of (a*a + b*b) + 1e-12), then
// sum over ci (outer) and tap k (inner) of (w * wNorm * g) * x[t - (K-1) + k].
void causal_conv1d(const float* in, int T, int c_in, int c_out, int K, const uint16_t* v, const uint16_t* g, float* out) {
  init_lut();
#pragma omp parallel for schedule(static)
  for (int co = 0; co < c_out; ++co) {
    const float gv = g_f16_lut[g[co]];
    const uint16_t* w = v + (size_t)co * c_in * K;
    float wn = 0.f;
    for (int p = 0; p < c_in * K / 2; ++p) {
      const float a = g_f16_lut[w[2 * p]], b = g_f16_lut[w[2 * p + 1]];
      wn += a * a + b * b;
    }
    wn = 1.0f / sqrtf(wn + 1e-12f);
    for (int t = 0; t < T; ++t) {
      float sum = 0.f;
      for (int ci = 0; ci < c_in; ++ci)
        for (int k = 0; k < K; ++k) {
          const int ti = t - (K - 1) + k;
          if (ti >= 0) sum += (g_f16_lut[w[ci * K + k]] * wn * gv) * in[(size_t)ti * c_in + ci];
        }
      out[(size_t)t * c_out + co] = sum;
    }
  }
}

// convTransposeNormScale + causalConvTranspose1d (src/shaders.ts:1004-1104), stride 2,
// 4 taps: scale[ci] = g[ci] / sqrt(sum of v[ci,:,:]^2 + 1e-12) (256-lane strided sums,
// tree reduction); out[t][co] = sum over taps k with t - k even and >= 0 (outer) and
// ci (inner) of (w[ci][co][k] * scale[ci]) * x[(t - k) / 2][ci].  T_out = 2 T_in.
void conv_transpose(const float* in, int T_in, const uint16_t* v, const uint16_t* g, float* out) {
  init_lut();
  const int C = kCDim, K = 4;
  std::vector<float> scale(C);
  for (int ci = 0; ci < C; ++ci) {
    float s[256];
    const uint16_t* w = v + (size_t)ci * C * K;
    for (int t = 0; t < 256; ++t) {
      float ss = 0.f;
      for (int i = t; i < C * K; i += 256) ss += g_f16_lut[w[i]] * g_f16_lut[w[i]];
      s[t] = ss;
    }
    for (int st = 128; st > 0; st >>= 1)
      for (int t = 0; t < st; ++t) s[t] += s[t + st];
    scale[ci] = g_f16_lut[g[ci]] * (1.0f / sqrtf(s[0] + 1e-12f));
  }
  const int T_out = 2 * T_in;
#pragma omp parallel for schedule(static)
  for (int co = 0; co < C; ++co)
    for (int t = 0; t < T_out; ++t) {
      float sum = 0.f;
      for (int k = 0; k < K; ++k) {
        const int diff = t - k;
        if (diff >= 0 && diff % 2 == 0) {
          const int ti = diff / 2;
          for (int ci = 0; ci < C; ++ci)
            sum += (g_f16_lut[v[((size_t)ci * C + co) * K + k]] * scale[ci]) * in[(size_t)ti * C + ci];
        }
      }
      out[(size_t)t * C + co] = sum;
    }
}

// batchedMatvecF16 (src/shaders.ts:1586-1633) = matvecF16 per frame.
void codec_matvec(const std::vector<uint16_t>& A, int M, int K, const float* x, int N, float* y) {
  std::vector<const float*> xs(N);
  std::vector<float*> ys(N);
  for (int n = 0; n < N; ++n) { xs[n] = x + (size_t)n * K; ys[n] = y + (size_t)n * M; }
  matvec_f16(A.data(), M, K, N, xs.data(), ys.data());
}

// qkNorm (src/shaders.ts:1795-1838), per (token, head): sequential sum of squares,
// rms = 1/sqrt(ss/128 + 1e-6), x = x * rms * w[h*128 + d].
void qk_norm(float* x, int N, const std::vector<uint16_t>& w) {
  for (int r = 0; r < N * kCHeads; ++r) {
    float* p = x + (size_t)r * kCHd;
    const int h = r % kCHeads;
    float ss = 0.f;
    for (int d = 0; d < kCHd; ++d) ss += p[d] * p[d];
    const float rms = 1.0f / sqrtf(ss / (float)kCHd + 1e-6f);
    for (int d = 0; d < kCHd; ++d) p[d] = p[d] * rms * g_f16_lut[w[h * kCHd + d]];
  }
}

// alibiAttnScore + codecSoftmax + codecAttnValue (src/shaders.ts:1432-1575).
void codec_attention(const float* q, const float* k, const float* v, int N, int W, float* out) {
  const float scale = 1.0f / sqrtf((float)kCHd);
#pragma omp parallel for schedule(static)
  for (int h = 0; h < kCHeads; ++h) {
    const float slope = powf(2.0f, -8.0f * (float)(h + 1) / (float)kCHeads);
    std::vector<float> sc(W);
    for (int qi = 0; qi < N; ++qi) {
      const int k0 = qi + 1 > W ? qi - W + 1 : 0;
      for (int s = 0; s < W; ++s) {
        const int ki = k0 + s;
        if (ki > qi) { sc[s] = -1e30f; continue; }
        float dot = 0.f;
        for (int d = 0; d < kCHd; ++d) dot += q[((size_t)qi * kCHeads + h) * kCHd + d] * k[((size_t)ki * kCHeads + h) * kCHd + d];
        sc[s] = dot * scale + (-slope * (float)(qi - ki));
      }
      float mx = -1e30f;
      for (int s = 0; s < W; ++s) mx = std::max(mx, sc[s]);
      float sum = 0.f;
      for (int s = 0; s < W; ++s) { sc[s] = expf(sc[s] - mx); sum += sc[s]; }
      for (int s = 0; s < W; ++s) sc[s] /= sum;
      for (int d = 0; d < kCHd; ++d) {
        float acc = 0.f;
        for (int s = 0; s < W; ++s) {
          const int ki = k0 + s;
          if (ki > qi) break;
          acc += sc[s] * v[((size_t)ki * kCHeads + h) * kCHd + d];
        }
        out[((size_t)qi * kCHeads + h) * kCHd + d] = acc;
      }
    }
  }
}

// One decoder transformer layer over N tokens (src/engine.ts:1501-1646).
void codec_layer(const CodecLayerW& L, std::vector<float>& cur, int N, int W) {
  const size_t n = (size_t)N * kCDim;
  std::vector<float> res(cur), nrm(n), q(n), k(n), v(n), att(n), o(n);
  for (int t = 0; t < N; ++t) rms_norm(&cur[(size_t)t * kCDim], L.attn_norm.data(), kCDim, 0.01f, &nrm[(size_t)t * kCDim]);
  codec_matvec(L.wq, kCDim, kCDim, nrm.data(), N, q.data());
  codec_matvec(L.wk, kCDim, kCDim, nrm.data(), N, k.data());
  codec_matvec(L.wv, kCDim, kCDim, nrm.data(), N, v.data());
  qk_norm(q.data(), N, L.q_norm);
  qk_norm(k.data(), N, L.k_norm);
  codec_attention(q.data(), k.data(), v.data(), N, W, att.data());
  codec_matvec(L.wo, kCDim, kCDim, att.data(), N, o.data());
  for (size_t i = 0; i < n; ++i) cur[i] = o[i] * g_f16_lut[L.attn_scale[i % kCDim]] + res[i];
  res = cur;
  for (int t = 0; t < N; ++t) rms_norm(&cur[(size_t)t * kCDim], L.ffn_norm.data(), kCDim, 0.01f, &nrm[(size_t)t * kCDim]);
  std::vector<float> gate((size_t)N * kCHidden), up((size_t)N * kCHidden);
  codec_matvec(L.w1, kCHidden, kCDim, nrm.data(), N, gate.data());
  codec_matvec(L.w3, kCHidden, kCDim, nrm.data(), N, up.data());
  for (size_t i = 0; i < gate.size(); ++i) gate[i] = swiglu(gate[i], up[i]);
  codec_matvec(L.w2, kCDim, kCHidden, gate.data(), N, o.data());
  for (size_t i = 0; i < n; ++i) cur[i] = o[i] * g_f16_lut[L.ffn_scale[i % kCDim]] + res[i];
}

}  // namespace

extern "C" {

struct orc_codec {
  CodecW w;
};

orc_codec* orc_codec_create(void) {
  init_lut();
  orc_codec* h = new orc_codec();
  CodecW& c = h->w;
  const std::string P = "audio_tokenizer.";
  gen_fill(c, c.sem_sum, P + "quantizer.semantic_codebook.embedding_sum", (size_t)8192 * 256, 0.f);
  gen_fill(c, c.usage, P + "quantizer.semantic_codebook.cluster_usage", 8192, 2.0f);
  gen_fill(c, c.in_v, P + "decoder_blocks.0.conv.parametrizations.weight.original1", (size_t)kCDim * 292 * 3, 0.f);
  gen_fill(c, c.in_g, P + "decoder_blocks.0.conv.parametrizations.weight.original0", kCDim, 1.0f);
  for (int s = 0; s < 4; ++s)
    for (int l = 0; l < 2; ++l) {
      CodecLayerW& L = c.L[2 * s + l];
      const std::string pre = P + "decoder_blocks." + std::to_string(1 + 2 * s) + ".layers." + std::to_string(l) + ".";
      const size_t DD = (size_t)kCDim * kCDim, DF = (size_t)kCDim * kCHidden;
      gen_fill(c, L.wq, pre + "attention.wq.weight", DD, 0.f);
      gen_fill(c, L.wk, pre + "attention.wk.weight", DD, 0.f);
      gen_fill(c, L.wv, pre + "attention.wv.weight", DD, 0.f);
      gen_fill(c, L.wo, pre + "attention.wo.weight", DD, 0.f);
      gen_fill(c, L.w1, pre + "feed_forward.w1.weight", DF, 0.f);
      gen_fill(c, L.w3, pre + "feed_forward.w3.weight", DF, 0.f);
      gen_fill(c, L.w2, pre + "feed_forward.w2.weight", DF, 0.f);
      gen_fill(c, L.attn_norm, pre + "attention_norm.weight", kCDim, 1.0f);
      gen_fill(c, L.ffn_norm, pre + "ffn_norm.weight", kCDim, 1.0f);
      gen_fill(c, L.q_norm, pre + "attention.q_norm.weight", kCDim, 1.0f);
      gen_fill(c, L.k_norm, pre + "attention.k_norm.weight", kCDim, 1.0f);
      gen_fill(c, L.attn_scale, pre + "attention_scale", kCDim, 0.1f);
      gen_fill(c, L.ffn_scale, pre + "ffn_scale", kCDim, 0.1f);
    }
  for (int s = 0; s < 3; ++s) {
    const std::string pre = P + "decoder_blocks." + std::to_string(2 + 2 * s) + ".conv.parametrizations.weight.";
    gen_fill(c, c.up_v[s], pre + "original1", (size_t)kCDim * kCDim * 4, 0.f);
    gen_fill(c, c.up_g[s], pre + "original0", kCDim, 1.0f);
  }
  gen_fill(c, c.out_v, P + "output_proj.conv.parametrizations.weight.original1", (size_t)240 * kCDim * 7, 0.f);
  gen_fill(c, c.out_g, P + "output_proj.conv.parametrizations.weight.original0", 240, 1.0f);
  codec_normalize(c);
  return h;
}

void orc_codec_destroy(orc_codec* h) { delete h; }

// Replace one tensor (f16 bits, full size) — e.g. to mirror a checkpoint loaded into the engine.
int orc_codec_set_tensor(orc_codec* h, const char* name, const uint16_t* data, size_t n) {
  for (auto& kv : h->w.named)
    if (kv.first == name) {
      if (kv.second->size() != n) return -2;
      memcpy(kv.second->data(), data, n * 2);
      codec_normalize(h->w);
      return 0;
    }
  return -1;
}

int orc_codec_get_tensor(orc_codec* h, const char* name, uint16_t* out, size_t n) {
  for (auto& kv : h->w.named)
    if (kv.first == name) {
      if (kv.second->size() != n) return -2;
      memcpy(out, kv.second->data(), n * 2);
      return 0;
    }
  return -1;
}

size_t orc_codec_debug_size(int T) { return T < 1 ? 0 : (size_t)T * (292 + 30 * kCDim + 8 * 240); }

// The decode with the intermediates in the engine's vx_codec_debug order (concat,
// after_input_conv, per stage the transformer output and the upsampled output, audio).
int orc_codec_decode(orc_codec* h, const uint32_t* sem, const uint32_t* ac, int T, float* out, size_t n_out) {
  if (T < 1 || n_out != orc_codec_debug_size(T)) return -1;
  const CodecW& c = h->w;
  size_t off = 0;
  auto dump = [&](const float* p, size_t n) { memcpy(out + off, p, n * 4); off += n; };
  // vqLookup + fsqDequant + concat (src/shaders.ts:817-848, 890-917, 1840-1867)
  std::vector<float> x0((size_t)T * 292);
  for (int t = 0; t < T; ++t) {
    for (int d = 0; d < 256; ++d)
      x0[(size_t)t * 292 + d] = sem[t] < 8192 ? g_f16_lut[c.cb[(size_t)sem[t] * 256 + d]] : 0.f;
    for (int i = 0; i < 36; ++i) {
      const uint32_t code = ac[(size_t)t * 36 + i] - 2u;
      x0[(size_t)t * 292 + 256 + i] = (float)code * 2.0f / 20.0f - 1.0f;
    }
  }
  dump(x0.data(), x0.size());
  std::vector<float> cur((size_t)T * kCDim);
  causal_conv1d(x0.data(), T, 292, kCDim, 3, c.in_v.data(), c.in_g.data(), cur.data());
  dump(cur.data(), cur.size());
  for (int s = 0; s < 4; ++s) {
    const int N = T << s, W = 2 << s;
    for (int l = 0; l < 2; ++l) codec_layer(c.L[2 * s + l], cur, N, W);
    dump(cur.data(), cur.size());
    if (s < 3) {
      std::vector<float> up((size_t)2 * N * kCDim);
      conv_transpose(cur.data(), N, c.up_v[s].data(), c.up_g[s].data(), up.data());
      cur.swap(up);
      dump(cur.data(), cur.size());
    }
  }
  std::vector<float> audio((size_t)8 * T * 240);
  causal_conv1d(cur.data(), 8 * T, kCDim, 240, 7, c.out_v.data(), c.out_g.data(), audio.data());
  dump(audio.data(), audio.size());
  return off == n_out ? 0 : -3;
}

}  // extern "C"
