// k_misc.cuh — the small kernels around the weight-streaming GEMVs:
// synthetic weight init, embeddings, final norm, FM sequence assembly,
// 3-token attention, CFG/Euler/FSQ tail, masked semantic argmax, LM-head argmax.
// All are launched with programmatic dependent launch: each calls
// griddep_launch() early and griddep_wait() before touching data produced by
// the previous kernel.
#pragma once
#include "vx_common.cuh"
#include "vx_rng.h"

namespace vx {

// Per-utterance decode state in device memory, so that one captured CUDA graph
// serves every step of a slot.
struct SlotState {
  int32_t pos;          // tokens in the KV cache = position of the next backbone step
  int32_t frame;        // index of the frame being produced (code-ring row)
  int32_t mode;         // EmbMode of the next backbone step
  int32_t token;        // token id for the token modes
  uint32_t codes[37];   // semantic + 36 acoustic codes of the last frame (next multi-codebook input)
  int32_t prompt_len;
  uint64_t codes_key;   // synthetic feedback-code stream (backbone-only decode)
  uint64_t noise_key;   // FM noise stream
  int32_t noise_mode;   // 0: FM noise from noise_key, 1: from the host-written noise row
  int32_t max_frames;   // capacity of the code ring
};
static_assert(sizeof(SlotState) % 8 == 0, "SlotState layout");
constexpr int kPosStride = sizeof(SlotState) / 4;

enum EmbMode : int32_t {
  kEmbToken = 0,        // tok_embeddings[token]                     (src/engine.ts:832-841)
  kEmbAudioToken = 1,   // audio_embeddings[token]  (useAudioEmbedding)
  kEmbRow = 2,          // host-provided f32 row REPLACES the lookup  (src/engine.ts:843-854)
  kEmbCodes = 3,        // multiCodebookEmbed(slot.codes)             (src/shaders.ts:1878-1917)
  kEmbSynthCodes = 4,   // multiCodebookEmbed of synthetic codes for frame `frame`
  kEmbPrompt = 5,       // prompt[pos]: token id, or voice row when negative
};

// Host-side writes into a slot's state, passed by value and applied in stream
// order (no host buffer has to outlive the call).
struct SlotUpdate {
  int32_t set_mode, mode, token;
  int32_t set_codes;
  uint32_t codes[37];
  int32_t set_noise_mode, noise_mode;
  int32_t set_counters, pos, frame;
  int32_t set_keys;
  uint64_t codes_key, noise_key;
  int32_t set_prompt_len, prompt_len;
};
__global__ void k_slot_update(SlotState* slots, int slot, SlotUpdate u) {
  SlotState& s = slots[slot];
  if (threadIdx.x != 0) return;
  if (u.set_mode) { s.mode = u.mode; s.token = u.token; }
  if (u.set_codes) for (int k = 0; k < 37; ++k) s.codes[k] = u.codes[k];
  if (u.set_noise_mode) s.noise_mode = u.noise_mode;
  if (u.set_counters) { s.pos = u.pos; s.frame = u.frame; }
  if (u.set_keys) { s.codes_key = u.codes_key; s.noise_key = u.noise_key; }
  if (u.set_prompt_len) s.prompt_len = u.prompt_len;
}

constexpr int kSemValid = 8194;     // 8192 semantic codes + 2 specials (src/engine.ts:2559-2563)
constexpr int kAcBase = 8194, kAcStride = 23, kNumAc = 36;

// ------------------------------------------------------------------ weight init
__global__ void k_init_normal_f16(__half* dst, long long n, uint64_t key, float sigma) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(__fmul_rn(vx_normal(key, (uint64_t)i), sigma));
}
__global__ void k_fill_f16(__half* dst, long long n, float v) {
  const __half hv = __float2half_rn(v);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = hv;
}
// Synthetic init of a contiguous run: dst[i] = f16(normal(key, base + i) * sigma).
__global__ void k_init_normal_f16_off(__half* dst, long long n, long long base, uint64_t key, float sigma) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(__fmul_rn(vx_normal(key, (uint64_t)(base + i)), sigma));
}
__global__ void k_fill_normal_f16_kv(__half* pool, long long rows, uint64_t key) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < rows * 128; i += (long long)gridDim.x * blockDim.x)
    pool[i] = __float2half_rn(vx_normal(key, (uint64_t)i));
}

// Synthetic context for long-context runs: K/V of positions [0, npos) of every
// layer of one slot = f16(N(0,1)) from stream (seed, 2*layer + kv) at counter
// pos * kv_width + head * 128 + d (kv_width = all KV heads; head0 = first KV head
// held by this tensor-parallel rank).  The CPU oracle's fill (orc_fill_kv) draws the
// same values in f32.
struct FillKvParams {
  __half* pool;
  const int32_t* page_table;
  int slot, max_pages, n_layers, n_kv_local, head0, kv_width, npos, page_size;
  uint64_t seed;
};
__global__ void k_fill_kv_slot(const __grid_constant__ FillKvParams p) {
  const long long total = (long long)p.n_layers * 2 * p.npos * p.n_kv_local * 128;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i & 127);
    long long t = i >> 7;
    const int hl = (int)(t % p.n_kv_local);
    t /= p.n_kv_local;
    const int pos = (int)(t % p.npos);
    t /= p.npos;
    const int kv = (int)(t & 1), layer = (int)(t >> 1);
    const uint64_t key = vx_stream_key(p.seed, 2ull * layer + kv);
    const float v = vx_normal(key, (uint64_t)pos * p.kv_width + (uint64_t)(p.head0 + hl) * 128 + d);
    const int page = p.page_table[(long long)p.slot * p.max_pages + pos / p.page_size];
    const long long row =
        ((((long long)page * p.n_layers + layer) * 2 + kv) * p.n_kv_local + hl) * p.page_size + pos % p.page_size;
    p.pool[row * 128 + d] = __float2half_rn(v);
  }
}

// ------------------------------------------------------------------ checkpoint conversion
// Checkpoint tensors arrive as BF16 (the published checkpoint) or F32 and are stored
// as F16 with the reference loader's bit rules (src/weights.ts), so that both
// implementations hold identical weights:
//   BF16 -> F16 (convertBF16toF16, :94-138): sign kept; BF16 zero / subnormal -> signed
//   zero; Inf / NaN kept (NaN quieted to mantissa 0x200); exponent above F16 range ->
//   Inf; below -> F16 subnormal by right shift (truncating), or zero; else the 7-bit
//   mantissa extended with three zero bits.
//   F32 -> F16 (float32ToFloat16, :222-232): truncating; exponent <= 0 after rebias ->
//   signed zero (no subnormals); >= 31 -> Inf (NaN included).
__device__ __forceinline__ uint16_t bf16_bits_to_f16_bits(uint16_t b) {
  const uint16_t sign = (uint16_t)(b & 0x8000u);
  const int exp = (b >> 7) & 0xFF;
  const int mant = b & 0x7F;
  if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (mant ? 0x0200u : 0u));
  if (exp == 0) return sign;
  const int unbiased = exp - 127;
  if (unbiased > 15) return (uint16_t)(sign | 0x7C00u);
  if (unbiased < -14) {
    const int shift = -14 - unbiased;
    if (shift > 10) return sign;
    return (uint16_t)(sign | ((((0x80 | (mant << 1)) >> shift) >> 1) & 0x03FF));
  }
  return (uint16_t)(sign | ((unbiased + 15) << 10) | ((mant << 3) & 0x03FF));
}
__device__ __forceinline__ uint16_t f32_bits_to_f16_bits(uint32_t b) {
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
  const int exp = (int)((b >> 23) & 0xFF) - 127 + 15;
  const uint16_t frac = (uint16_t)((b >> 13) & 0x3FF);
  if (exp <= 0) return sign;
  if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
  return (uint16_t)(sign | (exp << 10) | frac);
}
// src [rows][cols] (dtype 0 F16, 1 BF16, 2 F32, packed) -> dst [rows] with row stride ld.
__global__ void k_convert_to_f16(const void* __restrict__ src, int dtype, long long rows, long long cols,
                                 uint16_t* __restrict__ dst, long long ld) {
  const long long n = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols, c = i % cols;
    uint16_t v;
    if (dtype == 1) v = bf16_bits_to_f16_bits(static_cast<const uint16_t*>(src)[i]);
    else if (dtype == 2) v = f32_bits_to_f16_bits(static_cast<const uint32_t*>(src)[i]);
    else v = static_cast<const uint16_t*>(src)[i];
    dst[r * ld + c] = v;
  }
}

// ------------------------------------------------------------------ embedding
struct EmbedParams {
  const __half* tok;   int vocab;
  const __half* audio; int audio_rows;
  SlotState* slots;
  const float* rows;          // [n_slots][D] host-provided rows
  const int32_t* prompt;      // [n_slots][max_seq] token ids, voice row r stored as -(r+1)
  const float* voice;         // [n_slots][max_voice][D]
  int max_seq, max_voice;
  uint32_t* code_ring;        // [n_slots][max_frames][37] (synthetic codes are recorded here)
  float* h;                   // [n_rows][D] output (row m <- slot slot0+m)
  int D, slot0;
};

__device__ __forceinline__ float h2f(const __half* t, long long idx) { return __half2float(t[idx]); }

__global__ void __launch_bounds__(256) k_embed(const __grid_constant__ EmbedParams p) {
  griddep_launch();
  griddep_wait();
  const int m = blockIdx.x, slot = p.slot0 + m;
  SlotState& st = p.slots[slot];
  __shared__ uint32_t codes[37];
  __shared__ int src_kind, src_row;    // 0 tok, 1 audio, 2 host row, 3 codes, 4 voice row, -1 bad
  if (threadIdx.x == 0) {
    int kind = -1, r = 0;
    switch (st.mode) {
      case kEmbToken: kind = 0; r = st.token; if (r < 0 || r >= p.vocab) kind = -1; break;
      case kEmbAudioToken: kind = 1; r = st.token; if (r < 0 || r >= p.audio_rows) kind = -1; break;
      case kEmbRow: kind = 2; break;
      case kEmbCodes: kind = 3; break;
      case kEmbSynthCodes: {
        // frame f >= 1 is fed the synthetic codes of counter base 37*(f-1)
        const uint64_t base = 37ull * (uint64_t)(st.frame - 1);
        st.codes[0] = 2u + (uint32_t)(vx_bits(st.codes_key, base) % 8192ull);
        for (int k = 0; k < kNumAc; ++k) st.codes[1 + k] = 2u + (uint32_t)(vx_bits(st.codes_key, base + 1 + k) % 21ull);
        if (st.frame >= 1 && st.frame - 1 < st.max_frames)
          for (int k = 0; k < 37; ++k) p.code_ring[((long long)slot * st.max_frames + st.frame - 1) * 37 + k] = st.codes[k];
        kind = 3;
        break;
      }
      case kEmbPrompt: {
        const int pos = st.pos;
        if (pos < 0 || pos >= p.max_seq || pos >= st.prompt_len) { kind = -1; break; }
        const int t = p.prompt[(long long)slot * p.max_seq + pos];
        if (t < 0) { kind = 4; r = -t - 1; if (r >= p.max_voice) kind = -1; }
        else { kind = 0; r = t; if (r >= p.vocab) kind = -1; }
        break;
      }
      default: kind = -1;
    }
    if (kind == 3) {
      for (int k = 0; k < 37; ++k) codes[k] = st.codes[k];
      bool okc = codes[0] < (uint32_t)p.audio_rows;
      for (int k = 0; k < kNumAc; ++k) okc = okc && (kAcBase + kAcStride * k + (int)codes[1 + k] < p.audio_rows);
      if (!okc) kind = -1;
    }
    if (kind < 0) set_error(kDevBadIndex);
    src_kind = kind;
    src_row = r;
  }
  __syncthreads();
  const int kind = src_kind, r = src_row;
  float* out = p.h + (long long)m * p.D;
  for (int i = threadIdx.x; i < p.D; i += blockDim.x) {
    float v = 0.f;
    if (kind == 0) v = h2f(p.tok, (long long)r * p.D + i);
    else if (kind == 1) v = h2f(p.audio, (long long)r * p.D + i);
    else if (kind == 2) v = p.rows[(long long)slot * p.D + i];
    else if (kind == 4) v = p.voice[((long long)slot * p.max_voice + r) * p.D + i];
    else if (kind == 3) {
      float s = 0.f;   // multiCodebookEmbed summation order: semantic row, then k = 0..35
      s += h2f(p.audio, (long long)codes[0] * p.D + i);
      for (int k = 0; k < kNumAc; ++k) s += h2f(p.audio, (long long)(kAcBase + kAcStride * k + codes[1 + k]) * p.D + i);
      v = s;
    }
    out[i] = v;
  }
}

// ------------------------------------------------------------------ norms
// Block-wide sum in a fixed order (deterministic).
__device__ __forceinline__ float block_sum_256(float v, float* sh) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += sh[w];
  __syncthreads();
  return t;
}

struct FinalNormParams {
  const float* h;       // [rows][D]
  const __half* w;
  float* out;           // [rows][D]
  int D;
  float eps;
  SlotState* slots;     // nullable: bookkeeping below
  int slot0;
  int inc_pos, inc_frame;
  float* normed_ring;   // nullable: [n_slots][max_frames][D] record of the frame's normed state
};

// rmsNorm (src/shaders.ts:137-183) of each row; optionally advances the slot's
// position / frame counters (the reference's `this.position++`, :2472, :2541).
__global__ void __launch_bounds__(256) k_final_norm(const __grid_constant__ FinalNormParams p) {
  griddep_launch();
  griddep_wait();
  __shared__ float sh[8];
  const int m = blockIdx.x;
  const float* x = p.h + (long long)m * p.D;
  float s = 0.f;
  for (int i = threadIdx.x; i < p.D; i += 256) s += x[i] * x[i];
  const float tot = block_sum_256(s, sh);
  const float rms = 1.0f / sqrtf(tot / (float)p.D + p.eps);
  float* o = p.out + (long long)m * p.D;
  float* ring = nullptr;
  if (p.slots && p.normed_ring) {
    const SlotState& st = p.slots[p.slot0 + m];
    if (st.frame >= 0 && st.frame < st.max_frames)
      ring = p.normed_ring + ((long long)(p.slot0 + m) * st.max_frames + st.frame) * p.D;
  }
  for (int i = threadIdx.x; i < p.D; i += 256) {
    const float v = x[i] * rms * __half2float(p.w[i]);
    o[i] = v;
    if (ring) ring[i] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0 && p.slots) {
    SlotState& st = p.slots[p.slot0 + m];
    if (p.inc_pos) st.pos += 1;
    if (p.inc_frame) st.frame += 1;
  }
}

// dst[m] = src[m] (copy) or RMSNorm(src[m]) * w — debug readbacks only.
__global__ void k_rows_copy_or_norm(const float* src, const __half* w, float* dst, int D, float eps) {
  griddep_launch();
  griddep_wait();
  __shared__ float sh[8];
  const float* x = src + (long long)blockIdx.x * D;
  float* o = dst + (long long)blockIdx.x * D;
  if (!w) {
    for (int i = threadIdx.x; i < D; i += blockDim.x) o[i] = x[i];
    return;
  }
  float s = 0.f;
  for (int i = threadIdx.x; i < D; i += 256) s += x[i] * x[i];
  const float tot = block_sum_256(s, sh);
  const float rms = 1.0f / sqrtf(tot / (float)D + eps);
  for (int i = threadIdx.x; i < D; i += 256) o[i] = x[i] * rms * __half2float(w[i]);
}

// ------------------------------------------------------------------ argmax
// LM-head argmax (src/shaders.ts:1154-1211): maximum value, lowest index on ties.
__global__ void __launch_bounds__(1024) k_argmax(const float* x, int n, int32_t* out) {
  griddep_launch();
  griddep_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    if (v > bv) { bv = v; bi = i; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    *out = bi;
  }
}

// ------------------------------------------------------------------ FM
struct FmParams {
  SlotState* slots;
  int slot;
  const float* head_out;     // [sem_vocab + D]: semantic logits then llm projection
  int sem_vocab, D;
  const float* host_noise;   // [36] (noise_mode 1)
  float* x;                  // [36] x_t
  const __half* w_in;        // [D][36] input_projection
  const float* tp;           // [7][D] time_projection(time_embedding(t_s)) table
  float* seq;                // [6][D]: cond (x_proj, t_proj, llm), uncond (x_proj, t_proj, 0)
  const float* qkv;          // [6][q+2kv]
  float* att;                // [6][q]
  int q_dim, kv_dim, n_heads, n_kv;
  const float* vel;          // [2][36] (cond, uncond)
  float alpha, dt;
  uint32_t* code_ring;       // [n_slots][max_frames][37]
  float* x_final;            // [36]
  int step;
};

// Masked semantic selection (mask index 0 and >= 8194, src/engine.ts:2559-2563)
// by argmax, then x_t <- noise.  One CTA.
__global__ void __launch_bounds__(1024) k_fm_prepare(const __grid_constant__ FmParams p) {
  griddep_launch();
  griddep_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  SlotState& st = p.slots[p.slot];
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const int n = min(kSemValid, p.sem_vocab);
  for (int i = 1 + threadIdx.x; i < n; i += blockDim.x) {
    const float v = p.head_out[i];
    if (v > bv) { bv = v; bi = i; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 32; ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    if (bi == 0x7fffffff) bi = 1;   // all -inf/NaN: the first unmasked index
    st.codes[0] = (uint32_t)bi;
    if (st.frame >= 0 && st.frame < st.max_frames)
      p.code_ring[((long long)p.slot * st.max_frames + st.frame) * 37] = (uint32_t)bi;
  }
  if (threadIdx.x < kNumAc) {
    p.x[threadIdx.x] = st.noise_mode ? p.host_noise[threadIdx.x]
                                     : vx_normal(st.noise_key, (uint64_t)st.frame * kNumAc + threadIdx.x);
  }
}

// x_proj = input_projection . x_t, and the two 3-token sequences
// (src/engine.ts:1310-1348).  grid D/256.
__global__ void __launch_bounds__(256) k_fm_assemble(const __grid_constant__ FmParams p) {
  griddep_launch();
  griddep_wait();
  __shared__ float xs[kNumAc];
  if (threadIdx.x < kNumAc) xs[threadIdx.x] = p.x[threadIdx.x];
  __syncthreads();
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= p.D) return;
  const __half* w = p.w_in + (long long)d * kNumAc;
  float s = 0.f;
  for (int k = 0; k < kNumAc; k += 2) s += __half2float(w[k]) * xs[k] + __half2float(w[k + 1]) * xs[k + 1];
  const float tpv = p.tp[(long long)p.step * p.D + d];
  const float llm = p.head_out[p.sem_vocab + d];
  p.seq[0 * (long long)p.D + d] = s;
  p.seq[1 * (long long)p.D + d] = tpv;
  p.seq[2 * (long long)p.D + d] = llm;
  p.seq[3 * (long long)p.D + d] = s;
  p.seq[4 * (long long)p.D + d] = tpv;
  p.seq[5 * (long long)p.D + d] = 0.f;
}

// biAttnScore / biSoftmax / biAttnValue (src/shaders.ts:684-807): bidirectional
// 3x3 attention inside each sequence, GQA 4:1, no RoPE.  One warp per
// (sequence, head); grid 2*n_heads/4, 128 threads.
__global__ void __launch_bounds__(128) k_fm_attn3(const __grid_constant__ FmParams p) {
  griddep_launch();
  griddep_wait();
  const int wg = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int seq = wg / p.n_heads, h = wg % p.n_heads;
  if (seq >= 2) return;
  const int kvh = h / (p.n_heads / p.n_kv);
  const long long ld = p.q_dim + 2LL * p.kv_dim;
  const float scale = 1.0f / sqrtf(128.0f);
  float q[3][4], k[3][4], v[3][4];
  for (int t = 0; t < 3; ++t) {
    const float* r = p.qkv + (3LL * seq + t) * ld;
    for (int e = 0; e < 4; ++e) {
      q[t][e] = r[h * 128 + lane * 4 + e];
      k[t][e] = r[p.q_dim + kvh * 128 + lane * 4 + e];
      v[t][e] = r[p.q_dim + p.kv_dim + kvh * 128 + lane * 4 + e];
    }
  }
  float sc[3][3];
  for (int qi = 0; qi < 3; ++qi)
    for (int ki = 0; ki < 3; ++ki) {
      float s = q[qi][0] * k[ki][0] + q[qi][1] * k[ki][1] + q[qi][2] * k[ki][2] + q[qi][3] * k[ki][3];
      sc[qi][ki] = warp_sum(s) * scale;
    }
  for (int qi = 0; qi < 3; ++qi) {
    float mx = -1e30f;
    for (int j = 0; j < 3; ++j) mx = fmaxf(mx, sc[qi][j]);
    float sum = 0.f;
    for (int j = 0; j < 3; ++j) { sc[qi][j] = expf(sc[qi][j] - mx); sum += sc[qi][j]; }
    for (int j = 0; j < 3; ++j) sc[qi][j] /= sum;
    float* o = p.att + (3LL * seq + qi) * p.q_dim + h * 128 + lane * 4;
    for (int e = 0; e < 4; ++e) o[e] = sc[qi][0] * v[0][e] + sc[qi][1] * v[1][e] + sc[qi][2] * v[2][e];
  }
}

// cfgCombine + eulerStep (src/shaders.ts:611-648); after the last step
// fsqQuantize (:653-673, WGSL round() = half-to-even) into the slot's codes and
// the code ring, then the frame counter advances.
__global__ void __launch_bounds__(64) k_fm_euler(const __grid_constant__ FmParams p, int last) {
  griddep_launch();
  griddep_wait();
  SlotState& st = p.slots[p.slot];
  const int i = threadIdx.x;
  if (i < kNumAc) {
    const float a = __fmul_rn(p.alpha, p.vel[i]);
    const float b = __fmul_rn(__fsub_rn(1.0f, p.alpha), p.vel[kNumAc + i]);
    const float v = __fadd_rn(a, b);
    const float x = __fadd_rn(p.x[i], __fmul_rn(v, p.dt));
    p.x[i] = x;
    if (last) {
      const float c = fminf(fmaxf(x, -1.0f), 1.0f);
      const float sc = rintf(__fmul_rn(__fmul_rn(__fadd_rn(c, 1.0f), 0.5f), 20.0f));
      const uint32_t code = (uint32_t)fminf(fmaxf(sc, 0.0f), 20.0f) + 2u;
      st.codes[1 + i] = code;
      if (st.frame >= 0 && st.frame < st.max_frames)
        p.code_ring[((long long)p.slot * st.max_frames + st.frame) * 37 + 1 + i] = code;
      if (p.x_final) p.x_final[i] = x;
    }
  }
  __syncthreads();
  if (last && i == 0) st.frame += 1;
}

// timeEmbedding (src/shaders.ts:579-602) for one t: [cos(t f_i) | sin(t f_i)],
// f_i = exp(-ln(1e4) * i / half) in f32.
__global__ void k_time_embed(float t, int D, float* out) {
  const int half = D / 2;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= half) return;
  const float freq = expf(__fdiv_rn(__fmul_rn(-9.210340371976184f, (float)i), (float)half));
  const float ang = __fmul_rn(t, freq);
  out[i] = cosf(ang);
  out[half + i] = sinf(ang);
}

}  // namespace vx
