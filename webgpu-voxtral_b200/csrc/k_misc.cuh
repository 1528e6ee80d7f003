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
  int32_t sample_mode;  // semantic code: 0 masked argmax, 1 temperature + top-p sampling
  int32_t sample_pad;
  double top_p, temperature;   // sampling parameters (doubles, as the reference's JS numbers)
  uint64_t sample_key;  // stream of the sampler's uniform draws (counter = frame)
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
  int32_t set_sampling, sample_mode;
  double top_p, temperature;
  uint64_t sample_key;
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
  if (u.set_sampling) {
    s.sample_mode = u.sample_mode;
    s.top_p = u.top_p;
    s.temperature = u.temperature;
    s.sample_key = u.sample_key;
  }
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

// Vocab-sharded LM head under tensor parallelism: this rank's argmax (index `local`
// into its logits, rows [row0, row0 + n) of the vocabulary) as a 64-bit key whose
// maximum over the ranks is the global argmax with k_argmax's rule (maximum value,
// lowest index on ties): high word = the value's bits mapped to an order-preserving
// unsigned, low word = ~(global index).
__global__ void k_argmax_key(const float* logits, const int32_t* local, int row0, unsigned long long* key) {
  griddep_launch();
  griddep_wait();
  if (threadIdx.x != 0) return;
  const int i = *local;
  const uint32_t b = __float_as_uint(logits[i]);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  *key = ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)(row0 + i));
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
  __half* att_hi;            // non-null: the attention rows go out as the f16 hi/lo operand
  __half* att_lo;            //   of the o_proj tensor-core GEMM instead of f32 [6][q]
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

// ------------------------------------------------------------------ top-p sampling
// sampleTopP (src/engine.ts:247-289) over the masked semantic logits (indices outside
// [valid_lo, valid_hi) are -Inf, :2559-2563), in one CTA of 1024 threads:
//   scaled = f32(logit / temperature) and probabilities f32(exp(f64(scaled) - max) /
//   sum), with the exponentials and their sum in f64 as the reference computes them.
// The reference then sorts by descending probability (stable: ties in index order),
// cuts at the first position whose running sum reaches top_p, and walks the kept
// prefix to the first position whose running sum reaches u * (sum of the kept).
// Here no full sort is made.  Running sums are carried in 2^-63 fixed point (64-bit
// integers, so every order of addition gives the same value).  The row is grouped by
// the first 12 bits of the key 0x7FFFFFFF - (probability bits) (a counting sort; the
// key ascends in the reference's order); the group in which the running sum reaches
// a target is found from the prefix sums of the grouped row, and only that group is
// put in exact order (pairwise ranking of (key, index); a group of more than 1024 is
// regrouped by two more digits of the key the same way, down to one run of equal
// probabilities, inside which the order is the index order).  The fixed-point sums differ from the reference's
// sequential f64 sums by < 1e-12, which changes the result only when a running sum
// lies that close to its threshold.
constexpr int kSortN = 16384;                 // largest row (>= semantic vocabulary)
constexpr int kTpPer = kSortN / 1024;         // thread t holds positions [t*kTpPer, (t+1)*kTpPer)
constexpr int kTpDigits = 4096;               // first digit: key bits 30..19
constexpr int kTpRankMax = 1024;              // largest group ordered by pairwise ranking
constexpr uint32_t kTpNone = 0xFFFFFFFFu;     // key of a position past the row
struct TopPSmem {
  uint32_t key[kSortN];                       // exponentials (f32 bits) first, then keys
  unsigned long long pk[kTpRankMax];          // the group being ranked: key << 16 | index
  uint16_t by_digit[kSortN];                  // row indices grouped by first digit
  uint16_t deep[kSortN];                      // a large group regrouped by its second digit
  uint16_t order[kSortN];                     // the ranked group in exact order / third-digit regrouping
  uint32_t cnt[kTpDigits];                    // first-digit counts, then fill counters
  uint32_t off[kTpDigits + 1];                // start of each digit in by_digit
  uint32_t sub_cnt[1024];
  uint32_t sub_off[1024];
};
constexpr size_t kSampleSmem = sizeof(TopPSmem);
constexpr uint64_t kSampleStream = 0x73616d706c65ull;   // stream id of the sampler's draws ("sample")

// Fixed-point (2^-63) value of the probability whose key is k, floor(p * 2^63), from
// the f32 fields: p = M * 2^(E - 150) (M with its hidden bit), so p * 2^63 = M << (E - 87).
__device__ __forceinline__ unsigned long long tp_fixed(uint32_t k) {
  const uint32_t b = 0x7FFFFFFFu - k;
  const int e = (int)(b >> 23);
  const unsigned long long m = (b & 0x7FFFFFu) | (e ? 0x800000u : 0u);
  const int sh = (e ? e : 1) - 87;
  return sh >= 0 ? (m << sh) : (sh > -64 ? (m >> -sh) : 0ull);
}

// f32(a / t) given r = f64(1 / t): a * r lies within 3 f64 ulps of the f64 quotient,
// so rounding it to f32 gives the same result unless it lies within a few f64 ulps of
// a tie between two f32 values (the 29 bits that f32 rounding drops are near
// 0x10000000) or outside the f32 normal range; those take the division.
__device__ __forceinline__ float tp_div_f32(double a, double r, double t) {
  const double d = a * r;
  const unsigned long long b = (unsigned long long)__double_as_longlong(d);
  const int e = (int)((b >> 52) & 0x7FF);
  const uint32_t low = (uint32_t)(b & 0x1FFFFFFFull);
  if (e > 1023 - 126 && e < 1023 + 127 && (low - 0x10000000u + 16u) > 32u) return (float)d;
  return (float)(a / t);
}

// Sum over the 1024 threads in a fixed order (the same value in every run).
__device__ __forceinline__ double block_sum_f64_1024(double v, double* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < 32; ++w) t += sh[w];
  __syncthreads();
  return t;
}

// Exclusive scan over the 1024 threads (sh: 32 scratch entries); *total = block sum.
template <typename T>
__device__ __forceinline__ T tp_excl_scan(T v, T* sh, T* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[w] = x;
  __syncthreads();
  if (w == 0) {
    T s = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    sh[lane] = s;
  }
  __syncthreads();
  const T off = w ? sh[w - 1] : T(0);
  if (total) *total = sh[31];
  __syncthreads();
  return off + x - v;
}

__device__ __forceinline__ int tp_block_min(int v, int* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    int x = sh[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = min(x, __shfl_xor_sync(0xffffffffu, x, o));
    if (threadIdx.x == 0) sh[0] = x;
  }
  __syncthreads();
  const int r = sh[0];
  __syncthreads();
  return r;
}

// ceil(u * x) exactly, for u in [0, 1) and x < 2^64.
__device__ __forceinline__ unsigned long long tp_ceil_mul(double u, unsigned long long x) {
  if (!(u > 0.0) || x == 0) return 0;
  const unsigned long long b = (unsigned long long)__double_as_longlong(u);
  const int e = (int)((b >> 52) & 0x7FF);
  const unsigned long long m = (b & ((1ull << 52) - 1)) | (e ? (1ull << 52) : 0ull);
  const int shift = (e ? 1075 - e : 1074);    // u = m * 2^-shift, shift >= 53
  const unsigned long long lo = m * x, hi = __umul64hi(m, x);
  if (shift >= 128) return (lo | hi) ? 1ull : 0ull;
  unsigned long long q;
  bool rem;
  if (shift >= 64) {
    const int s = shift - 64;
    q = s ? (hi >> s) : hi;
    rem = lo != 0 || (s && (hi & ((1ull << s) - 1)) != 0);
  } else {
    q = (hi << (64 - shift)) | (lo >> shift);
    rem = (lo & ((1ull << shift) - 1)) != 0;
  }
  return q + (rem ? 1ull : 0ull);
}

struct TpPos {
  int idx;                      // row index at the position (-1: the total never reaches the target)
  unsigned long long incl;      // running sum up to and including it
};

// Inside a group of c > kTpRankMax row indices `a` (one first digit; the running sum
// reaches target inside it, after `before` for the earlier groups): regroup by key
// bits 18..9, then by bits 8..0 (counting sorts), each time keeping the subgroup in
// which the running sum reaches target; the last subgroup holds one key, and in it
// the m-th element in index order is the answer (found by a scan of the whole row).
__device__ TpPos tp_select_deep(TopPSmem& s, const uint16_t* a, int c, unsigned long long before,
                                unsigned long long target) {
  __shared__ int shi[32];
  __shared__ uint32_t shu[32];
  __shared__ unsigned long long shs[32];
  __shared__ unsigned long long s_before;
  __shared__ int s_idx;
  const int t = threadIdx.x;
  const uint16_t* src = a;
#pragma unroll 1
  for (int level = 0; level < 2; ++level) {
    const int shift = level == 0 ? 9 : 0, nb = level == 0 ? 1024 : 512;
    uint16_t* dst = level == 0 ? s.deep : s.order;
    if (t < nb) s.sub_cnt[t] = 0;
    __syncthreads();
    for (int x = t; x < c; x += 1024) atomicAdd(&s.sub_cnt[(s.key[src[x]] >> shift) & (nb - 1)], 1u);
    __syncthreads();
    const uint32_t mine = t < nb ? s.sub_cnt[t] : 0u;
    const uint32_t o = tp_excl_scan<uint32_t>(mine, shu, nullptr);
    if (t < nb) { s.sub_off[t] = o; s.sub_cnt[t] = 0; }
    __syncthreads();
    for (int x = t; x < c; x += 1024) {
      const uint16_t i = src[x];
      const int d = (s.key[i] >> shift) & (nb - 1);
      dst[s.sub_off[d] + atomicAdd(&s.sub_cnt[d], 1u)] = i;
    }
    __syncthreads();
    // running sums over the regrouped indices: thread t holds [t*per, t*per + per)
    const int per = (c + 1023) / 1024, x0 = min(c, t * per), x1 = min(c, t * per + per);
    unsigned long long loc = 0;
    for (int x = x0; x < x1; ++x) loc += tp_fixed(s.key[dst[x]]);
    const unsigned long long ex = before + tp_excl_scan<unsigned long long>(loc, shs, nullptr);
    unsigned long long run = ex;
    int cand = 0x7fffffff;
    for (int x = x0; x < x1; ++x) {
      run += tp_fixed(s.key[dst[x]]);
      if (run >= target) { cand = x; break; }
    }
    const int xpos = tp_block_min(cand, shi);
    if (xpos == 0x7fffffff) return TpPos{-1, 0};   // not reached (uniform across the block)
    const int d = (s.key[dst[xpos]] >> shift) & (nb - 1);
    const int st = (int)s.sub_off[d];
    const int cn = (int)s.sub_cnt[d];
    if (x0 <= st && st < x1) {
      unsigned long long acc = ex;
      for (int x = x0; x < st; ++x) acc += tp_fixed(s.key[dst[x]]);
      s_before = acc;
    }
    __syncthreads();
    before = s_before;
    src = dst + st;
    c = cn;
    __syncthreads();
  }
  // one key left: its m-th element in index order reaches the target
  const uint32_t key = s.key[src[0]];
  const unsigned long long q = tp_fixed(key), tg = target - before;
  unsigned long long m = (q == 0 || tg == 0) ? 1ull : (tg + q - 1) / q;
  if (m > (unsigned long long)c) m = c;
  int cm = 0;
#pragma unroll 4
  for (int j = 0; j < kTpPer; ++j) cm += s.key[t * kTpPer + j] == key;
  int total;
  const int exm = tp_excl_scan<int>(cm, shi, &total);
  if ((unsigned long long)exm < m && m <= (unsigned long long)(exm + cm)) {
    int r = (int)(m - exm);
    for (int j = 0; j < kTpPer; ++j)
      if (s.key[t * kTpPer + j] == key && --r == 0) { s_idx = t * kTpPer + j; break; }
  }
  __syncthreads();
  const TpPos res{s_idx, before + m * q};
  __syncthreads();
  return res;
}

// First position of the reference's sorted order whose running sum reaches target.
// pre = this thread's exclusive prefix over the grouped row (positions [t*kTpPer, ...)).
__device__ TpPos tp_select(TopPSmem& s, int n, unsigned long long pre, unsigned long long target) {
  __shared__ int shi[32];
  __shared__ unsigned long long shs[32];
  __shared__ unsigned long long s_before, s_incl;
  __shared__ int s_idx;
  const int t = threadIdx.x;
  // the group: the one holding the first grouped position whose running sum reaches target
  unsigned long long run = pre;
  int cand = 0x7fffffff;
#pragma unroll 4
  for (int j = 0; j < kTpPer; ++j) {
    const int pos = t * kTpPer + j;
    if (pos < n) {
      run += tp_fixed(s.key[s.by_digit[pos]]);
      if (cand == 0x7fffffff && run >= target) cand = pos;
    }
  }
  const int ipos = tp_block_min(cand, shi);
  if (ipos == 0x7fffffff) return TpPos{-1, 0};
  const uint32_t digit = s.key[s.by_digit[ipos]] >> 19;
  const int start = (int)s.off[digit], c = (int)s.off[digit + 1] - start;
  if (t == start / kTpPer) {
    unsigned long long acc = pre;
    for (int pos = t * kTpPer; pos < start; ++pos) acc += tp_fixed(s.key[s.by_digit[pos]]);
    s_before = acc;
  }
  __syncthreads();
  const unsigned long long before = s_before;
  if (c > kTpRankMax) return tp_select_deep(s, s.by_digit + start, c, before, target);
  // exact order inside the group: rank of (key, index) among the group, one warp per element
  for (int x = t; x < c; x += 1024) {
    const uint32_t ix = s.by_digit[start + x];
    s.pk[x] = ((unsigned long long)s.key[ix] << 16) | ix;
  }
  __syncthreads();
  const int lane = t & 31, w = t >> 5;
  for (int x = w; x < c; x += 32) {
    const unsigned long long kx = s.pk[x];
    uint32_t r = 0;
    for (int y = lane; y < c; y += 32) r += s.pk[y] < kx;
    r = __reduce_add_sync(0xffffffffu, r);
    if (lane == 0) s.order[r] = (uint16_t)(kx & 0xFFFF);
  }
  __syncthreads();
  // running sums inside the group (one element per thread)
  const unsigned long long v = t < c ? tp_fixed(s.key[s.order[t]]) : 0ull;
  const unsigned long long ex = tp_excl_scan<unsigned long long>(v, shs, nullptr);
  const int hit = (t < c && before + ex + v >= target) ? t : 0x7fffffff;
  const int first = tp_block_min(hit, shi);
  if (t == first) { s_idx = s.order[t]; s_incl = before + ex + v; }
  __syncthreads();
  const TpPos res{s_idx, s_incl};
  __syncthreads();
  return res;
}

// Returns the sampled index (all threads).  1 <= n <= kSortN.
__device__ int top_p_sample_block(const float* logits, int n, int valid_lo, int valid_hi, double top_p,
                                  double temperature, double u, TopPSmem& s) {
  __shared__ double shd[32];
  __shared__ float shf[32];
  __shared__ unsigned long long shs[32];
  __shared__ uint32_t shu[32];
  const int t = threadIdx.x;
  for (int b = t; b < kTpDigits; b += 1024) s.cnt[b] = 0;
  // this thread's logits (masked ones -Inf); the maximum of the scaled logits:
  // f32(x / t) does not decrease with x, so it is the scaled maximum logit
  float lg[kTpPer];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kTpPer; ++j) {
    const int i = t * kTpPer + j;
    lg[j] = (i < n && i >= valid_lo && i < valid_hi) ? logits[i] : -INFINITY;
    mx = fmaxf(mx, lg[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((t & 31) == 0) shf[t >> 5] = mx;
  __syncthreads();
  mx = shf[0];
  for (int w = 1; w < 32; ++w) mx = fmaxf(mx, shf[w]);
  const double max_scaled = (double)(float)((double)mx / temperature);
  const double rt = 1.0 / temperature;
  // exponentials (f32 values, f64 arithmetic) and their f64 sum
  double part = 0.0;
#pragma unroll
  for (int j = 0; j < kTpPer; ++j) {
    float v = 0.f;
    if (lg[j] != -INFINITY) {
      const float sc = tp_div_f32((double)lg[j], rt, temperature);
      if (sc != -INFINITY) v = (float)exp((double)sc - max_scaled);
    }
    s.key[t * kTpPer + j] = __float_as_uint(v);
    part += (double)v;
  }
  const double sum = block_sum_f64_1024(part, shd);
  const double rs = 1.0 / sum;
  // keys and first-digit counts
  unsigned long long tot = 0;
#pragma unroll 4
  for (int j = 0; j < kTpPer; ++j) {
    const int i = t * kTpPer + j;
    uint32_t k = kTpNone;
    if (i < n) {
      const float pr = tp_div_f32((double)__uint_as_float(s.key[i]), rs, sum);
      k = 0x7FFFFFFFu - (pr > 0.f ? __float_as_uint(pr) : 0u);   // NaN (no finite logit) counts as 0
      atomicAdd(&s.cnt[k >> 19], 1u);
      tot += tp_fixed(k);
    }
    s.key[i] = k;
  }
  __syncthreads();
  // digit offsets (thread t owns digits [4t, 4t + 4)), then the grouped row
  uint32_t c4[4], loc = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) { c4[i] = s.cnt[4 * t + i]; loc += c4[i]; }
  uint32_t o = tp_excl_scan<uint32_t>(loc, shu, nullptr);
#pragma unroll
  for (int i = 0; i < 4; ++i) { s.off[4 * t + i] = o; o += c4[i]; s.cnt[4 * t + i] = 0; }
  if (t == 0) s.off[kTpDigits] = (uint32_t)n;
  __syncthreads();
#pragma unroll 4
  for (int j = 0; j < kTpPer; ++j) {
    const int i = t * kTpPer + j;
    if (i < n) {
      const uint32_t d = s.key[i] >> 19;
      s.by_digit[s.off[d] + atomicAdd(&s.cnt[d], 1u)] = (uint16_t)i;
    }
  }
  __syncthreads();
  unsigned long long loc_sum = 0;
#pragma unroll 4
  for (int j = 0; j < kTpPer; ++j) {
    const int pos = t * kTpPer + j;
    if (pos < n) loc_sum += tp_fixed(s.key[s.by_digit[pos]]);
  }
  unsigned long long total;
  const unsigned long long pre = tp_excl_scan<unsigned long long>(loc_sum, shs, &total);
  // cutoff: the first position whose running sum reaches top_p (all n when none does)
  const double tp_scaled = top_p * 9223372036854775808.0;
  const unsigned long long t_cut = !(tp_scaled > 0.0) ? 0ull
                                   : (tp_scaled >= 18446744073709551616.0 ? ~0ull : (unsigned long long)ceil(tp_scaled));
  const TpPos cut = tp_select(s, n, pre, t_cut);
  const unsigned long long re_sum = cut.idx >= 0 ? cut.incl : total;
  // walk: the first position whose running sum reaches u * re_sum (at or before the cutoff)
  TpPos pick = tp_select(s, n, pre, tp_ceil_mul(u, re_sum));
  if (pick.idx < 0) pick = tp_select(s, n, pre, 0);
  return pick.idx;
}

// Semantic code of the frame by top-p sampling when the slot samples (sample_mode 1);
// the uniform draw is counter `frame` of the slot's sample_key stream.  Runs after
// k_fm_prepare (which wrote the masked argmax) and replaces its choice.
__global__ void __launch_bounds__(1024, 1) k_fm_sample(const __grid_constant__ FmParams p) {
  extern __shared__ __align__(16) unsigned char tp_smem[];
  griddep_launch();
  griddep_wait();
  SlotState& st = p.slots[p.slot];
  if (st.sample_mode != 1) return;
  const double u = vx_uniform01(st.sample_key, (uint64_t)st.frame);
  const int n = min(p.sem_vocab, kSortN);
  int idx = top_p_sample_block(p.head_out, n, 1, kSemValid, st.top_p, st.temperature, u,
                               *reinterpret_cast<TopPSmem*>(tp_smem));
  if (idx < 0 || idx >= n) idx = 0;   // only non-finite logits get here; keep the code a valid row
  if (threadIdx.x == 0) {
    st.codes[0] = (uint32_t)idx;
    if (st.frame >= 0 && st.frame < st.max_frames)
      p.code_ring[((long long)p.slot * st.max_frames + st.frame) * 37] = (uint32_t)idx;
  }
}

// Test support: top-p sampling of a logit row, CTA b with the uniform draw u[b].
__global__ void __launch_bounds__(1024, 1) k_top_p_test(const float* logits, int n, int valid_lo, int valid_hi,
                                                     double top_p, double temperature, const double* u, int32_t* out) {
  extern __shared__ __align__(16) unsigned char tp_smem[];
  const int idx = top_p_sample_block(logits, n, valid_lo, valid_hi, top_p, temperature, u[blockIdx.x],
                                     *reinterpret_cast<TopPSmem*>(tp_smem));
  if (threadIdx.x == 0) out[blockIdx.x] = idx;
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
    const long long o = (3LL * seq + qi) * p.q_dim + h * 128 + lane * 4;
    for (int e = 0; e < 4; ++e) {
      const float a = sc[qi][0] * v[0][e] + sc[qi][1] * v[1][e] + sc[qi][2] * v[2][e];
      if (p.att_hi) {
        const __half hv = __float2half_rn(a);
        p.att_hi[o + e] = hv;
        p.att_lo[o + e] = __float2half_rn(a - __half2float(hv));
      } else {
        p.att[o + e] = a;
      }
    }
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
