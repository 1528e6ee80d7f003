// k_codec.cuh — kernels of the codec decoder (codes -> 24 kHz waveform), the step
// that follows the frame loop in generate() (codecDecode, src/engine.ts:1402-1713).
//
// Every projection and convolution of the decoder runs as a tensor-core GEMM
// (tc::k_gemm) over the tokens of a stage; the kernels here are what sits between
// those GEMMs:
//   - weight preparation (once per checkpoint): the normalised VQ codebook, the
//     weight-norm scales of the convolutions, and the convolution weights
//     re-ordered so that a convolution is one GEMM over an im2col operand;
//   - k_codec_embed: VQ lookup + FSQ dequantisation + concat, written directly as
//     the im2col operand of the input convolution;
//   - k_codec_row: one token row after a GEMM — layer scale + residual, then the
//     next GEMM's operand (RMSNorm, the transposed-convolution operand, or the
//     output-convolution im2col operand);
//   - k_codec_qknorm / k_codec_attn: per-head QK RMSNorm and the windowed causal
//     ALiBi attention;
//   - k_codec_audio: output-convolution weight-norm scale -> waveform.
// Activations are f32 [tokens, channels] (time-major, as in the reference); GEMM
// operands are f16 hi/lo pairs (k_gemm.cuh).  Every kernel waits for its predecessor
// (programmatic dependent launch) before touching memory.
#pragma once
#include "k_gemm.cuh"

namespace vx {
namespace codec {

constexpr int kDim = 1024;          // codec.dim
constexpr int kHidden = 4096;       // codec.hidden_dim
constexpr int kHeads = 8, kHeadDim = 128;
constexpr int kSemDim = 256, kNumAc = 36, kSemEntries = 8192;
constexpr int kInCh = kSemDim + kNumAc;   // 292
constexpr int kInChPad = 320;             // padded to a multiple of the GEMM's K step / 8
constexpr int kInTaps = 3, kOutTaps = 7, kUpTaps = 4;
constexpr int kPatch = 240;               // output channels = samples per output step
constexpr int kPatchPad = 256;
constexpr float kNormEps = 0.01f, kQkEps = 1e-6f;

__device__ __forceinline__ void split_pair(__half* hi, __half* lo, long long i, float x) {
  const __half h = __float2half_rn(x);
  hi[i] = h;
  lo[i] = __float2half_rn(x - __half2float(h));
}

// ---------------------------------------------------------------- weight preparation
// normalizeCodebook (src/shaders.ts:856-888): codebook = embedding_sum / max(usage, 1e-5),
// rounded to f16.
__global__ void k_cb_normalize(const __half* __restrict__ sum, const __half* __restrict__ usage, __half* cb) {
  griddep_launch();
  griddep_wait();
  const long long n = (long long)kSemEntries * kSemDim;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float u = fmaxf(__half2float(usage[i / kSemDim]), 1e-5f);
    cb[i] = __float2half_rn(__half2float(sum[i]) / u);
  }
}

// Weight norm of a causal convolution (src/shaders.ts:924-941): per output channel,
// scale = g / sqrt(sum of squares of v[co, :, :] + 1e-12), the squares summed over
// consecutive pairs in order as the shader does.  One thread per channel.
__global__ void k_conv_out_scale(const __half* __restrict__ v, const __half* __restrict__ g, int c_out, int per,
                                 float* scale) {
  griddep_launch();
  griddep_wait();
  const int co = blockIdx.x * blockDim.x + threadIdx.x;
  if (co >= c_out) return;
  const __half* w = v + (long long)co * per;
  float ss = 0.f;
  for (int p = 0; p < per / 2; ++p) {
    const float a = __half2float(w[2 * p]), b = __half2float(w[2 * p + 1]);
    ss += a * a + b * b;
  }
  scale[co] = __half2float(g[co]) * (1.0f / sqrtf(ss + 1e-12f));
}

// Weight norm of a transposed convolution (convTransposeNormScale, src/shaders.ts:1004-1052):
// per input channel, scale = g[ci] / sqrt(sum over [c_out, kernel] of v^2 + 1e-12), with the
// shader's 256-lane strided partial sums and tree reduction.  One CTA of 256 per channel.
__global__ void __launch_bounds__(256) k_convT_in_scale(const __half* __restrict__ v, const __half* __restrict__ g,
                                                         int per, float* scale) {
  griddep_launch();
  griddep_wait();
  __shared__ float s[256];
  const int ci = blockIdx.x, t = threadIdx.x;
  const __half* w = v + (long long)ci * per;
  float ss = 0.f;
  for (int i = t; i < per; i += 256) {
    const float a = __half2float(w[i]);
    ss += a * a;
  }
  s[t] = ss;
  __syncthreads();
  for (int st = 128; st > 0; st >>= 1) {
    if (t < st) s[t] += s[t + st];
    __syncthreads();
  }
  if (t == 0) scale[ci] = __half2float(g[ci]) * (1.0f / sqrtf(s[0] + 1e-12f));
}

// Causal convolution weight [c_out, c_in, taps] -> GEMM weight [c_out_pad, taps * c_in_pad]
// with row co = (tap 0 channels, tap 1 channels, ...), zero padding.  The GEMM's X row t
// is then (x[t - taps + 1], ..., x[t]) over the padded channels.
__global__ void k_conv_reorder(const __half* __restrict__ v, int c_out, int c_in, int taps, int c_out_pad,
                               int c_in_pad, __half* dst) {
  griddep_launch();
  griddep_wait();
  const long long n = (long long)c_out_pad * taps * c_in_pad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int ci = (int)(i % c_in_pad);
    const int k = (int)((i / c_in_pad) % taps);
    const int co = (int)(i / ((long long)c_in_pad * taps));
    dst[i] = (co < c_out && ci < c_in) ? v[((long long)co * c_in + ci) * taps + k] : __float2half_rn(0.f);
  }
}

// Transposed convolution weight v[c_in][c_out][4] (stride 2) -> two GEMM weights, one
// per output parity: output 2m + par = sum over j in {0, 1} of W_par[:, j] . x[m - 1 + j],
// with tap k = 2 - 2j + par (par 0: taps 2, 0; par 1: taps 3, 1).  dst[par][co][j*C + ci].
__global__ void k_convT_reorder(const __half* __restrict__ v, __half* dst) {
  griddep_launch();
  griddep_wait();
  const long long n = 2LL * kDim * 2 * kDim;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int ci = (int)(i % kDim);
    const int j = (int)((i / kDim) % 2);
    const int co = (int)((i / (2LL * kDim)) % kDim);
    const int par = (int)(i / (2LL * kDim * kDim));
    const int k = 2 - 2 * j + par;
    dst[i] = v[((long long)ci * kDim + co) * kUpTaps + k];
  }
}

// ---------------------------------------------------------------- input
// vqLookup + fsqDequant + concatCodecInput (src/shaders.ts:817-848, 890-917, 1840-1867):
// x[t] = (codebook[sem[t]] (256), (ac[t, i] - 2) * 2 / 20 - 1 (36)).  The reference
// indexes its 8192-row codebook with the raw semantic code; codes 8192 and 8193 (which
// generate() can produce) lie past its end, where the reference's read is left to the
// WebGPU implementation — here they give a zero row.  The FSQ subtraction is u32, as in
// the shader.  Written as the f32 concat row (for debugging) and as the im2col operand of
// the 3-tap input convolution: X[t][k * 320 + c] = x[t - 2 + k][c] (zero before t = 0 and
// for the padding channels).
__global__ void k_codec_embed(const uint32_t* __restrict__ sem, const uint32_t* __restrict__ ac,
                              const __half* __restrict__ cb, int T, float* concat, __half* hi, __half* lo) {
  griddep_launch();
  griddep_wait();
  const long long n = (long long)T * kInTaps * kInChPad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % kInChPad);
    const int k = (int)((i / kInChPad) % kInTaps);
    const int t = (int)(i / ((long long)kInChPad * kInTaps));
    const int ts = t - (kInTaps - 1) + k;
    float x = 0.f;
    if (ts >= 0 && c < kInCh) {
      if (c < kSemDim) {
        const uint32_t code = sem[ts];
        x = code < (uint32_t)kSemEntries ? __half2float(cb[(long long)code * kSemDim + c]) : 0.f;
      } else {
        const uint32_t code = ac[(long long)ts * kNumAc + (c - kSemDim)] - 2u;
        x = (float)code * 2.0f / 20.0f - 1.0f;
      }
      if (k == kInTaps - 1 && concat) concat[(long long)ts * kInCh + c] = x;
    }
    split_pair(hi, lo, i, x);
  }
}

// ---------------------------------------------------------------- token rows
enum RowOut : int {
  kOpNorm = 0,    // RMSNorm(cur) * w -> operand row [t][1024]
  kOpConvT = 1,   // cur * s_in -> operand rows t ([1024, 2048)) and t + 1 ([0, 1024)), [2T_in rows, 2048]
  kOpOutConv = 2, // cur -> im2col operand of the 7-tap output convolution [t + j][(6 - j) * 1024 + c]
};
struct RowParams {
  const float* y;          // GEMM output rows
  long long ldy;
  const __half* scale;     // layer scale [1024] (f16) or null
  const float* fscale;     // weight-norm scale [1024] (f32) or null
  int residual;            // 1: cur = y * scale + cur (batchedLayerScale, src/shaders.ts:1763-1790)
  float* cur;              // residual stream [N, 1024]
  int n_rows;
  int out;                 // RowOut
  const __half* norm_w;    // kOpNorm
  const float* op_scale;   // kOpConvT: per-input-channel weight norm
  __half* hi;
  __half* lo;
};

// One CTA of 256 threads per token row; thread t holds channels t, t+256, t+512, t+768
// (the strided lanes of batchedRmsNorm, src/shaders.ts:1645-1690: partial sums of
// squares, tree reduction, rms = 1/sqrt(ss/dim + eps), y = x * rms * w).
__global__ void __launch_bounds__(256) k_codec_row(const __grid_constant__ RowParams p) {
  griddep_launch();
  griddep_wait();
  __shared__ float s[256];
  const int r = blockIdx.x, t = threadIdx.x;
  float v[4];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = t + 256 * j;
    float x = p.y[(long long)r * p.ldy + c];
    if (p.scale) x = x * __half2float(p.scale[c]);
    if (p.fscale) x = x * p.fscale[c];
    if (p.residual) x = x + p.cur[(long long)r * kDim + c];
    p.cur[(long long)r * kDim + c] = x;
    v[j] = x;
    ss += x * x;
  }
  if (p.out == kOpNorm) {
    s[t] = ss;
    __syncthreads();
    for (int st = 128; st > 0; st >>= 1) {
      if (t < st) s[t] += s[t + st];
      __syncthreads();
    }
    const float rms = 1.0f / sqrtf(s[0] / (float)kDim + kNormEps);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = t + 256 * j;
      split_pair(p.hi, p.lo, (long long)r * kDim + c, v[j] * rms * __half2float(p.norm_w[c]));
    }
  } else if (p.out == kOpConvT) {
    const long long ld = 2 * kDim;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = t + 256 * j;
      const float u = v[j] * p.op_scale[c];
      split_pair(p.hi, p.lo, (long long)r * ld + kDim + c, u);
      if (r + 1 < p.n_rows) split_pair(p.hi, p.lo, (long long)(r + 1) * ld + c, u);
      if (r == 0) split_pair(p.hi, p.lo, c, 0.f);
    }
  } else {
    const long long ld = (long long)kOutTaps * kDim;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = t + 256 * j;
      for (int d = 0; d < kOutTaps; ++d) {
        if (r + d < p.n_rows) split_pair(p.hi, p.lo, (long long)(r + d) * ld + (kOutTaps - 1 - d) * kDim + c, v[j]);
        if (d < kOutTaps - 1 - r) split_pair(p.hi, p.lo, (long long)r * ld + d * kDim + c, 0.f);
      }
    }
  }
}

// qkNorm (src/shaders.ts:1795-1838) on the q and k parts of QKV rows [N, 3 * 1024], in place:
// per (token, head), rms over the 128 values, x * rms * w[h * 128 + d].  One warp per
// (token, head, q|k); lane l holds d = l, l + 32, l + 64, l + 96.
__global__ void __launch_bounds__(256) k_codec_qknorm(float* qkv, int N, const __half* __restrict__ q_w,
                                                      const __half* __restrict__ k_w) {
  griddep_launch();
  griddep_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N * kHeads * 2) return;
  const int which = warp & 1, h = (warp >> 1) % kHeads, row = (warp >> 1) / kHeads;
  float* x = qkv + (long long)row * 3 * kDim + which * kDim + h * kHeadDim;
  const __half* w = (which ? k_w : q_w) + h * kHeadDim;
  float v[4], ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = x[lane + 32 * j];
    ss += v[j] * v[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rms = 1.0f / sqrtf(ss / (float)kHeadDim + kQkEps);
#pragma unroll
  for (int j = 0; j < 4; ++j) x[lane + 32 * j] = v[j] * rms * __half2float(w[lane + 32 * j]);
}

// alibiAttnScore + codecSoftmax + codecAttnValue (src/shaders.ts:1432-1575): query qi of
// head h attends to keys ki in [max(0, qi - W + 1), qi]:
//   score = (q . k) / sqrt(128) - 2^-(h+1) * (qi - ki); softmax (max from -1e30);
//   out = sum over the window of p * v.
// One warp per (token, head); the output row goes out as the hi/lo operand of wo.
__global__ void __launch_bounds__(256) k_codec_attn(const float* __restrict__ qkv, int N, int W, __half* hi,
                                                    __half* lo) {
  griddep_launch();
  griddep_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N * kHeads) return;
  const int h = warp % kHeads, qi = warp / kHeads;
  const float* q = qkv + (long long)qi * 3 * kDim + h * kHeadDim;
  float qv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) qv[j] = q[lane + 32 * j];
  const int k0 = max(0, qi - W + 1), nk = qi - k0 + 1;   // nk <= W <= 16
  const float scale = 1.0f / sqrtf((float)kHeadDim);
  const float slope = ldexpf(1.0f, -(h + 1));            // pow(2, -8 (h + 1) / 8)
  float sc[16];
  float mx = -1e30f;
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    sc[s] = -1e30f;
    if (s < nk) {
      const int ki = k0 + s;
      const float* k = qkv + (long long)ki * 3 * kDim + kDim + h * kHeadDim;
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) d += qv[j] * k[lane + 32 * j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
      sc[s] = d * scale + (-slope * (float)(qi - ki));
    }
    mx = fmaxf(mx, sc[s]);
  }
  float sum = 0.f;
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    sc[s] = s < nk ? expf(sc[s] - mx) : 0.f;
    sum += sc[s];
  }
  float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    if (s < nk) {
      const float pr = sc[s] / sum;
      const float* v = qkv + (long long)(k0 + s) * 3 * kDim + 2 * kDim + h * kHeadDim;
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] += pr * v[lane + 32 * j];
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) split_pair(hi, lo, (long long)qi * kDim + h * kHeadDim + lane + 32 * j, o[j]);
}

// Output convolution epilogue: audio[t * 240 + c] = y[t][c] * scale[c] ([T_out, 240]
// time-major is the waveform, src/engine.ts:1700-1702).
__global__ void k_codec_audio(const float* __restrict__ y, long long ldy, const float* __restrict__ scale, int n_rows,
                              float* audio) {
  griddep_launch();
  griddep_wait();
  const long long n = (long long)n_rows * kPatch;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / kPatch;
    const int c = (int)(i % kPatch);
    audio[i] = y[t * ldy + c] * scale[c];
  }
}

}  // namespace codec
}  // namespace vx
