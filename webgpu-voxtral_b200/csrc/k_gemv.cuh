// k_gemv.cuh — weight-streaming GEMV/skinny-GEMM for the decode path.
//
// Replaces matvecF16 / matvecF16Offset (src/shaders.ts:21-71, :1221-1272) and the
// elementwise passes that follow them in src/engine.ts (rmsNorm before the
// projections, RoPE + kvCacheWrite after Q/K/V, addInPlace after o_proj / down,
// swiGLU after gate/up: :867-1005, FM :1057-1225).
//
//   y[m][row] (op)= sum_k W[row][col0+k] * x'[m][col0+k]     m < M activation rows
//   x' = x, or RMSNorm(x) * gain when the kernel carries the norm prologue.
//
// Design (B200): the op is bound by streaming f16 weights from HBM.  One CTA per
// SM (persistent over tiles), 10 warps:
//   warp 0    producer: one lane issues 1-D TMA bulk copies (cp.async.bulk) of
//             whole weight tiles (R rows x kc columns) into a 6-stage shared
//             memory ring (6 x 36 KB), L2 evict-first;
//   warps 1-8 consumers: each owns a fixed 1/8 of the columns (128-column chunks,
//             8 bytes per lane per row -> conflict-free), keeps its slice of x'
//             in registers, accumulates f32 FMAs, reduces the R*M partial sums
//             across lanes with a transposed butterfly and hands them to
//   warp 9    epilogue: sums the 8 warp partials in a fixed order (bit-
//             reproducible) and applies the fused op: store, residual add,
//             SwiGLU, or RoPE + q store + paged f16 KV append.
// The kernel triggers programmatic dependent launch at entry and the producer
// never waits on the previous kernel (weights are constant), so the next
// GEMV's ring fills while this one drains; only x / outputs wait
// (griddepcontrol.wait).
#pragma once
#include "vx_common.cuh"

namespace vx {
namespace gemv {

constexpr int kCW = 8;                       // consumer warps
constexpr int kThreads = (kCW + 2) * 32;     // + producer + epilogue warps
constexpr int kStages = 6;
constexpr int kStageBytes = 36864;           // 36 KB
constexpr int kRedSlots = 4;
constexpr int kMaxVals = 32;                 // R * M per tile
constexpr int kMaxM = 8;
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + (2 * kStages + 2 * kRedSlots) * 8 +
                              (size_t)kRedSlots * kCW * kMaxVals * 4 + kMaxM * kCW * 4;

enum Epi { kStore = 0, kResid = 1, kSwiglu = 2, kQkv = 3 };

// Paged KV cache geometry shared with the attention kernel.  Row index of
// (page, layer, kv in {0=K,1=V}, head, slot-in-page) in a [rows, head_dim] f16 pool:
//   (((page * n_layers + layer) * 2 + kv) * n_kv + head) * page_size + slot
struct KvGeom {
  __half* pool;
  const int32_t* page_table;   // [n_slots][max_pages]
  int max_pages, n_layers, n_kv, page_size;
};
__host__ __device__ __forceinline__ long long kv_row(const KvGeom& g, int page, int layer, int kv, int head, int slot) {
  return ((((long long)page * g.n_layers + layer) * 2 + kv) * g.n_kv + head) * g.page_size + slot;
}

struct SlotState;  // defined in k_misc.cuh

struct QkvOut {
  float* q;                    // [M][ldq]
  long long ldq;
  int q_dim, kv_dim;           // rows [0,q_dim) -> q, [q_dim, q_dim+kv_dim) -> K, rest -> V
  KvGeom kv;
  int layer;
  const int32_t* pos;          // &slot_state[0].pos, stride pos_stride ints
  int pos_stride;
  int slot0;                   // activation row m belongs to slot slot0 + m
  const float* rope_freq;      // [head_dim / 2]
};

struct Params {
  const __half* W;             // weight rows, row stride ldw elements
  long long ldw;
  long long second_off;        // kSwiglu: element offset of the "up" rows (w3) from W (w1)
  int rows;                    // output rows
  int col0, kc;                // column slice [col0, col0 + kc)
  const float* x;              // [M][ldx]
  long long ldx;
  const __half* norm_w;        // RMSNorm gain (NORM variants)
  float eps;
  int norm_dim;
  float* y;                    // [M][ldy]
  long long ldy;
  QkvOut qkv;
};

// Transposed butterfly: P values per lane -> one fully reduced value per lane,
// P - 1 + (5 - log2 P) shuffles instead of 5 P.  Lane holds index
// sum_k bit_k(lane) * (P >> (k+1)).
template <int P>
__device__ __forceinline__ float transpose_reduce(float (&v)[P], int lane) {
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    if ((P >> k) > 1) {
      const bool upper = (lane >> k) & 1;
#pragma unroll
      for (int i = 0; i < ((P >> k) / 2); ++i) {
        const int h = (P >> k) / 2;
        const float send = upper ? v[i] : v[i + h];
        const float keep = upper ? v[i + h] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 1 << k);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1 << k);
    }
  }
  return v[0];
}
template <int P>
__device__ __forceinline__ int transpose_index(int lane) {
  int idx = 0;
#pragma unroll
  for (int k = 0; k < 5; ++k)
    if ((P >> k) > 1) idx += ((lane >> k) & 1) * ((P >> k) / 2);
  return idx;
}
template <int N>
struct Pow2 {
  static constexpr int v = N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : N <= 8 ? 8 : N <= 16 ? 16 : 32;
};

template <int M, int R, int CPL, int EPI, bool NORM>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(const __grid_constant__ Params p) {
  static_assert(R * M <= kMaxVals && M <= kMaxM, "tile too large");
  static_assert(EPI != kSwiglu || (R % 2) == 0, "SwiGLU tiles hold gate+up row pairs");
  static_assert(EPI != kQkv || (R % 2) == 0, "RoPE pairs must not straddle tiles");
  constexpr int ORT = (EPI == kSwiglu) ? R / 2 : R;   // output rows per tile
  constexpr int P = Pow2<R * M>::v;

  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* rfull = empty + kStages;
  uint64_t* rempty = rfull + kRedSlots;
  float* red = reinterpret_cast<float*>(rempty + kRedSlots);     // [kRedSlots][kCW][kMaxVals]
  float* ssq = red + kRedSlots * kCW * kMaxVals;                  // [M][kCW]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (p.rows + ORT - 1) / ORT;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], kCW); }
#pragma unroll
    for (int s = 0; s < kRedSlots; ++s) { mbar_init(&rfull[s], kCW); mbar_init(&rempty[s], 1); }
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint32_t rowbytes = (uint32_t)p.kc * 2u;
      // L2 prefetch of the tiles kAhead iterations ahead keeps DRAM busy beyond the ring
      constexpr int kAhead = 8;
      auto prefetch_tile = [&](int tt) {
        const int r0 = tt * ORT;
        const int nr = min(ORT, p.rows - r0);
        const __half* src = p.W + (long long)r0 * p.ldw + p.col0;
        if (p.kc == p.ldw) {
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"((uint32_t)nr * rowbytes) : "memory");
          if (EPI == kSwiglu)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src + p.second_off),
                         "r"((uint32_t)nr * rowbytes) : "memory");
        }
      };
      for (int k = 0; k < kAhead; ++k)
        if (blockIdx.x + k * (int)gridDim.x < ntiles) prefetch_tile(blockIdx.x + k * gridDim.x);
      int it = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        if (t + kAhead * (int)gridDim.x < ntiles) prefetch_tile(t + kAhead * gridDim.x);
        const int s = it % kStages;
        const uint32_t ph = (uint32_t)(it / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, kDevTimeoutEmpty)) break;
        const int r0 = t * ORT;
        const int nr = min(ORT, p.rows - r0);
        const uint32_t bytes = (uint32_t)nr * rowbytes * (EPI == kSwiglu ? 2u : 1u);
        mbar_arrive_expect_tx(&full[s], bytes);
        uint8_t* dst = stages + (size_t)s * kStageBytes;
        const __half* src = p.W + (long long)r0 * p.ldw + p.col0;
        if (p.kc == p.ldw) {
          bulk_g2s(dst, src, (uint32_t)nr * rowbytes, &full[s], pol);
          if (EPI == kSwiglu)
            bulk_g2s(dst + (size_t)ORT * rowbytes, src + p.second_off, (uint32_t)nr * rowbytes, &full[s], pol);
        } else {
          for (int r = 0; r < nr; ++r) {
            bulk_g2s(dst + (size_t)r * rowbytes, src + (long long)r * p.ldw, rowbytes, &full[s], pol);
            if (EPI == kSwiglu)
              bulk_g2s(dst + (size_t)(ORT + r) * rowbytes, src + p.second_off + (long long)r * p.ldw, rowbytes,
                       &full[s], pol);
          }
        }
      }
      // Drain: every issued copy must land before the CTA's shared memory is released.
      const int first = it > kStages ? it - kStages : 0;
      for (int i = first; i < it; ++i)
        if (!mbar_wait_drain(&full[i % kStages], (uint32_t)(i / kStages) & 1u)) break;
    }
    griddep_wait();
    return;
  }

  if (warp <= kCW) {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1;
    griddep_wait();
    float rms[M];
#pragma unroll
    for (int m = 0; m < M; ++m) rms[m] = 1.0f;
    if constexpr (NORM) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float* xm = p.x + (long long)m * p.ldx;
        float s = 0.f;
        for (int i = cw * 32 + lane; i < p.norm_dim; i += kCW * 32) s += xm[i] * xm[i];
        s = warp_sum(s);
        if (lane == 0) ssq[m * kCW + cw] = s;
      }
      named_bar_sync(1, kCW * 32);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kCW; ++w) tot += ssq[m * kCW + w];
        rms[m] = 1.0f / sqrtf(tot / (float)p.norm_dim + p.eps);
      }
    }
    // This warp's slice of x' in registers: chunk c = cw + 8j (128 columns), lane -> 4 columns.
    // kc/128 chunks need not divide by 8: chunks beyond the slice are skipped.
    const int nch = p.kc >> 7;
    float xr[M][CPL][4];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      if (cw + kCW * j >= nch) {
#pragma unroll
        for (int m = 0; m < M; ++m) xr[m][j][0] = xr[m][j][1] = xr[m][j][2] = xr[m][j][3] = 0.f;
        continue;
      }
      const int col = p.col0 + (cw + kCW * j) * 128 + lane * 4;
      float4 g = make_float4(1.f, 1.f, 1.f, 1.f);
      if constexpr (NORM) {
        const __half2* w2 = reinterpret_cast<const __half2*>(p.norm_w + col);
        const float2 a = __half22float2(w2[0]), b = __half22float2(w2[1]);
        g = make_float4(a.x, a.y, b.x, b.y);
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float4 v = *reinterpret_cast<const float4*>(p.x + (long long)m * p.ldx + col);
        if constexpr (NORM) {
          xr[m][j][0] = v.x * rms[m] * g.x;
          xr[m][j][1] = v.y * rms[m] * g.y;
          xr[m][j][2] = v.z * rms[m] * g.z;
          xr[m][j][3] = v.w * rms[m] * g.w;
        } else {
          xr[m][j][0] = v.x; xr[m][j][1] = v.y; xr[m][j][2] = v.z; xr[m][j][3] = v.w;
        }
      }
    }
    const int my_idx = transpose_index<P>(lane);
    const bool writer = lane < P && my_idx < R * M;
    const uint32_t rowbytes = (uint32_t)p.kc * 2u;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int s = it % kStages;
      if (!mbar_wait(&full[s], (uint32_t)(it / kStages) & 1u, kDevTimeoutFull)) break;
      float acc[R][M];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
      const uint8_t* base = stages + (size_t)s * kStageBytes + (size_t)(cw * 128 + lane * 4) * 2;
#pragma unroll
      for (int r = 0; r < R; ++r) {
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          if (cw + kCW * j >= nch) continue;
          const uint2 wv = *reinterpret_cast<const uint2*>(base + (size_t)r * rowbytes + (size_t)j * kCW * 256);
          const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
          const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float a = acc[r][m];
            a = fmaf(w01.x, xr[m][j][0], a);
            a = fmaf(w01.y, xr[m][j][1], a);
            a = fmaf(w23.x, xr[m][j][2], a);
            a = fmaf(w23.y, xr[m][j][3], a);
            acc[r][m] = a;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      float v[P];
#pragma unroll
      for (int i = 0; i < P; ++i) v[i] = (i < R * M) ? acc[i / M][i % M] : 0.f;
      const float red_v = transpose_reduce<P>(v, lane);
      const int rs = it % kRedSlots;
      if (!mbar_wait(&rempty[rs], ((uint32_t)(it / kRedSlots) & 1u) ^ 1u, kDevTimeoutRed)) break;
      if (writer) red[(rs * kCW + cw) * kMaxVals + my_idx] = red_v;
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfull[rs]);
    }
    return;
  }

  // -------------------------------------------------------------- epilogue warp
  griddep_wait();
  int it = 0;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
    const int rs = it % kRedSlots;
    if (!mbar_wait(&rfull[rs], (uint32_t)(it / kRedSlots) & 1u, kDevTimeoutRed)) break;
    const int i = lane;
    float val = 0.f;
    if (i < R * M) {
#pragma unroll
      for (int w = 0; w < kCW; ++w) val += red[(rs * kCW + w) * kMaxVals + i];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&rempty[rs]);
    const int r = i / M, m = i % M;
    if constexpr (EPI == kStore || EPI == kResid) {
      const int row = t * ORT + r;
      if (i < R * M && row < p.rows) {
        float* yp = p.y + (long long)m * p.ldy + row;
        if constexpr (EPI == kStore) *yp = val;
        else *yp = *yp + val;
      }
    } else if constexpr (EPI == kSwiglu) {
      const float up = __shfl_down_sync(0xffffffffu, val, ORT * M);
      const int row = t * ORT + r;
      if (r < ORT && i < R * M && row < p.rows) p.y[(long long)m * p.ldy + row] = swiglu(val, up);
    } else {  // kQkv: RoPE on q and k (interleaved pairs), q -> p.qkv.q, k/v -> paged f16 cache
      const int partner_lane = ((r ^ 1) * M + m) & 31;
      const float other = __shfl_sync(0xffffffffu, val, partner_lane);
      const int row = t * R + r;
      if (i < R * M && row < p.rows) {
        const QkvOut& o = p.qkv;
        const int slot = o.slot0 + m;
        const int pos = o.pos[(long long)slot * o.pos_stride];
        float out = val;
        if (row < o.q_dim + o.kv_dim) {
          const int pair = (row & 127) >> 1;
          const float ang = (float)pos * o.rope_freq[pair];
          float sn, cs;
          sincosf(ang, &sn, &cs);
          const bool even = (row & 1) == 0;
          const float x0 = even ? val : other, x1 = even ? other : val;
          out = even ? __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn))
                     : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
        if (row < o.q_dim) {
          o.q[(long long)m * o.ldq + row] = out;
        } else {
          const int kvr = row - o.q_dim;
          const int kv = kvr >= o.kv_dim ? 1 : 0;
          const int rr = kvr - kv * o.kv_dim;
          const int head = rr >> 7, d = rr & 127;
          const int lp = pos / o.kv.page_size;
          if (lp >= o.kv.max_pages) {
            set_error(kDevBadIndex);
          } else {
            const int page = o.kv.page_table[(long long)slot * o.kv.max_pages + lp];
            const long long prow = kv_row(o.kv, page, o.layer, kv, head, pos % o.kv.page_size);
            o.kv.pool[prow * 128 + d] = __float2half_rn(out);
          }
        }
      }
    }
  }
}

}  // namespace gemv
}  // namespace vx
