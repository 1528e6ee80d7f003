// k_gemm.cuh — tcgen05 / TMEM tensor-core GEMM for token batches, and the
// element-wise kernels around it.
//
// A token batch is N activation rows that all go through the same layer: the N
// prompt positions of one utterance (batched prefill, replacing the reference's
// token-by-token prefill loop src/engine.ts:2457-2472), or the current position
// of N utterances (batched decode).  Each projection of backboneStep
// (src/engine.ts:882-1005, matvecF16 src/shaders.ts:21-71) becomes
//
//     Y[n, m] (=|+=) sum_k W[m, k] * X[n, k]        W: f16 [M, K] (checkpoint layout)
//
// on the 5th-generation tensor cores.  The reference computes with f32
// activations; tensor-core operands of kind::f16 are f16 on both sides, so X is
// carried as an f16 pair (hi = f16(x), lo = f16(x - hi)) and each K step issues
// two MMAs into the same f32 accumulator: W*hi + W*lo keeps ~22 bits of x and
// every product is exact in f32.  Weight rows are the MMA's M side (128 TMEM
// lanes), tokens its N side (TMEM columns).
//
// CTA = one 128 x BN output tile (and one K range when split-K is on), 4 warps:
//   warp 0 lane 0  TMA producer: W tile [128 x 64] and the hi/lo X tiles [BN x 64]
//                  per stage (128-byte swizzle), into a kStages-deep ring;
//   warp 1 lane 0  MMA issuer: 4 K-steps x (hi, lo) tcgen05.mma per stage, then
//                  tcgen05.commit frees the stage; a final commit marks the
//                  accumulator complete;
//   warp 2         allocates / frees the TMEM accumulator (BN columns);
//   all 4 warps    epilogue: tcgen05.ld (warp w reads TMEM lanes 32w..32w+31),
//                  stores Y[n, m] with m along the lanes (coalesced).
// Split-K: every split writes its f32 partial tile to a workspace and
// k_splitk_reduce (the next launch) sums the partials in split order 0..S-1 over
// the whole output at once, so the result does not depend on CTA timing.
#pragma once
#include "vx_common.cuh"
#include "vx_rng.h"

namespace vx {
namespace tc {

constexpr int kBM = 128;       // weight rows per tile (UMMA M = TMEM lanes)
constexpr int kBK = 64;        // K per stage = one 128-byte swizzle row of f16
constexpr int kThreads = 128;

template <int BN>
struct Cfg {
  static_assert(BN == 16 || BN == 64 || BN == 128 || BN == 256, "BN");
  static constexpr int kA = kBM * kBK * 2;                   // 16 KB
  static constexpr int kB = BN * kBK * 2;                    // per hi / lo operand
  static constexpr int kStage = kA + 2 * kB;
  static constexpr int kStages = (196 * 1024) / kStage;       // BN=16: 9, 64: 6, 128: 4, 256: 2
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;    // TMEM allocations are powers of 2 >= 32
  static constexpr size_t kSmem = (size_t)kStages * kStage + 1024 /*align*/ + 256 /*barriers*/;
  // instruction descriptor (kind::f16): D f32 (bit 4), A = B = f16, both K-major,
  // N >> 3 at bit 17, M >> 4 at bit 24
  static constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
};

struct Params {
  float* y;              // Y[n * ldy + m]
  long long ldy;
  float* ws;             // split-K partials [m_tiles * n_tiles][splits][BN][kBM]
  int M, N, K;
  int chunks_per_split;  // K chunks (kBK each) per split
  int accumulate;        // 0: Y = acc, 1: Y += acc (residual)
};

// ---------------------------------------------------------------- tcgen05 wrappers
// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride
// byte offset), descriptor version 1, layout type 2 (SWIZZLE_128B).  A K step of
// 16 f16 inside the 128-byte row advances the start address by 32 bytes; the
// tile base is 1024-byte aligned so the swizzle phase is that of the row.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 16 consecutive f32 columns of this thread's TMEM lane (warp-wide, .sync.aligned);
// the wait is in the same statement so no register is read before it lands.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- the GEMM
template <int BN>
__global__ void __launch_bounds__(kThreads, 1) k_gemm(const __grid_constant__ CUtensorMap wmap,
                                                      const __grid_constant__ CUtensorMap xhi_map,
                                                      const __grid_constant__ CUtensorMap xlo_map,
                                                      const __grid_constant__ Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStage);
  uint64_t* empty = full + C::kStages;
  uint64_t* accb = empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y, split = blockIdx.z, splits = gridDim.z;
  const int m0 = m_tile * kBM, n0 = n_tile * BN;
  const int kc0 = split * p.chunks_per_split;
  const int nk = max(0, min(p.chunks_per_split, p.K / kBK - kc0));

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    fence_mbar_init();
    prefetch_tmap(&wmap);
    prefetch_tmap(&xhi_map);
    prefetch_tmap(&xlo_map);
  }
  if (warp == 2) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_launch();
  // The weight tiles do not depend on the previous kernel: the first ring's worth of them
  // starts streaming before the dependency wait, under the previous kernel's tail.
  const int pre = min(nk, C::kStages);
  if (warp == 0 && lane == 0)
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], C::kStage);   // W now, X after the wait: one phase
      tma_load_2d(smem + i * C::kStage, &wmap, (kc0 + i) * kBK, m0, &full[i]);
    }
  griddep_wait();   // X (and Y when accumulating) come from the previous kernel

  if (warp == 0 && lane == 0) {
    // ---- TMA producer
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      if (i >= C::kStages && !mbar_wait(&empty[s], (uint32_t)((i / C::kStages) - 1) & 1u, kDevTimeoutEmpty)) break;
      uint8_t* st = smem + s * C::kStage;
      const int kx = (kc0 + i) * kBK;
      if (i >= pre) {
        mbar_arrive_expect_tx(&full[s], C::kStage);
        tma_load_2d(st, &wmap, kx, m0, &full[s]);
      }
      tma_load_2d(st + C::kA, &xhi_map, kx, n0, &full[s]);
      tma_load_2d(st + C::kA + C::kB, &xlo_map, kx, n0, &full[s]);
      issued = i + 1;
    }
    // After an error the MMA warp may stop consuming: every copy still in flight must
    // land before the CTA's shared memory is released (each stage's last use is exact).
    if (issued < nk || error_set())
      for (int i = issued > C::kStages ? issued - C::kStages : 0; i < issued; ++i)
        if (!mbar_wait_drain(&full[i % C::kStages], (uint32_t)(i / C::kStages) & 1u)) break;
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      if (!mbar_wait(&full[s], (uint32_t)(i / C::kStages) & 1u, kDevTimeoutFull)) break;
      tc_fence_after();
      const uint32_t a = smem_u32(smem + s * C::kStage);
      const uint32_t bh = a + C::kA, bl = bh + C::kB;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        const uint64_t ad = sw128_desc(a + kk * 32);
        tc_mma(tmem, ad, sw128_desc(bh + kk * 32), C::kIdesc, (i | kk) != 0 ? 1u : 0u);
        tc_mma(tmem, ad, sw128_desc(bl + kk * 32), C::kIdesc, 1u);
      }
      tc_commit(&empty[s]);   // the stage is free once these MMAs have read it
    }
    tc_commit(accb);          // accumulator complete
  }
  __syncwarp();

  // ---- epilogue: TMEM -> registers -> global
  const bool acc_ok = mbar_wait(accb, 0u, kDevTimeoutAcc);
  tc_fence_after();
  const int row = warp * 32 + lane;          // TMEM lane = weight row inside the tile
  const int m = m0 + row;
  const uint32_t tbase = tmem + ((uint32_t)(warp * 32) << 16);
  const bool live = acc_ok && nk > 0;
  if (splits == 1) {
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      tmem_ld16(tbase + c, v);
      if (live && m < p.M) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = n0 + c + j;
          if (n < p.N) {
            float* yp = p.y + (long long)n * p.ldy + m;
            *yp = p.accumulate ? *yp + v[j] : v[j];
          }
        }
      }
    }
  } else {
    const int tile = m_tile * gridDim.x + n_tile;
    float* wst = p.ws + (long long)tile * splits * (BN * kBM);
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      tmem_ld16(tbase + c, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) wst[(long long)split * BN * kBM + (c + j) * kBM + row] = live ? v[j] : 0.f;
    }
  }

  // ---- teardown: every tcgen05.ld has completed (wait::ld above)
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Sum of the split-K partials of k_gemm, in split order, into Y (= or +=).  One
// thread per 4 consecutive output rows m of one token n (float4 along m).
struct ReduceParams {
  const float* ws;
  float* y;
  long long ldy;
  int M, N, splits, n_tiles, bn, accumulate;
};
__global__ void __launch_bounds__(256) k_splitk_reduce(const __grid_constant__ ReduceParams p) {
  griddep_launch();
  griddep_wait();
  const long long total = (long long)p.N * (p.M / 4);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / (p.M / 4)), m = (int)(i % (p.M / 4)) * 4;
    const int tile = (m / kBM) * p.n_tiles + n / p.bn;
    const float* src = p.ws + ((long long)tile * p.splits * p.bn + n % p.bn) * kBM + m % kBM;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < p.splits; ++s) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + (long long)s * p.bn * kBM));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    float4* yp = reinterpret_cast<float4*>(p.y + (long long)n * p.ldy + m);
    if (p.accumulate) {
      const float4 y = *yp;
      acc.x += y.x; acc.y += y.y; acc.z += y.z; acc.w += y.w;
    }
    *yp = acc;
  }
}

// ---------------------------------------------------------------- token batches
// Which (slot, position) each activation row belongs to.
//   mode 0: the N consecutive prompt positions of slot `slot`, starting at the
//           slot's current position (batched prefill);
//   mode 1: row r is slot `slot` + r at its current position (batched decode).
struct TokRows {
  const int32_t* pos;   // &SlotState[0].pos
  int pos_stride;       // ints between consecutive slots' states
  int mode, slot;
};
__device__ __forceinline__ int tok_slot(const TokRows& t, int r) { return t.mode == 0 ? t.slot : t.slot + r; }
__device__ __forceinline__ int tok_pos(const TokRows& t, int r) {
  return t.mode == 0 ? t.pos[(long long)t.slot * t.pos_stride] + r : t.pos[(long long)(t.slot + r) * t.pos_stride];
}

__device__ __forceinline__ void split_store(__half* hi, __half* lo, long long i, float x) {
  const __half h = __float2half_rn(x);
  hi[i] = h;
  lo[i] = __float2half_rn(x - __half2float(h));
}

// X[N, K] f32 -> hi/lo pair (attention output feeding o_proj).
__global__ void k_tb_split(const float* __restrict__ x, long long n, __half* hi, __half* lo) {
  griddep_launch();
  griddep_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    split_store(hi, lo, i, x[i]);
}

// swiGLU (src/shaders.ts:483-501) of Y13[N, 2F] (gate rows [0,F), up rows [F,2F)
// of the stacked [w1; w3] projection) into the hi/lo pair of G[N, F].
__global__ void k_tb_swiglu_split(const float* __restrict__ y13, int N, int F, __half* hi, __half* lo) {
  griddep_launch();
  griddep_wait();
  const long long n = (long long)N * F;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / F, c = i % F;
    const float* yr = y13 + r * 2 * F;
    split_store(hi, lo, i, swiglu(yr[c], yr[F + c]));
  }
}

// RoPE (src/shaders.ts:224-256, interleaved pairs, angle = pos * freq) on the q
// and k parts of a QKV row [q_dim + 2 kv_dim], q -> Q[N, q_dim] (f32), K/V appended
// to the paged f16 cache at the row's position (src/shaders.ts:452-473), with the
// rotation arithmetic of the decode kernels' QKV epilogue (k_tb_row, kRowQkv).
struct RopeKvParams {
  const float* qkv;
  float* q;
  int q_dim, kv_dim, N;
  __half* pool;
  const int32_t* page_table;
  int max_pages, n_layers, n_kv, page_size, layer;
  const float* rope_freq;
  TokRows rows;
};
// Per-row epilogue of a token-batch GEMM, one CTA per activation row n: sums the split-K partials of the row in split order (splits == 0: the
// GEMM wrote its result to Y itself) and then
//   kRowResidNorm: h[n] += partials; x' = RMSNorm(h[n]) * w (src/shaders.ts:137-183:
//                  x * (1/sqrt(mean(x^2) + eps)) * w) -> hi/lo operand pair of the
//                  next GEMM (norm_w null: no operand output);
//   kRowQkv:       RoPE on the q / k parts, q -> Q[n], K/V appended to the paged
//                  cache at the row's position.
enum RowMode { kRowResidNorm = 0, kRowQkv = 1 };
struct RowParams {
  const float* ws;
  int splits, n_tiles, bn;   // partial layout of k_gemm: [tile][split][bn][kBM]
  float* y;                  // h [N][ldy] (kRowResidNorm) or the QKV rows (kRowQkv, splits == 0)
  long long ldy;
  int M;
  int mode;
  const __half* norm_w;
  float eps;
  __half *hi, *lo;           // [N][M]
  RopeKvParams rope;         // kRowQkv (rope.qkv unused)
  const float* add;          // kRowResidNorm with splits == 0: h[n] += add[n] ([N][M], e.g. an all-reduced
                             // tensor-parallel partial); null: Y already holds h[n]
};
// Launched with M / 4, M / 8 or M / 12 threads per row (a multiple of 32, at most
// 1024): each thread owns 1-3 float4 groups and issues the loads of every split at
// once (up to kMaxRowSplits in flight).
constexpr int kMaxRowSplits = 8;
__global__ void __launch_bounds__(1024) k_tb_row(const __grid_constant__ RowParams p) {
  griddep_launch();
  griddep_wait();
  __shared__ float sh[32];
  const int n = blockIdx.x;
  const int nt = blockDim.x;
  const int G = p.M / (4 * nt);   // float4 groups per thread
  float4 v[3];
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (u >= G) continue;
    const int m = (threadIdx.x + nt * u) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.splits == 0) {
      acc = *reinterpret_cast<const float4*>(p.y + (long long)n * p.ldy + m);
      if (p.mode == kRowResidNorm && p.add) {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(p.add + (long long)n * p.M + m));
        acc = make_float4(acc.x + a.x, acc.y + a.y, acc.z + a.z, acc.w + a.w);
        *reinterpret_cast<float4*>(p.y + (long long)n * p.ldy + m) = acc;
      }
    } else {
      const int tile = (m / kBM) * p.n_tiles + n / p.bn;
      const float* src = p.ws + ((long long)tile * p.splits * p.bn + n % p.bn) * kBM + m % kBM;
      float4 w[kMaxRowSplits];
#pragma unroll
      for (int s = 0; s < kMaxRowSplits; ++s)
        if (s < p.splits) w[s] = __ldcg(reinterpret_cast<const float4*>(src + (long long)s * p.bn * kBM));
#pragma unroll
      for (int s = 0; s < kMaxRowSplits; ++s)
        if (s < p.splits) { acc.x += w[s].x; acc.y += w[s].y; acc.z += w[s].z; acc.w += w[s].w; }
      if (p.mode == kRowResidNorm) {
        const float4 h = *reinterpret_cast<const float4*>(p.y + (long long)n * p.ldy + m);
        acc = make_float4(h.x + acc.x, h.y + acc.y, h.z + acc.z, h.w + acc.w);
        *reinterpret_cast<float4*>(p.y + (long long)n * p.ldy + m) = acc;
      }
    }
    v[u] = acc;
  }
  if (p.mode == kRowResidNorm) {
    if (!p.norm_w) return;
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 3; ++u)
      if (u < G) ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (nt >> 5); ++i) tot += sh[i];
    const float rms = 1.0f / sqrtf(tot / (float)p.M + p.eps);
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      if (u >= G) continue;
      const int m = (threadIdx.x + nt * u) * 4;
      const __half2* w2 = reinterpret_cast<const __half2*>(p.norm_w + m);
      const float2 wa = __half22float2(w2[0]), wb = __half22float2(w2[1]);
      const long long o = (long long)n * p.M + m;
      split_store(p.hi, p.lo, o + 0, v[u].x * rms * wa.x);
      split_store(p.hi, p.lo, o + 1, v[u].y * rms * wa.y);
      split_store(p.hi, p.lo, o + 2, v[u].z * rms * wb.x);
      split_store(p.hi, p.lo, o + 3, v[u].w * rms * wb.y);
    }
    return;
  }
  // kRowQkv: RoPE pairs are (m, m+1) inside each float4
  const RopeKvParams& r = p.rope;
  const int slot = tok_slot(r.rows, n), pos = tok_pos(r.rows, n);
  const int lp = pos / r.page_size;
  const bool page_ok = pos >= 0 && lp < r.max_pages;
  if (!page_ok && threadIdx.x == 0) set_error(kDevBadIndex);
  const int page = page_ok ? r.page_table[(long long)slot * r.max_pages + lp] : 0;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    if (u >= G) continue;
    const int m = (threadIdx.x + nt * u) * 4;
    float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
    if (m < r.q_dim + r.kv_dim) {
#pragma unroll
      for (int q = 0; q < 4; q += 2) {
        const int pair = ((m + q) & 127) >> 1;
        const float ang = (float)pos * r.rope_freq[pair];
        float sn, cs;
        sincosf(ang, &sn, &cs);
        const float x0 = e[q], x1 = e[q + 1];
        e[q] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        e[q + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
      }
    }
    if (m < r.q_dim) {
      *reinterpret_cast<float4*>(r.q + (long long)n * r.q_dim + m) = make_float4(e[0], e[1], e[2], e[3]);
    } else if (page_ok && m < r.q_dim + 2 * r.kv_dim) {
      const int kvr = m - r.q_dim;
      const int kv = kvr >= r.kv_dim ? 1 : 0;
      const int rr = kvr - kv * r.kv_dim;
      const int head = rr >> 7, d = rr & 127;
      const long long prow =
          ((((long long)page * r.n_layers + r.layer) * 2 + kv) * r.n_kv + head) * r.page_size + pos % r.page_size;
      __half2* dst = reinterpret_cast<__half2*>(r.pool + prow * 128 + d);
      dst[0] = __floats2half2_rn(e[0], e[1]);
      dst[1] = __floats2half2_rn(e[2], e[3]);
    }
  }
}

// Input rows of a prefill batch: prompt[pos] is a token id (tok_embeddings row,
// src/engine.ts:832-841) or -(r+1) for voice row r, which replaces the lookup
// (src/engine.ts:843-854).
struct TbEmbedParams {
  const __half* tok;
  int vocab;
  const int32_t* prompt;   // [n_slots][max_seq]
  const float* voice;      // [n_slots][max_voice][D]
  int max_seq, max_voice, D;
  float* h;                // [N][D]
  TokRows rows;
};
__global__ void __launch_bounds__(256) k_tb_embed(const __grid_constant__ TbEmbedParams p) {
  griddep_launch();
  griddep_wait();
  const int r = blockIdx.x;
  const int slot = tok_slot(p.rows, r), pos = tok_pos(p.rows, r);
  int kind = -1, idx = 0;
  if (pos >= 0 && pos < p.max_seq) {
    const int t = p.prompt[(long long)slot * p.max_seq + pos];
    if (t < 0) { kind = 1; idx = -t - 1; if (idx >= p.max_voice) kind = -1; }
    else if (t < p.vocab) { kind = 0; idx = t; }
  }
  if (kind < 0 && threadIdx.x == 0) set_error(kDevBadIndex);
  float* out = p.h + (long long)r * p.D;
  for (int i = threadIdx.x; i < p.D; i += 256) {
    float v = 0.f;
    if (kind == 0) v = __half2float(p.tok[(long long)idx * p.D + i]);
    else if (kind == 1) v = p.voice[((long long)slot * p.max_voice + idx) * p.D + i];
    out[i] = v;
  }
}

// Advance a slot's position by n after a batched prefill (the reference's
// `this.position++` per prompt token, src/engine.ts:2472).
__global__ void k_tb_advance(int32_t* pos, int n) {
  griddep_launch();
  griddep_wait();
  if (threadIdx.x == 0) *pos += n;
}

// ---------------------------------------------------------------- self-test support
// Reference product on CUDA cores in f32 from the same f16 W and f32 X (the X
// the tensor-core path splits into hi/lo), for vx_selftest_gemm.
__global__ void k_ref_gemm(const __half* W, const float* X, int M, int N, int K, float* Y) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x, n = blockIdx.y;
  if (m >= M) return;
  float acc = 0.f;
  for (int k = 0; k < K; ++k) acc = fmaf(__half2float(W[(long long)m * K + k]), X[(long long)n * K + k], acc);
  Y[(long long)n * M + m] = acc;
}
__global__ void k_selftest_fill(__half* W, long long nw, float* X, long long nx, uint64_t key) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nw + nx;
       i += (long long)gridDim.x * blockDim.x) {
    if (i < nw) W[i] = __float2half_rn(0.02f * vx_normal(key, (uint64_t)i));
    else X[i - nw] = vx_normal(key, (uint64_t)i);
  }
}

}  // namespace tc
}  // namespace vx
