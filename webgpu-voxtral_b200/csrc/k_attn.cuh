// k_attn.cuh — split-KV flash-decode GQA attention over the paged f16 KV cache.
//
// Replaces attnScore / softmax / attnValue (src/shaders.ts:306-447, dispatched at
// src/engine.ts:918-944): out[h] = softmax(q_h . K[0..pos, h/4]^T / sqrt(128)) V.
// The reference materialises the [32, seq] score matrix in global memory and
// reads the f32 KV cache three times; here one pass reads each f16 K/V page once.
//
// Grid (kv_head, split, batch row), 4 warps.  A batch row is either one slot at
// its current position or (rows_consecutive) one of a batch of consecutive
// prompt positions of a single slot, attending causally up to its own position.  A split owns a contiguous range of
// 64-position pages; one thread streams K and V pages (2-D TMA tiles, 128-byte
// swizzle, double-buffered) and each warp takes 16 positions of the page.
// The 4 query heads that share a KV head form the rows of an m16n8k16 MMA:
// rows 0-3 hold q in f16 (hi), rows 4-7 the f16 remainder (lo) of the same q,
// so q.K keeps ~22 bits of q.  Online softmax in f32; P is split hi/lo the same
// way for P.V.  Each split writes (max, sum, unnormalised O) and the last split
// CTA of a (row, kv_head) merges all splits (atomic ticket) and writes
// attn_out — no separate combine launch.
#pragma once
#include "k_gemv.cuh"
#include "vx_common.cuh"

namespace vx {
namespace attn {

constexpr int kThreads = 128;
constexpr int kGqa = 4;              // query heads per KV head
constexpr int kHd = 128;
constexpr int kPage = 64;
constexpr int kStageBytes = 4 * 8192;  // K box0, K box1, V box0, V box1 (64 rows x 64 cols f16 each)
constexpr int kPartStride = 4 + kHd;   // (m, l, -, -, o[128]) per head: o 16-byte aligned
constexpr int kMaxSplits = 64;         // splits per (row, kv head); the combine holds one weight per split
constexpr size_t kSmemBytes = 2 * (size_t)kStageBytes + 1024 /*align slack*/ + 64;

struct Params {
  const float* q;            // [rows][ldq], row m = slot slot0 + m
  long long ldq;
  float* out;                // [rows][ldo]
  long long ldo;
  float* part;               // [rows][n_kv][n_splits][kGqa][kPartStride]
  int* tickets;              // [rows][n_kv], zero between launches
  gemv::KvGeom kv;
  int layer;
  const int32_t* pos;        // current position of each slot (stride pos_stride)
  int pos_stride;
  int slot0;
  int n_splits;
  float scale;
  int rows_consecutive;      // 1: every row is slot slot0, row m at position pos(slot0) + m (batched prefill)
  __half* out_hi;            // nullable: out also as an f16 hi / lo pair [rows][ldo] (tensor-core GEMM operand)
  __half* out_lo;
};

// Byte offset of 16-byte chunk (row, col/8) inside a K or V page tile made of
// two 64x64 f16 TMA boxes with the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz(int row, int col) {
  const int box = col >> 6;
  const int chunk = (col & 63) >> 3;
  return (uint32_t)(box * 8192 + row * 128 + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kThreads) k_attn_decode(const __grid_constant__ CUtensorMap kvmap,
                                                          const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStageBytes);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x, split = blockIdx.y, row = blockIdx.z;
  const int slot = p.rows_consecutive ? p.slot0 : p.slot0 + row;

  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_mbar_init();
    prefetch_tmap(&kvmap);
  }
  __syncthreads();
  griddep_launch();
  griddep_wait();   // q and the K/V of the current position come from the previous kernel

  const int seq = p.pos[(long long)slot * p.pos_stride] + (p.rows_consecutive ? row : 0) + 1;
  const int npages = (seq + kPage - 1) / kPage;
  const int pps = (npages + p.n_splits - 1) / p.n_splits;
  const int pg0 = split * pps, pg1 = min(npages, pg0 + pps);
  const int32_t* ptab = p.kv.page_table + (long long)slot * p.kv.max_pages;

  auto issue = [&](int pg, int st) {
    const int phys = ptab[pg];
    const int krow = (int)gemv::kv_row(p.kv, phys, p.layer, 0, kvh, 0);
    const int vrow = (int)gemv::kv_row(p.kv, phys, p.layer, 1, kvh, 0);
    uint8_t* dst = smem + st * kStageBytes;
    mbar_arrive_expect_tx(&full[st], kStageBytes);
    tma_load_2d(dst, &kvmap, 0, krow, &full[st]);
    tma_load_2d(dst + 8192, &kvmap, 64, krow, &full[st]);
    tma_load_2d(dst + 16384, &kvmap, 0, vrow, &full[st]);
    tma_load_2d(dst + 24576, &kvmap, 64, vrow, &full[st]);
  };
  const bool bad = pg1 > p.kv.max_pages;
  if (bad && threadIdx.x == 0) set_error(kDevBadIndex);
  int issued = 0;   // pages issued so far (meaningful in thread 0)
  if (threadIdx.x == 0 && !bad) {
    if (pg0 < pg1) { issue(pg0, 0); issued = 1; }
    if (pg0 + 1 < pg1) { issue(pg0 + 1, 1); issued = 2; }
  }

  // A fragments of q: row g = lane/4 -> head g%4, hi (g<4) or lo (g>=4) half.
  const int g = lane >> 2, hq = g & 3;
  const bool lo_part = g >= 4;
  const float* qh = p.q + (long long)row * p.ldq + (long long)(kvh * kGqa + hq) * kHd;
  uint32_t qa0[8], qa2[8];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int c = kk * 16 + (lane & 3) * 2;
    float v0 = qh[c], v1 = qh[c + 1], v8 = qh[c + 8], v9 = qh[c + 9];
    if (lo_part) {
      v0 -= __half2float(__float2half_rn(v0));
      v1 -= __half2float(__float2half_rn(v1));
      v8 -= __half2float(__float2half_rn(v8));
      v9 -= __half2float(__float2half_rn(v9));
    }
    qa0[kk] = pack_half2(v0, v1);
    qa2[kk] = pack_half2(v8, v9);
  }

  float m_run = -INFINITY, l_run = 0.f;
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

  bool ok = !bad;
  for (int pg = pg0, i = 0; ok && pg < pg1; ++pg, ++i) {
    const int st = i & 1;
    // every thread leaves the loop together if any wait expired
    if (!__syncthreads_and(mbar_wait(&full[st], (uint32_t)(i >> 1) & 1u, kDevTimeoutFull))) { ok = false; break; }
    {
      const uint32_t kbase = smem_u32(smem + st * kStageBytes);
      const uint32_t vbase = kbase + 16384;
      // ---- S = Q K^T for this warp's 16 positions (two n8 tiles)
      float s[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      const int mat = lane >> 3, r8 = lane & 7;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int prow = warp * 16 + (mat >> 1) * 8 + r8;
        const int col = kk * 16 + (mat & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3, kbase + swz(prow, col));
        mma_16816(s[0], qa0[kk], 0u, qa2[kk], 0u, b0, b1);
        mma_16816(s[1], qa0[kk], 0u, qa2[kk], 0u, b2, b3);
      }
      // full score = hi row + lo row (lanes l and l^16), scaled, masked
      float sc[2][2];
      float mloc = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float full_dot = s[j][e] + __shfl_xor_sync(0xffffffffu, s[j][e], 16);
          const int ppos = pg * kPage + warp * 16 + j * 8 + (lane & 3) * 2 + e;
          const float v = ppos < seq ? full_dot * p.scale : -INFINITY;
          sc[j][e] = v;
          mloc = fmaxf(mloc, v);
        }
      mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 1));
      mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 2));
      const float m_new = fmaxf(m_run, mloc);
      const float corr = (m_new == -INFINITY) ? 1.f : expf(m_run - m_new);
      float psum = 0.f;
      uint32_t pa0, pa2;
      float pv[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pe = (sc[j][e] == -INFINITY) ? 0.f : expf(sc[j][e] - m_new);
          psum += pe;
          pv[j][e] = lo_part ? pe - __half2float(__float2half_rn(pe)) : pe;
        }
      pa0 = pack_half2(pv[0][0], pv[0][1]);
      pa2 = pack_half2(pv[1][0], pv[1][1]);
      l_run = l_run * corr + psum;
      m_run = m_new;
#pragma unroll
      for (int j = 0; j < 16; ++j) { o[j][0] *= corr; o[j][1] *= corr; }
      // ---- O += P V (16 positions x 128 dims)
#pragma unroll
      for (int dt2 = 0; dt2 < 8; ++dt2) {
        const int prow = warp * 16 + (mat & 1) * 8 + r8;
        const int col = dt2 * 16 + (mat >> 1) * 8;
        uint32_t v0, v1, v2, v3;
        ldmatrix_x4_trans(v0, v1, v2, v3, vbase + swz(prow, col));
        mma_16816(o[2 * dt2], pa0, 0u, pa2, 0u, v0, v1);
        mma_16816(o[2 * dt2 + 1], pa0, 0u, pa2, 0u, v2, v3);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && pg + 2 < pg1) { issue(pg + 2, st); issued = i + 3; }
  }
  if (!ok && threadIdx.x == 0) {
    // Drain any copy still in flight before the shared memory is released.
    for (int i = issued > 2 ? issued - 2 : 0; i < issued; ++i)
      if (!mbar_wait_drain(&full[i & 1], (uint32_t)(i >> 1) & 1u)) break;
  }

  // ---- per-warp state -> shared, merge the 4 warps, write this split's partial
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    o[j][0] += __shfl_xor_sync(0xffffffffu, o[j][0], 16);
    o[j][1] += __shfl_xor_sync(0xffffffffu, o[j][1], 16);
  }
  __syncthreads();   // stage memory is free: reuse it as merge scratch
  float* ws = reinterpret_cast<float*>(smem);   // [4 warps][kGqa][kPartStride]
  if (lane < 16) {
    float* w = ws + (warp * kGqa + hq) * kPartStride;
    if ((lane & 3) == 0) { w[0] = m_run; w[1] = l_run; }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = j * 8 + (lane & 3) * 2;
      w[2 + d] = o[j][0];
      w[2 + d + 1] = o[j][1];
    }
  }
  __syncthreads();
  float* part = p.part + (((long long)row * p.kv.n_kv + kvh) * p.n_splits + split) * (kGqa * kPartStride);
  for (int idx = threadIdx.x; idx < kGqa * kHd; idx += kThreads) {
    const int h = idx / kHd, d = idx % kHd;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, ws[(w * kGqa + h) * kPartStride]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float* ww = ws + (w * kGqa + h) * kPartStride;
        const float f = (ww[0] == -INFINITY) ? 0.f : expf(ww[0] - M);
        L += ww[1] * f;
        O += ww[2 + d] * f;
      }
    }
    if (p.n_splits == 1) {
      // one split: this CTA holds the whole softmax, write the output directly
      const float v = L > 0.f ? O / L : 0.f;
      const long long oi = (long long)row * p.ldo + (long long)(kvh * kGqa + h) * kHd + d;
      p.out[oi] = v;
      if (p.out_hi) {
        const __half hh = __float2half_rn(v);
        p.out_hi[oi] = hh;
        p.out_lo[oi] = __float2half_rn(v - __half2float(hh));
      }
      continue;
    }
    part[h * kPartStride + 2 + d] = O;
    if (d == 0) { part[h * kPartStride] = M; part[h * kPartStride + 1] = L; }
  }
  if (p.n_splits == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int t = atomicAdd(&p.tickets[row * p.kv.n_kv + kvh], 1);
    s_last = (t == p.n_splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- last split CTA: merge the splits that hold positions into attn_out.
  // Warp h reduces head h's (max, sum) over the splits in parallel; then every
  // thread sums its (head, dim) outputs with independent loads.
  const float* pb = p.part + ((long long)row * p.kv.n_kv + kvh) * p.n_splits * (kGqa * kPartStride);
  const int n_used = min(p.n_splits, (npages + pps - 1) / pps);
  __shared__ float s_w[kMaxSplits][kGqa];
  {
    const int h = warp;
    float ms[2], ls[2];
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int sp = lane + 32 * j;
      ms[j] = sp < n_used ? __ldcg(pb + sp * kGqa * kPartStride + h * kPartStride) : -INFINITY;
      ls[j] = sp < n_used ? __ldcg(pb + sp * kGqa * kPartStride + h * kPartStride + 1) : 0.f;
      M = fmaxf(M, ms[j]);
    }
    M = warp_max(M);
    float f[2], L = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      f[j] = (ms[j] == -INFINITY) ? 0.f : expf(ms[j] - M);
      L += ls[j] * f[j];
    }
    L = warp_sum(L);
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (lane + 32 * j < n_used) s_w[lane + 32 * j][h] = f[j] / L;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < kGqa * kHd; idx += kThreads) {
    const int h = idx / kHd, d = idx % kHd;
    float O = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < n_used; ++sp) O += __ldcg(pb + sp * kGqa * kPartStride + h * kPartStride + 2 + d) * s_w[sp][h];
    const long long oi = (long long)row * p.ldo + (long long)(kvh * kGqa + h) * kHd + d;
    p.out[oi] = O;
    if (p.out_hi) {
      const __half hh = __float2half_rn(O);
      p.out_hi[oi] = hh;
      p.out_lo[oi] = __float2half_rn(O - __half2float(hh));
    }
  }
  if (threadIdx.x == 0) p.tickets[row * p.kv.n_kv + kvh] = 0;
}

}  // namespace attn
}  // namespace vx
