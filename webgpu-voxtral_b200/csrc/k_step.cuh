// k_step.cuh — persistent decode megakernel: many backbone steps in one launch.
//
// Replaces the reference's per-token command stream (backboneStep, src/engine.ts:814-1042:
// ~450 dispatches per token, one queue.submit per token in the prefill loop :2457-2472
// and per frame in the decode loop :2498-2541) with ONE cooperative launch that runs
// `n_frames` consecutive backbone steps of one utterance.
//
// Each step is a fixed program of phases separated by grid-wide barriers:
//   EMBED | 26 x ( QKV+RoPE+KV-append | ATTENTION | O+residual | W13+SwiGLU | W2+residual ) | FINAL-NORM
// Grid: one CTA per SM, 10 warps.
//   warp 0  producer: walks every GEMV phase of every step and streams the weight
//           tiles assigned to this CTA through a 4-stage ring (TMA bulk copies).
//           Weights never depend on activations, so it never waits on a barrier:
//           while the consumers wait at a phase boundary the ring keeps filling,
//           and HBM stays busy across all phases, layers and steps.
//   warps 1-8 consumers: GEMV partial sums from the ring (x' slice in registers),
//           attention (mma.sync over TMA-loaded f16 KV pages), embedding and final
//           norm slices.
//   warp 9  epilogue: per-tile sums, fused epilogue (RoPE + KV append, residual,
//           SwiGLU), and this CTA's arrival at the grid barrier of each GEMV phase.
// Tiles of GEMV phase p are dealt round-robin starting at CTA (sum of earlier tile
// counts) mod G, so every CTA's cumulative share of the weight stream stays within
// one tile of the others.
// Tensor parallelism (template degree N > 1, one kernel per GPU): each rank holds
// 1/N of the q / KV heads and FFN columns.  The o_proj and down epilogues store the
// rank's partial rows straight into every rank's receive buffer (peer memory over
// NVLink) as 8-byte words {value, all-reduce index + 1}; the next phase's prologue
// polls those words until every rank's tag has arrived (no fence, no counter, no
// grid barrier on this transition) and forms h = h_old + sum of the N partials in
// rank order, so every rank holds the same residual stream (the reference's
// single-device step, split over N GPUs with 2 all-reduces per layer fused into the
// kernel).
// Every wait is bounded (vx_common.cuh): an expired wait records a device error and
// the kernel unwinds instead of hanging.
#pragma once
#include "k_attn.cuh"
#include "k_gemv.cuh"
#include "k_misc.cuh"

namespace vx {
namespace mk {

constexpr int kCW = 8;
constexpr int kThreads = (kCW + 2) * 32;
constexpr int kStages = 4;
constexpr int kStageBytes = 36864;
constexpr int kRedSlots = 4;
constexpr int kMaxVals = 32;
constexpr int D = 3072, HD = 128, GQA = 4;
constexpr int kMaxTp = 8;
// Per-rank dimensions and tile geometry of tensor-parallel degree N.  O and W2
// tiles keep ~32-36 KB per stage: RO / RW2 rows of the rank's K columns; WKO /
// WKW2 consumer warps split K (8 / WK warps split the rows).
template <int N>
struct Tp {
  static_assert(N == 1 || N == 2 || N == 4 || N == 8, "tensor-parallel degree");
  static constexpr int QD = 4096 / N, KVD = 1024 / N, QKVD = QD + 2 * KVD, F = 9216 / N, NKV = 8 / N;
  static constexpr int RO = 4 * N, WKO = N == 8 ? 4 : 8, CPLO = QD / 128 / WKO;
  static constexpr int RW2 = 2 * N, WKW2 = 8 / N, CPLW2 = F / 128 / WKW2;
  static constexpr int TQKV = QKVD / 6, TO = D / RO, TW13 = F / 3, TW2 = D / RW2;
  static constexpr int TLayer = TQKV + TO + TW13 + TW2;
  static_assert(RO * QD * 2 <= 36864 && RW2 * F * 2 <= 36864, "tile fits a stage");
};

// shared memory map (offsets from a 1024-aligned base)
constexpr int kOffRing = 0;
constexpr int kOffAttn = kStages * kStageBytes;            // 147456, 1024-aligned
constexpr int kAttnBytes = 65536;                          // a pair of K/V pages
constexpr int kOffBars = kOffAttn + kAttnBytes;            // mbarriers
constexpr int kOffRed = kOffBars + 256;
constexpr int kOffScratch = kOffRed + kRedSlots * kCW * kMaxVals * 4;
constexpr int kScratchBytes = 4096;   // [0,256) norm partials, [256,768) q of the attention item, [768,805) codes
constexpr size_t kSmemBytes = (size_t)kOffScratch + kScratchBytes + 1024;   // + alignment slack

// tiles per reduction group (group outputs TG * rows-per-tile <= 32)
constexpr int kTgQKV = 1, kTgO = 1, kTgW13 = 1, kTgW2 = 1;

struct LayerPtrs {
  const __half *wqkv, *wo, *w13, *w2, *attn_norm, *ffn_norm;
};

struct StepParams {
  const LayerPtrs* layers;
  int n_layers;
  const __half* tok; int vocab;
  const __half* audio; int audio_rows;
  const float* rows_in;
  const int32_t* prompt; const float* voice; int max_seq, max_voice;
  uint32_t* code_ring;
  float *h, *q, *att, *g, *normed, *normed_ring;
  const __half* final_norm;
  float eps;
  gemv::KvGeom kv;
  float* part; int* tickets; int n_splits;
  const float* rope_freq;
  SlotState* slots; int slot;
  unsigned* bar;          // grid barrier counter, zero at launch
  unsigned long long* trace;  // nullable: [G][kTraceFrames][phases][kTraceSlots] (see trace_mark)
  int prefetch_ahead;     // weight tiles prefetched into L2 ahead of the ring (0..kMaxPrefetchAhead)
  int early_kv;           // copy each CTA's first K/V pair during the QKV phase (preload_kv)
  int n_frames;
  int mode0, token0;      // embedding of the first step
  int mode_next;          // embedding of later steps
  int inc_frame, record;  // advance the frame counter / record normed states per step
  // Per-layer record (debugBackboneLayerByLayer, src/engine.ts:2106-2287) of step dbg_frame
  // of this launch: dbg [(4L+3)][D] = embed, per layer {attn_norm, attn_out, ffn_norm,
  // ffn_out}, final_norm, hidden.  Null: no record.
  float* dbg;
  int dbg_frame;
  // Polls before a bounded wait of this kernel gives up (0: the built-in limits).
  uint32_t wait_limit;
  // tensor parallelism (N > 1)
  int rank;
  float* h2;                          // second residual buffer (h alternates per all-reduce)
  unsigned long long* recv;           // this rank's receive words [2 parity][N source][D]: tag << 32 | f32 bits
  unsigned long long* peer_recv[kMaxTp];   // every rank's receive words (index = rank; own one included)
  unsigned long long* hx;             // local tagged words of the summed residual [2 parity][D]
  unsigned long long ar_base;         // all-reduces completed before this launch
  // AR kernels: the QKV epilogues' outputs as tagged words [QD + 2 KVD] (K / V rows
  // f16-rounded; local memory, zeroed at allocation), read by the attention phase
  unsigned long long* qkv_t;
};

struct Smem {
  uint8_t* ring;
  uint8_t* attn;
  uint64_t *full, *empty, *rfull, *rempty, *afull;
  float* red;
  float* scratch;
};

__device__ __forceinline__ Smem smem_map(uint8_t* raw) {
  uint8_t* b = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  Smem s;
  s.ring = b + kOffRing;
  s.attn = b + kOffAttn;
  uint64_t* bars = reinterpret_cast<uint64_t*>(b + kOffBars);
  s.full = bars; s.empty = bars + kStages; s.rfull = bars + 2 * kStages; s.rempty = s.rfull + kRedSlots;
  s.afull = s.rempty + kRedSlots;
  s.red = reinterpret_cast<float*>(b + kOffRed);
  s.scratch = reinterpret_cast<float*>(b + kOffScratch);
  return s;
}

// ---------------------------------------------------------------- grid barrier
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Generic-proxy stores to shared memory ordered before later TMA writes to it.
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Tagged all-reduce words: 8-byte single-copy-atomic stores / loads, so a reader
// that sees the expected tag also sees the value stored with it.
__device__ __forceinline__ void st_tagged(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_tagged2(const unsigned long long* p) {
  ulonglong2 v;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Value of a tagged word once its tag is `tag` (bounded poll, as below).
// Default poll limits of the kernel's waits (StepParams::wait_limit overrides both).
constexpr uint32_t kTagPolls = 1u << 24, kBarPolls = 1u << 27;
__device__ __forceinline__ float wait_tagged(const unsigned long long* p, uint32_t tag, uint32_t limit) {
  unsigned long long w = ld_tagged(p);
  for (uint32_t i = 0; (uint32_t)(w >> 32) != tag; ++i) {
    if (i > limit || ((i & 1023u) == 1023u && error_set())) {
      if (i > limit) set_error(kDevTimeoutPeer);
      break;
    }
    w = ld_tagged(p);
  }
  return __uint_as_float((uint32_t)w);
}
// Four consecutive tagged words (two 16-byte loads), once all carry `tag` (bounded
// poll: an expired wait records an error and returns the words' current values).
__device__ __forceinline__ float4 wait_tagged4(const unsigned long long* p, uint32_t tag, uint32_t limit) {
  ulonglong2 a = ld_tagged2(p), b = ld_tagged2(p + 2);
  for (uint32_t i = 0; (uint32_t)(a.x >> 32) != tag || (uint32_t)(a.y >> 32) != tag || (uint32_t)(b.x >> 32) != tag ||
                       (uint32_t)(b.y >> 32) != tag;
       ++i) {
    if (i > limit || ((i & 1023u) == 1023u && error_set())) {
      if (i > limit) set_error(kDevTimeoutPeer);
      break;
    }
    a = ld_tagged2(p);
    b = ld_tagged2(p + 2);
  }
  return make_float4(__uint_as_float((uint32_t)a.x), __uint_as_float((uint32_t)a.y), __uint_as_float((uint32_t)b.x),
                     __uint_as_float((uint32_t)b.y));
}
// Consumers (256 threads) wait until `target` CTA-phase arrivals are counted.  One
// thread polls (relaxed loads, then one acquire fence); the named barrier releases
// the others.  Writers publish with bar.sync + one red.release (no full fence).
// skip_grid (tensor parallelism, the phase after an all-reduce): the phase needs only
// the all-reduced residual, whose words carry their own tags, so the consumers only
// synchronise inside the CTA.
template <int N>
__device__ __forceinline__ void grid_wait(const StepParams& p, unsigned target, int ctid, bool skip_grid = false) {
  if (ctid == 0 && !skip_grid) {
    const uint32_t limit = p.wait_limit ? p.wait_limit : kBarPolls;
    uint32_t i = 0;
    while (ld_relaxed(p.bar) < target) {
      if (++i > limit || ((i & 1023u) == 0 && error_set())) {
        if (i > limit) set_error(kDevTimeoutBarrier);
        break;
      }
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  named_bar_sync(1, kCW * 32);
}
// Arrival of this CTA for the current phase, by the warp that wrote its outputs.
template <int N>
__device__ __forceinline__ void grid_arrive_warp(const StepParams& p, int lane, bool kv_written) {
  if (kv_written) fence_proxy_async_global();   // KV rows (st.global) are read by TMA next phase
  __syncwarp();
  if (lane == 0) red_release_add(p.bar, 1u);
}
// Phase trace for the first kTraceFrames steps when p.trace is set, per [cta][step][phase]:
// globaltimer stamps (ns) [0] = consumers released, [1] = consumers done, [2] = epilogue
// arrival, [3] = consumers' x' prologue done (GEMV phases); SM cycles spent waiting
// [4] = consumer warp 0 on weight stages, [5] = consumer warp 0 on reduction slots,
// [6] = epilogue warp on reduction results.  Attention phase, stamps of the CTA's
// first item: [4] K/V pair in shared memory, [5] split partial stored, [6] merge
// ticket taken.
constexpr int kTraceFrames = 2, kTraceSlots = 8;
__device__ __forceinline__ void trace_val(const StepParams& p, int c, int f, int kl, int which, int L, int t0,
                                          unsigned long long v) {
  if (p.trace && f < kTraceFrames && t0 == 0)
    p.trace[(((long long)c * kTraceFrames + f) * (2 + 5 * L) + kl) * kTraceSlots + which] = v;
}
__device__ __forceinline__ void trace_mark(const StepParams& p, int c, int f, int kl, int which, int L, int t0) {
  if (p.trace && f < kTraceFrames && t0 == 0) trace_val(p, c, f, kl, which, L, t0, globaltimer());
}
__device__ __forceinline__ long long clk() { return clock64(); }

__device__ __forceinline__ int first_tile(int c, int off, int G) { return (c - off % G + G) % G; }

// ---------------------------------------------------------------- producer
// Position in this CTA's sequence of weight tiles: (frame, layer, GEMV kind, tile).
constexpr int kMaxPrefetchAhead = 32;   // bound on StepParams::prefetch_ahead
template <int N>
__device__ __forceinline__ int tiles_of(int k) {
  return k == 0 ? Tp<N>::TQKV : k == 1 ? Tp<N>::TO : k == 2 ? Tp<N>::TW13 : Tp<N>::TW2;
}
struct Cursor {
  int f, l, k, t;
  int off;                    // dealing offset of the current phase: (tiles of earlier phases) mod G
  const __half *w0, *w1, *w2, *w3;   // weights of layer l (cached: no global load per tile)
};
__device__ __forceinline__ void cursor_layer(const StepParams& p, Cursor& x) {
  const LayerPtrs& W = p.layers[x.l];
  x.w0 = W.wqkv; x.w1 = W.wo; x.w2 = W.w13; x.w3 = W.w2;
}
template <int N>
__device__ __forceinline__ void cursor_fix(const StepParams& p, Cursor& x, int c, int G, int L) {
  while (x.t >= tiles_of<N>(x.k)) {
    x.off = (x.off + tiles_of<N>(x.k)) % G;
    if (++x.k == 4) {
      x.k = 0;
      if (++x.l == L) { x.l = 0; ++x.f; }
      if (x.f < p.n_frames) cursor_layer(p, x);
    }
    x.t = first_tile(c, x.off, G);
  }
}
template <int N>
__device__ __forceinline__ void cursor_start(const StepParams& p, Cursor& x, int c, int G, int L) {
  x.f = 0; x.l = 0; x.k = 0; x.off = 0; x.t = first_tile(c, 0, G);
  cursor_layer(p, x);
  cursor_fix<N>(p, x, c, G, L);
}
template <int N>
__device__ __forceinline__ void cursor_next(const StepParams& p, Cursor& x, int c, int G, int L) {
  x.t += G;
  cursor_fix<N>(p, x, c, G, L);
}
// Source of a tile: first chunk (and the SwiGLU "up" chunk), bytes per chunk.
// Every phase's row count is a multiple of its tile height, so tiles are full.
template <int N>
__device__ __forceinline__ void tile_src(const StepParams& p, const Cursor& x, const __half*& a, const __half*& b,
                                         uint32_t& bytes, int& ort) {
  using T = Tp<N>;
  b = nullptr;
  switch (x.k) {
    case 0: ort = 6; a = x.w0 + (long long)x.t * 6 * D; bytes = 6 * D * 2; break;
    case 1: ort = T::RO; a = x.w1 + (long long)x.t * T::RO * T::QD; bytes = T::RO * T::QD * 2; break;
    case 2: ort = 3; a = x.w2 + (long long)x.t * 3 * D; b = a + (long long)T::F * D; bytes = 3 * D * 2; break;
    default: ort = T::RW2; a = x.w3 + (long long)x.t * T::RW2 * T::F; bytes = T::RW2 * T::F * 2; break;
  }
}
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- consumer GEMV phase
// Tiles are consumed in groups of TG: each ring stage is released right after its
// FMAs, but the cross-lane reduction, the reduction-slot handoff and the epilogue run
// once per group (TG*R <= 32 outputs), which amortises their latency over TG tiles.
// Inputs of a phase that follows a tensor-parallel all-reduce.  At N = 8 the
// reduction runs in two stages inside the rank: (A) CTA c sums its slice [e0, e1) of
// the row over the N sources (h_old + partials in rank order), stores it to h_new and
// publishes it as tagged words in hx; (B) every CTA reads the whole summed row from
// hx.  A CTA only ever reads back its own slice of h_old / h_new, so those need no
// synchronisation.  At N <= 4 every CTA sums the whole row itself (ar_sum4) and CTA 0
// stores it to h_new.
struct ArIn {
  const float* h_old;
  const unsigned long long* recv;   // [N source][D] tagged words of this all-reduce's parity
  float* h_new;
  uint32_t tag;
  unsigned long long* hx;           // [D] tagged words of the summed row (this parity)
  int e0, e1;
  uint32_t limit;                   // polls before a wait for a peer's words gives up
};
__device__ __forceinline__ bool tags_are(const ulonglong2& a, const ulonglong2& b, uint32_t tag) {
  return (uint32_t)(a.x >> 32) == tag && (uint32_t)(a.y >> 32) == tag && (uint32_t)(b.x >> 32) == tag &&
         (uint32_t)(b.y >> 32) == tag;
}
// One-stage form (N <= 4): h_old + sum over source ranks 0..N-1 (in that order) of 4
// consecutive columns, read by every CTA for the whole row.  The loads of up to 4
// sources are issued before any tag is checked.
template <int N>
__device__ __forceinline__ float4 ar_sum4(const ArIn& a, int col) {
  constexpr int GS = N < 4 ? N : 4;
  float4 v = __ldcg(reinterpret_cast<const float4*>(a.h_old + col));
#pragma unroll
  for (int r0 = 0; r0 < N; r0 += GS) {
    ulonglong2 w[GS][2];
#pragma unroll
    for (int g = 0; g < GS; ++g) {
      const unsigned long long* q = a.recv + (long long)(r0 + g) * D + col;
      w[g][0] = ld_tagged2(q);
      w[g][1] = ld_tagged2(q + 2);
    }
#pragma unroll
    for (int g = 0; g < GS; ++g) {
      const float4 x = tags_are(w[g][0], w[g][1], a.tag)
                           ? make_float4(__uint_as_float((uint32_t)w[g][0].x), __uint_as_float((uint32_t)w[g][0].y),
                                         __uint_as_float((uint32_t)w[g][1].x), __uint_as_float((uint32_t)w[g][1].y))
                           : wait_tagged4(a.recv + (long long)(r0 + g) * D + col, a.tag, a.limit);
      v.x += x.x; v.y += x.y; v.z += x.z; v.w += x.w;
    }
  }
  return v;
}
// Two stages for N = 8, where every CTA reading all N x D words is the cost.
template <int N>
constexpr bool kArTwoStage = N >= 8;
// Stage A for thread t of the CTA's consumers: element e0 + t of the slice (the N
// source loads are issued before any tag is checked).
template <int N>
__device__ __forceinline__ void ar_stage_a(const ArIn& a, int t) {
  for (int i = a.e0 + t; i < a.e1; i += kCW * 32) {
    float v = __ldcg(a.h_old + i);
    unsigned long long w[N];
#pragma unroll
    for (int r = 0; r < N; ++r) w[r] = ld_tagged(a.recv + (long long)r * D + i);
#pragma unroll
    for (int r = 0; r < N; ++r)
      v += (uint32_t)(w[r] >> 32) == a.tag ? __uint_as_float((uint32_t)w[r]) : wait_tagged(a.recv + (long long)r * D + i, a.tag, a.limit);
    a.h_new[i] = v;
    st_tagged(a.hx + i, v, a.tag);
  }
}
// Stage B: CPL groups of 4 summed columns (all loads issued before the tag checks).
template <int CPL>
__device__ __forceinline__ void ar_stage_b(const ArIn& a, const int (&col)[CPL], float4 (&v)[CPL]) {
  ulonglong2 w[CPL][2];
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    w[j][0] = ld_tagged2(a.hx + col[j]);
    w[j][1] = ld_tagged2(a.hx + col[j] + 2);
  }
#pragma unroll
  for (int j = 0; j < CPL; ++j)
    v[j] = tags_are(w[j][0], w[j][1], a.tag)
               ? make_float4(__uint_as_float((uint32_t)w[j][0].x), __uint_as_float((uint32_t)w[j][0].y),
                             __uint_as_float((uint32_t)w[j][1].x), __uint_as_float((uint32_t)w[j][1].y))
               : wait_tagged4(a.hx + col[j], a.tag, a.limit);
}
// WK consumer warps split the tile's K columns (chunk j of warp (wr, wk) is
// column block wk + WK*j), the 8/WK row groups split its R rows.
template <int R, int CPL, bool NORM, int TG, int WK = kCW, int N = 1>
__device__ __forceinline__ bool consume(const StepParams& p, Smem& s, uint32_t& it, uint32_t& rit, const float* x,
                                       const __half* norm_w, int kc, int T, int off, int c, int G, int cw, int lane,
                                       int pos, int f, int kl, const ArIn* ar = nullptr, int rec_row = -1) {
  constexpr int RW = R / (kCW / WK);   // rows per warp
  static_assert(RW * (kCW / WK) == R && RW * TG <= kMaxVals, "tile rows");
  static_assert(!NORM || WK == kCW, "RMSNorm phases partition the row over all warps");
  constexpr int P = gemv::Pow2<RW * TG>::v;
  const int wr = cw / WK, wk = cw % WK;
  // x' slice in registers.  For the RMSNorm variants each warp's slice (CPL x 128
  // columns; the 8 slices partition the row) also gives its partial sum of squares,
  // so the norm costs one load round and one named barrier.
  float xr[CPL][4];
  float2 wn[CPL][2];
  float ss = 0.f;
  float4 hv[CPL];
  if (ar) {
    // all-reduce: h = h_old + partials of ranks 0..N-1, the same order on every rank
    int cols[CPL];
#pragma unroll
    for (int j = 0; j < CPL; ++j) cols[j] = (wk + WK * j) * 128 + lane * 4;
    if constexpr (kArTwoStage<N>) {
      ar_stage_a<N>(*ar, cw * 32 + lane);
      ar_stage_b<CPL>(*ar, cols, hv);
    } else {
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        hv[j] = ar_sum4<N>(*ar, cols[j]);
        if (c == 0) *reinterpret_cast<float4*>(ar->h_new + cols[j]) = hv[j];
      }
    }
  }
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int col = (wk + WK * j) * 128 + lane * 4;
    float4 v;
    if (ar) {
      v = hv[j];
    } else {
      v = *reinterpret_cast<const float4*>(x + col);
    }
    xr[j][0] = v.x; xr[j][1] = v.y; xr[j][2] = v.z; xr[j][3] = v.w;
    if (NORM) {
      const __half2* w2 = reinterpret_cast<const __half2*>(norm_w + col);
      wn[j][0] = __half22float2(w2[0]);
      wn[j][1] = __half22float2(w2[1]);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  }
  if (NORM) {
    ss = warp_sum(ss);
    if (lane == 0) s.scratch[cw] = ss;
    named_bar_sync(1, kCW * 32);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kCW; ++w) tot += s.scratch[w];
    const float rms = 1.0f / sqrtf(tot / (float)(CPL * kCW * 128) + p.eps);
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      xr[j][0] = xr[j][0] * rms * wn[j][0].x; xr[j][1] = xr[j][1] * rms * wn[j][0].y;
      xr[j][2] = xr[j][2] * rms * wn[j][1].x; xr[j][3] = xr[j][3] * rms * wn[j][1].y;
    }
  }
  if (NORM && rec_row >= 0 && p.dbg && f == p.dbg_frame && c == 0) {
    // per-layer record: the input row (rec_row) and its RMSNorm output (rec_row + 1)
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int col = (wk + WK * j) * 128 + lane * 4;
      const float4 raw = ar ? hv[j] : *reinterpret_cast<const float4*>(x + col);
      *reinterpret_cast<float4*>(p.dbg + (long long)rec_row * D + col) = raw;
      *reinterpret_cast<float4*>(p.dbg + (long long)(rec_row + 1) * D + col) =
          make_float4(xr[j][0], xr[j][1], xr[j][2], xr[j][3]);
    }
  }
  trace_mark(p, c, f, kl, 3, p.n_layers, cw * 32 + lane);
  const int my_idx = gemv::transpose_index<P>(lane);
  const bool writer = lane < P && my_idx < RW * TG;
  const uint32_t rowbytes = (uint32_t)kc * 2u;
  const bool tw = p.trace && f < kTraceFrames;   // wait accounting for the trace
  long long w_full = 0, w_red = 0;
  for (int g0 = first_tile(c, off, G); g0 < T; g0 += TG * G, ++rit) {
    float acc[TG][RW];
#pragma unroll
    for (int u = 0; u < TG; ++u)
#pragma unroll
      for (int r = 0; r < RW; ++r) acc[u][r] = 0.f;
#pragma unroll
    for (int u = 0; u < TG; ++u) {
      if (g0 + u * G >= T) break;
      const int st = it % kStages;
      const long long t0 = tw ? clk() : 0;
      if (!mbar_wait(&s.full[st], (it / kStages) & 1u, kDevTimeoutFull)) return false;
      if (tw) w_full += clk() - t0;
      const uint8_t* base =
          s.ring + (size_t)st * kStageBytes + (size_t)(wk * 128 + lane * 4) * 2 + (size_t)(wr * RW) * rowbytes;
#pragma unroll
      for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const uint2 wv = *reinterpret_cast<const uint2*>(base + (size_t)r * rowbytes + (size_t)j * WK * 256);
          const float2 w01 = __half22float2(*reinterpret_cast<const __half2*>(&wv.x));
          const float2 w23 = __half22float2(*reinterpret_cast<const __half2*>(&wv.y));
          float a = acc[u][r];
          a = fmaf(w01.x, xr[j][0], a);
          a = fmaf(w01.y, xr[j][1], a);
          a = fmaf(w23.x, xr[j][2], a);
          a = fmaf(w23.y, xr[j][3], a);
          acc[u][r] = a;
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[st]);
      ++it;
    }
    float v[P];
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] = i < RW * TG ? acc[i / RW][i % RW] : 0.f;
    const float rv = gemv::transpose_reduce<P>(v, lane);
    const int rs = rit % kRedSlots;
    const long long t1 = tw ? clk() : 0;
    if (!mbar_wait(&s.rempty[rs], ((rit / kRedSlots) & 1u) ^ 1u, kDevTimeoutRed)) return false;
    if (tw) w_red += clk() - t1;
    if (writer) s.red[(rs * kCW + cw) * kMaxVals + my_idx] = rv;
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.rfull[rs]);
  }
  trace_val(p, c, f, kl, 4, p.n_layers, cw * 32 + lane, (unsigned long long)w_full);
  trace_val(p, c, f, kl, 5, p.n_layers, cw * 32 + lane, (unsigned long long)w_red);
  return true;
}

// ---------------------------------------------------------------- epilogue GEMV phase
// EPI: gemv::kQkv (rows -> q / K / V with RoPE), kResid (y += ), kSwiglu (g = silu(a)*b)
// kPeer (tensor parallelism): the tile's rows are this rank's partial of an
// all-reduce; they are stored into every rank's receive buffer (slot `rank` of
// parity `par`) and summed by the next phase's prologue.
constexpr int kPeer = 100;
template <int R, int EPI, int TG, int WK = kCW, int N = 1>
__device__ __forceinline__ bool epilogue(const StepParams& p, Smem& s, uint32_t& rit, float* y, int rows, int T,
                                         int off, int c, int G, int lane, int layer, int pos, int f, int kl,
                                         unsigned long long ar_k = 0) {
  const bool tw = p.trace && f < kTraceFrames;
  long long w_red = 0;
  using TD = Tp<N>;
  constexpr int ORT = EPI == gemv::kSwiglu ? R / 2 : R;
  constexpr int RW = R / (kCW / WK);
  for (int g0 = first_tile(c, off, G); g0 < T; g0 += TG * G, ++rit) {
    const int rs = rit % kRedSlots;
    // lane -> (tile u of the group, row r of the tile)
    const int u = lane / R, r = lane % R;
    const int t = g0 + u * G;
    const bool live = lane < R * TG && t < T;
    float yold = 0.f;   // residual row loaded before the wait so its latency overlaps it
    if constexpr (EPI == gemv::kResid) {
      const int row = t * ORT + r;
      if (live && row < rows) yold = y[row];
    }
    const long long t0 = tw ? clk() : 0;
    if (!mbar_wait(&s.rfull[rs], (rit / kRedSlots) & 1u, kDevTimeoutRed)) return false;
    if (tw) w_red += clk() - t0;
    float val = 0.f;
    if (lane < R * TG) {
      // row r of tile u: written by the WK warps of row group r / RW at index u*RW + r%RW
      const int wr = r / RW, idx = u * RW + r % RW;
#pragma unroll
      for (int k = 0; k < WK; ++k) val += s.red[(rs * kCW + wr * WK + k) * kMaxVals + idx];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.rempty[rs]);
    if constexpr (EPI == kPeer) {
      const int row = t * R + r;
      if (live && row < rows)
#pragma unroll
        for (int q = 0; q < N; ++q)
          st_tagged(p.peer_recv[q] + ((long long)(ar_k & 1) * N + p.rank) * D + row, val, (uint32_t)(ar_k + 1));
    } else if constexpr (EPI == gemv::kResid) {
      const int row = t * ORT + r;
      if (live && row < rows) y[row] = yold + val;
    } else if constexpr (EPI == gemv::kSwiglu) {
      const float up = __shfl_down_sync(0xffffffffu, val, ORT);
      const int row = t * ORT + r;
      if (live && r < ORT && row < rows) y[row] = swiglu(val, up);
    } else {
      const float other = __shfl_xor_sync(0xffffffffu, val, 1);
      const int row = t * R + r;
      if (live && row < rows) {
        float out = val;
        if (row < TD::QD + TD::KVD) {
          const float ang = (float)pos * p.rope_freq[(row & 127) >> 1];
          float sn, cs;
          sincosf(ang, &sn, &cs);
          const bool even = (row & 1) == 0;
          const float x0 = even ? val : other, x1 = even ? other : val;
          out = even ? __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn)) : __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
        const uint32_t tag = (uint32_t)(ar_k + 1);
        if (row < TD::QD) {
          if (p.qkv_t) st_tagged(p.qkv_t + row, out, tag);
          else p.q[row] = out;
        } else {
          const int kvr = row - TD::QD;
          const int kv = kvr >= TD::KVD ? 1 : 0;
          const int rr = kvr - kv * TD::KVD;
          const int lp = pos / p.kv.page_size;
          if (lp >= p.kv.max_pages) {
            set_error(kDevBadIndex);
          } else {
            const int page = p.kv.page_table[(long long)p.slot * p.kv.max_pages + lp];
            const long long prow = gemv::kv_row(p.kv, page, layer, kv, rr >> 7, pos % p.kv.page_size);
            const __half hv = __float2half_rn(out);
            p.kv.pool[prow * HD + (rr & 127)] = hv;
            if (p.qkv_t) st_tagged(p.qkv_t + row, __half2float(hv), tag);
          }
        }
      }
    }
  }
  trace_val(p, c, f, kl, 6, p.n_layers, lane, (unsigned long long)w_red);
  grid_arrive_warp<N>(p, lane, EPI == gemv::kQkv);
  return true;
}

// ---------------------------------------------------------------- attention phase
// Split-KV flash decode over the pages of (kv head, split) items dealt to this CTA.
// 8 warps: warps 0-3 take page 2i of a pair, warps 4-7 page 2i+1, 16 positions each.
// Split plan of a step: splits of >= 2 pages (one TMA pair), at most p.n_splits per KV
// head; n_used splits hold positions.  Partials live at
// part[((kvh * p.n_splits + split) * GQA + head) * kPartStride] = {max, sum, -, -, o[128]}.
constexpr int PS = attn::kPartStride;
constexpr int kMaxUsed = 9;   // splits per KV head: the last split merges them in one load round
__device__ __forceinline__ void split_plan(const StepParams& p, int pos, int& npages, int& pps, int& n_used) {
  npages = (pos + 1 + 63) / 64;
  const int cap = min(p.n_splits, kMaxUsed);
  pps = max(2, (npages + cap - 1) / cap);
  n_used = (npages + pps - 1) / pps;
}

// TMA of K/V pages [pp, pp+npair) of one KV head into the attention buffer (thread 0).
__device__ __forceinline__ void issue_pair(const StepParams& p, const CUtensorMap* kvmap, Smem& s, int layer, int kvh,
                                           int pp, int npair) {
  const int32_t* ptab = p.kv.page_table + (long long)p.slot * p.kv.max_pages;
  mbar_arrive_expect_tx(s.afull, (uint32_t)npair * 32768u);
  for (int k = 0; k < npair; ++k) {
    const int phys = ptab[pp + k];
    const int krow = (int)gemv::kv_row(p.kv, phys, layer, 0, kvh, 0);
    const int vrow = (int)gemv::kv_row(p.kv, phys, layer, 1, kvh, 0);
    uint8_t* dst = s.attn + k * 32768;
    tma_load_2d(dst, kvmap, 0, krow, s.afull);
    tma_load_2d(dst + 8192, kvmap, 64, krow, s.afull);
    tma_load_2d(dst + 16384, kvmap, 0, vrow, s.afull);
    tma_load_2d(dst + 24576, kvmap, 64, vrow, s.afull);
  }
}
// Called by the consumers at the start of the QKV phase.  With p.early_kv, thread 0
// copies the first K/V pair of this CTA's first attention item into the attention
// buffer, so that the copy runs under the QKV phase instead of after the barrier that
// ends it; the row of `pos` in that pair is stale (this phase writes it) and the
// attention phase patches it in shared memory from the KV pool.  The other pages of
// this CTA's items are prefetched into L2, so that their TMA loads hit L2.  Returns
// whether the first pair was issued early (the same value on every thread).
template <int N>
__device__ __forceinline__ bool preload_kv(const StepParams& p, const CUtensorMap* kvmap, Smem& s, int layer, int pos,
                                           int c, int G, int ctid, uint32_t ait, bool& a_pending, uint32_t& a_par) {
  int npages, pps, n_used;
  split_plan(p, pos, npages, pps, n_used);
  const bool pre = p.early_kv && c < Tp<N>::NKV * p.n_splits && c % p.n_splits < n_used;
  if (ctid != 0) return pre;
  const int32_t* ptab = p.kv.page_table + (long long)p.slot * p.kv.max_pages;
  for (int item = c; item < Tp<N>::NKV * p.n_splits; item += G) {
    const int kvh = item / p.n_splits, split = item % p.n_splits;
    if (split >= n_used) continue;
    const int pg0 = split * pps, pg1 = min(npages, pg0 + pps);
    int pg = pg0;
    if (item == c && pre) {
      const int npair = min(2, pg1 - pg0);
      if (!error_set()) {
        a_pending = true;
        a_par = ait & 1u;
        issue_pair(p, kvmap, s, layer, kvh, pg0, npair);
      }
      pg += npair;
    }
    for (; pg < pg1; ++pg) {
      const int phys = ptab[pg];
      prefetch_l2(p.kv.pool + gemv::kv_row(p.kv, phys, layer, 0, kvh, 0) * HD, 64u * HD * 2u);
      prefetch_l2(p.kv.pool + gemv::kv_row(p.kv, phys, layer, 1, kvh, 0) * HD, 64u * HD * 2u);
    }
  }
  return pre;
}

// Value pair of two consecutive tagged words, once both carry `tag` (bounded poll).
__device__ __forceinline__ float2 tagged_pair(ulonglong2 w, const unsigned long long* p, uint32_t tag, uint32_t limit) {
  const float x = (uint32_t)(w.x >> 32) == tag ? __uint_as_float((uint32_t)w.x) : wait_tagged(p, tag, limit);
  const float y = (uint32_t)(w.y >> 32) == tag ? __uint_as_float((uint32_t)w.y) : wait_tagged(p + 1, tag, limit);
  return make_float2(x, y);
}

// Control flow is uniform across the 256 consumer threads (every named barrier is
// reached by all of them); after a device error the work is skipped, not the barriers.
// TQ (the AR kernels): no grid barrier before this phase; q and the current position's
// K / V rows arrive as tagged words from the QKV epilogues (p.qkv_t, tag `tag`), so an
// item starts as soon as the words of its KV head have landed.  !TQ: q from p.q after
// the QKV barrier.  Either way the splits' partials go to p.part, the last split to
// take a ticket merges them into p.att, and the phase ends at a grid barrier.
template <int N, bool TQ>
__device__ __forceinline__ void attention(const StepParams& p, const CUtensorMap* kvmap, Smem& s, uint32_t& ait,
                                          bool& a_pending, uint32_t& a_par, bool pre, int layer, int pos, int c,
                                          int G, int cw, int lane, int ctid, int f, int kl, uint32_t tag) {
  using TD = Tp<N>;
  const int seq = pos + 1;
  int npages, pps, n_used;
  split_plan(p, pos, npages, pps, n_used);
  const int32_t* ptab = p.kv.page_table + (long long)p.slot * p.kv.max_pages;
  const uint32_t limit = p.wait_limit ? p.wait_limit : kTagPolls;
  const float scale = 0.08838834764831845f;   // 1/sqrt(128) rounded to f32
  // mma operands: query columns n = 2 head + (0: f16 part, 1: f16 remainder), 8 per KV
  // head; this lane supplies query column lane / 4 and holds head lane % 4's results
  const int qn = lane >> 2, hd = lane & 3;
  const int half_pair = cw >> 2, grp = cw & 3;
  for (int item = c; item < TD::NKV * p.n_splits; item += G) {
    const int kvh = item / p.n_splits, split = item % p.n_splits;
    if (split >= n_used) continue;   // uniform: no positions in this split
    const int pg0 = split * pps, pg1 = min(npages, pg0 + pps);
    float m_run = -INFINITY, l_run = 0.f;
    float ot[8][4];   // O^T: 8 tiles of 16 dims x 8 query columns
    uint32_t qb0[8], qb1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ot[i][0] = ot[i][1] = ot[i][2] = ot[i][3] = 0.f;
    for (int pp = pg0; pp < pg1; pp += 2) {
      const int npair = min(2, pg1 - pp);
      const bool go = !error_set();
      const bool early = pre && item == c && pp == pg0;   // issued by preload_kv
      if (ctid == 0 && go && !early) {
        a_pending = true;
        a_par = ait & 1u;
        issue_pair(p, kvmap, s, layer, kvh, pp, npair);
      }
      // The pair holding position pos may hold a stale copy of its row: copied before
      // the QKV phase wrote it (early pair; TAG: any pair, as no barrier precedes this
      // phase).  The row is stored over it after the copy lands: TAG from the tagged
      // words (f16-rounded values), else from the KV pool.
      const int lp = pos >> 6;
      const bool patch = (TQ || early) && lp >= pp && lp < pp + npair;
      uint4 nrow = make_uint4(0u, 0u, 0u, 0u);
      ulonglong2 trow = make_ulonglong2(0ull, 0ull);
      const unsigned long long* trow_p =
          TQ ? p.qkv_t + TD::QD + (ctid >> 6) * TD::KVD + kvh * HD + (ctid & 63) * 2 : nullptr;
      if constexpr (TQ) {
        if (patch && go && ctid < 128) trow = ld_tagged2(trow_p);
      } else {
        if (patch && go && ctid < 32)
          nrow = __ldcg(reinterpret_cast<const uint4*>(
                            p.kv.pool + gemv::kv_row(p.kv, ptab[lp], layer, ctid >> 4, kvh, pos & 63) * HD) +
                        (ctid & 15));
      }
      if (pp == pg0) {
        // Q^T fragments (the B operand of S^T = K Q^T) for the 4 heads of this KV head,
        // loaded while the first K/V pair is in flight
        float qv[8][4];
        if constexpr (TQ) {
          // the 512 words of q of this KV head: two per thread, staged in shared memory
          float* qs = s.scratch + 256;
          const unsigned long long* qt = p.qkv_t + (long long)kvh * GQA * HD + ctid * 2;
          const float2 v = go ? tagged_pair(ld_tagged2(qt), qt, tag, limit) : make_float2(0.f, 0.f);
          qs[ctid * 2] = v.x;
          qs[ctid * 2 + 1] = v.y;
          named_bar_sync(1, kCW * 32);
          const float* qh = qs + (qn >> 1) * HD;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int cc = kk * 16 + (lane & 3) * 2;
            qv[kk][0] = qh[cc]; qv[kk][1] = qh[cc + 1]; qv[kk][2] = qh[cc + 8]; qv[kk][3] = qh[cc + 9];
          }
        } else {
          const float* qh = p.q + (long long)(kvh * GQA + (qn >> 1)) * HD;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int cc = kk * 16 + (lane & 3) * 2;
            qv[kk][0] = qh[cc]; qv[kk][1] = qh[cc + 1]; qv[kk][2] = qh[cc + 8]; qv[kk][3] = qh[cc + 9];
          }
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          float v0 = qv[kk][0], v1 = qv[kk][1], v8 = qv[kk][2], v9 = qv[kk][3];
          if (qn & 1) {
            v0 -= __half2float(__float2half_rn(v0)); v1 -= __half2float(__float2half_rn(v1));
            v8 -= __half2float(__float2half_rn(v8)); v9 -= __half2float(__float2half_rn(v9));
          }
          qb0[kk] = pack_half2(v0, v1);
          qb1[kk] = pack_half2(v8, v9);
        }
      }
      const bool w_ok = go && mbar_wait(s.afull, ait & 1u, kDevTimeoutFull);
      if (w_ok && ctid == 0) a_pending = false;
      ++ait;
      if (item == c && pp == pg0) trace_mark(p, c, f, kl, 4, p.n_layers, ctid);
      if (patch) {
        if constexpr (TQ) {
          if (w_ok && ctid < 128) {
            const float2 v = tagged_pair(trow, trow_p, tag, limit);
            const int col = (ctid & 63) * 2;
            *reinterpret_cast<__half2*>(s.attn + (lp - pp) * 32768 + (ctid >> 6) * 16384 + attn::swz(pos & 63, col) +
                                        (col & 7) * 2) = __floats2half2_rn(v.x, v.y);
            fence_proxy_async_shared();   // the next TMA into this buffer is ordered after the store
          }
        } else {
          if (w_ok && ctid < 32) {
            *reinterpret_cast<uint4*>(s.attn + (lp - pp) * 32768 + (ctid >> 4) * 16384 +
                                      attn::swz(pos & 63, (ctid & 15) * 8)) = nrow;
            fence_proxy_async_shared();
          }
        }
        named_bar_sync(1, kCW * 32);
      }
      if (w_ok && half_pair < npair) {
        const int pg = pp + half_pair;
        const uint32_t kbase = smem_u32(s.attn + half_pair * 32768);
        const uint32_t vbase = kbase + 16384;
        const int mat = lane >> 3, r8 = lane & 7;
        // S^T = K Q^T over the warp's 16 positions (rows) and the 8 query columns
        float st[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(a0, a1, a2, a3, kbase + attn::swz(grp * 16 + (mat & 1) * 8 + r8, kk * 16 + (mat >> 1) * 8));
          mma_16816(st, a0, a1, a2, a3, qb0[kk], qb1[kk]);
        }
        // head hd at positions p0 and p0 + 8: the two query columns of the head summed
        const int p0 = pg * 64 + grp * 16 + qn;
        const float s0 = p0 < seq ? (st[0] + st[1]) * scale : -INFINITY;
        const float s1 = p0 + 8 < seq ? (st[2] + st[3]) * scale : -INFINITY;
        float mloc = fmaxf(s0, s1);
        mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 4));
        mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 8));
        mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 16));
        const float m_new = fmaxf(m_run, mloc);
        const float corr = (m_new == -INFINITY) ? 1.f : expf(m_run - m_new);
        const float e0 = s0 == -INFINITY ? 0.f : expf(s0 - m_new);
        const float e1 = s1 == -INFINITY ? 0.f : expf(s1 - m_new);
        l_run = l_run * corr + (e0 + e1);
        m_run = m_new;
        // P^T (the B operand of O^T += V^T P^T): (f16 part, remainder) pairs in S^T's
        // layout, each 8x8 tile transposed in registers
        const uint32_t pb0 = movmatrix_trans(pack_half2(e0, e0 - __half2float(__float2half_rn(e0))));
        const uint32_t pb1 = movmatrix_trans(pack_half2(e1, e1 - __half2float(__float2half_rn(e1))));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          ot[i][0] *= corr; ot[i][1] *= corr; ot[i][2] *= corr; ot[i][3] *= corr;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(a0, a1, a2, a3, vbase + attn::swz(grp * 16 + (mat >> 1) * 8 + r8, i * 16 + (mat & 1) * 8));
          mma_16816(ot[i], a0, a1, a2, a3, pb0, pb1);
        }
      }
      named_bar_sync(1, kCW * 32);   // the pair buffer is free again
    }
    // merge the 8 warps (reuse the pair buffer as scratch): l over the head's 8 lanes
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 4);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 8);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 16);
    float* ws = reinterpret_cast<float*>(s.attn);     // [8 warps][4 heads][130]
    {
      float* w = ws + (cw * GQA + hd) * attn::kPartStride;
      if (lane < 4) { w[0] = m_run; w[1] = l_run; }
#pragma unroll
      for (int i = 0; i < 8; ++i) {   // f16 part + remainder columns of head hd
        w[2 + i * 16 + qn] = ot[i][0] + ot[i][1];
        w[2 + i * 16 + qn + 8] = ot[i][2] + ot[i][3];
      }
      fence_proxy_async_shared();   // scratch in the pair buffer, which TMA overwrites next
    }
    named_bar_sync(1, kCW * 32);
    float* part = p.part + ((long long)kvh * p.n_splits + split) * (GQA * PS);
    for (int idx = ctid; idx < GQA * HD; idx += kCW * 32) {
      const int h = idx / HD, d = idx % HD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kCW; ++w) M = fmaxf(M, ws[(w * GQA + h) * attn::kPartStride]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kCW; ++w) {
          const float* ww = ws + (w * GQA + h) * attn::kPartStride;
          const float fw = ww[0] == -INFINITY ? 0.f : expf(ww[0] - M);
          L += ww[1] * fw;
          O += ww[2 + d] * fw;
        }
      }
      part[h * PS + 4 + d] = O;
      if (d == 0) { part[h * PS] = M; part[h * PS + 1] = L; }
    }
    named_bar_sync(1, kCW * 32);
    if (item == c) trace_mark(p, c, f, kl, 5, p.n_layers, ctid);
    // The last split of this KV head to finish merges all n_used splits into att.
    // Each thread owns 2 output dims of one head and issues all its loads at once.
    int* s_flag = reinterpret_cast<int*>(s.scratch + 1020);
    if (ctid == 0) *s_flag = (atom_add_acq_rel(&p.tickets[kvh], 1) == n_used - 1);
    named_bar_sync(1, kCW * 32);
    if (item == c) trace_mark(p, c, f, kl, 6, p.n_layers, ctid);
    if (*s_flag) {
      const int h = ctid >> 6, d0 = (ctid & 63) * 2;
      const float* base = p.part + ((long long)kvh * p.n_splits * GQA + h) * PS;
      float mm[kMaxUsed], ll[kMaxUsed];
      float2 oo[kMaxUsed];
#pragma unroll
      for (int sp = 0; sp < kMaxUsed; ++sp) {
        if (sp < n_used) {
          const float* b = base + (long long)sp * GQA * PS;
          mm[sp] = __ldcg(b);
          ll[sp] = __ldcg(b + 1);
          oo[sp] = __ldcg(reinterpret_cast<const float2*>(b + 4 + d0));
        } else {
          mm[sp] = -INFINITY; ll[sp] = 0.f; oo[sp] = make_float2(0.f, 0.f);
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int sp = 0; sp < kMaxUsed; ++sp) M = fmaxf(M, mm[sp]);
      float L = 0.f, a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int sp = 0; sp < kMaxUsed; ++sp) {
        const float w = mm[sp] == -INFINITY ? 0.f : expf(mm[sp] - M);
        L += ll[sp] * w;
        a0 += w * oo[sp].x;
        a1 += w * oo[sp].y;
      }
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      *reinterpret_cast<float2*>(p.att + (kvh * GQA + h) * HD + d0) = make_float2(a0 * inv, a1 * inv);
      if (ctid == 0) p.tickets[kvh] = 0;
    }
    named_bar_sync(1, kCW * 32);
  }
}

// ---------------------------------------------------------------- embedding / final norm slices
__device__ __forceinline__ int embed_source(const StepParams& p, int mode, int token, int pos, int frame,
                                            uint32_t* codes, int& row) {
  SlotState& st = p.slots[p.slot];
  switch (mode) {
    case kEmbToken: row = token; return (row >= 0 && row < p.vocab) ? 0 : -1;
    case kEmbAudioToken: row = token; return (row >= 0 && row < p.audio_rows) ? 1 : -1;
    case kEmbRow: return 2;
    case kEmbCodes:
      for (int k = 0; k < 37; ++k) codes[k] = st.codes[k];
      break;
    case kEmbSynthCodes: {
      const uint64_t base = 37ull * (uint64_t)(frame - 1);
      codes[0] = 2u + (uint32_t)(vx_bits(st.codes_key, base) % 8192ull);
      for (int k = 0; k < kNumAc; ++k) codes[1 + k] = 2u + (uint32_t)(vx_bits(st.codes_key, base + 1 + k) % 21ull);
      break;
    }
    case kEmbPrompt: {
      if (pos < 0 || pos >= p.max_seq || pos >= st.prompt_len) return -1;
      const int t = p.prompt[(long long)p.slot * p.max_seq + pos];
      if (t < 0) { row = -t - 1; return row < p.max_voice ? 4 : -1; }
      row = t;
      return row < p.vocab ? 0 : -1;
    }
    default: return -1;
  }
  bool ok = codes[0] < (uint32_t)p.audio_rows;
  for (int k = 0; k < kNumAc; ++k) ok = ok && (kAcBase + kAcStride * k + (int)codes[1 + k] < p.audio_rows);
  return ok ? 3 : -1;
}

// ---------------------------------------------------------------- the kernel
// AR: the residual stream is handed from the o_proj / down epilogues to the next phase
// as tagged words (the all-reduce protocol above; with N = 1 a one-source all-reduce),
// so the phase after each residual update starts without a grid barrier.  !AR (N = 1
// only): the epilogues add into h and the next phase waits at a grid barrier.
template <int N, bool AR>
__global__ void __launch_bounds__(kThreads, 1) k_decode_steps(const __grid_constant__ CUtensorMap kvmap,
                                                              const __grid_constant__ StepParams p) {
  static_assert(AR || N == 1, "tensor parallelism hands the residual over as tagged words");
  using TD = Tp<N>;
  extern __shared__ uint8_t smem_raw[];
  Smem s = smem_map(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x, G = gridDim.x;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) { mbar_init(&s.full[i], 1); mbar_init(&s.empty[i], kCW); }
    for (int i = 0; i < kRedSlots; ++i) { mbar_init(&s.rfull[i], kCW); mbar_init(&s.rempty[i], 1); }
    mbar_init(s.afull, 1);
    fence_mbar_init();
    prefetch_tmap(&kvmap);
  }
  __syncthreads();
  const int pos0 = p.slots[p.slot].pos;
  const int frame0 = p.slots[p.slot].frame;
  const int L = p.n_layers;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t it = 0;
      Cursor cur, ahead;
      cursor_start<N>(p, cur, c, G, L);
      cursor_start<N>(p, ahead, c, G, L);
      int dist = 0;   // tiles the L2 lookahead runs ahead of the ring
      for (; dist < p.prefetch_ahead && ahead.f < p.n_frames; ++dist) {
        const __half *a, *b; uint32_t bytes; int ort;
        tile_src<N>(p, ahead, a, b, bytes, ort);
        prefetch_l2(a, bytes);
        if (b) prefetch_l2(b, bytes);
        cursor_next<N>(p, ahead, c, G, L);
      }
      while (cur.f < p.n_frames) {
        const int st = it % kStages;
        if (!mbar_wait(&s.empty[st], ((it / kStages) & 1u) ^ 1u, kDevTimeoutEmpty)) break;
        const __half *a, *b; uint32_t bytes; int ort;
        tile_src<N>(p, cur, a, b, bytes, ort);
        mbar_arrive_expect_tx(&s.full[st], bytes * (b ? 2u : 1u));
        uint8_t* dst = s.ring + (size_t)st * kStageBytes;
        bulk_g2s(dst, a, bytes, &s.full[st], pol);
        if (b) bulk_g2s(dst + (size_t)ort * D * 2, b, bytes, &s.full[st], pol);   // SwiGLU up rows after the gate rows
        ++it;
        cursor_next<N>(p, cur, c, G, L);
        if (dist > 0) --dist;
        while (dist < p.prefetch_ahead && ahead.f < p.n_frames) {
          tile_src<N>(p, ahead, a, b, bytes, ort);
          prefetch_l2(a, bytes);
          if (b) prefetch_l2(b, bytes);
          cursor_next<N>(p, ahead, c, G, L);
          ++dist;
        }
      }
      // drain the copies still in flight
      const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0u;
      for (uint32_t i = first; i < it; ++i)
        if (!mbar_wait_drain(&s.full[i % kStages], (i / kStages) & 1u)) break;
    }
    return;
  }

  uint32_t rit = 0;
  if (warp == kCW + 1) {
    // ------------------------------------------------------------ epilogue warp
    long long tiles_before = 0;
    for (int f = 0; f < p.n_frames; ++f) {
      const int pos = pos0 + f;
      const unsigned long long kf = p.ar_base + 2ull * L * f;   // all-reduce index of layer 0's o_proj
      for (int l = 0; l < L; ++l) {
        const int o0 = (int)(tiles_before % G);
        const int o1 = (int)((tiles_before + TD::TQKV) % G);
        const int o2 = (int)((tiles_before + TD::TQKV + TD::TO) % G);
        const int o3 = (int)((tiles_before + TD::TQKV + TD::TO + TD::TW13) % G);
        const int kl = 1 + 5 * l;
        const unsigned long long k_o = kf + 2 * l, k_w2 = kf + 2 * l + 1;
        if (!epilogue<6, gemv::kQkv, kTgQKV, kCW, N>(p, s, rit, nullptr, TD::QKVD, TD::TQKV, o0, c, G, lane, l, pos, f, kl,
                                                     k_o))
          return;
        trace_mark(p, c, f, kl, 2, L, lane);
        if constexpr (!AR) {
          if (!epilogue<4, gemv::kResid, kTgO>(p, s, rit, p.h, D, TD::TO, o1, c, G, lane, l, pos, f, kl + 2)) return;
        } else {
          if (!epilogue<TD::RO, kPeer, 1, TD::WKO, N>(p, s, rit, nullptr, D, TD::TO, o1, c, G, lane, l, pos, f, kl + 2, k_o))
            return;
        }
        trace_mark(p, c, f, kl + 2, 2, L, lane);
        if (!epilogue<6, gemv::kSwiglu, kTgW13, kCW, N>(p, s, rit, p.g, TD::F, TD::TW13, o2, c, G, lane, l, pos, f, kl + 3)) return;
        trace_mark(p, c, f, kl + 3, 2, L, lane);
        if constexpr (!AR) {
          if (!epilogue<2, gemv::kResid, kTgW2>(p, s, rit, p.h, D, TD::TW2, o3, c, G, lane, l, pos, f, kl + 4)) return;
        } else {
          if (!epilogue<TD::RW2, kPeer, 1, TD::WKW2, N>(p, s, rit, nullptr, D, TD::TW2, o3, c, G, lane, l, pos, f, kl + 4, k_w2))
            return;
        }
        trace_mark(p, c, f, kl + 4, 2, L, lane);
        tiles_before += TD::TLayer;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers (warps 1-8)
  const int cw = warp - 1, ctid = threadIdx.x - 32;
  uint32_t it = 0, ait = 0;
  unsigned phase = 0;                     // CTA-phase arrivals required before the next phase
  long long tiles_before = 0;
  const int per = (D + G - 1) / G;        // embedding / norm slice of this CTA
  const int e0 = c * per, e1 = min(D, e0 + per);
  uint32_t* codes = reinterpret_cast<uint32_t*>(s.scratch + 768);
  bool a_pending = false;   // an attention TMA pair is in flight (thread 0) ...
  uint32_t a_par = 0;       // ... and the parity of its completion on s.afull
  // tensor parallelism: the residual alternates between p.h and p.h2 per all-reduce
  // (all-reduce k reads h[k & 1] and its parity k & 1 of the receive buffer, writes
  // h[(k + 1) & 1]); every launch starts at an even all-reduce index, so EMBED
  // writes p.h and the last all-reduce of a launch leaves the residual in p.h.
  float* const hb[2] = {p.h, AR ? p.h2 : p.h};
  auto ar_in = [&](unsigned long long k) {
    return ArIn{hb[k & 1], p.recv + (long long)(k & 1) * N * D, hb[(k + 1) & 1], (uint32_t)(k + 1),
                p.hx + (long long)(k & 1) * D, e0, e1, p.wait_limit ? p.wait_limit : kTagPolls};
  };
  for (int f = 0; f < p.n_frames; ++f) {
    const int pos = pos0 + f, frame = frame0 + f;
    const unsigned long long kf = p.ar_base + 2ull * L * f;
    const bool rec = p.dbg && f == p.dbg_frame;   // per-layer record of this step
    // ---- EMBED
    grid_wait<N>(p, phase * G, ctid);
    trace_mark(p, c, f, 0, 0, L, ctid);
    {
      int row = 0, kind = -1;
      __shared__ int s_kind, s_row;
      if (ctid == 0) {
        kind = embed_source(p, f == 0 ? p.mode0 : p.mode_next, p.token0, pos, frame, codes, row);
        if (kind < 0) set_error(kDevBadIndex);
        s_kind = kind;
        s_row = row;
        if (kind == 3 && c == 0 && p.inc_frame && frame >= 1 && frame - 1 < p.slots[p.slot].max_frames &&
            (f == 0 ? p.mode0 : p.mode_next) == kEmbSynthCodes)
          for (int k = 0; k < 37; ++k)
            p.code_ring[((long long)p.slot * p.slots[p.slot].max_frames + frame - 1) * 37 + k] = codes[k];
      }
      named_bar_sync(1, kCW * 32);
      kind = s_kind;
      row = s_row;
      for (int i = e0 + ctid; i < e1; i += kCW * 32) {
        float v = 0.f;
        if (kind == 0) v = __half2float(p.tok[(long long)row * D + i]);
        else if (kind == 1) v = __half2float(p.audio[(long long)row * D + i]);
        else if (kind == 2) v = p.rows_in[(long long)p.slot * D + i];
        else if (kind == 4) v = p.voice[((long long)p.slot * p.max_voice + row) * D + i];
        else if (kind == 3) {
          // all 37 rows loaded first (one memory round trip), summed in the reference's order
          __half r[37];
          r[0] = p.audio[(long long)codes[0] * D + i];
#pragma unroll
          for (int k = 0; k < kNumAc; ++k) r[1 + k] = p.audio[(long long)(kAcBase + kAcStride * k + codes[1 + k]) * D + i];
          float a = 0.f;
#pragma unroll
          for (int k = 0; k < 37; ++k) a += __half2float(r[k]);
          v = a;
        }
        p.h[i] = v;
        if (rec) p.dbg[i] = v;
      }
      named_bar_sync(1, kCW * 32);
      if (ctid == 0) red_release_add(p.bar, 1u);
      ++phase;
    }
    for (int l = 0; l < L; ++l) {
      const LayerPtrs& W = p.layers[l];
      const int o0 = (int)(tiles_before % G);
      const int o1 = (int)((tiles_before + TD::TQKV) % G);
      const int o2 = (int)((tiles_before + TD::TQKV + TD::TO) % G);
      const int o3 = (int)((tiles_before + TD::TQKV + TD::TO + TD::TW13) % G);
      const int kl = 1 + 5 * l;
      const unsigned long long k_o = kf + 2 * l, k_prev = kf + 2 * l - 1;   // k_prev: layer l-1's down
      // ---- QKV (+ RoPE + KV append in the epilogue warp); TP: h = all-reduce of layer l-1's down
      const bool ar_qkv = AR && l > 0;
      grid_wait<N>(p, phase * G, ctid, ar_qkv);
      trace_mark(p, c, f, kl, 0, L, ctid);
      const bool kv_pre = preload_kv<N>(p, &kvmap, s, l, pos, c, G, ctid, ait, a_pending, a_par);
      {
        const ArIn a = ar_qkv ? ar_in(k_prev) : ArIn{};
        consume<6, 3, true, kTgQKV, kCW, N>(p, s, it, rit, hb[0], W.attn_norm, D, TD::TQKV, o0, c, G, cw, lane, pos, f,
                                            kl, ar_qkv ? &a : nullptr, 4 * l);
      }
      trace_mark(p, c, f, kl, 1, L, ctid);
      ++phase;
      // ---- attention (AR: its inputs arrive as tagged words, no grid barrier before it)
      if constexpr (!AR) grid_wait<N>(p, phase * G, ctid);
      trace_mark(p, c, f, kl + 1, 0, L, ctid);
      attention<N, AR>(p, &kvmap, s, ait, a_pending, a_par, kv_pre, l, pos, c, G, cw, lane, ctid, f, kl + 1,
                       (uint32_t)(k_o + 1));
      trace_mark(p, c, f, kl + 1, 1, L, ctid);
      if (ctid == 0) red_release_add(p.bar, 1u);
      ++phase;
      // ---- o_proj + residual (TP: partial rows to every rank)
      grid_wait<N>(p, phase * G, ctid);
      trace_mark(p, c, f, kl + 2, 0, L, ctid);
      consume<TD::RO, TD::CPLO, false, kTgO, TD::WKO, N>(p, s, it, rit, p.att, nullptr, TD::QD, TD::TO, o1, c, G, cw,
                                                         lane, pos, f, kl + 2);
      trace_mark(p, c, f, kl + 2, 1, L, ctid);
      ++phase;
      // ---- gate/up + SwiGLU; TP: h = all-reduce of o_proj
      grid_wait<N>(p, phase * G, ctid, AR);
      trace_mark(p, c, f, kl + 3, 0, L, ctid);
      {
        const ArIn a = AR ? ar_in(k_o) : ArIn{};
        consume<6, 3, true, kTgW13, kCW, N>(p, s, it, rit, hb[0], W.ffn_norm, D, TD::TW13, o2, c, G, cw, lane, pos, f,
                                            kl + 3, AR ? &a : nullptr, 4 * l + 2);
      }
      trace_mark(p, c, f, kl + 3, 1, L, ctid);
      ++phase;
      // ---- down + residual (TP: partial rows to every rank)
      grid_wait<N>(p, phase * G, ctid);
      trace_mark(p, c, f, kl + 4, 0, L, ctid);
      consume<TD::RW2, TD::CPLW2, false, kTgW2, TD::WKW2, N>(p, s, it, rit, p.g, nullptr, TD::F, TD::TW2, o3, c, G, cw,
                                                             lane, pos, f, kl + 4);
      trace_mark(p, c, f, kl + 4, 1, L, ctid);
      ++phase;
      tiles_before += TD::TLayer;
    }
    // ---- FINAL norm (each CTA: full sum of squares, its slice of the output);
    // TP: h = all-reduce of the last layer's down (CTA 0 stores it to p.h)
    const unsigned long long k_last = kf + 2ull * L - 1;
    grid_wait<N>(p, phase * G, ctid, AR);
    trace_mark(p, c, f, 1 + 5 * L, 0, L, ctid);
    {
      const ArIn fa = AR ? ar_in(k_last) : ArIn{};
      // TP, two stages: stage A leaves this CTA's slice in fa.h_new (= p.h), written by
      // the same threads that read it back in the slice pass below.  One stage: the
      // summed row is staged in the (idle) attention buffer for the slice pass.
      float* hs = reinterpret_cast<float*>(s.attn);
      auto hval = [&](int i) -> float { return !AR ? p.h[i] : kArTwoStage<N> ? fa.h_new[i] : hs[i]; };
      float ss = 0.f;
      if constexpr (!AR) {
        for (int i = ctid; i < D; i += kCW * 32) ss += p.h[i] * p.h[i];
      } else {
        constexpr int U = D / (kCW * 32 * 4);
        int cols[U];
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) cols[u] = (ctid + kCW * 32 * u) * 4;
        if constexpr (kArTwoStage<N>) {
          ar_stage_a<N>(fa, ctid);
          ar_stage_b<U>(fa, cols, v);
        } else {
#pragma unroll
          for (int u = 0; u < U; ++u) {
            v[u] = ar_sum4<N>(fa, cols[u]);
            *reinterpret_cast<float4*>(hs + cols[u]) = v[u];
            if (c == 0) *reinterpret_cast<float4*>(fa.h_new + cols[u]) = v[u];
          }
          fence_proxy_async_shared();   // hs lies in the attention buffer, which TMA overwrites next
        }
#pragma unroll
        for (int u = 0; u < U; ++u) ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
      }
      ss = warp_sum(ss);
      if (lane == 0) s.scratch[cw] = ss;
      named_bar_sync(1, kCW * 32);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) tot += s.scratch[w];
      const float rms = 1.0f / sqrtf(tot / (float)D + p.eps);
      SlotState& st = p.slots[p.slot];
      float* ring = (p.record && frame >= 0 && frame < st.max_frames)
                        ? p.normed_ring + ((long long)p.slot * st.max_frames + frame) * D : nullptr;
      for (int i = e0 + ctid; i < e1; i += kCW * 32) {
        const float hi = hval(i);
        const float v = hi * rms * __half2float(p.final_norm[i]);
        p.normed[i] = v;
        if (ring) ring[i] = v;
        if (rec) {   // last layer's ffn_out, final_norm, hidden
          p.dbg[(long long)(4 * L) * D + i] = hi;
          p.dbg[(long long)(4 * L + 1) * D + i] = v;
          p.dbg[(long long)(4 * L + 2) * D + i] = hi;
        }
      }
      named_bar_sync(1, kCW * 32);
      if (ctid == 0) red_release_add(p.bar, 1u);
      ++phase;
    }
  }
  // an attention copy left in flight by an error must land before the CTA exits
  if (ctid == 0 && a_pending) mbar_wait_drain(s.afull, a_par);
  // slot bookkeeping once every CTA has finished the last step
  if (c == 0) {
    grid_wait<N>(p, phase * G, ctid);
    if (ctid == 0 && !error_set()) {
      SlotState& st = p.slots[p.slot];
      st.pos = pos0 + p.n_frames;
      if (p.inc_frame) st.frame = frame0 + p.n_frames;
      const int lm = p.n_frames > 1 ? p.mode_next : p.mode0;
      if (lm == kEmbSynthCodes)
        for (int k = 0; k < 37; ++k) st.codes[k] = codes[k];
    }
  }
}

}  // namespace mk
}  // namespace vx
