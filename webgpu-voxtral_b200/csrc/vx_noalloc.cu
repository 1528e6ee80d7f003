// vx_noalloc.cu — LM-head argmax for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at all: a real-time audio callback cannot
// risk it (cudaMalloc may synchronise the device and block for an unbounded time),
// and a host framework that owns every byte of device memory through its own
// arena forbids libraries from allocating behind its back.  Such callers cannot
// create a vx_handle (vx_create allocates the weights, KV cache and work buffers),
// but they can hold the weight matrix and vectors in their own memory.
//
// vx_lm_head_argmax_noalloc computes argmax_r (W[r,:] . x) — the greedy token choice of
// backboneStepAndRead's tied LM head — in ONE kernel that allocates nothing.  Its
// only scratch (per-CTA partial maxima and a completion ticket) lives in the
// file-scope array below, whose device address is looked up once per device.  The
// handle-based path (vx_backbone_step with argmax_out) computes the same result with
// a 512 KB logits buffer allocated at vx_create.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "../../include/voxtral_b200.h"

namespace {

constexpr int kRowsPerBlock = 256;                  // rows of W per CTA
constexpr int kMaxBlocks = 8192;                    // CTA partials the scratch holds
constexpr int kMaxRows = kRowsPerBlock * kMaxBlocks;  // 2,097,152 rows
constexpr int kMaxDim = 16384;                      // x is staged in 64 KB of shared memory
constexpr size_t kScratchBytes = 256 + (size_t)kMaxBlocks * 8;   // ticket + partials = 65,792 B
constexpr int kMaxDevices = 64;

// Shared by every call on a device, kept until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
unsigned char* g_scratch_ptr[kMaxDevices] = {nullptr};

struct Best {
  float v;
  int i;
};
__device__ __forceinline__ Best better(Best a, Best b) {
  // maximum value, lowest index on ties (the rule of k_argmax)
  return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a;
}

__global__ void __launch_bounds__(256) k_lm_head_argmax_noalloc(const __half* __restrict__ W, const float* __restrict__ x,
                                                                 int rows, int dim, int32_t* out_idx, float* out_val,
                                                                 unsigned char* scratch) {
  extern __shared__ float xs[];
  __shared__ Best wbest[8];
  __shared__ int s_last;
  unsigned* ticket = reinterpret_cast<unsigned*>(scratch);
  Best* part = reinterpret_cast<Best*>(scratch + 256);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) xs[i] = x[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Best best{-INFINITY, 0x7fffffff};
  const int r0 = blockIdx.x * kRowsPerBlock;
  for (int r = r0 + warp; r < min(rows, r0 + kRowsPerBlock); r += 8) {
    const __half* w = W + (long long)r * dim;
    float acc = 0.f;
    for (int k = lane * 8; k < dim; k += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(w + k);
      const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h2[j]);
        acc = fmaf(f.x, xs[k + 2 * j], acc);
        acc = fmaf(f.y, xs[k + 2 * j + 1], acc);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    best = better(best, Best{acc, r});
  }
  if (lane == 0) wbest[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    Best b = wbest[0];
    for (int w = 1; w < 8; ++w) b = better(b, wbest[w]);
    part[blockIdx.x] = b;
    __threadfence();
    s_last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  // the last CTA to finish reduces every CTA's partial
  __threadfence();
  Best b{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) {
    const Best* pi = part + i;
    b = better(b, Best{__ldcg(&pi->v), __ldcg(&pi->i)});
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const Best ob{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
    b = better(b, ob);
  }
  if (lane == 0) wbest[warp] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    Best f = wbest[0];
    for (int w = 1; w < 8; ++w) f = better(f, wbest[w]);
    // NaN products never win; if every product is NaN no row was chosen: report -1
    const bool none = f.i == 0x7fffffff;
    *out_idx = none ? -1 : f.i;
    if (out_val) *out_val = none ? __int_as_float(0x7fc00000) : f.v;
  }
}

void put_err(char* err, size_t n, const char* msg) {
  if (err && n) snprintf(err, n, "%s", msg);
}

}  // namespace

extern "C" int vx_lm_head_argmax_noalloc(const uint16_t* weight, const float* x, int32_t rows, int32_t dim,
                                         int32_t* out_index, float* out_value, void* stream, char* err,
                                         size_t err_len) {
  if (!weight || !x || !out_index) {
    put_err(err, err_len, "weight, x and out_index must be device pointers");
    return VX_E_INVALID;
  }
  if (rows < 1 || rows > kMaxRows) {
    char m[160];
    snprintf(m, sizeof m, "rows %d outside [1, %d]: the static scratch holds %d CTA partials of %d rows", rows,
             kMaxRows, kMaxBlocks, kRowsPerBlock);
    put_err(err, err_len, m);
    return VX_E_RANGE;
  }
  if (dim < 8 || dim > kMaxDim || dim % 8) {
    char m[128];
    snprintf(m, sizeof m, "dim %d must be a multiple of 8 in [8, %d]", dim, kMaxDim);
    put_err(err, err_len, m);
    return VX_E_RANGE;
  }
  if ((reinterpret_cast<uintptr_t>(weight) & 15) || (reinterpret_cast<uintptr_t>(x) & 3)) {
    put_err(err, err_len, "weight must be 16-byte aligned and x 4-byte aligned");
    return VX_E_INVALID;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    put_err(err, err_len, "no current CUDA device");
    return VX_E_CUDA;
  }
  unsigned char* scratch = nullptr;
  {
    // Set-up, once per device (with that device current): the host cannot use the
    // array's name as a device address, so look the address up.
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) {
        char m[160];
        snprintf(m, sizeof m, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        put_err(err, err_len, m);
        return VX_E_CUDA;
      }
      g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
    }
    scratch = g_scratch_ptr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the completion ticket must start at zero (the array keeps the last call's contents)
  cudaError_t e = cudaMemsetAsync(scratch, 0, 4, s);
  const int blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  const size_t smem = (size_t)dim * sizeof(float);
  if (e == cudaSuccess && smem > 48 * 1024)
    e = cudaFuncSetAttribute(k_lm_head_argmax_noalloc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) {
    k_lm_head_argmax_noalloc<<<blocks, 256, smem, s>>>(reinterpret_cast<const __half*>(weight), x, rows, dim,
                                                      out_index, out_value, scratch);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    char m[160];
    snprintf(m, sizeof m, "launch: %s", cudaGetErrorString(e));
    put_err(err, err_len, m);
    return VX_E_CUDA;
  }
  put_err(err, err_len, "");
  return VX_OK;
}
