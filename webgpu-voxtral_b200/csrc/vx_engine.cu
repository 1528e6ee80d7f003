// vx_engine.cu — the B200 decode engine behind include/voxtral_b200.h.
//
// Replaces the WebGPU orchestration of the reference's VoxtralEngine
// (src/engine.ts: createWorkBuffers :453-508, createKVCaches :510-530,
// organizeWeights :659-743, backboneStep :814-1042, fmTransformerPass :1057-1225,
// fmForward :1240-1380, generate :2416-2616).
//
// Memory (HBM): one arena holds all weights in streaming order per layer
//   [wq;wk;wv] [6144,3072] | wo [3072,4096] | [w1;w3] [18432,3072] | w2 [3072,9216] | norms
// so that every projection is one contiguous weight stream; a paged f16 KV pool
// (pages of 64 positions, page table per slot); f32 activations per slot.
// Each backbone step / FM pass / decode frame is one CUDA graph whose kernels
// read the slot's position and inputs from device memory (SlotState), so one
// captured graph serves every step.  Kernels are chained with programmatic
// dependent launch.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/voxtral_b200.h"
#include "k_attn.cuh"
#include "k_codec.cuh"
#include "k_gemm.cuh"
#include "k_gemv.cuh"
#include "k_misc.cuh"
#include "k_step.cuh"

using namespace vx;

namespace {

constexpr int kPage = 64;
constexpr int kAudioKick = 24;   // AUDIO token fed through the text embedding after prefill

struct LayerW {
  __half *wqkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr, *attn_norm = nullptr, *ffn_norm = nullptr;
};

// One checkpoint tensor and where its (shard of) values live on the device.
struct TensorSlot {
  __half* dst;
  long long ld;               // destination row stride (elements)
  long long rows, cols;       // local block
  long long full_rows, full_cols;
  long long row0, col0;       // block origin inside the full tensor
  bool is_norm;
  float fill = 0.f;           // synthetic weights: 0 = N(0, sigma) values, else this constant
};

struct NcclApi {
  void* lib = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  const char* (*getErrorString)(ncclResult_t) = nullptr;
  bool load(const char* path, std::string& err) {
    if (lib) return true;
    lib = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!lib) { err = std::string("cannot load NCCL: ") + dlerror(); return false; }
    getUniqueId = (decltype(getUniqueId))dlsym(lib, "ncclGetUniqueId");
    commInitRank = (decltype(commInitRank))dlsym(lib, "ncclCommInitRank");
    allReduce = (decltype(allReduce))dlsym(lib, "ncclAllReduce");
    commDestroy = (decltype(commDestroy))dlsym(lib, "ncclCommDestroy");
    getErrorString = (decltype(getErrorString))dlsym(lib, "ncclGetErrorString");
    if (!getUniqueId || !commInitRank || !allReduce || !commDestroy) { err = "NCCL symbols missing"; return false; }
    return true;
  }
};
NcclApi g_nccl;

}  // namespace

struct CodecState;   // vx_codec.cuh

struct vx_handle {
  vx_config cfg{};
  int dev = 0, num_sms = 148;
  cudaStream_t own_stream = nullptr, stream = nullptr;
  std::string err;
  long long launches = 0;

  // dims (local to this TP rank where sharded)
  int D = 0, L = 0, HD = 128, F = 0, FL = 0, NH = 0, NKV = 0, QD = 0, KVD = 0, QKVD = 0;
  int V = 0, AV = 0, NAC = 36, SEMV = 0, Fl = 0;   // Fl: local FFN width
  int tp = 1, rank = 0;

  // weights
  void* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<LayerW> layers, fm_layers;
  __half *tok_emb = nullptr, *audio_emb = nullptr, *final_norm = nullptr;
  __half *fm_in = nullptr, *fm_head = nullptr, *fm_time = nullptr, *fm_norm = nullptr, *fm_ac = nullptr;
  std::unordered_map<std::string, TensorSlot> tensors;
  bool weights_ready = false, tp_table_ready = false;
  CodecState* codec = nullptr;   // codec decoder (vx_codec.cuh), when enabled

  // KV cache
  __half* kv_pool = nullptr;
  long long kv_rows = 0;
  int max_pages = 0, n_splits = 1;
  int32_t* page_table = nullptr;
  CUtensorMap kv_map;
  float* attn_part = nullptr;
  int* attn_tickets = nullptr;
  float* rope_freq = nullptr;

  // slots and activations
  int B = 1;
  SlotState* slots = nullptr;
  float *h = nullptr, *q = nullptr, *att = nullptr, *g = nullptr, *normed = nullptr, *rows_in = nullptr;
  int32_t* prompt = nullptr;
  float* voice = nullptr;
  uint32_t* code_ring = nullptr;
  float* normed_ring = nullptr;
  float* logits = nullptr;
  int32_t* argmax_dev = nullptr;
  float* dbg = nullptr;
  // FM work buffers (per slot)
  float *fm_head_out = nullptr, *fm_seq = nullptr, *fm_qkv = nullptr, *fm_att = nullptr, *fm_g = nullptr;
  float *fm_vel = nullptr, *fm_x = nullptr, *fm_noise = nullptr, *fm_xfinal = nullptr, *tp_table = nullptr,
        *te_tmp = nullptr;
  // checkpoint copies
  SlotState* ck_slots = nullptr;
  float* ck_normed = nullptr;
  std::vector<int> ck_pos_host, ck_frame_host;

  std::vector<int> pos_host, frame_host, prompt_len_host;

  // graphs: per slot
  struct G {
    cudaGraphExec_t exec = nullptr;
    long long kernels = 0;
  };
  std::vector<G> g_step, g_fm, g_frame_fm, g_frame_bb;

  // staging
  uint8_t* pinned = nullptr;
  void* load_stage = nullptr;   // vx_load_tensor_typed staging (allocated by the first call)
  size_t pinned_bytes = 0;

  // TP
  ncclComm_t comm = nullptr;
  // TP persistent kernel: tagged receive words in peer-accessible memory (CUDA IPC),
  // the residual's second buffer, and all-reduces completed so far
  void* p2p_buf = nullptr;
  void* p2p_peer[mk::kMaxTp] = {nullptr};
  bool p2p_ready = false;
  float* h2 = nullptr;
  unsigned long long ar_base = 0;
  // persistent kernel (AR form): q / K / V rows handed to its attention phase as tagged words
  unsigned long long* mk_tags = nullptr;
  bool coop = false;

  // persistent decode kernel (k_step.cuh): layer table and grid-barrier counter
  bool use_mk = true;
  mk::LayerPtrs* d_layers = nullptr;
  unsigned* d_bar = nullptr;
  unsigned long long* d_trace = nullptr;   // phase trace of the next persistent launch (vx_trace)
  int prefetch_ahead = 2;   // persistent kernel: L2 lookahead in weight tiles (option l2_prefetch_tiles; measured best)
  bool early_kv = true;     // persistent kernel: first K/V pair copied during the QKV phase (option early_kv_pair)
  uint32_t wait_limit = 0;  // persistent kernel: polls before a barrier / peer wait gives up (option wait_limit; 0 = built-in)
  bool tp_loopback = false; // option tp_loopback: every peer receive buffer is this handle's own (test support)
  bool tagged = true;       // tp 1: residual handed over as tagged words (option residual_handoff)
  bool trace_armed = false;

  // token batches on the tensor cores (k_gemm.cuh): batched prefill
  bool use_tb = true;                  // token-batch path (tensor-core GEMMs)
  bool prefill_tokenwise = false;      // option batched_prefill = 0: token-by-token prefill
  int tb_cap = 0;                      // rows per batch
  struct TbLayerMaps { CUtensorMap wqkv, wo, w13, w2; };
  std::vector<TbLayerMaps> tb_wmaps;   // per backbone layer
  std::vector<TbLayerMaps> fm_wmaps;   // per acoustic-transformer layer (its 6 sequence rows on the tensor cores)
  CUtensorMap tb_xhi[3], tb_xlo[3];    // operand pair for K = D, QD, Fl (128-row boxes)
  CUtensorMap tb_xhi64[3], tb_xlo64[3];  // the same with 64-row boxes (batches of <= 64 rows)
  CUtensorMap tb_xhi16[3], tb_xlo16[3];  // and 16-row boxes (the acoustic transformer's 6 rows)
  std::unordered_map<long long, G> g_batch;   // batched decode step graphs, key (slot0, n)
  void* tb_buf = nullptr;
  float *tb_h = nullptr, *tb_y = nullptr, *tb_q = nullptr, *tb_att = nullptr, *tb_part = nullptr, *tb_ws = nullptr;
  float* tb_ar = nullptr;              // tp > 1: [tb_cap][D] partial rows of o_proj / down, all-reduced in place
  int* tb_att_tickets = nullptr;
  __half *tb_hi = nullptr, *tb_lo = nullptr;
  size_t tb_ws_floats = 0;

  // vx_profile_step: which kernels a captured step contains, and the GEMV bytes it moves
  int parts = 7;          // kPartMisc | kPartGemv | kPartAttn
  bool profiling = false;
  double prof_bytes = 0;

  int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    err = buf;
    return code;
  }
};

#define CK(...)                                                                                 \
  do {                                                                                          \
    cudaError_t e_ = (__VA_ARGS__);                                                                  \
    if (e_ != cudaSuccess) return h->fail(VX_E_CUDA, "%s: %s", #__VA_ARGS__, cudaGetErrorString(e_)); \
  } while (0)

namespace {

template <typename... KArgs, typename... Args>
cudaError_t launch(vx_handle* h, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = h->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  h->launches++;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <int M, int R, int CPL, int EPI, bool NORM>
cudaError_t gemv_attr() {
  return cudaFuncSetAttribute(gemv::k_gemv<M, R, CPL, EPI, NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)gemv::kSmemBytes);
}

template <int BN>
cudaError_t tc_attr() {
  return cudaFuncSetAttribute(tc::k_gemm<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::Cfg<BN>::kSmem);
}

// Every GEMV instantiation the programs use gets its shared-memory opt-in at
// engine creation, before any stream capture.
int prime_kernel_attrs(vx_handle* h) {
  using namespace gemv;
  CK(gemv_attr<1, 6, 3, kQkv, true>());
  CK(gemv_attr<1, 4, 4, kResid, false>()); CK(gemv_attr<1, 4, 4, kStore, false>());
  CK(gemv_attr<1, 8, 2, kResid, false>()); CK(gemv_attr<1, 8, 2, kStore, false>());
  CK(gemv_attr<1, 8, 1, kResid, false>()); CK(gemv_attr<1, 8, 1, kStore, false>());
  CK(gemv_attr<1, 6, 3, kSwiglu, true>());
  CK(gemv_attr<1, 2, 9, kResid, false>()); CK(gemv_attr<1, 2, 9, kStore, false>());
  CK(gemv_attr<1, 2, 5, kResid, false>()); CK(gemv_attr<1, 2, 5, kStore, false>());
  CK(gemv_attr<1, 6, 3, kResid, false>()); CK(gemv_attr<1, 6, 3, kStore, false>());
  CK(gemv_attr<6, 4, 3, kStore, true>()); CK(gemv_attr<6, 4, 4, kResid, false>());
  CK(gemv_attr<6, 4, 3, kSwiglu, true>()); CK(gemv_attr<6, 4, 3, kResid, false>());
  CK(gemv_attr<2, 6, 3, kStore, true>());
  CK(cudaFuncSetAttribute(attn::k_attn_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn::kSmemBytes));
  CK(cudaFuncSetAttribute(mk::k_decode_steps<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mk::kSmemBytes));
  CK(cudaFuncSetAttribute(mk::k_decode_steps<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mk::kSmemBytes));
  CK(cudaFuncSetAttribute(mk::k_decode_steps<2, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mk::kSmemBytes));
  CK(cudaFuncSetAttribute(mk::k_decode_steps<4, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mk::kSmemBytes));
  CK(cudaFuncSetAttribute(mk::k_decode_steps<8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mk::kSmemBytes));
  CK(cudaFuncSetAttribute(k_fm_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSampleSmem));
  CK(cudaFuncSetAttribute(k_top_p_test, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSampleSmem));
  CK(tc_attr<16>()); CK(tc_attr<64>()); CK(tc_attr<128>()); CK(tc_attr<256>());
  return VX_OK;
}

// n_frames consecutive backbone steps of one slot in ONE cooperative launch of the
// persistent decode kernel (k_step.cuh).
// Peer-accessible block of the TP persistent kernel: tagged receive words
// [2 parity][tp source][D] (8 bytes each; zero = no tag yet), then this rank's own
// tagged words of the summed residual [2 parity][D] (read only locally).
constexpr size_t kP2pHxOff = 2ull * mk::kMaxTp * 3072 * 8;
// Highest tensor-parallel degree at which the persistent decode kernel runs.  At degree 8
// its per-layer record of a 2-layer model differs from the golden fixture from layer 0's
// attention output on (the per-op path and the 1-layer kernel match), so degree 8 decodes
// through the per-op kernels with NCCL all-reduces.
constexpr int kMkMaxTp = 4;
constexpr size_t kP2pBytes = kP2pHxOff + 2ull * 3072 * 8;

int launch_steps(vx_handle* h, int slot, int n_frames, int mode0, int token0, int mode_next, bool inc_frame,
                 bool record, float* dbg = nullptr, int dbg_frame = -1) {
  if (n_frames <= 0) return VX_OK;
  mk::StepParams sp{};
  sp.layers = h->d_layers; sp.n_layers = h->L;
  sp.tok = h->tok_emb; sp.vocab = h->V; sp.audio = h->audio_emb; sp.audio_rows = h->AV;
  sp.rows_in = h->rows_in; sp.prompt = h->prompt; sp.voice = h->voice;
  sp.max_seq = h->cfg.max_seq_len; sp.max_voice = h->cfg.max_voice_rows; sp.code_ring = h->code_ring;
  const long long D = h->D;
  sp.h = h->h + slot * D; sp.q = h->q + (long long)slot * h->QD; sp.att = h->att + (long long)slot * h->QD;
  sp.g = h->g + (long long)slot * h->Fl; sp.normed = h->normed + slot * D; sp.normed_ring = h->normed_ring;
  sp.final_norm = h->final_norm; sp.eps = h->cfg.norm_eps;
  sp.kv = gemv::KvGeom{h->kv_pool, h->page_table, h->max_pages, h->L, h->NKV, kPage};
  sp.part = h->attn_part + (long long)slot * h->NKV * h->n_splits * attn::kGqa * attn::kPartStride;
  sp.tickets = h->attn_tickets + (long long)slot * h->NKV;
  sp.n_splits = h->n_splits; sp.rope_freq = h->rope_freq;
  sp.slots = h->slots; sp.slot = slot; sp.bar = h->d_bar;
  sp.trace = h->trace_armed ? h->d_trace : nullptr;
  sp.prefetch_ahead = h->prefetch_ahead;
  sp.early_kv = h->early_kv ? 1 : 0;
  sp.dbg = dbg; sp.dbg_frame = dbg_frame;
  sp.wait_limit = h->wait_limit;
  h->trace_armed = false;
  sp.n_frames = n_frames; sp.mode0 = mode0; sp.token0 = token0; sp.mode_next = mode_next;
  sp.inc_frame = inc_frame ? 1 : 0; sp.record = record ? 1 : 0;
  CK(cudaMemsetAsync(h->d_bar, 0, sizeof(unsigned), h->stream));
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(h->num_sms);
  cfg.blockDim = dim3(mk::kThreads);
  cfg.dynamicSmemBytes = mk::kSmemBytes;
  cfg.stream = h->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const bool ar = h->tp > 1 || h->tagged;
  if (ar) {
    if (!h->p2p_ready) return h->fail(VX_E_STATE, "tensor-parallel persistent kernel needs vx_tp_p2p_open");
    sp.rank = h->rank;
    sp.h2 = h->h2 + slot * D;
    sp.recv = reinterpret_cast<unsigned long long*>(h->p2p_buf);
    for (int r = 0; r < h->tp; ++r) sp.peer_recv[r] = reinterpret_cast<unsigned long long*>(h->p2p_peer[r]);
    sp.hx = reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(h->p2p_buf) + kP2pHxOff);
    sp.ar_base = h->ar_base;
    sp.qkv_t = h->mk_tags;
  }
  h->launches++;
  switch (h->tp) {
    case 1:
      if (ar) CK(cudaLaunchKernelEx(&cfg, mk::k_decode_steps<1, true>, h->kv_map, sp));
      else CK(cudaLaunchKernelEx(&cfg, mk::k_decode_steps<1, false>, h->kv_map, sp));
      break;
    case 2: CK(cudaLaunchKernelEx(&cfg, mk::k_decode_steps<2, true>, h->kv_map, sp)); break;
    case 4: CK(cudaLaunchKernelEx(&cfg, mk::k_decode_steps<4, true>, h->kv_map, sp)); break;
    default: CK(cudaLaunchKernelEx(&cfg, mk::k_decode_steps<8, true>, h->kv_map, sp)); break;
  }
  if (ar) h->ar_base += 2ull * h->L * (unsigned long long)n_frames;
  return VX_OK;
}

template <int M, int R, int CPL, int EPI, bool NORM>
int run_gemv(vx_handle* h, const gemv::Params& p) {
  auto kern = gemv::k_gemv<M, R, CPL, EPI, NORM>;
  constexpr int ORT = EPI == gemv::kSwiglu ? R / 2 : R;
  if (p.kc % 128 || (p.kc / 128 + gemv::kCW - 1) / gemv::kCW != CPL || (long long)R * p.kc * 2 > gemv::kStageBytes ||
      p.col0 % 128 ||
      p.col0 + p.kc > p.ldw || p.rows <= 0)
    return h->fail(VX_E_INVALID, "gemv shape: rows %d kc %d col0 %d ldw %lld (CPL %d R %d)", p.rows, p.kc, p.col0,
                   p.ldw, CPL, R);
  const int ntiles = (p.rows + ORT - 1) / ORT;
  const int grid = std::min(ntiles, h->num_sms);
  if (h->profiling) {
    // algorithmic bytes: the weight slice once, x once, y written (read too for residual adds)
    const double w = (double)p.rows * p.kc * 2.0 * (EPI == gemv::kSwiglu ? 2.0 : 1.0);
    const double xy = (double)M * p.kc * 4.0 + (double)M * p.rows * 4.0 * (EPI == gemv::kResid ? 2.0 : 1.0);
    h->prof_bytes += w + xy;
  }
  if (!(h->parts & 2)) return VX_OK;
  CK(launch(h, kern, dim3(grid), dim3(gemv::kThreads), gemv::kSmemBytes, p));
  return VX_OK;
}

void* carve(uint8_t*& cur, size_t bytes) {
  void* p = cur;
  cur += (bytes + 255) & ~size_t(255);
  return p;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int make_kv_map(vx_handle* h) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (!fn || q != cudaDriverEntryPointSuccess) return h->fail(VX_E_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {128, (cuuint64_t)h->kv_rows};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t es[2] = {1, 1};
  CUresult r = ((EncodeTiledFn)fn)(&h->kv_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, h->kv_pool, dims, strides, box, es,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return h->fail(VX_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VX_OK;
}

// 2-D f16 tensor map, 128-byte swizzle, K innermost: `rows` rows of `inner`
// elements, `row_bytes` apart; box = box_inner x box_rows.
int encode_f16_2d(vx_handle* h, CUtensorMap* map, const void* base, long long inner, long long rows, long long row_bytes,
                  int box_inner, int box_rows) {
  static void* fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess) { fn = nullptr; return h->fail(VX_E_CUDA, "cuTensorMapEncodeTiled unavailable"); }
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = ((EncodeTiledFn)fn)(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                                   es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return h->fail(VX_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VX_OK;
}

// -------------------------------------------------------------------- programs
int check_device_error(vx_handle* h) {
  int e = 0;
  CK(cudaMemcpyFromSymbol(&e, vx::vx_dev_error, sizeof(int)));
  if (e) {
    int z = 0;
    cudaMemcpyToSymbol(vx::vx_dev_error, &z, sizeof(int));
    static const char* names[] = {"ok", "TMA stage wait expired", "free-stage wait expired",
                                  "reduction slot wait expired", "drain wait expired", "index out of range",
                                  "tensor-core accumulator wait expired",
                                  "tensor-parallel peer wait expired (a peer's all-reduce words did not arrive)",
                                  "grid barrier wait expired"};
    return h->fail(VX_E_DEVICE, "device-side error: %s", (e > 0 && e < 9) ? names[e] : "unknown");
  }
  return VX_OK;
}

int allreduce_inplace(vx_handle* h, float* buf, size_t n) {
  if (h->tp == 1) return VX_OK;
  ncclResult_t r = g_nccl.allReduce(buf, buf, n, ncclFloat32, ncclSum, h->comm, h->stream);
  if (r != ncclSuccess)
    return h->fail(VX_E_NCCL, "ncclAllReduce: %s", g_nccl.getErrorString ? g_nccl.getErrorString(r) : "error");
  return VX_OK;
}

struct DebugSink {
  float* base = nullptr;   // [(4L+3)][D] on device
};

int dbg_rows(vx_handle* h, const float* src, const __half* w, float* dst) {
  CK(launch(h, k_rows_copy_or_norm, dim3(1), dim3(256), 0, src, w, dst, h->D, h->cfg.norm_eps));
  return VX_OK;
}

// backboneStep for one slot: embed -> L x (norm+QKV+RoPE+KV append, attention,
// o_proj+residual, norm+gate/up+SwiGLU, down+residual) -> final norm.
int enqueue_backbone(vx_handle* h, int slot, bool inc_frame, bool record, const DebugSink* dbg) {
  const int D = h->D;
  int rc;
  EmbedParams ep{};
  ep.tok = h->tok_emb; ep.vocab = h->V; ep.audio = h->audio_emb; ep.audio_rows = h->AV;
  ep.slots = h->slots; ep.rows = h->rows_in; ep.prompt = h->prompt; ep.voice = h->voice;
  ep.max_seq = h->cfg.max_seq_len; ep.max_voice = h->cfg.max_voice_rows; ep.code_ring = h->code_ring;
  ep.h = h->h + (long long)slot * D; ep.D = D; ep.slot0 = slot;
  if (h->parts & 1) CK(launch(h, k_embed, dim3(1), dim3(256), 0, ep));
  if (dbg && (rc = dbg_rows(h, ep.h, nullptr, dbg->base))) return rc;

  float* hs = h->h + (long long)slot * D;
  float* qs = h->q + (long long)slot * h->QD;
  float* as = h->att + (long long)slot * h->QD;
  float* gs = h->g + (long long)slot * h->Fl;
  gemv::KvGeom kg{h->kv_pool, h->page_table, h->max_pages, h->L, h->NKV, kPage};
  for (int l = 0; l < h->L; ++l) {
    const LayerW& W = h->layers[l];
    if (dbg && (rc = dbg_rows(h, hs, W.attn_norm, dbg->base + (size_t)(1 + 4 * l) * D))) return rc;
    {  // RMSNorm + [wq;wk;wv] + RoPE + q store + K/V append
      gemv::Params p{};
      p.W = W.wqkv; p.ldw = D; p.rows = h->QKVD; p.col0 = 0; p.kc = D;
      p.x = hs; p.ldx = D; p.norm_w = W.attn_norm; p.eps = h->cfg.norm_eps; p.norm_dim = D;
      p.qkv.q = qs; p.qkv.ldq = h->QD; p.qkv.q_dim = h->QD; p.qkv.kv_dim = h->KVD; p.qkv.kv = kg; p.qkv.layer = l;
      p.qkv.pos = &h->slots[0].pos; p.qkv.pos_stride = kPosStride; p.qkv.slot0 = slot; p.qkv.rope_freq = h->rope_freq;
      if ((rc = run_gemv<1, 6, 3, gemv::kQkv, true>(h, p))) return rc;
    }
    {  // split-KV flash-decode
      attn::Params ap{};
      ap.q = qs; ap.ldq = h->QD; ap.out = as; ap.ldo = h->QD;
      ap.part = h->attn_part + (long long)slot * h->NKV * h->n_splits * attn::kGqa * attn::kPartStride;
      ap.tickets = h->attn_tickets + (long long)slot * h->NKV;
      ap.kv = kg; ap.layer = l; ap.pos = &h->slots[0].pos; ap.pos_stride = kPosStride; ap.slot0 = slot;
      ap.n_splits = h->n_splits; ap.scale = 1.0f / sqrtf((float)h->HD);
      if (h->parts & 4)
      CK(launch(h, attn::k_attn_decode, dim3(h->NKV, h->n_splits, 1), dim3(attn::kThreads), attn::kSmemBytes,
                h->kv_map, ap));
    }
    {  // o_proj + residual (TP: rank-local partial, then allreduce of h)
      gemv::Params p{};
      p.W = W.wo; p.ldw = h->QD; p.rows = D; p.col0 = 0; p.kc = h->QD; p.x = as; p.ldx = h->QD; p.y = hs; p.ldy = D;
      if (h->QD == 4096) rc = (h->rank == 0) ? run_gemv<1, 4, 4, gemv::kResid, false>(h, p) : run_gemv<1, 4, 4, gemv::kStore, false>(h, p);
      else if (h->QD == 2048) rc = (h->rank == 0) ? run_gemv<1, 8, 2, gemv::kResid, false>(h, p) : run_gemv<1, 8, 2, gemv::kStore, false>(h, p);
      else if (h->QD == 1024) rc = (h->rank == 0) ? run_gemv<1, 8, 1, gemv::kResid, false>(h, p) : run_gemv<1, 8, 1, gemv::kStore, false>(h, p);
      else if (h->QD == 512) rc = (h->rank == 0) ? run_gemv<1, 8, 1, gemv::kResid, false>(h, p) : run_gemv<1, 8, 1, gemv::kStore, false>(h, p);
      else rc = h->fail(VX_E_INVALID, "unsupported local q width %d", h->QD);
      if (rc) return rc;
      if ((h->parts & 2) && (rc = allreduce_inplace(h, hs, D))) return rc;
    }
    if (dbg && (rc = dbg_rows(h, hs, nullptr, dbg->base + (size_t)(2 + 4 * l) * D))) return rc;
    if (dbg && (rc = dbg_rows(h, hs, W.ffn_norm, dbg->base + (size_t)(3 + 4 * l) * D))) return rc;
    {  // RMSNorm + [w1;w3] + SwiGLU
      gemv::Params p{};
      p.W = W.w13; p.ldw = D; p.second_off = (long long)h->Fl * D; p.rows = h->Fl; p.col0 = 0; p.kc = D;
      p.x = hs; p.ldx = D; p.norm_w = W.ffn_norm; p.eps = h->cfg.norm_eps; p.norm_dim = D; p.y = gs; p.ldy = h->Fl;
      if ((rc = run_gemv<1, 6, 3, gemv::kSwiglu, true>(h, p))) return rc;
    }
    {  // down + residual
      gemv::Params p{};
      p.W = W.w2; p.ldw = h->Fl; p.rows = D; p.col0 = 0; p.kc = h->Fl; p.x = gs; p.ldx = h->Fl; p.y = hs; p.ldy = D;
      if (h->Fl == 9216) rc = (h->rank == 0) ? run_gemv<1, 2, 9, gemv::kResid, false>(h, p) : run_gemv<1, 2, 9, gemv::kStore, false>(h, p);
      else if (h->Fl == 4608) rc = (h->rank == 0) ? run_gemv<1, 2, 5, gemv::kResid, false>(h, p) : run_gemv<1, 2, 5, gemv::kStore, false>(h, p);
      else if (h->Fl == 2304) rc = (h->rank == 0) ? run_gemv<1, 6, 3, gemv::kResid, false>(h, p) : run_gemv<1, 6, 3, gemv::kStore, false>(h, p);
      else if (h->Fl == 1152) rc = (h->rank == 0) ? run_gemv<1, 8, 2, gemv::kResid, false>(h, p) : run_gemv<1, 8, 2, gemv::kStore, false>(h, p);
      else rc = h->fail(VX_E_INVALID, "unsupported local FFN width %d", h->Fl);
      if (rc) return rc;
      if ((h->parts & 2) && (rc = allreduce_inplace(h, hs, D))) return rc;
    }
    if (dbg && (rc = dbg_rows(h, hs, nullptr, dbg->base + (size_t)(4 + 4 * l) * D))) return rc;
  }
  FinalNormParams fp{};
  fp.h = hs; fp.w = h->final_norm; fp.out = h->normed + (long long)slot * D; fp.D = D; fp.eps = h->cfg.norm_eps;
  fp.slots = h->slots; fp.slot0 = slot; fp.inc_pos = 1; fp.inc_frame = inc_frame ? 1 : 0;
  fp.normed_ring = record ? h->normed_ring : nullptr;
  if (h->parts & 1) CK(launch(h, k_final_norm, dim3(1), dim3(256), 0, fp));
  if (dbg) {
    if ((rc = dbg_rows(h, fp.out, nullptr, dbg->base + (size_t)(1 + 4 * h->L) * D))) return rc;
    if ((rc = dbg_rows(h, hs, nullptr, dbg->base + (size_t)(2 + 4 * h->L) * D))) return rc;
  }
  return VX_OK;
}

FmParams fm_params(vx_handle* h, int slot) {
  FmParams f{};
  const int D = h->D;
  f.slots = h->slots; f.slot = slot;
  f.head_out = h->fm_head_out + (long long)slot * (h->SEMV + D);
  f.sem_vocab = h->SEMV; f.D = D;
  f.host_noise = h->fm_noise + (long long)slot * 36;
  f.x = h->fm_x + (long long)slot * 36;
  f.w_in = h->fm_in; f.tp = h->tp_table;
  f.seq = h->fm_seq + (long long)slot * 6 * D;
  f.qkv = h->fm_qkv + (long long)slot * 6 * (4096 + 2048);
  f.att = h->fm_att + (long long)slot * 6 * 4096;
  f.q_dim = h->QD; f.kv_dim = h->KVD; f.n_heads = h->NH; f.n_kv = h->NKV;   // this rank's heads
  f.vel = h->fm_vel + (long long)slot * 72;
  f.alpha = h->cfg.fm_cfg_alpha; f.dt = (float)(1.0 / (h->cfg.fm_nfe - 1));
  f.code_ring = h->code_ring;
  f.x_final = h->fm_xfinal + (long long)slot * 36;
  return f;
}

int enqueue_fm_layers_tc(vx_handle* h, const FmParams& f);

// fmForward for one slot on its normed state.  Under tensor parallelism the acoustic
// transformer's heads and FFN columns are sharded like the backbone's, with an NCCL
// all-reduce of the 6 sequence rows after o_proj and after down; the heads around it
// (semantic head, input projection, acoustic head, Euler step) are replicated.
int enqueue_fm(vx_handle* h, int slot) {
  const int D = h->D;
  int rc;
  {  // semantic head + llm projection in one weight stream ([8320 + 3072] rows)
    gemv::Params p{};
    p.W = h->fm_head; p.ldw = D; p.rows = h->SEMV + D; p.col0 = 0; p.kc = D;
    p.x = h->normed + (long long)slot * D; p.ldx = D; p.y = h->fm_head_out + (long long)slot * (h->SEMV + D); p.ldy = 0;
    if ((rc = run_gemv<1, 6, 3, gemv::kStore, false>(h, p))) return rc;
  }
  FmParams f = fm_params(h, slot);
  CK(launch(h, k_fm_prepare, dim3(1), dim3(1024), 0, f));
  CK(launch(h, k_fm_sample, dim3(1), dim3(1024), kSampleSmem, f));   // returns at once unless the slot samples
  const int steps = h->cfg.fm_nfe - 1;
  for (int s = 0; s < steps; ++s) {
    f.step = s;
    CK(launch(h, k_fm_assemble, dim3((D + 255) / 256), dim3(256), 0, f));
    if (h->tp > 1 && !h->comm) return h->fail(VX_E_STATE, "tensor-parallel acoustic transformer needs vx_tp_init (NCCL)");
    if ((rc = enqueue_fm_layers_tc(h, f))) return rc;
    {  // final norm of position 0 of both sequences + acoustic_codebook_output
      gemv::Params p{};
      p.W = h->fm_ac; p.ldw = D; p.rows = 36; p.col0 = 0; p.kc = D; p.x = f.seq; p.ldx = 3LL * D;
      p.norm_w = h->fm_norm; p.eps = 1e-5f; p.norm_dim = D; p.y = const_cast<float*>(f.vel); p.ldy = 36;
      if ((rc = run_gemv<2, 6, 3, gemv::kStore, true>(h, p))) return rc;
    }
    CK(launch(h, k_fm_euler, dim3(1), dim3(64), 0, f, (int)(s == steps - 1)));
  }
  return VX_OK;
}

// time_projection(time_embedding(t_s)) for the 7 Euler times: frame-independent,
// so computed once instead of once per step of every frame.
int build_tp_table(vx_handle* h) {
  const int D = h->D, steps = h->cfg.fm_nfe - 1;
  for (int s = 0; s < steps; ++s) {
    const float t = (float)((double)s / steps);
    k_time_embed<<<(D / 2 + 255) / 256, 256, 0, h->stream>>>(t, D, h->te_tmp);
    h->launches++;
    CK(cudaGetLastError());
    gemv::Params p{};
    p.W = h->fm_time; p.ldw = D; p.rows = D; p.col0 = 0; p.kc = D; p.x = h->te_tmp; p.ldx = D;
    p.y = h->tp_table + (long long)s * D; p.ldy = D;
    int rc = run_gemv<1, 6, 3, gemv::kStore, false>(h, p);
    if (rc) return rc;
  }
  CK(cudaStreamSynchronize(h->stream));
  h->tp_table_ready = true;
  return VX_OK;
}

enum Prog { kProgStep = 0, kProgFm = 1, kProgFrameFm = 2, kProgFrameBb = 3 };

int enqueue_prog(vx_handle* h, int prog, int slot) {
  int rc;
  switch (prog) {
    case kProgStep: return enqueue_backbone(h, slot, false, false, nullptr);
    case kProgFm: return enqueue_fm(h, slot);
    case kProgFrameFm: {
      // frame f > 0: multiCodebookEmbed(frame f-1 codes) -> backbone -> FM
      if ((rc = enqueue_backbone(h, slot, false, true, nullptr))) return rc;
      return enqueue_fm(h, slot);
    }
    case kProgFrameBb: return enqueue_backbone(h, slot, true, true, nullptr);
  }
  return h->fail(VX_E_INVALID, "bad program");
}

int run_prog(vx_handle* h, int prog, int slot) {
  std::vector<vx_handle::G>* tab = prog == kProgStep ? &h->g_step : prog == kProgFm ? &h->g_fm
                                 : prog == kProgFrameFm ? &h->g_frame_fm : &h->g_frame_bb;
  vx_handle::G& g = (*tab)[slot];
  if (!g.exec) {
    cudaGraph_t graph;
    const long long before = h->launches;
    CK(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_prog(h, prog, slot);
    cudaError_t ce = cudaStreamEndCapture(h->stream, &graph);
    if (rc) { if (ce == cudaSuccess) cudaGraphDestroy(graph); return rc; }
    if (ce != cudaSuccess) return h->fail(VX_E_CUDA, "graph capture: %s", cudaGetErrorString(ce));
    cudaError_t ie = cudaGraphInstantiate(&g.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return h->fail(VX_E_CUDA, "graph instantiate: %s", cudaGetErrorString(ie));
    g.kernels = h->launches - before;
    h->launches = before;
  }
  CK(cudaGraphLaunch(g.exec, h->stream));
  h->launches += g.kernels;
  return VX_OK;
}

int check_slot(vx_handle* h, int slot) {
  if (!h) return VX_E_INVALID;
  if (slot < 0 || slot >= h->B) return h->fail(VX_E_RANGE, "slot %d out of range [0,%d)", slot, h->B);
  if (!h->weights_ready) return h->fail(VX_E_STATE, "Engine not initialized. Call init() and loadWeights() first.");
  return VX_OK;
}

int slot_update(vx_handle* h, int slot, const SlotUpdate& u) {
  k_slot_update<<<1, 32, 0, h->stream>>>(h->slots, slot, u);
  h->launches++;
  CK(cudaGetLastError());
  return VX_OK;
}

// ---------------------------------------------------------------- token batches (k_gemm.cuh)
// Y[N, M] (=|+=) X[N, K] W[M, K]^T on the tensor cores.  Split-K fills the SMs
// when the output has fewer tiles than SMs: floor(SMs / tiles) splits (at most
// `max_splits`), so that the CTAs form one whole wave.
template <int BN>
int run_tc_gemm_ws(vx_handle* h, const CUtensorMap& w, const CUtensorMap& xhi, const CUtensorMap& xlo, float* y,
                   long long ldy, int M, int N, int K, int accumulate, float* ws, size_t ws_floats, int max_splits = 8,
                   int* splits_out = nullptr) {
  if (N < 1 || M < 1 || K < tc::kBK || K % tc::kBK) return h->fail(VX_E_INVALID, "tensor-core GEMM shape %dx%dx%d", M, N, K);
  const int n_tiles = (N + BN - 1) / BN, m_tiles = (M + tc::kBM - 1) / tc::kBM;
  const int chunks = K / tc::kBK;
  const int tiles = n_tiles * m_tiles;
  int splits = 1;
  if (tiles < h->num_sms) splits = std::max(1, std::min({chunks, max_splits, h->num_sms / tiles}));
  if (M % 4 || ldy % 4) splits = 1;   // the split-K reduction writes float4 along m
  while (splits > 1 && (size_t)tiles * splits * BN * tc::kBM > ws_floats) --splits;
  const int cps = (chunks + splits - 1) / splits;
  splits = (chunks + cps - 1) / cps;
  tc::Params p{y, ldy, ws, M, N, K, cps, accumulate};
  CK(launch(h, tc::k_gemm<BN>, dim3(n_tiles, m_tiles, splits), dim3(tc::kThreads), tc::Cfg<BN>::kSmem, w, xhi, xlo, p));
  if (splits_out) {
    *splits_out = splits > 1 ? splits : 0;   // the caller's row kernel sums the partials
  } else if (splits > 1) {
    tc::ReduceParams rp{ws, y, ldy, M, N, splits, n_tiles, BN, accumulate};
    const long long n4 = (long long)N * (M / 4);
    CK(launch(h, tc::k_splitk_reduce, dim3((unsigned)std::min<long long>((n4 + 255) / 256, 4L * h->num_sms)), dim3(256),
              0, rp));
  }
  return VX_OK;
}

template <int BN>
int run_tc_gemm(vx_handle* h, const CUtensorMap& w, const CUtensorMap& xhi, const CUtensorMap& xlo, float* y,
                long long ldy, int M, int N, int K, int accumulate, int max_splits = 8, int* splits_out = nullptr) {
  return run_tc_gemm_ws<BN>(h, w, xhi, xlo, y, ldy, M, N, K, accumulate, h->tb_ws, h->tb_ws_floats, max_splits,
                            splits_out);
}

// Per-row epilogue launch (k_tb_row): split-K sum + residual + RMSNorm -> hi/lo, or
// split-K sum + RoPE + K/V append.
int tb_row(vx_handle* h, int n, int mode, int splits, int n_tiles, int bn, float* y, long long ldy, int M,
           const __half* norm_w, const tc::RopeKvParams* rope, const float* add = nullptr) {
  tc::RowParams rp{};
  rp.add = add;
  rp.ws = h->tb_ws; rp.splits = splits; rp.n_tiles = n_tiles; rp.bn = bn; rp.y = y; rp.ldy = ldy; rp.M = M;
  rp.mode = mode; rp.norm_w = norm_w; rp.eps = h->cfg.norm_eps; rp.hi = h->tb_hi; rp.lo = h->tb_lo;
  if (rope) rp.rope = *rope;
  // threads per row: as many as the row allows (one float4 group each), for latency
  int nt = 0;
  for (int g = 1; g <= 3 && !nt; ++g)
    if (M % (4 * g) == 0 && M / (4 * g) <= 1024 && (M / (4 * g)) % 32 == 0) nt = M / (4 * g);
  if (!nt) return h->fail(VX_E_INVALID, "row width %d", M);
  if (splits > tc::kMaxRowSplits) return h->fail(VX_E_INVALID, "%d split-K partials per row", splits);
  CK(launch(h, tc::k_tb_row, dim3(n), dim3(nt), 0, rp));
  return VX_OK;
}

// The 3 acoustic-transformer layers of one Euler step (fmTransformerPass, src/engine.ts:1057-1225)
// on the tensor cores: the 6 sequence rows (3 positions x cond/uncond) are a token batch
// of 6 through tcgen05 GEMMs (16-row tiles, 9-stage weight pipeline), with the pre-norms, residual adds and split-K
// sums in k_tb_row, SwiGLU in k_tb_swiglu_split and the 3-token attention in k_fm_attn3.
int enqueue_fm_layers_tc(vx_handle* h, const FmParams& f) {
  const int D = h->D, n = 6;
  int rc, sp = 0;
  if ((rc = tb_row(h, n, tc::kRowResidNorm, 0, 1, 16, f.seq, D, D, h->fm_layers[0].attn_norm, nullptr))) return rc;
  for (int l = 0; l < h->FL; ++l) {
    const LayerW& W = h->fm_layers[l];
    const vx_handle::TbLayerMaps& m = h->fm_wmaps[l];
    const __half* next = l + 1 < h->FL ? h->fm_layers[l + 1].attn_norm : nullptr;
    if ((rc = run_tc_gemm<16>(h, m.wqkv, h->tb_xhi16[0], h->tb_xlo16[0], const_cast<float*>(f.qkv), h->QKVD, h->QKVD, n,
                              D, 0)))
      return rc;
    FmParams fa = f;   // attention output straight into the o_proj operand
    fa.att_hi = h->tb_hi;
    fa.att_lo = h->tb_lo;
    CK(launch(h, k_fm_attn3, dim3(2 * h->NH / 4), dim3(128), 0, fa));   // (sequence, head) per warp
    if (h->tp == 1) {
      if ((rc = run_tc_gemm<16>(h, m.wo, h->tb_xhi16[1], h->tb_xlo16[1], f.seq, D, D, n, h->QD, 1, 8, &sp))) return rc;
      if ((rc = tb_row(h, n, tc::kRowResidNorm, sp, 1, 16, f.seq, D, D, W.ffn_norm, nullptr))) return rc;
    } else {
      // this rank's heads: o_proj partial, summed over the ranks (NCCL), then the residual + ffn norm
      if ((rc = run_tc_gemm<16>(h, m.wo, h->tb_xhi16[1], h->tb_xlo16[1], h->tb_ar, D, D, n, h->QD, 0))) return rc;
      if ((rc = allreduce_inplace(h, h->tb_ar, (size_t)n * D))) return rc;
      if ((rc = tb_row(h, n, tc::kRowResidNorm, 0, 1, 16, f.seq, D, D, W.ffn_norm, nullptr, h->tb_ar))) return rc;
    }
    if ((rc = run_tc_gemm<16>(h, m.w13, h->tb_xhi16[0], h->tb_xlo16[0], h->tb_y, 2LL * h->Fl, 2 * h->Fl, n, D, 0)))
      return rc;
    const long long ng = (long long)n * h->Fl;
    CK(launch(h, tc::k_tb_swiglu_split, dim3((unsigned)std::min<long long>((ng + 255) / 256, 8L * h->num_sms)),
              dim3(256), 0, (const float*)h->tb_y, n, h->Fl, h->tb_hi, h->tb_lo));
    if (h->tp == 1) {
      if ((rc = run_tc_gemm<16>(h, m.w2, h->tb_xhi16[2], h->tb_xlo16[2], f.seq, D, D, n, h->Fl, 1, 8, &sp))) return rc;
      if ((rc = tb_row(h, n, tc::kRowResidNorm, sp, 1, 16, f.seq, D, D, next, nullptr))) return rc;
    } else {
      if ((rc = run_tc_gemm<16>(h, m.w2, h->tb_xhi16[2], h->tb_xlo16[2], h->tb_ar, D, D, n, h->Fl, 0))) return rc;
      if ((rc = allreduce_inplace(h, h->tb_ar, (size_t)n * D))) return rc;
      if ((rc = tb_row(h, n, tc::kRowResidNorm, 0, 1, 16, f.seq, D, D, next, nullptr, h->tb_ar))) return rc;
    }
  }
  return VX_OK;
}


// The L layers for a batch of n activation rows in tb_h (rows described by `tr`):
// on entry tb_hi/tb_lo must hold RMSNorm(tb_h) * attention_norm of layer 0; on
// exit tb_h holds the last layer's residual stream.  Per layer:
//   GEMM [wq;wk;wv] -> row kernel (split-K sum, RoPE, q, K/V append) -> attention
//   (writes the hi/lo operand of o_proj) -> GEMM wo -> row kernel (h +=, RMSNorm
//   ffn_norm -> hi/lo) -> GEMM [w1;w3] -> SwiGLU -> GEMM w2 -> row kernel (h +=,
//   RMSNorm of the next layer's attention_norm -> hi/lo).
template <int BN>
int tb_layers(vx_handle* h, int n, const tc::TokRows& tr, int slot0, int rows_consecutive, int nsb) {
  const int D = h->D;
  int rc, sp = 0;
  const CUtensorMap* xh = BN == 64 ? h->tb_xhi64 : h->tb_xhi;
  const CUtensorMap* xl = BN == 64 ? h->tb_xlo64 : h->tb_xlo;
  const int n_tiles = (n + BN - 1) / BN;
  gemv::KvGeom kg{h->kv_pool, h->page_table, h->max_pages, h->L, h->NKV, kPage};
  for (int l = 0; l < h->L; ++l) {
    const LayerW& W = h->layers[l];
    const vx_handle::TbLayerMaps& mp = h->tb_wmaps[l];
    if ((rc = run_tc_gemm<BN>(h, mp.wqkv, xh[0], xl[0], h->tb_y, h->QKVD, h->QKVD, n, D, 0, 8, &sp))) return rc;
    tc::RopeKvParams rp{nullptr, h->tb_q, h->QD, h->KVD, n, h->kv_pool, h->page_table, h->max_pages, h->L, h->NKV,
                        kPage, l, h->rope_freq, tr};
    if ((rc = tb_row(h, n, tc::kRowQkv, sp, n_tiles, BN, h->tb_y, h->QKVD, h->QKVD, nullptr, &rp))) return rc;
    attn::Params ap{};
    ap.q = h->tb_q; ap.ldq = h->QD; ap.out = h->tb_att; ap.ldo = h->QD;
    ap.part = h->tb_part; ap.tickets = h->tb_att_tickets;
    ap.kv = kg; ap.layer = l; ap.pos = &h->slots[0].pos; ap.pos_stride = kPosStride; ap.slot0 = slot0;
    ap.n_splits = nsb; ap.scale = 1.0f / sqrtf((float)h->HD); ap.rows_consecutive = rows_consecutive;
    ap.out_hi = h->tb_hi; ap.out_lo = h->tb_lo;
    CK(launch(h, attn::k_attn_decode, dim3(h->NKV, nsb, n), dim3(attn::kThreads), attn::kSmemBytes, h->kv_map, ap));
    const __half* next_norm = l + 1 < h->L ? h->layers[l + 1].attn_norm : nullptr;
    if (h->tp == 1) {
      if ((rc = run_tc_gemm<BN>(h, mp.wo, xh[1], xl[1], h->tb_h, D, D, n, h->QD, 1, 8, &sp))) return rc;
      if ((rc = tb_row(h, n, tc::kRowResidNorm, sp, n_tiles, BN, h->tb_h, D, D, W.ffn_norm, nullptr))) return rc;
    } else {
      // tensor parallelism: this rank's o_proj partial over its heads, summed over the
      // ranks (NCCL all-reduce), then h += sum and the ffn norm
      if ((rc = run_tc_gemm<BN>(h, mp.wo, xh[1], xl[1], h->tb_ar, D, D, n, h->QD, 0))) return rc;
      if ((rc = allreduce_inplace(h, h->tb_ar, (size_t)n * D))) return rc;
      if ((rc = tb_row(h, n, tc::kRowResidNorm, 0, n_tiles, BN, h->tb_h, D, D, W.ffn_norm, nullptr, h->tb_ar)))
        return rc;
    }
    if ((rc = run_tc_gemm<BN>(h, mp.w13, xh[0], xl[0], h->tb_y, 2LL * h->Fl, 2 * h->Fl, n, D, 0))) return rc;
    const long long ng = (long long)n * h->Fl;
    CK(launch(h, tc::k_tb_swiglu_split, dim3((unsigned)std::min<long long>((ng + 255) / 256, 8L * h->num_sms)),
              dim3(256), 0, (const float*)h->tb_y, n, h->Fl, h->tb_hi, h->tb_lo));
    if (h->tp == 1) {
      if ((rc = run_tc_gemm<BN>(h, mp.w2, xh[2], xl[2], h->tb_h, D, D, n, h->Fl, 1, 8, &sp))) return rc;
      if ((rc = tb_row(h, n, tc::kRowResidNorm, sp, n_tiles, BN, h->tb_h, D, D, next_norm, nullptr))) return rc;
    } else {
      if ((rc = run_tc_gemm<BN>(h, mp.w2, xh[2], xl[2], h->tb_ar, D, D, n, h->Fl, 0))) return rc;
      if ((rc = allreduce_inplace(h, h->tb_ar, (size_t)n * D))) return rc;
      if ((rc = tb_row(h, n, tc::kRowResidNorm, 0, n_tiles, BN, h->tb_h, D, D, next_norm, nullptr, h->tb_ar)))
        return rc;
    }
  }
  return VX_OK;
}

// The N prompt positions of a slot through the backbone as token batches of up
// to tb_cap rows: every projection is one tensor-core GEMM over the batch
// instead of N weight-streaming steps (the reference runs one backboneStep per
// prompt token, src/engine.ts:2457-2472).  Leaves the slot as the token-by-token
// prefill does: K/V of every position cached, position advanced by N, the last
// position's final-norm state in `normed` and its residual stream in `h`.
int prefill_tb(vx_handle* h, int slot, int n) {
  const int D = h->D;
  int rc;
  tc::TokRows tr{&h->slots[0].pos, kPosStride, 0, slot};
  int nc = 0;
  for (int c0 = 0; c0 < n; c0 += h->tb_cap) {
    nc = std::min(h->tb_cap, n - c0);
    tc::TbEmbedParams ep{h->tok_emb, h->V, h->prompt, h->voice, h->cfg.max_seq_len, h->cfg.max_voice_rows, D, h->tb_h, tr};
    CK(launch(h, tc::k_tb_embed, dim3(nc), dim3(256), 0, ep));
    if ((rc = tb_row(h, nc, tc::kRowResidNorm, 0, 0, 128, h->tb_h, D, D, h->layers[0].attn_norm, nullptr))) return rc;
    if ((rc = tb_layers<128>(h, nc, tr, slot, 1, 1))) return rc;
    CK(launch(h, tc::k_tb_advance, dim3(1), dim3(32), 0, &h->slots[slot].pos, nc));
  }
  // last position: final norm into `normed`, residual stream into `h`
  FinalNormParams fp{};
  fp.h = h->tb_h + (long long)(nc - 1) * D; fp.w = h->final_norm; fp.out = h->normed + (long long)slot * D; fp.D = D;
  fp.eps = h->cfg.norm_eps;
  CK(launch(h, k_final_norm, dim3(1), dim3(256), 0, fp));
  CK(cudaMemcpyAsync(h->h + (long long)slot * D, fp.h, (size_t)D * 4, cudaMemcpyDeviceToDevice, h->stream));
  return VX_OK;
}

// One backbone step of slots [slot0, slot0 + n) in lockstep, each at its own
// position (the reference's per-frame backboneStep, src/engine.ts:814-1042, for n
// utterances at once): embedding per slot, the token-batch layers (weights streamed
// once per step for all slots), final norm per slot with the position / frame
// advance and the normed-state record.
template <int BN>
int enqueue_decode_batch_bn(vx_handle* h, int slot0, int n, int nsb) {
  const int D = h->D;
  int rc;
  tc::TokRows tr{&h->slots[0].pos, kPosStride, 1, slot0};
  EmbedParams ep{};
  ep.tok = h->tok_emb; ep.vocab = h->V; ep.audio = h->audio_emb; ep.audio_rows = h->AV;
  ep.slots = h->slots; ep.rows = h->rows_in; ep.prompt = h->prompt; ep.voice = h->voice;
  ep.max_seq = h->cfg.max_seq_len; ep.max_voice = h->cfg.max_voice_rows; ep.code_ring = h->code_ring;
  ep.h = h->tb_h; ep.D = D; ep.slot0 = slot0;
  CK(launch(h, k_embed, dim3(n), dim3(256), 0, ep));
  if ((rc = tb_row(h, n, tc::kRowResidNorm, 0, 0, BN, h->tb_h, D, D, h->layers[0].attn_norm, nullptr))) return rc;
  if ((rc = tb_layers<BN>(h, n, tr, slot0, 0, nsb))) return rc;
  FinalNormParams fp{};
  fp.h = h->tb_h; fp.w = h->final_norm; fp.out = h->normed + (long long)slot0 * D; fp.D = D; fp.eps = h->cfg.norm_eps;
  fp.slots = h->slots; fp.slot0 = slot0; fp.inc_pos = 1; fp.inc_frame = 1; fp.normed_ring = h->normed_ring;
  CK(launch(h, k_final_norm, dim3(n), dim3(256), 0, fp));
  return VX_OK;
}

// Attention splits of a batched step: enough (slot, KV head, split) items for ~2
// waves of 3 CTAs per SM once the context is long, at least 8 pages per split (at
// short context one split per item, which writes its output without a merge).  The
// partials hold tb_cap x n_kv x 1 split, so n rows x nsb splits must fit.
int batch_attn_splits(vx_handle* h, int slot0, int n) {
  int max_pos = 0;
  for (int s = slot0; s < slot0 + n; ++s) max_pos = std::max(max_pos, h->pos_host[s]);
  const int pages = max_pos / kPage + 1;
  const int want = std::max(1, std::min((6 * h->num_sms + h->NKV * n - 1) / (h->NKV * n), pages / 8));
  return std::max(1, std::min({want, h->tb_cap / n, attn::kMaxSplits}));
}

int run_decode_batch(vx_handle* h, int slot0, int n) {
  const int nsb = batch_attn_splits(h, slot0, n);
  vx_handle::G& g = h->g_batch[((long long)slot0 << 32) | ((long long)n << 8) | nsb];
  if (!g.exec) {
    cudaGraph_t graph;
    const long long before = h->launches;
    CK(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    int rc = n <= 64 ? enqueue_decode_batch_bn<64>(h, slot0, n, nsb) : enqueue_decode_batch_bn<128>(h, slot0, n, nsb);
    cudaError_t ce = cudaStreamEndCapture(h->stream, &graph);
    if (rc) { if (ce == cudaSuccess) cudaGraphDestroy(graph); return rc; }
    if (ce != cudaSuccess) return h->fail(VX_E_CUDA, "graph capture: %s", cudaGetErrorString(ce));
    cudaError_t ie = cudaGraphInstantiate(&g.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return h->fail(VX_E_CUDA, "graph instantiate: %s", cudaGetErrorString(ie));
    g.kernels = h->launches - before;
    h->launches = before;
  }
  CK(cudaGraphLaunch(g.exec, h->stream));
  h->launches += g.kernels;
  return VX_OK;
}

// Buffers and tensor maps of the token-batch path (tp == 1).
int setup_tb(vx_handle* h) {
  const long long D = h->D;
  h->tb_cap = 512;
  const long long cap = h->tb_cap;
  const long long kmax = std::max<long long>({D, (long long)h->QD, (long long)h->Fl});
  const long long ymax = std::max<long long>(h->QKVD, 2LL * h->Fl);
  h->tb_ws_floats = (size_t)8 << 20;
  size_t bytes = 0;
  auto add = [&](size_t b) { bytes += (b + 255) & ~size_t(255); };
  add(cap * D * 4); add(cap * ymax * 4); add(cap * h->QD * 4); add(cap * h->QD * 4);
  add(cap * h->NKV * attn::kGqa * attn::kPartStride * 4); add(h->tb_ws_floats * 4);
  add(cap * h->NKV * 4); add(cap * kmax * 2); add(cap * kmax * 2);
  if (h->tp > 1) add(cap * D * 4);
  if (cudaMalloc(&h->tb_buf, bytes) != cudaSuccess) return h->fail(VX_E_NOMEM, "token-batch buffers (%.1f MB)", bytes / 1e6);
  CK(cudaMemset(h->tb_buf, 0, bytes));
  uint8_t* cur = (uint8_t*)h->tb_buf;
  h->tb_h = (float*)carve(cur, cap * D * 4);
  h->tb_y = (float*)carve(cur, cap * ymax * 4);
  h->tb_q = (float*)carve(cur, cap * h->QD * 4);
  h->tb_att = (float*)carve(cur, cap * h->QD * 4);
  h->tb_part = (float*)carve(cur, cap * h->NKV * attn::kGqa * attn::kPartStride * 4);
  h->tb_ws = (float*)carve(cur, h->tb_ws_floats * 4);
  h->tb_att_tickets = (int*)carve(cur, cap * h->NKV * 4);
  h->tb_hi = (__half*)carve(cur, cap * kmax * 2);
  h->tb_lo = (__half*)carve(cur, cap * kmax * 2);
  if (h->tp > 1) h->tb_ar = (float*)carve(cur, cap * D * 4);
  int rc;
  const long long ks[3] = {D, (long long)h->QD, (long long)h->Fl};
  for (int i = 0; i < 3; ++i) {
    if ((rc = encode_f16_2d(h, &h->tb_xhi[i], h->tb_hi, ks[i], cap, ks[i] * 2, tc::kBK, 128))) return rc;
    if ((rc = encode_f16_2d(h, &h->tb_xlo[i], h->tb_lo, ks[i], cap, ks[i] * 2, tc::kBK, 128))) return rc;
    if ((rc = encode_f16_2d(h, &h->tb_xhi64[i], h->tb_hi, ks[i], cap, ks[i] * 2, tc::kBK, 64))) return rc;
    if ((rc = encode_f16_2d(h, &h->tb_xlo64[i], h->tb_lo, ks[i], cap, ks[i] * 2, tc::kBK, 64))) return rc;
    if ((rc = encode_f16_2d(h, &h->tb_xhi16[i], h->tb_hi, ks[i], cap, ks[i] * 2, tc::kBK, 16))) return rc;
    if ((rc = encode_f16_2d(h, &h->tb_xlo16[i], h->tb_lo, ks[i], cap, ks[i] * 2, tc::kBK, 16))) return rc;
  }
  h->tb_wmaps.resize(h->L);
  for (int l = 0; l < h->L; ++l) {
    const LayerW& W = h->layers[l];
    vx_handle::TbLayerMaps& m = h->tb_wmaps[l];
    if ((rc = encode_f16_2d(h, &m.wqkv, W.wqkv, D, h->QKVD, D * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &m.wo, W.wo, h->QD, D, h->QD * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &m.w13, W.w13, D, 2LL * h->Fl, D * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &m.w2, W.w2, h->Fl, D, (long long)h->Fl * 2, tc::kBK, tc::kBM))) return rc;
  }
  // acoustic transformer (this rank's shard, the backbone's shapes)
  h->fm_wmaps.resize(h->FL);
  for (int l = 0; l < h->FL; ++l) {
    const LayerW& W = h->fm_layers[l];
    vx_handle::TbLayerMaps& m = h->fm_wmaps[l];
    if ((rc = encode_f16_2d(h, &m.wqkv, W.wqkv, D, h->QKVD, D * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &m.wo, W.wo, h->QD, D, h->QD * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &m.w13, W.w13, D, 2LL * h->Fl, D * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &m.w2, W.w2, h->Fl, D, (long long)h->Fl * 2, tc::kBK, tc::kBM))) return rc;
  }
  return VX_OK;
}

int set_slot_fields(vx_handle* h, int slot, int mode, int token) {
  SlotUpdate u{};
  u.set_mode = 1; u.mode = mode; u.token = token;
  return slot_update(h, slot, u);
}

int need_positions(vx_handle* h, int slot, int n) {
  if (h->pos_host[slot] + n > h->cfg.max_seq_len)
    return h->fail(VX_E_RANGE, "position %d + %d exceeds maxSeqLen %d", h->pos_host[slot], n, h->cfg.max_seq_len);
  return VX_OK;
}

int finish(vx_handle* h) {
  CK(cudaStreamSynchronize(h->stream));
  return check_device_error(h);
}

}  // namespace

#include "vx_codec.cuh"

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

void vx_default_config(vx_config* c) {
  memset(c, 0, sizeof(*c));
  c->dim = 3072; c->n_layers = 26; c->head_dim = 128; c->hidden_dim = 9216; c->n_heads = 32; c->n_kv_heads = 8;
  c->vocab_size = 131072; c->rope_theta = 1.0e6f; c->norm_eps = 1e-5f;
  c->fm_n_layers = 3; c->fm_nfe = 8; c->fm_cfg_alpha = 1.2f; c->fm_n_acoustic = 36; c->fm_semantic_vocab = 8320;
  c->acoustic_levels = 21; c->audio_vocab = 9088;
  c->max_seq_len = 4096; c->max_slots = 1; c->max_frames = 2048; c->max_voice_rows = 256;
  c->enable_fm = 1; c->device = 0; c->tp_size = 1; c->tp_rank = 0;
  c->enable_codec = 1;
}

const char* vx_last_error(const vx_handle* h) { return h ? h->err.c_str() : "null handle"; }

int64_t vx_launch_count(const vx_handle* h) { return h ? h->launches : 0; }

static void add_tensor(vx_handle* h, const std::string& name, __half* dst, long long ld, long long rows, long long cols,
                       long long full_rows, long long full_cols, long long row0, long long col0, bool norm) {
  h->tensors[name] = TensorSlot{dst, ld, rows, cols, full_rows, full_cols, row0, col0, norm, norm ? 1.0f : 0.f};
}

int vx_create(const vx_config* cfg, vx_handle** out) {
  if (!cfg || !out) return VX_E_INVALID;
  *out = nullptr;
  vx_handle* h = new vx_handle();
  h->cfg = *cfg;
  const vx_config& c = h->cfg;
  auto bad = [&](const char* m) { h->err = m; return VX_E_INVALID; };
  int rc = VX_OK;
  if (c.dim != 3072 || c.head_dim != 128 || c.hidden_dim != 9216 || c.n_heads != 32 || c.n_kv_heads != 8)
    rc = bad("this build is specialised for the Ministral-3B shape (dim 3072, 32/8 heads of 128, FFN 9216)");
  else if (c.n_layers < 1 || c.max_seq_len < 1 || c.max_slots < 1 || c.max_frames < 1 || c.max_voice_rows < 0)
    rc = bad("bad sizes");
  else if (!(c.tp_size == 1 || c.tp_size == 2 || c.tp_size == 4 || c.tp_size == 8) || c.tp_rank < 0 ||
           c.tp_rank >= c.tp_size)
    rc = bad("tp_size must be 1, 2, 4 or 8 with 0 <= tp_rank < tp_size");
  else if (c.vocab_size < 1 || c.vocab_size % c.tp_size)
    rc = bad("vocab_size must be a positive multiple of tp_size (the LM head is vocab-sharded)");
  else if (c.fm_nfe < 2 || c.fm_n_acoustic != 36 || c.fm_semantic_vocab < 8194 || c.audio_vocab < 9022)
    rc = bad("bad acoustic-transformer config");
  if (rc) { *out = h; return rc; }

  h->dev = c.device;
  if (cudaSetDevice(h->dev) != cudaSuccess) { *out = h; return h->fail(VX_E_CUDA, "cudaSetDevice(%d) failed", h->dev); }
  cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, h->dev);
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, h->dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, h->dev);
  if (major != 10) { *out = h; return h->fail(VX_E_CUDA, "needs an sm_100 (B200) GPU, found sm_%d%d", major, minor); }
  if (cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
    *out = h; return h->fail(VX_E_CUDA, "stream create failed");
  }
  h->stream = h->own_stream;

  h->tp = c.tp_size; h->rank = c.tp_rank;
  h->D = c.dim; h->L = c.n_layers; h->HD = c.head_dim; h->F = c.hidden_dim;
  h->NH = c.n_heads / h->tp; h->NKV = c.n_kv_heads / h->tp;
  h->QD = h->NH * h->HD; h->KVD = h->NKV * h->HD; h->QKVD = h->QD + 2 * h->KVD; h->Fl = h->F / h->tp;
  h->V = c.vocab_size; h->AV = c.audio_vocab; h->SEMV = c.fm_semantic_vocab; h->FL = c.enable_fm ? c.fm_n_layers : 0;
  h->B = c.max_slots;
  const long long D = h->D;

  // ---------------------------------------------------------- weight arena
  const size_t layer_elems = (size_t)h->QKVD * D + D * (size_t)h->QD + 2 * (size_t)h->Fl * D + D * (size_t)h->Fl + 2 * D;
  // the acoustic transformer's layers are sharded like the backbone's (same shapes)
  const size_t fm_layer_elems = layer_elems;
  size_t elems = layer_elems * h->L + (size_t)h->V * D + (size_t)h->AV * D + D;
  if (c.enable_fm)
    elems += fm_layer_elems * h->FL + D * 36 + (size_t)(h->SEMV + D) * D + D * D + D + 36 * D;
  h->arena_bytes = elems * 2 + 64 * 256 * (h->L + h->FL + 16);
  if (cudaMalloc(&h->arena, h->arena_bytes) != cudaSuccess) {
    *out = h; return h->fail(VX_E_NOMEM, "cannot allocate %.2f GB of weights", h->arena_bytes / 1e9);
  }
  uint8_t* cur = (uint8_t*)h->arena;
  auto alloc_h = [&](size_t n) { return (__half*)carve(cur, n * 2); };
  const long long Q = c.n_heads * (long long)c.head_dim, KV = c.n_kv_heads * (long long)c.head_dim, Fm = c.hidden_dim;
  h->layers.resize(h->L);
  for (int l = 0; l < h->L; ++l) {
    LayerW& W = h->layers[l];
    const std::string pre = "layers." + std::to_string(l) + ".";
    W.wqkv = alloc_h((size_t)h->QKVD * D);
    W.wo = alloc_h(D * (size_t)h->QD);
    W.w13 = alloc_h(2 * (size_t)h->Fl * D);
    W.w2 = alloc_h(D * (size_t)h->Fl);
    W.attn_norm = alloc_h(D);
    W.ffn_norm = alloc_h(D);
    const long long r = h->rank;
    add_tensor(h, pre + "attention.wq.weight", W.wqkv, D, h->QD, D, Q, D, r * h->QD, 0, false);
    add_tensor(h, pre + "attention.wk.weight", W.wqkv + (size_t)h->QD * D, D, h->KVD, D, KV, D, r * h->KVD, 0, false);
    add_tensor(h, pre + "attention.wv.weight", W.wqkv + (size_t)(h->QD + h->KVD) * D, D, h->KVD, D, KV, D,
               r * h->KVD, 0, false);
    add_tensor(h, pre + "attention.wo.weight", W.wo, h->QD, D, h->QD, D, Q, 0, r * h->QD, false);
    add_tensor(h, pre + "feed_forward.w1.weight", W.w13, D, h->Fl, D, Fm, D, r * h->Fl, 0, false);
    add_tensor(h, pre + "feed_forward.w3.weight", W.w13 + (size_t)h->Fl * D, D, h->Fl, D, Fm, D, r * h->Fl, 0, false);
    add_tensor(h, pre + "feed_forward.w2.weight", W.w2, h->Fl, D, h->Fl, D, Fm, 0, r * h->Fl, false);
    add_tensor(h, pre + "attention_norm.weight", W.attn_norm, D, 1, D, 1, D, 0, 0, true);
    add_tensor(h, pre + "ffn_norm.weight", W.ffn_norm, D, 1, D, 1, D, 0, 0, true);
  }
  h->tok_emb = alloc_h((size_t)h->V * D);
  h->audio_emb = alloc_h((size_t)h->AV * D);
  h->final_norm = alloc_h(D);
  add_tensor(h, "mm_audio_embeddings.tok_embeddings.weight", h->tok_emb, D, h->V, D, h->V, D, 0, 0, false);
  add_tensor(h, "mm_audio_embeddings.audio_codebook_embeddings.embeddings.weight", h->audio_emb, D, h->AV, D, h->AV, D,
             0, 0, false);
  add_tensor(h, "norm.weight", h->final_norm, D, 1, D, 1, D, 0, 0, true);
  if (c.enable_fm) {
    const std::string p = "acoustic_transformer.";
    h->fm_layers.resize(h->FL);
    for (int l = 0; l < h->FL; ++l) {
      LayerW& W = h->fm_layers[l];
      const std::string pre = p + "layers." + std::to_string(l) + ".";
      W.wqkv = alloc_h((size_t)h->QKVD * D);
      W.wo = alloc_h(D * (size_t)h->QD);
      W.w13 = alloc_h(2 * (size_t)h->Fl * D);
      W.w2 = alloc_h(D * (size_t)h->Fl);
      W.attn_norm = alloc_h(D);
      W.ffn_norm = alloc_h(D);
      const long long r = h->rank;
      add_tensor(h, pre + "attention.wq.weight", W.wqkv, D, h->QD, D, Q, D, r * h->QD, 0, false);
      add_tensor(h, pre + "attention.wk.weight", W.wqkv + (size_t)h->QD * D, D, h->KVD, D, KV, D, r * h->KVD, 0, false);
      add_tensor(h, pre + "attention.wv.weight", W.wqkv + (size_t)(h->QD + h->KVD) * D, D, h->KVD, D, KV, D,
                 r * h->KVD, 0, false);
      add_tensor(h, pre + "attention.wo.weight", W.wo, h->QD, D, h->QD, D, Q, 0, r * h->QD, false);
      add_tensor(h, pre + "feed_forward.w1.weight", W.w13, D, h->Fl, D, Fm, D, r * h->Fl, 0, false);
      add_tensor(h, pre + "feed_forward.w3.weight", W.w13 + (size_t)h->Fl * D, D, h->Fl, D, Fm, D, r * h->Fl, 0, false);
      add_tensor(h, pre + "feed_forward.w2.weight", W.w2, h->Fl, D, h->Fl, D, Fm, 0, r * h->Fl, false);
      add_tensor(h, pre + "attention_norm.weight", W.attn_norm, D, 1, D, 1, D, 0, 0, true);
      add_tensor(h, pre + "ffn_norm.weight", W.ffn_norm, D, 1, D, 1, D, 0, 0, true);
    }
    h->fm_in = alloc_h(D * 36);
    h->fm_head = alloc_h((size_t)(h->SEMV + D) * D);
    h->fm_time = alloc_h(D * D);
    h->fm_norm = alloc_h(D);
    h->fm_ac = alloc_h(36 * D);
    add_tensor(h, p + "input_projection.weight", h->fm_in, 36, D, 36, D, 36, 0, 0, false);
    add_tensor(h, p + "semantic_codebook_output.weight", h->fm_head, D, h->SEMV, D, h->SEMV, D, 0, 0, false);
    add_tensor(h, p + "llm_projection.weight", h->fm_head + (size_t)h->SEMV * D, D, D, D, D, D, 0, 0, false);
    add_tensor(h, p + "time_projection.weight", h->fm_time, D, D, D, D, D, 0, 0, false);
    add_tensor(h, p + "norm.weight", h->fm_norm, D, 1, D, 1, D, 0, 0, true);
    add_tensor(h, p + "acoustic_codebook_output.weight", h->fm_ac, D, 36, D, 36, D, 0, 0, false);
  }
  if (c.enable_codec && (rc = codec_create(h))) { *out = h; return rc; }

  // ---------------------------------------------------------- KV cache + activations
  h->max_pages = (c.max_seq_len + kPage - 1) / kPage;
  const long long total_pages = (long long)h->B * h->max_pages;
  h->kv_rows = total_pages * h->L * 2 * h->NKV * kPage;
  // one attention item per CTA: (kv heads x splits) <= SMs
  h->n_splits = std::max(1, std::min(std::min(h->max_pages, attn::kMaxSplits), h->num_sms / h->NKV));
  size_t act = 0;
  auto f32n = [&](size_t n) { act += ((n * 4 + 255) & ~size_t(255)); };
  f32n(64);  // rope
  f32n((size_t)h->B * D * 3 + (size_t)h->B * h->QD * 2 + (size_t)h->B * h->Fl);
  f32n((size_t)h->B * D);  // h2
  f32n((size_t)h->B * h->NKV * h->n_splits * attn::kGqa * attn::kPartStride);
  f32n((size_t)h->B * h->NKV);
  f32n((size_t)h->B * c.max_seq_len);
  f32n((size_t)h->B * c.max_voice_rows * D);
  f32n((size_t)h->B * c.max_frames * 37);
  f32n((size_t)h->B * c.max_frames * D);
  f32n((size_t)h->V + 16);
  f32n((size_t)(4 * h->L + 3) * D);
  f32n((size_t)h->B * D);  // checkpoint normed
  if (c.enable_fm) {
    f32n((size_t)h->B * (h->SEMV + D));
    f32n((size_t)h->B * 6 * D);
    f32n((size_t)h->B * 6 * 6144);
    f32n((size_t)h->B * 6 * 4096);
    f32n((size_t)h->B * 6 * Fm);
    f32n((size_t)h->B * (72 + 36 * 3));
    f32n((size_t)8 * D + D);
  }
  act += 2 * ((sizeof(SlotState) * h->B + 255) & ~size_t(255));
  act += ((size_t)h->B * h->max_pages * 4 + 255) & ~size_t(255);
  void* abuf = nullptr;
  if (cudaMalloc(&abuf, act + 4096) != cudaSuccess ||
      cudaMalloc((void**)&h->kv_pool, (size_t)h->kv_rows * 256) != cudaSuccess) {
    *out = h; return h->fail(VX_E_NOMEM, "cannot allocate KV cache (%.2f GB) / work buffers", h->kv_rows * 256 / 1e9);
  }
  cudaMemset(abuf, 0, act + 4096);
  cudaMemset(h->kv_pool, 0, (size_t)h->kv_rows * 256);   // masked positions must hold finite values
  uint8_t* ac = (uint8_t*)abuf;
  auto fa = [&](size_t n) { return (float*)carve(ac, n * 4); };
  h->rope_freq = fa(64);
  h->h = fa((size_t)h->B * D); h->normed = fa((size_t)h->B * D); h->rows_in = fa((size_t)h->B * D);
  h->h2 = fa((size_t)h->B * D);
  h->q = fa((size_t)h->B * h->QD); h->att = fa((size_t)h->B * h->QD); h->g = fa((size_t)h->B * h->Fl);
  h->attn_part = fa((size_t)h->B * h->NKV * h->n_splits * attn::kGqa * attn::kPartStride);
  h->attn_tickets = (int*)fa((size_t)h->B * h->NKV);
  h->prompt = (int32_t*)fa((size_t)h->B * c.max_seq_len);
  h->voice = fa((size_t)h->B * c.max_voice_rows * D);
  h->code_ring = (uint32_t*)fa((size_t)h->B * c.max_frames * 37);
  h->normed_ring = fa((size_t)h->B * c.max_frames * D);
  h->logits = fa((size_t)h->V + 16);
  h->argmax_dev = (int32_t*)(h->logits + h->V);
  h->dbg = fa((size_t)(4 * h->L + 3) * D);
  h->ck_normed = fa((size_t)h->B * D);
  if (c.enable_fm) {
    h->fm_head_out = fa((size_t)h->B * (h->SEMV + D));
    h->fm_seq = fa((size_t)h->B * 6 * D);
    h->fm_qkv = fa((size_t)h->B * 6 * 6144);
    h->fm_att = fa((size_t)h->B * 6 * 4096);
    h->fm_g = fa((size_t)h->B * 6 * Fm);
    float* small = fa((size_t)h->B * (72 + 36 * 3));
    h->fm_vel = small; h->fm_x = small + (size_t)h->B * 72; h->fm_noise = h->fm_x + (size_t)h->B * 36;
    h->fm_xfinal = h->fm_noise + (size_t)h->B * 36;
    h->tp_table = fa((size_t)8 * D + D);
    h->te_tmp = h->tp_table + (size_t)8 * D;
  }
  h->slots = (SlotState*)carve(ac, sizeof(SlotState) * h->B);
  h->ck_slots = (SlotState*)carve(ac, sizeof(SlotState) * h->B);
  h->page_table = (int32_t*)carve(ac, (size_t)h->B * h->max_pages * 4);

  // rope frequencies 1/theta^(2i/head_dim), formed in double and rounded once
  std::vector<float> freq(64, 0.f);
  for (int i = 0; i < h->HD / 2; ++i) freq[i] = (float)(1.0 / pow((double)c.rope_theta, (double)(2 * i) / h->HD));
  std::vector<int32_t> ptab((size_t)h->B * h->max_pages);
  for (size_t i = 0; i < ptab.size(); ++i) ptab[i] = (int32_t)i;   // slot s owns pages [s*max_pages, (s+1)*max_pages)
  std::vector<SlotState> st(h->B);
  memset(st.data(), 0, sizeof(SlotState) * h->B);
  for (int s = 0; s < h->B; ++s) {
    st[s].max_frames = c.max_frames;
    st[s].codes_key = vx_stream_key(VX_SEED_CODES, s);
    st[s].noise_key = vx_stream_key(VX_SEED_FM_NOISE, s);
  }
  if (cudaMemcpy(h->rope_freq, freq.data(), 64 * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(h->page_table, ptab.data(), ptab.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(h->slots, st.data(), sizeof(SlotState) * h->B, cudaMemcpyHostToDevice) != cudaSuccess) {
    *out = h; return h->fail(VX_E_CUDA, "init copies failed");
  }
  h->pinned_bytes = std::max<size_t>((size_t)(4 * h->L + 3) * D * 4, (size_t)(h->SEMV + 64) * 4) + (size_t)c.max_frames * 37 * 4 +
                    (size_t)c.max_seq_len * 4 + 65536;
  if (cudaMallocHost(&h->pinned, h->pinned_bytes) != cudaSuccess) { *out = h; return h->fail(VX_E_NOMEM, "pinned"); }
  h->pos_host.assign(h->B, 0); h->frame_host.assign(h->B, 0); h->prompt_len_host.assign(h->B, 0);
  h->ck_pos_host.assign(h->B, 0);
  h->ck_frame_host.assign(h->B, 0);
  h->g_step.resize(h->B); h->g_fm.resize(h->B); h->g_frame_fm.resize(h->B); h->g_frame_bb.resize(h->B);
  if ((rc = make_kv_map(h))) { *out = h; return rc; }
  if ((rc = prime_kernel_attrs(h))) { *out = h; return rc; }
  {
    std::vector<mk::LayerPtrs> lp(h->L);
    for (int l = 0; l < h->L; ++l)
      lp[l] = mk::LayerPtrs{h->layers[l].wqkv, h->layers[l].wo, h->layers[l].w13, h->layers[l].w2,
                            h->layers[l].attn_norm, h->layers[l].ffn_norm};
    if (cudaMalloc((void**)&h->d_layers, sizeof(mk::LayerPtrs) * h->L + 256) != cudaSuccess ||
        cudaMemcpy(h->d_layers, lp.data(), sizeof(mk::LayerPtrs) * h->L, cudaMemcpyHostToDevice) != cudaSuccess) {
      *out = h; return h->fail(VX_E_NOMEM, "layer table");
    }
    h->d_bar = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(h->d_layers) + sizeof(mk::LayerPtrs) * h->L);
    h->d_bar = reinterpret_cast<unsigned*>((reinterpret_cast<uintptr_t>(h->d_bar) + 127) & ~uintptr_t(127));
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, h->dev);
    h->coop = coop != 0;
    h->use_mk = h->coop && h->tp == 1;   // TP: enabled by vx_tp_p2p_open
    if (h->coop) {
      // the QKV epilogues' outputs as tagged words for the attention phase (tag 0 never matches)
      const size_t words = (size_t)h->QKVD;
      if (cudaMalloc((void**)&h->mk_tags, words * 8) != cudaSuccess || cudaMemset(h->mk_tags, 0, words * 8) != cudaSuccess) {
        *out = h; return h->fail(VX_E_NOMEM, "tagged q / K / V words");
      }
    }
    if (h->coop && h->tp == 1) {
      // the persistent kernel's tagged residual words (a one-rank all-reduce)
      if (cudaMalloc(&h->p2p_buf, kP2pBytes) != cudaSuccess || cudaMemset(h->p2p_buf, 0, kP2pBytes) != cudaSuccess) {
        *out = h; return h->fail(VX_E_NOMEM, "tagged residual words");
      }
      h->p2p_peer[0] = h->p2p_buf;
      h->p2p_ready = true;
    }
  }
  {
    // token batches on the tensor cores; under tensor parallelism their all-reduces
    // need the NCCL communicator of vx_tp_init
    h->use_tb = true;
    if ((rc = setup_tb(h))) { *out = h; return rc; }
  }
  *out = h;
  return VX_OK;
}

void vx_destroy(vx_handle* h) {
  if (!h) return;
  cudaSetDevice(h->dev);
  if (h->stream) cudaStreamSynchronize(h->stream);
  codec_destroy(h);
  for (auto* tab : {&h->g_step, &h->g_fm, &h->g_frame_fm, &h->g_frame_bb})
    for (auto& g : *tab)
      if (g.exec) cudaGraphExecDestroy(g.exec);
  for (auto& kv : h->g_batch)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  if (h->comm && g_nccl.commDestroy) g_nccl.commDestroy(h->comm);
  for (int r = 0; r < mk::kMaxTp; ++r)
    if (h->p2p_peer[r] && h->p2p_peer[r] != h->p2p_buf) cudaIpcCloseMemHandle(h->p2p_peer[r]);
  if (h->p2p_buf) cudaFree(h->p2p_buf);
  if (h->mk_tags) cudaFree(h->mk_tags);
  if (h->arena) cudaFree(h->arena);
  if (h->d_layers) cudaFree(h->d_layers);
  if (h->d_trace) cudaFree(h->d_trace);
  if (h->kv_pool) cudaFree(h->kv_pool);
  if (h->tb_buf) cudaFree(h->tb_buf);
  if (h->load_stage) cudaFree(h->load_stage);
  if (h->rope_freq) cudaFree(h->rope_freq);   // base of the activation block
  if (h->pinned) cudaFreeHost(h->pinned);
  if (h->own_stream) cudaStreamDestroy(h->own_stream);
  delete h;
}

// Test support, no counterpart in the reference: the tensor-core GEMM of the
// batched paths against an f32 CUDA-core product of the same seeded operands.
int vx_selftest_gemm(vx_handle* h, int32_t M, int32_t N, int32_t K, int32_t bn, int32_t max_splits, uint64_t seed,
                     double* out_rel_err) {
  if (!h || !out_rel_err) return VX_E_INVALID;
  if (!h->use_tb) return h->fail(VX_E_STATE, "token-batch path is off");
  if (M < 1 || N < 1 || K < 64 || K % 64 || !(bn == 16 || bn == 64 || bn == 128 || bn == 256) || max_splits < 1 ||
      (long long)M * K > (1LL << 28) || (long long)N * K > (1LL << 26) || (long long)N * M > (1LL << 26))
    return h->fail(VX_E_INVALID, "selftest shape M=%d N=%d K=%d bn=%d", M, N, K, bn);
  CK(cudaSetDevice(h->dev));
  __half *W = nullptr, *hi = nullptr, *lo = nullptr;
  float *X = nullptr, *Y = nullptr, *R = nullptr;
  int rc = VX_OK;
  const size_t nw = (size_t)M * K, nx = (size_t)N * K, ny = (size_t)N * M;
  if (cudaMalloc(&W, nw * 2) != cudaSuccess || cudaMalloc(&hi, nx * 2) != cudaSuccess ||
      cudaMalloc(&lo, nx * 2) != cudaSuccess || cudaMalloc(&X, nx * 4) != cudaSuccess ||
      cudaMalloc(&Y, ny * 4) != cudaSuccess || cudaMalloc(&R, ny * 4) != cudaSuccess)
    rc = h->fail(VX_E_NOMEM, "selftest buffers");
  CUtensorMap wm, xh, xl;
  if (!rc) rc = encode_f16_2d(h, &wm, W, K, M, (long long)K * 2, tc::kBK, tc::kBM);
  if (!rc) rc = encode_f16_2d(h, &xh, hi, K, N, (long long)K * 2, tc::kBK, bn);
  if (!rc) rc = encode_f16_2d(h, &xl, lo, K, N, (long long)K * 2, tc::kBK, bn);
  std::vector<float> y(ny), r(ny);
  if (!rc) {
    const uint64_t key = vx_stream_key(seed, 77);
    if (launch(h, tc::k_selftest_fill, dim3(4 * h->num_sms), dim3(256), 0, W, (long long)nw, X, (long long)nx, key) !=
            cudaSuccess ||
        launch(h, tc::k_tb_split, dim3(4 * h->num_sms), dim3(256), 0, (const float*)X, (long long)nx, hi, lo) !=
            cudaSuccess)
      rc = h->fail(VX_E_CUDA, "selftest fill");
  }
  for (int pass = 0; pass < 2 && !rc; ++pass) {
    if (bn == 16) rc = run_tc_gemm<16>(h, wm, xh, xl, Y, M, M, N, K, pass, max_splits);
    else if (bn == 64) rc = run_tc_gemm<64>(h, wm, xh, xl, Y, M, M, N, K, pass, max_splits);
    else if (bn == 128) rc = run_tc_gemm<128>(h, wm, xh, xl, Y, M, M, N, K, pass, max_splits);
    else rc = run_tc_gemm<256>(h, wm, xh, xl, Y, M, M, N, K, pass, max_splits);
    if (!rc && pass == 0) {
      tc::k_ref_gemm<<<dim3((M + 127) / 128, N), 128, 0, h->stream>>>(W, X, M, N, K, R);
      if (cudaGetLastError() != cudaSuccess) rc = h->fail(VX_E_CUDA, "reference GEMM launch");
    }
    if (!rc && cudaMemcpyAsync(y.data(), Y, ny * 4, cudaMemcpyDeviceToHost, h->stream) != cudaSuccess)
      rc = h->fail(VX_E_CUDA, "selftest copy");
    if (!rc && pass == 0 && cudaMemcpyAsync(r.data(), R, ny * 4, cudaMemcpyDeviceToHost, h->stream) != cudaSuccess)
      rc = h->fail(VX_E_CUDA, "selftest copy");
    if (!rc) rc = finish(h);
    if (!rc) {
      double emax = 0, rmax = 0;
      const double f = pass + 1.0;
      for (size_t i = 0; i < ny; ++i) {
        emax = std::max(emax, std::fabs((double)y[i] - f * r[i]));
        rmax = std::max(rmax, std::fabs(f * r[i]));
      }
      out_rel_err[pass] = rmax > 0 ? emax / rmax : emax;
    }
  }
  cudaStreamSynchronize(h->stream);
  for (void* ptr : {(void*)W, (void*)hi, (void*)lo, (void*)X, (void*)Y, (void*)R})
    if (ptr) cudaFree(ptr);
  return rc;
}

// Test support: the device top-p sampler (k_top_p_test) on a host logit row with
// explicit uniform draws, one CTA per draw.
int vx_selftest_top_p(vx_handle* h, const float* logits, int32_t n, int32_t valid_lo, int32_t valid_hi, double top_p,
                      double temperature, const double* u, int32_t n_draws, int32_t* out) {
  if (!h || !logits || !u || !out) return VX_E_INVALID;
  if (n < 1 || n > kSortN || n_draws < 1 || n_draws > 65535 || !(temperature > 0) || !std::isfinite(temperature) ||
      !std::isfinite(top_p))
    return h->fail(VX_E_INVALID, "top-p selftest n=%d draws=%d", n, n_draws);
  for (int i = 0; i < n_draws; ++i)
    if (!(u[i] >= 0.0 && u[i] < 1.0)) return h->fail(VX_E_INVALID, "draw %d = %g outside [0, 1)", i, u[i]);
  CK(cudaSetDevice(h->dev));
  float* dl = nullptr;
  double* du = nullptr;
  int32_t* dout = nullptr;
  int rc = VX_OK;
  if (cudaMalloc(&dl, (size_t)n * 4) != cudaSuccess || cudaMalloc(&du, (size_t)n_draws * 8) != cudaSuccess ||
      cudaMalloc(&dout, (size_t)n_draws * 4) != cudaSuccess)
    rc = h->fail(VX_E_NOMEM, "selftest buffers");
  if (!rc && (cudaMemcpyAsync(dl, logits, (size_t)n * 4, cudaMemcpyHostToDevice, h->stream) != cudaSuccess ||
              cudaMemcpyAsync(du, u, (size_t)n_draws * 8, cudaMemcpyHostToDevice, h->stream) != cudaSuccess))
    rc = h->fail(VX_E_CUDA, "selftest copy");
  if (!rc) {
    k_top_p_test<<<n_draws, 1024, kSampleSmem, h->stream>>>(dl, n, valid_lo, valid_hi, top_p, temperature, du, dout);
    h->launches++;
    if (cudaGetLastError() != cudaSuccess) rc = h->fail(VX_E_CUDA, "top-p selftest launch");
  }
  if (!rc && cudaMemcpyAsync(out, dout, (size_t)n_draws * 4, cudaMemcpyDeviceToHost, h->stream) != cudaSuccess)
    rc = h->fail(VX_E_CUDA, "selftest copy");
  if (!rc) rc = finish(h);
  cudaStreamSynchronize(h->stream);
  for (void* ptr : {(void*)dl, (void*)du, (void*)dout})
    if (ptr) cudaFree(ptr);
  return rc;
}

int vx_set_stream(vx_handle* h, void* stream) {
  if (!h) return VX_E_INVALID;
  h->stream = stream ? (cudaStream_t)stream : h->own_stream;
  return VX_OK;
}

int vx_synchronize(vx_handle* h) {
  if (!h) return VX_E_INVALID;
  cudaSetDevice(h->dev);
  return finish(h);
}

int vx_init_random_weights(vx_handle* h, uint64_t seed) {
  if (!h || !h->arena) return VX_E_STATE;
  CK(cudaSetDevice(h->dev));
  for (auto& kv : h->tensors) {
    const TensorSlot& t = kv.second;
    if (t.fill != 0.f) {
      k_fill_f16<<<4, 256, 0, h->stream>>>(t.dst, t.rows * t.cols, t.fill);
      CK(cudaGetLastError());
      continue;
    }
    const uint64_t key = vx_stream_key(seed, vx_fnv1a(kv.first.c_str()));
    if (t.cols == t.full_cols && t.ld == t.cols) {
      // the block spans whole rows: element i is element row0*C + i of the full tensor
      k_init_normal_f16_off<<<2048, 256, 0, h->stream>>>(t.dst, t.rows * t.cols, t.row0 * t.full_cols, key,
                                                         VX_WEIGHT_SIGMA);
      CK(cudaGetLastError());
    } else {
      for (long long r = 0; r < t.rows; ++r) {
        k_init_normal_f16_off<<<(int)std::min(1024LL, t.cols / 256 + 1), 256, 0, h->stream>>>(
            t.dst + r * t.ld, t.cols, (t.row0 + r) * t.full_cols + t.col0, key, VX_WEIGHT_SIGMA);
        CK(cudaGetLastError());
      }
    }
  }
  CK(cudaStreamSynchronize(h->stream));
  h->weights_ready = true;
  int rc;
  if (h->codec && (rc = codec_prepare(h))) return rc;
  if (h->cfg.enable_fm) return build_tp_table(h);
  return VX_OK;
}

int vx_load_tensor_typed(vx_handle* h, const char* name, const void* data, int32_t dtype, size_t n) {
  if (!h || !name || !data) return VX_E_INVALID;
  if (dtype < 0 || dtype > 2) return h->fail(VX_E_INVALID, "dtype %d (0 F16, 1 BF16, 2 F32)", dtype);
  auto it = h->tensors.find(name);
  if (it == h->tensors.end()) return h->fail(VX_E_INVALID, "Missing weight: %s", name);
  const TensorSlot& t = it->second;
  if ((long long)n != t.full_rows * t.full_cols)
    return h->fail(VX_E_INVALID, "%s: expected %lld elements, got %zu", name, t.full_rows * t.full_cols, n);
  CK(cudaSetDevice(h->dev));
  const size_t es = dtype == 2 ? 4 : 2;
  // The rank's block goes through a bounded device staging buffer, a chunk of rows at a time.
  constexpr size_t kStage = 64ull << 20;
  if (!h->load_stage) CK(cudaMalloc(&h->load_stage, kStage));
  const long long rows_per = std::max<long long>(1, (long long)(kStage / (t.cols * es)));
  const uint8_t* base = static_cast<const uint8_t*>(data) + ((size_t)t.row0 * t.full_cols + t.col0) * es;
  for (long long r0 = 0; r0 < t.rows; r0 += rows_per) {
    const long long nr = std::min(rows_per, t.rows - r0);
    CK(cudaMemcpy2DAsync(h->load_stage, t.cols * es, base + (size_t)r0 * t.full_cols * es, t.full_cols * es,
                         t.cols * es, nr, cudaMemcpyHostToDevice, h->stream));
    const long long cnt = nr * t.cols;
    CK(launch(h, k_convert_to_f16, dim3((unsigned)std::min<long long>((cnt + 255) / 256, 16L * h->num_sms)), dim3(256),
              0, (const void*)h->load_stage, dtype, nr, t.cols, reinterpret_cast<uint16_t*>(t.dst + r0 * t.ld), t.ld));
  }
  return finish(h);
}

size_t vx_tensor_names(const vx_handle* h, char* buf, size_t len) {
  if (!h) return 0;
  std::vector<std::string> names;
  for (const auto& kv : h->tensors) names.push_back(kv.first);
  std::sort(names.begin(), names.end());
  std::string all;
  for (const auto& n : names) { all += n; all += '\n'; }
  if (buf && len) {
    const size_t k = std::min(len - 1, all.size());
    memcpy(buf, all.data(), k);
    buf[k] = 0;
  }
  return all.size() + 1;
}

size_t vx_tensor_numel(const vx_handle* h, const char* name) {
  if (!h || !name) return 0;
  auto it = h->tensors.find(name);
  if (it == h->tensors.end()) return 0;
  return (size_t)(it->second.full_rows * it->second.full_cols);
}

int vx_load_tensor(vx_handle* h, const char* name, const uint16_t* f16, size_t n) {
  if (!h || !name || !f16) return VX_E_INVALID;
  auto it = h->tensors.find(name);
  if (it == h->tensors.end()) return h->fail(VX_E_INVALID, "Missing weight: %s", name);
  const TensorSlot& t = it->second;
  if ((long long)n != t.full_rows * t.full_cols)
    return h->fail(VX_E_INVALID, "%s: expected %lld elements, got %zu", name, t.full_rows * t.full_cols, n);
  CK(cudaSetDevice(h->dev));
  const uint16_t* src = f16 + t.row0 * t.full_cols + t.col0;
  CK(cudaMemcpy2D(t.dst, t.ld * 2, src, t.full_cols * 2, t.cols * 2, t.rows, cudaMemcpyHostToDevice));
  return VX_OK;
}

int vx_read_tensor(vx_handle* h, const char* name, uint16_t* out, size_t n) {
  if (!h || !name || !out) return VX_E_INVALID;
  auto it = h->tensors.find(name);
  if (it == h->tensors.end()) return h->fail(VX_E_INVALID, "Missing weight: %s", name);
  const TensorSlot& t = it->second;
  if (t.rows != t.full_rows || t.cols != t.full_cols) return h->fail(VX_E_STATE, "tensor is sharded");
  if ((long long)n != t.rows * t.cols) return h->fail(VX_E_INVALID, "size mismatch");
  CK(cudaSetDevice(h->dev));
  CK(cudaMemcpy2D(out, t.cols * 2, t.dst, t.ld * 2, t.cols * 2, t.rows, cudaMemcpyDeviceToHost));
  return VX_OK;
}

int vx_mark_weights_loaded(vx_handle* h) {
  if (!h) return VX_E_INVALID;
  h->weights_ready = true;
  int rc;
  if (h->codec && (rc = codec_prepare(h))) return rc;
  if (h->cfg.enable_fm) return build_tp_table(h);
  return VX_OK;
}

int vx_reset(vx_handle* h, int32_t slot) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  CK(cudaSetDevice(h->dev));
  SlotUpdate u{};
  u.set_counters = 1;   // pos = frame = 0
  if ((rc = slot_update(h, slot, u))) return rc;
  h->pos_host[slot] = 0;
  h->frame_host[slot] = 0;
  return finish(h);
}

int vx_get_position(vx_handle* h, int32_t slot, int32_t* pos) {
  if (!h || !pos) return VX_E_INVALID;
  if (slot < 0 || slot >= h->B) return h->fail(VX_E_RANGE, "slot out of range");
  *pos = h->pos_host[slot];
  return VX_OK;
}

int vx_set_streams(vx_handle* h, int32_t slot, uint64_t noise_seed, uint64_t codes_seed, int32_t utt) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  CK(cudaSetDevice(h->dev));
  SlotUpdate u{};
  u.set_keys = 1;
  u.noise_key = vx_stream_key(noise_seed, (uint64_t)utt);
  u.codes_key = vx_stream_key(codes_seed, (uint64_t)utt);
  u.set_noise_mode = 1;
  u.noise_mode = 0;
  if ((rc = slot_update(h, slot, u))) return rc;
  return finish(h);
}

int vx_set_sampling(vx_handle* h, int32_t slot, int32_t mode, double top_p, double temperature, uint64_t seed) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (mode != 0 && mode != 1) return h->fail(VX_E_INVALID, "sampling mode %d (0 argmax, 1 top-p)", mode);
  if (mode == 1 && !(std::isfinite(top_p) && std::isfinite(temperature) && temperature > 0))
    return h->fail(VX_E_INVALID, "top_p %g / temperature %g", top_p, temperature);
  if (mode == 1 && h->SEMV > kSortN) return h->fail(VX_E_RANGE, "semantic vocabulary %d > %d", h->SEMV, kSortN);
  CK(cudaSetDevice(h->dev));
  SlotUpdate u{};
  u.set_sampling = 1;
  u.sample_mode = mode;
  u.top_p = top_p;
  u.temperature = temperature;
  u.sample_key = vx_stream_key(seed, kSampleStream);
  if ((rc = slot_update(h, slot, u))) return rc;
  return finish(h);
}

int vx_prefill(vx_handle* h, int32_t slot, const int32_t* tokens, int32_t n, int32_t audio_start, int32_t audio_count,
               const float* voice) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (!tokens || n < 0) return h->fail(VX_E_INVALID, "tokens");
  if (audio_count < 0 || (audio_count > 0 && (!voice || audio_start < 0 || audio_start + audio_count > n)))
    return h->fail(VX_E_INVALID, "voice span [%d, %d) does not fit the prompt", audio_start, audio_start + audio_count);
  if (voice && audio_count > h->cfg.max_voice_rows)
    return h->fail(VX_E_RANGE, "%d voice rows exceed max_voice_rows %d", audio_count, h->cfg.max_voice_rows);
  if ((rc = need_positions(h, slot, n))) return rc;
  CK(cudaSetDevice(h->dev));
  const int p0 = h->pos_host[slot];
  std::vector<int32_t> pt(n);
  for (int i = 0; i < n; ++i) {
    const bool is_voice = voice && i >= audio_start && i < audio_start + audio_count;
    if (!is_voice && (tokens[i] < 0 || tokens[i] >= h->V)) return h->fail(VX_E_RANGE, "token %d out of range", tokens[i]);
    pt[i] = is_voice ? -(i - audio_start) - 1 : tokens[i];
  }
  if (n == 0) return VX_OK;
  // pageable sources: cudaMemcpyAsync stages them before returning, ordered in the stream
  CK(cudaMemcpyAsync(h->prompt + (size_t)slot * h->cfg.max_seq_len + p0, pt.data(), (size_t)n * 4,
                     cudaMemcpyHostToDevice, h->stream));
  if (voice && audio_count)
    CK(cudaMemcpyAsync(h->voice + (size_t)slot * h->cfg.max_voice_rows * h->D, voice, (size_t)audio_count * h->D * 4,
                       cudaMemcpyHostToDevice, h->stream));
  SlotUpdate u{};
  u.set_mode = 1; u.mode = kEmbPrompt; u.token = 0;
  u.set_prompt_len = 1; u.prompt_len = p0 + n;
  if ((rc = slot_update(h, slot, u))) return rc;
  if (h->use_tb && !h->prefill_tokenwise && (h->tp == 1 || h->comm)) {
    if ((rc = prefill_tb(h, slot, n))) return rc;
  } else if (h->use_mk) {
    if ((rc = launch_steps(h, slot, n, kEmbPrompt, 0, kEmbPrompt, false, false))) return rc;
  } else {
    for (int i = 0; i < n; ++i)
      if ((rc = run_prog(h, kProgStep, slot))) return rc;
  }
  h->pos_host[slot] += n;
  return finish(h);
}

static int step_common(vx_handle* h, int slot, float* normed_out, int32_t* argmax_out) {
  int rc;
  if ((rc = run_prog(h, kProgStep, slot))) return rc;
  h->pos_host[slot] += 1;
  if (argmax_out) {
    // tied LM head (src/engine.ts:1017-1041); under tensor parallelism each rank scores
    // its 1/tp of the vocabulary and a max all-reduce of 64-bit keys picks the winner
    const int vs = h->V / h->tp, r0 = h->rank * vs;
    gemv::Params p{};
    p.W = h->tok_emb + (size_t)r0 * h->D; p.ldw = h->D; p.rows = vs; p.col0 = 0; p.kc = h->D;
    p.x = h->normed + (size_t)slot * h->D; p.ldx = h->D; p.y = h->logits; p.ldy = 0;
    if ((rc = run_gemv<1, 6, 3, gemv::kStore, false>(h, p))) return rc;
    CK(launch(h, k_argmax, dim3(1), dim3(1024), 0, (const float*)h->logits, vs, h->argmax_dev));
    if (h->tp == 1) {
      CK(cudaMemcpyAsync(h->pinned, h->argmax_dev, 4, cudaMemcpyDeviceToHost, h->stream));
    } else {
      unsigned long long* key = reinterpret_cast<unsigned long long*>(h->argmax_dev + 4);
      CK(launch(h, k_argmax_key, dim3(1), dim3(32), 0, (const float*)h->logits, (const int32_t*)h->argmax_dev, r0, key));
      ncclResult_t r = g_nccl.allReduce(key, key, 1, ncclUint64, ncclMax, h->comm, h->stream);
      if (r != ncclSuccess) return h->fail(VX_E_NCCL, "ncclAllReduce (LM-head argmax): %s", g_nccl.getErrorString(r));
      CK(cudaMemcpyAsync(h->pinned, key, 8, cudaMemcpyDeviceToHost, h->stream));
    }
  }
  if (normed_out)
    CK(cudaMemcpyAsync(h->pinned + 64, h->normed + (size_t)slot * h->D, (size_t)h->D * 4, cudaMemcpyDeviceToHost,
                       h->stream));
  if ((rc = finish(h))) return rc;
  if (argmax_out) {
    if (h->tp == 1) {
      memcpy(argmax_out, h->pinned, 4);
    } else {
      unsigned long long key;
      memcpy(&key, h->pinned, 8);
      *argmax_out = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
    }
  }
  if (normed_out) memcpy(normed_out, h->pinned + 64, (size_t)h->D * 4);
  return VX_OK;
}

int vx_backbone_step(vx_handle* h, int32_t slot, int32_t token, int32_t use_audio, const float* embed,
                     float* normed_out, int32_t* argmax_out) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if ((rc = need_positions(h, slot, 1))) return rc;
  if (!embed && (token < 0 || token >= (use_audio ? h->AV : h->V)))
    return h->fail(VX_E_RANGE, "token %d out of range", token);
  CK(cudaSetDevice(h->dev));
  if (embed) {
    CK(cudaMemcpyAsync(h->rows_in + (size_t)slot * h->D, embed, (size_t)h->D * 4, cudaMemcpyHostToDevice, h->stream));
    if ((rc = set_slot_fields(h, slot, kEmbRow, 0))) return rc;
  } else if ((rc = set_slot_fields(h, slot, use_audio ? kEmbAudioToken : kEmbToken, token))) {
    return rc;
  }
  return step_common(h, slot, normed_out, argmax_out);
}

int vx_backbone_step_codes(vx_handle* h, int32_t slot, uint32_t sem, const uint32_t* ac, float* normed_out) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (!ac) return h->fail(VX_E_INVALID, "acoustic codes");
  if ((rc = need_positions(h, slot, 1))) return rc;
  if ((int)sem >= h->AV) return h->fail(VX_E_RANGE, "semantic code %u out of range", sem);
  for (int k = 0; k < 36; ++k)
    if (8194 + 23 * k + (int)ac[k] >= h->AV) return h->fail(VX_E_RANGE, "acoustic code %u out of range", ac[k]);
  CK(cudaSetDevice(h->dev));
  SlotUpdate u{};
  u.set_codes = 1;
  u.codes[0] = sem;
  memcpy(u.codes + 1, ac, 36 * 4);
  u.set_mode = 1; u.mode = kEmbCodes; u.token = 0;
  if ((rc = slot_update(h, slot, u))) return rc;
  return step_common(h, slot, normed_out, nullptr);
}

int vx_fm_step(vx_handle* h, int32_t slot, const float* noise, float* sem_logits, uint32_t* sem_code,
               uint32_t* ac_codes, float* x_final) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (!h->cfg.enable_fm) return h->fail(VX_E_STATE, "engine created without the acoustic transformer");
  CK(cudaSetDevice(h->dev));
  {
    SlotUpdate u{};
    u.set_noise_mode = 1;
    u.noise_mode = noise ? 1 : 0;
    if ((rc = slot_update(h, slot, u))) return rc;
  }
  if (noise)
    CK(cudaMemcpyAsync(h->fm_noise + (size_t)slot * 36, noise, 36 * 4, cudaMemcpyHostToDevice, h->stream));
  if ((rc = run_prog(h, kProgFm, slot))) return rc;
  // frame counter advanced by the FM tail: the codes of this call are in ring row frame_host
  const int fr = h->frame_host[slot];
  uint8_t* pb = h->pinned + 1024;
  const size_t nl = (size_t)h->SEMV * 4;
  CK(cudaMemcpyAsync(pb, h->fm_head_out + (size_t)slot * (h->SEMV + h->D), nl, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaMemcpyAsync(pb + nl, reinterpret_cast<uint8_t*>(&h->slots[slot]) + offsetof(SlotState, codes), 37 * 4,
                     cudaMemcpyDeviceToHost, h->stream));
  CK(cudaMemcpyAsync(pb + nl + 256, h->fm_xfinal + (size_t)slot * 36, 36 * 4, cudaMemcpyDeviceToHost, h->stream));
  if ((rc = finish(h))) return rc;
  h->frame_host[slot] = fr + 1;
  if (noise) {  // back to the seeded stream for device-resident decode
    SlotUpdate u{};
    u.set_noise_mode = 1;
    u.noise_mode = 0;
    if ((rc = slot_update(h, slot, u))) return rc;
  }
  const uint32_t* codes = reinterpret_cast<const uint32_t*>(pb + nl);
  if (sem_logits) memcpy(sem_logits, pb, nl);
  if (sem_code) *sem_code = codes[0];
  if (ac_codes) memcpy(ac_codes, codes + 1, 36 * 4);
  if (x_final) memcpy(x_final, pb + nl + 256, 36 * 4);
  return VX_OK;
}

int vx_debug_layers(vx_handle* h, int32_t slot, int32_t token, float* out) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (!out) return h->fail(VX_E_INVALID, "out");
  if (token < 0 || token >= h->V) return h->fail(VX_E_RANGE, "token out of range");
  if ((rc = need_positions(h, slot, 1))) return rc;
  CK(cudaSetDevice(h->dev));
  if (h->use_mk) {
    // the persistent decode kernel that vx_decode / vx_prefill run, recording this step
    if ((rc = launch_steps(h, slot, 1, kEmbToken, token, kEmbToken, false, false, h->dbg, 0))) return rc;
  } else {
    if ((rc = set_slot_fields(h, slot, kEmbToken, token))) return rc;
    DebugSink sink{h->dbg};
    if ((rc = enqueue_backbone(h, slot, false, false, &sink))) return rc;
  }
  h->pos_host[slot] += 1;
  const size_t n = (size_t)(4 * h->L + 3) * h->D;
  CK(cudaMemcpyAsync(out, h->dbg, n * 4, cudaMemcpyDeviceToHost, h->stream));
  return finish(h);
}

int vx_decode(vx_handle* h, int32_t slot, int32_t n_frames, int32_t with_fm) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (n_frames < 0) return h->fail(VX_E_INVALID, "n_frames");
  if (with_fm && !h->cfg.enable_fm) return h->fail(VX_E_STATE, "engine created without the acoustic transformer");
  int f0 = h->frame_host[slot];
  if (f0 + n_frames > h->cfg.max_frames)
    return h->fail(VX_E_RANGE, "frames %d + %d exceed the code ring (%d)", f0, n_frames, h->cfg.max_frames);
  // backbone steps this call will run
  const int steps = with_fm ? (f0 == 0 ? std::max(0, n_frames - 1) : n_frames) : n_frames;
  if ((rc = need_positions(h, slot, steps))) return rc;
  CK(cudaSetDevice(h->dev));
  if (h->use_mk && !with_fm) {
    // all frames in one launch: frame 0 is the AUDIO kick, later frames the synthetic codes
    if (f0 == 0) rc = launch_steps(h, slot, n_frames, kEmbToken, kAudioKick, kEmbSynthCodes, true, true);
    else rc = launch_steps(h, slot, n_frames, kEmbSynthCodes, 0, kEmbSynthCodes, true, true);
    if (rc) return rc;
    h->pos_host[slot] += n_frames;
    h->frame_host[slot] = f0 + n_frames;
    return VX_OK;
  }
  for (int i = 0; i < n_frames; ++i) {
    const int f = f0 + i;
    if (with_fm) {
      if (f == 0) {
        if ((rc = run_prog(h, kProgFm, slot))) return rc;
      } else if (h->use_mk) {
        if ((rc = launch_steps(h, slot, 1, kEmbCodes, 0, kEmbCodes, false, true))) return rc;
        if ((rc = run_prog(h, kProgFm, slot))) return rc;
        h->pos_host[slot] += 1;
      } else {
        if (i == 0 || f0 + i == 1) {
          if ((rc = set_slot_fields(h, slot, kEmbCodes, 0))) return rc;
        }
        if ((rc = run_prog(h, kProgFrameFm, slot))) return rc;
        h->pos_host[slot] += 1;
      }
    } else {
      if (f == 0) {
        if ((rc = set_slot_fields(h, slot, kEmbToken, kAudioKick))) return rc;
      } else if (i == 0 || f == 1) {
        if ((rc = set_slot_fields(h, slot, kEmbSynthCodes, 0))) return rc;
      }
      if ((rc = run_prog(h, kProgFrameBb, slot))) return rc;
      h->pos_host[slot] += 1;
    }
  }
  h->frame_host[slot] = f0 + n_frames;
  return VX_OK;
}

int vx_decode_record(vx_handle* h, int32_t slot, int32_t n_frames, int32_t record_frame, float* out) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (!out || n_frames < 1 || record_frame < 0 || record_frame >= n_frames)
    return h->fail(VX_E_INVALID, "record_frame %d outside [0, n_frames %d)", record_frame, n_frames);
  if (!h->use_mk) return h->fail(VX_E_STATE, "vx_decode_record needs the persistent decode kernel");
  const int f0 = h->frame_host[slot];
  if (f0 + n_frames > h->cfg.max_frames)
    return h->fail(VX_E_RANGE, "frames %d + %d exceed the code ring (%d)", f0, n_frames, h->cfg.max_frames);
  if ((rc = need_positions(h, slot, n_frames))) return rc;
  CK(cudaSetDevice(h->dev));
  if (f0 == 0) rc = launch_steps(h, slot, n_frames, kEmbToken, kAudioKick, kEmbSynthCodes, true, true, h->dbg, record_frame);
  else rc = launch_steps(h, slot, n_frames, kEmbSynthCodes, 0, kEmbSynthCodes, true, true, h->dbg, record_frame);
  if (rc) return rc;
  h->pos_host[slot] += n_frames;
  h->frame_host[slot] = f0 + n_frames;
  CK(cudaMemcpyAsync(out, h->dbg, (size_t)(4 * h->L + 3) * h->D * 4, cudaMemcpyDeviceToHost, h->stream));
  return finish(h);
}

int vx_fill_kv(vx_handle* h, int32_t slot, int32_t n_positions, uint64_t seed) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (n_positions < 1 || n_positions > h->cfg.max_seq_len)
    return h->fail(VX_E_RANGE, "n_positions %d outside [1, maxSeqLen %d]", n_positions, h->cfg.max_seq_len);
  CK(cudaSetDevice(h->dev));
  FillKvParams fp{h->kv_pool, h->page_table, slot, h->max_pages, h->L, h->NKV, h->rank * h->NKV,
                  h->cfg.n_kv_heads * h->HD, n_positions, kPage, seed};
  CK(launch(h, k_fill_kv_slot, dim3(16 * h->num_sms), dim3(256), 0, fp));
  SlotUpdate u{};
  u.set_counters = 1; u.pos = n_positions; u.frame = 0;
  u.set_prompt_len = 1; u.prompt_len = n_positions;
  if ((rc = slot_update(h, slot, u))) return rc;
  h->pos_host[slot] = n_positions;
  h->frame_host[slot] = 0;
  return finish(h);
}

int vx_decode_batch(vx_handle* h, int32_t slot0, int32_t n_slots, int32_t n_frames) {
  if (!h) return VX_E_INVALID;
  int rc;
  if (n_slots < 1 || slot0 < 0 || slot0 + n_slots > h->B)
    return h->fail(VX_E_RANGE, "slots [%d, %d) outside [0, %d)", slot0, slot0 + n_slots, h->B);
  if (n_frames < 0) return h->fail(VX_E_INVALID, "n_frames");
  if ((rc = check_slot(h, slot0))) return rc;
  if (!h->use_tb) return h->fail(VX_E_STATE, "batched decode needs the token-batch path");
  if (h->tp > 1 && !h->comm) return h->fail(VX_E_STATE, "tensor-parallel batched decode needs vx_tp_init (NCCL)");
  if (n_slots > h->tb_cap) return h->fail(VX_E_RANGE, "%d slots exceed the batch capacity %d", n_slots, h->tb_cap);
  if (n_frames == 0) return VX_OK;
  for (int s = slot0; s < slot0 + n_slots; ++s) {
    if ((rc = need_positions(h, s, n_frames))) return rc;
    if (h->frame_host[s] + n_frames > h->cfg.max_frames)
      return h->fail(VX_E_RANGE, "slot %d: frames %d + %d exceed the code ring (%d)", s, h->frame_host[s], n_frames,
                     h->cfg.max_frames);
  }
  CK(cudaSetDevice(h->dev));
  // frame 0 of a slot is the AUDIO kick; later frames are fed the synthetic codes
  bool any_kick = false;
  for (int s = slot0; s < slot0 + n_slots; ++s) {
    const bool kick = h->frame_host[s] == 0;
    any_kick |= kick;
    if ((rc = set_slot_fields(h, s, kick ? kEmbToken : kEmbSynthCodes, kick ? kAudioKick : 0))) return rc;
  }
  for (int f = 0; f < n_frames; ++f) {
    if ((rc = run_decode_batch(h, slot0, n_slots))) return rc;
    for (int s = slot0; s < slot0 + n_slots; ++s) {
      h->pos_host[s] += 1;
      h->frame_host[s] += 1;
    }
    if (f == 0 && any_kick)
      for (int s = slot0; s < slot0 + n_slots; ++s)
        if ((rc = set_slot_fields(h, s, kEmbSynthCodes, 0))) return rc;
  }
  return VX_OK;
}

int vx_read_codes(vx_handle* h, int32_t slot, int32_t frame0, int32_t n, uint32_t* out) {
  if (!h || !out) return VX_E_INVALID;
  if (slot < 0 || slot >= h->B || frame0 < 0 || n < 0 || frame0 + n > h->cfg.max_frames)
    return h->fail(VX_E_RANGE, "frame range");
  CK(cudaSetDevice(h->dev));
  CK(cudaMemcpyAsync(out, h->code_ring + ((size_t)slot * h->cfg.max_frames + frame0) * 37, (size_t)n * 37 * 4,
                     cudaMemcpyDeviceToHost, h->stream));
  return finish(h);
}

int vx_read_normed(vx_handle* h, int32_t slot, int32_t frame0, int32_t n, float* out) {
  if (!h || !out) return VX_E_INVALID;
  if (slot < 0 || slot >= h->B || frame0 < 0 || n < 0 || frame0 + n > h->cfg.max_frames)
    return h->fail(VX_E_RANGE, "frame range");
  CK(cudaSetDevice(h->dev));
  CK(cudaMemcpyAsync(out, h->normed_ring + ((size_t)slot * h->cfg.max_frames + frame0) * h->D, (size_t)n * h->D * 4,
                     cudaMemcpyDeviceToHost, h->stream));
  return finish(h);
}

int vx_checkpoint(vx_handle* h, int32_t slot) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  CK(cudaSetDevice(h->dev));
  CK(cudaMemcpyAsync(&h->ck_slots[slot], &h->slots[slot], sizeof(SlotState), cudaMemcpyDeviceToDevice, h->stream));
  CK(cudaMemcpyAsync(h->ck_normed + (size_t)slot * h->D, h->normed + (size_t)slot * h->D, (size_t)h->D * 4,
                     cudaMemcpyDeviceToDevice, h->stream));
  h->ck_pos_host[slot] = h->pos_host[slot];
  h->ck_frame_host[slot] = h->frame_host[slot];
  return finish(h);
}

int vx_rewind(vx_handle* h, int32_t slot) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  CK(cudaSetDevice(h->dev));
  CK(cudaMemcpyAsync(&h->slots[slot], &h->ck_slots[slot], sizeof(SlotState), cudaMemcpyDeviceToDevice, h->stream));
  CK(cudaMemcpyAsync(h->normed + (size_t)slot * h->D, h->ck_normed + (size_t)slot * h->D, (size_t)h->D * 4,
                     cudaMemcpyDeviceToDevice, h->stream));
  h->pos_host[slot] = h->ck_pos_host[slot];
  h->frame_host[slot] = h->ck_frame_host[slot];
  return VX_OK;
}

// Capture one backbone step restricted to `parts` as a graph (not cached).
static int capture_parts(vx_handle* h, int slot, int parts, cudaGraphExec_t* exec) {
  cudaGraph_t graph;
  h->parts = parts;
  h->profiling = (parts == 2);
  if (h->profiling) h->prof_bytes = 0;
  const long long before = h->launches;
  cudaError_t ce = cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal);
  int rc = ce == cudaSuccess ? enqueue_backbone(h, slot, false, false, nullptr) : VX_E_CUDA;
  cudaError_t ee = cudaStreamEndCapture(h->stream, &graph);
  h->parts = 7;
  h->profiling = false;
  h->launches = before;
  if (rc || ce != cudaSuccess || ee != cudaSuccess) {
    if (ee == cudaSuccess) cudaGraphDestroy(graph);
    return rc ? rc : h->fail(VX_E_CUDA, "profile capture failed");
  }
  cudaError_t ie = cudaGraphInstantiate(exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) return h->fail(VX_E_CUDA, "profile instantiate: %s", cudaGetErrorString(ie));
  return VX_OK;
}

int vx_profile_step(vx_handle* h, int32_t slot, int32_t reps, float* out_ms, double* out_bytes) {
  int rc = check_slot(h, slot);
  if (rc) return rc;
  if (!out_ms || reps < 1) return h->fail(VX_E_INVALID, "profile args");
  if ((rc = need_positions(h, slot, reps))) return rc;
  CK(cudaSetDevice(h->dev));
  // the slot's decode state is saved and restored around the measurement
  SlotState saved;
  CK(cudaMemcpyAsync(&saved, &h->slots[slot], sizeof(SlotState), cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  if ((rc = set_slot_fields(h, slot, kEmbSynthCodes, 0))) return rc;
  cudaGraphExec_t g[3] = {nullptr, nullptr, nullptr};
  const int parts[3] = {7, 2, 4};
  double gemv_bytes = 0;
  for (int k = 0; k < 3 && !rc; ++k) {
    rc = capture_parts(h, slot, parts[k], &g[k]);
    if (parts[k] == 2) gemv_bytes = h->prof_bytes;
  }
  cudaEvent_t a = nullptr, b = nullptr;
  if (!rc) { cudaEventCreate(&a); cudaEventCreate(&b); }
  for (int k = 0; k < 3 && !rc; ++k) {
    // one untimed launch, then `reps` timed launches back to back
    if (cudaGraphLaunch(g[k], h->stream) != cudaSuccess) { rc = h->fail(VX_E_CUDA, "profile launch"); break; }
    cudaEventRecord(a, h->stream);
    for (int i = 0; i < reps; ++i) cudaGraphLaunch(g[k], h->stream);
    cudaEventRecord(b, h->stream);
    if (cudaEventSynchronize(b) != cudaSuccess) { rc = h->fail(VX_E_CUDA, "profile sync"); break; }
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    out_ms[k] = ms / reps;
    // restore the position advanced by the full-step graph
    CK(cudaMemcpyAsync(&h->slots[slot], &saved, sizeof(SlotState), cudaMemcpyHostToDevice, h->stream));
    if ((rc = set_slot_fields(h, slot, kEmbSynthCodes, 0))) break;
  }
  for (auto& x : g) if (x) cudaGraphExecDestroy(x);
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  CK(cudaMemcpyAsync(&h->slots[slot], &saved, sizeof(SlotState), cudaMemcpyHostToDevice, h->stream));
  if (rc) return rc;
  if (out_bytes) out_bytes[0] = gemv_bytes;
  return finish(h);
}

int vx_trace(vx_handle* h, int32_t mode, uint64_t* out, size_t n, int32_t* dims) {
  if (!h) return VX_E_INVALID;
  CK(cudaSetDevice(h->dev));
  const size_t per = (size_t)mk::kTraceFrames * (2 + 5 * h->L) * mk::kTraceSlots;
  const size_t total = per * h->num_sms;
  if (dims) { dims[0] = h->num_sms; dims[1] = mk::kTraceFrames; dims[2] = 2 + 5 * h->L; dims[3] = mk::kTraceSlots; }
  if (mode == 2) return VX_OK;   // dimensions only
  if (mode == 1) {
    if (!h->d_trace && cudaMalloc((void**)&h->d_trace, total * 8) != cudaSuccess) return h->fail(VX_E_NOMEM, "trace");
    CK(cudaMemsetAsync(h->d_trace, 0, total * 8, h->stream));
    h->trace_armed = true;
    return VX_OK;
  }
  if (!out || !h->d_trace) return h->fail(VX_E_STATE, "no trace recorded");
  CK(cudaMemcpyAsync(out, h->d_trace, std::min(n, total) * 8, cudaMemcpyDeviceToHost, h->stream));
  return finish(h);
}

int vx_set_option(vx_handle* h, const char* name, int64_t value) {
  if (!h || !name) return VX_E_INVALID;
  const std::string n = name;
  if (n == "persistent_decode") {
    if (value != 0 && value != 1) return h->fail(VX_E_INVALID, "persistent_decode must be 0 or 1");
    if (value && !h->coop) return h->fail(VX_E_STATE, "the device has no cooperative launch");
    if (value && h->tp > 1 && !h->p2p_ready) return h->fail(VX_E_STATE, "tensor parallelism: call vx_tp_p2p_open first");
    if (value && h->tp > kMkMaxTp)
      return h->fail(VX_E_STATE, "the persistent decode kernel runs at tensor-parallel degree <= %d", kMkMaxTp);
    h->use_mk = value != 0;
  } else if (n == "residual_handoff") {
    if (value != 0 && value != 1) return h->fail(VX_E_INVALID, "residual_handoff must be 0 or 1");
    if (h->tp > 1 && value == 0) return h->fail(VX_E_STATE, "tensor parallelism needs residual_handoff 1");
    h->tagged = value != 0;
  } else if (n == "batched_prefill") {
    if (value != 0 && value != 1) return h->fail(VX_E_INVALID, "batched_prefill must be 0 or 1");
    if (value && !h->use_tb) return h->fail(VX_E_STATE, "the token-batch path is off");
    h->prefill_tokenwise = value == 0;
  } else if (n == "l2_prefetch_tiles") {
    if (value < 0 || value > mk::kMaxPrefetchAhead)
      return h->fail(VX_E_RANGE, "l2_prefetch_tiles must lie in [0, %d]", mk::kMaxPrefetchAhead);
    h->prefetch_ahead = (int)value;
  } else if (n == "early_kv_pair") {
    if (value != 0 && value != 1) return h->fail(VX_E_INVALID, "early_kv_pair must be 0 or 1");
    h->early_kv = value != 0;
  } else if (n == "wait_limit") {
    if (value < 0 || value > 0xffffffffll) return h->fail(VX_E_RANGE, "wait_limit must lie in [0, 2^32)");
    h->wait_limit = (uint32_t)value;
  } else if (n == "tp_loopback") {
    if (value != 1) return h->fail(VX_E_INVALID, "tp_loopback can only be switched on");
    if (h->tp < 2 || h->tp > kMkMaxTp) return h->fail(VX_E_STATE, "tp_loopback needs tp_size 2..%d", kMkMaxTp);
    if (h->p2p_ready) return h->fail(VX_E_STATE, "peer buffers are already open");
    if (!h->coop) return h->fail(VX_E_STATE, "the device has no cooperative launch");
    CK(cudaSetDevice(h->dev));
    if (!h->p2p_buf) {
      CK(cudaMalloc(&h->p2p_buf, kP2pBytes));
      CK(cudaMemset(h->p2p_buf, 0, kP2pBytes));
      CK(cudaDeviceSynchronize());
    }
    for (int r = 0; r < h->tp; ++r) h->p2p_peer[r] = h->p2p_buf;
    h->tp_loopback = true;
    h->p2p_ready = true;
    h->use_mk = true;
  } else {
    return h->fail(VX_E_INVALID, "unknown option '%s'", name);
  }
  return VX_OK;
}

int vx_nccl_unique_id(const char* lib, uint8_t out[128]) {
  std::string err;
  if (!out || !g_nccl.load(lib, err)) return VX_E_NCCL;
  ncclUniqueId id;
  if (g_nccl.getUniqueId(&id) != ncclSuccess) return VX_E_NCCL;
  memcpy(out, id.internal, 128);
  return VX_OK;
}

int vx_tp_init(vx_handle* h, const char* lib, const uint8_t id_bytes[128]) {
  if (!h || !id_bytes) return VX_E_INVALID;
  if (h->tp == 1) return VX_OK;
  std::string err;
  if (!g_nccl.load(lib, err)) return h->fail(VX_E_NCCL, "%s", err.c_str());
  CK(cudaSetDevice(h->dev));
  ncclUniqueId id;
  memcpy(id.internal, id_bytes, 128);
  ncclResult_t r = g_nccl.commInitRank(&h->comm, h->tp, id, h->rank);
  if (r != ncclSuccess) return h->fail(VX_E_NCCL, "ncclCommInitRank: %s", g_nccl.getErrorString(r));
  return VX_OK;
}

int vx_tp_p2p_handle(vx_handle* h, uint8_t out[64]) {
  if (!h || !out) return VX_E_INVALID;
  if (h->tp < 2) return h->fail(VX_E_STATE, "tp_size is 1");
  CK(cudaSetDevice(h->dev));
  if (!h->p2p_buf) {
    CK(cudaMalloc(&h->p2p_buf, kP2pBytes));
    CK(cudaMemset(h->p2p_buf, 0, kP2pBytes));   // tag 0 never matches an all-reduce (tags start at 1)
    CK(cudaDeviceSynchronize());
  }
  cudaIpcMemHandle_t mh;
  CK(cudaIpcGetMemHandle(&mh, h->p2p_buf));
  static_assert(sizeof(mh) == 64, "IPC handle size");
  memcpy(out, &mh, 64);
  return VX_OK;
}

int vx_tp_p2p_open(vx_handle* h, const uint8_t* handles) {
  if (!h || !handles) return VX_E_INVALID;
  if (h->tp < 2 || !h->p2p_buf) return h->fail(VX_E_STATE, "call vx_tp_p2p_handle first");
  CK(cudaSetDevice(h->dev));
  for (int r = 0; r < h->tp; ++r) {
    if (r == h->rank) { h->p2p_peer[r] = h->p2p_buf; continue; }
    if (h->p2p_peer[r]) continue;
    cudaIpcMemHandle_t mh;
    memcpy(&mh, handles + 64 * r, 64);
    void* ptr = nullptr;
    CK(cudaIpcOpenMemHandle(&ptr, mh, cudaIpcMemLazyEnablePeerAccess));
    h->p2p_peer[r] = ptr;
  }
  h->p2p_ready = true;
  h->use_mk = h->coop && h->tp <= kMkMaxTp;
  return VX_OK;
}

}  // extern "C"

