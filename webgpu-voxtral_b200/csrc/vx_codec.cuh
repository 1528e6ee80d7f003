// vx_codec.cuh — host side of the codec decoder (codecDecode, src/engine.ts:1402-1713;
// debugCodecDecode :1719-1975).  Included by vx_engine.cu (it uses the handle's
// launch, tensor-map and GEMM helpers).
//
// Weights: one arena holding the checkpoint tensors under their reference names
// (organizeWeights, src/engine.ts:700-775) plus what is derived from them once they
// are loaded (codec_prepare): the normalised VQ codebook, weight-norm scales, and the
// convolution weights re-ordered as GEMM weights.
//
// Decode of T frames (stage s has T * 2^s tokens, attention window 2^(s+1)):
//   embed + input-conv im2col -> GEMM [T, 960] x [1024, 960]^T -> row (weight norm, RMSNorm)
//   per stage, 2 layers: GEMM qkv -> qknorm -> windowed ALiBi attention -> GEMM wo ->
//     row (layer scale + residual, RMSNorm) -> GEMM w1|w3 -> SwiGLU -> GEMM w2 ->
//     row (layer scale + residual, next operand)
//   stages 0-2: transposed conv as two GEMMs [T_s, 2048] x [1024, 2048]^T (even / odd
//     output steps) -> row (RMSNorm of the next stage)
//   output conv: GEMM [8T, 7168] x [240, 7168]^T -> weight-norm scale -> waveform.

struct CodecLayer {
  __half *wqkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr;
  __half *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  __half *attn_scale = nullptr, *ffn_scale = nullptr;
  CUtensorMap m_wqkv, m_wo, m_w13, m_w2;
};

constexpr int kCodecKs[5] = {codec::kInTaps * codec::kInChPad, codec::kDim, 2 * codec::kDim, codec::kHidden,
                             codec::kOutTaps * codec::kDim};
constexpr int kCodecMaxFrames = 8192;
constexpr int kCodecBN = 128;

struct CodecState {
  void* arena = nullptr;
  __half *sem_sum = nullptr, *usage = nullptr, *in_v = nullptr, *in_g = nullptr, *out_v = nullptr, *out_g = nullptr;
  __half *up_v[3] = {nullptr, nullptr, nullptr}, *up_g[3] = {nullptr, nullptr, nullptr};
  CodecLayer layers[8];
  // derived (codec_prepare)
  __half *cb = nullptr, *in_w = nullptr, *out_w = nullptr, *up_w[3] = {nullptr, nullptr, nullptr};
  float *in_scale = nullptr, *out_scale = nullptr, *up_scale[3] = {nullptr, nullptr, nullptr};
  CUtensorMap m_in, m_out, m_up[3][2];
  bool prepared = false;
  // work buffers for up to `cap` frames
  void* work = nullptr;
  int cap = 0;
  float *cur = nullptr, *y = nullptr, *ws = nullptr, *concat = nullptr, *audio = nullptr;
  __half *hi = nullptr, *lo = nullptr;
  uint32_t *sem = nullptr, *ac = nullptr;
  size_t ws_floats = 0;
  CUtensorMap xhi[5], xlo[5];
};

namespace {

int codec_kidx(int K) {
  for (int i = 0; i < 5; ++i)
    if (kCodecKs[i] == K) return i;
  return -1;
}

void codec_add(vx_handle* h, const std::string& name, __half* dst, long long rows, long long cols, float fill,
               long long row0 = 0, long long full_rows = -1) {
  TensorSlot t{dst, cols, rows, cols, full_rows < 0 ? rows : full_rows, cols, row0, 0, false};
  t.fill = fill;
  h->tensors[name] = t;
}

// Arena, tensor registration and weight tensor maps.
int codec_create(vx_handle* h) {
  using namespace codec;
  CodecState* c = new CodecState();
  h->codec = c;
  const size_t layer_elems = (size_t)3 * kDim * kDim + (size_t)kDim * kDim + (size_t)2 * kHidden * kDim +
                             (size_t)kDim * kHidden + 6 * kDim;
  const size_t elems = 8 * layer_elems + 2 * (size_t)kSemEntries * kSemDim + kSemEntries +
                       (size_t)kDim * kInCh * kInTaps + kDim + 3 * ((size_t)kDim * kDim * kUpTaps + kDim) +
                       (size_t)kPatch * kDim * kOutTaps + kPatch + (size_t)kDim * kInTaps * kInChPad +
                       3 * (size_t)2 * kDim * 2 * kDim + (size_t)kPatchPad * kOutTaps * kDim;
  const size_t bytes = elems * 2 + (size_t)(kDim * 4 + kPatchPad) * 4 + 256 * 160;
  if (cudaMalloc(&c->arena, bytes) != cudaSuccess) return h->fail(VX_E_NOMEM, "codec weights (%.2f GB)", bytes / 1e9);
  cudaMemset(c->arena, 0, bytes);
  uint8_t* cur = (uint8_t*)c->arena;
  auto ah = [&](size_t n) { return (__half*)carve(cur, n * 2); };
  auto af = [&](size_t n) { return (float*)carve(cur, n * 4); };
  const std::string P = "audio_tokenizer.";
  c->sem_sum = ah((size_t)kSemEntries * kSemDim);
  c->usage = ah(kSemEntries);
  codec_add(h, P + "quantizer.semantic_codebook.embedding_sum", c->sem_sum, kSemEntries, kSemDim, 0.f);
  codec_add(h, P + "quantizer.semantic_codebook.cluster_usage", c->usage, 1, kSemEntries, 2.0f);
  c->in_v = ah((size_t)kDim * kInCh * kInTaps);
  c->in_g = ah(kDim);
  codec_add(h, P + "decoder_blocks.0.conv.parametrizations.weight.original1", c->in_v, kDim, kInCh * kInTaps, 0.f);
  codec_add(h, P + "decoder_blocks.0.conv.parametrizations.weight.original0", c->in_g, 1, kDim, 1.0f);
  for (int s = 0; s < 4; ++s)
    for (int l = 0; l < 2; ++l) {
      CodecLayer& L = c->layers[2 * s + l];
      const std::string pre = P + "decoder_blocks." + std::to_string(1 + 2 * s) + ".layers." + std::to_string(l) + ".";
      L.wqkv = ah((size_t)3 * kDim * kDim);
      L.wo = ah((size_t)kDim * kDim);
      L.w13 = ah((size_t)2 * kHidden * kDim);
      L.w2 = ah((size_t)kDim * kHidden);
      L.attn_norm = ah(kDim); L.ffn_norm = ah(kDim); L.q_norm = ah(kDim); L.k_norm = ah(kDim);
      L.attn_scale = ah(kDim); L.ffn_scale = ah(kDim);
      codec_add(h, pre + "attention.wq.weight", L.wqkv, kDim, kDim, 0.f);
      codec_add(h, pre + "attention.wk.weight", L.wqkv + (size_t)kDim * kDim, kDim, kDim, 0.f);
      codec_add(h, pre + "attention.wv.weight", L.wqkv + (size_t)2 * kDim * kDim, kDim, kDim, 0.f);
      codec_add(h, pre + "attention.wo.weight", L.wo, kDim, kDim, 0.f);
      codec_add(h, pre + "feed_forward.w1.weight", L.w13, kHidden, kDim, 0.f);
      codec_add(h, pre + "feed_forward.w3.weight", L.w13 + (size_t)kHidden * kDim, kHidden, kDim, 0.f);
      codec_add(h, pre + "feed_forward.w2.weight", L.w2, kDim, kHidden, 0.f);
      codec_add(h, pre + "attention_norm.weight", L.attn_norm, 1, kDim, 1.0f);
      codec_add(h, pre + "ffn_norm.weight", L.ffn_norm, 1, kDim, 1.0f);
      codec_add(h, pre + "attention.q_norm.weight", L.q_norm, 1, kDim, 1.0f);
      codec_add(h, pre + "attention.k_norm.weight", L.k_norm, 1, kDim, 1.0f);
      codec_add(h, pre + "attention_scale", L.attn_scale, 1, kDim, 0.1f);
      codec_add(h, pre + "ffn_scale", L.ffn_scale, 1, kDim, 0.1f);
    }
  for (int s = 0; s < 3; ++s) {
    const std::string pre = P + "decoder_blocks." + std::to_string(2 + 2 * s) + ".conv.parametrizations.weight.";
    c->up_v[s] = ah((size_t)kDim * kDim * kUpTaps);
    c->up_g[s] = ah(kDim);
    codec_add(h, pre + "original1", c->up_v[s], kDim, kDim * kUpTaps, 0.f);
    codec_add(h, pre + "original0", c->up_g[s], 1, kDim, 1.0f);
  }
  c->out_v = ah((size_t)kPatch * kDim * kOutTaps);
  c->out_g = ah(kPatch);
  codec_add(h, P + "output_proj.conv.parametrizations.weight.original1", c->out_v, kPatch, kDim * kOutTaps, 0.f);
  codec_add(h, P + "output_proj.conv.parametrizations.weight.original0", c->out_g, 1, kPatch, 1.0f);
  // derived
  c->cb = ah((size_t)kSemEntries * kSemDim);
  c->in_w = ah((size_t)kDim * kInTaps * kInChPad);
  for (int s = 0; s < 3; ++s) c->up_w[s] = ah((size_t)2 * kDim * 2 * kDim);
  c->out_w = ah((size_t)kPatchPad * kOutTaps * kDim);
  c->in_scale = af(kDim);
  for (int s = 0; s < 3; ++s) c->up_scale[s] = af(kDim);
  c->out_scale = af(kPatchPad);
  if ((size_t)(cur - (uint8_t*)c->arena) > bytes) return h->fail(VX_E_INVALID, "codec arena overflow");
  int rc;
  for (auto& L : c->layers) {
    if ((rc = encode_f16_2d(h, &L.m_wqkv, L.wqkv, kDim, 3 * kDim, kDim * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &L.m_wo, L.wo, kDim, kDim, kDim * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &L.m_w13, L.w13, kDim, 2 * kHidden, kDim * 2, tc::kBK, tc::kBM))) return rc;
    if ((rc = encode_f16_2d(h, &L.m_w2, L.w2, kHidden, kDim, kHidden * 2, tc::kBK, tc::kBM))) return rc;
  }
  const int kin = kInTaps * kInChPad, kout = kOutTaps * kDim;
  if ((rc = encode_f16_2d(h, &c->m_in, c->in_w, kin, kDim, kin * 2, tc::kBK, tc::kBM))) return rc;
  if ((rc = encode_f16_2d(h, &c->m_out, c->out_w, kout, kPatchPad, (long long)kout * 2, tc::kBK, tc::kBM))) return rc;
  for (int s = 0; s < 3; ++s)
    for (int par = 0; par < 2; ++par)
      if ((rc = encode_f16_2d(h, &c->m_up[s][par], c->up_w[s] + (size_t)par * kDim * 2 * kDim, 2 * kDim, kDim,
                              4LL * kDim, tc::kBK, tc::kBM)))
        return rc;
  return VX_OK;
}

// What is derived from the loaded checkpoint (normalizeVQCodebook src/engine.ts:593-614,
// precomputeConvTransposeScales :621-654, the conv weight norms, GEMM weight layouts).
int codec_prepare(vx_handle* h) {
  using namespace codec;
  CodecState* c = h->codec;
  cudaStream_t st = h->stream;
  const int g = 4 * h->num_sms;
  k_cb_normalize<<<g, 256, 0, st>>>(c->sem_sum, c->usage, c->cb);
  k_conv_out_scale<<<(kDim + 255) / 256, 256, 0, st>>>(c->in_v, c->in_g, kDim, kInCh * kInTaps, c->in_scale);
  k_conv_reorder<<<g, 256, 0, st>>>(c->in_v, kDim, kInCh, kInTaps, kDim, kInChPad, c->in_w);
  for (int s = 0; s < 3; ++s) {
    k_convT_in_scale<<<kDim, 256, 0, st>>>(c->up_v[s], c->up_g[s], kDim * kUpTaps, c->up_scale[s]);
    k_convT_reorder<<<g, 256, 0, st>>>(c->up_v[s], c->up_w[s]);
  }
  k_conv_out_scale<<<1, 256, 0, st>>>(c->out_v, c->out_g, kPatch, kDim * kOutTaps, c->out_scale);
  k_conv_reorder<<<g, 256, 0, st>>>(c->out_v, kPatch, kDim, kOutTaps, kPatchPad, kDim, c->out_w);
  h->launches += 14;
  CK(cudaGetLastError());
  CK(cudaStreamSynchronize(st));
  c->prepared = true;
  return VX_OK;
}

// Work buffers and operand tensor maps for up to `frames` frames (grown on demand).
int codec_work(vx_handle* h, int frames) {
  using namespace codec;
  CodecState* c = h->codec;
  if (frames <= c->cap) return VX_OK;
  const int cap = std::max(frames, std::min(2 * c->cap, kCodecMaxFrames));
  const size_t R = 8 * (size_t)cap;
  const size_t ws_floats = (size_t)h->num_sms * kCodecBN * tc::kBM;
  const size_t bytes = R * kDim * 4 + R * 2 * kHidden * 4 + ws_floats * 4 + (size_t)cap * kInCh * 4 +
                       R * kPatch * 4 + 2 * R * kOutTaps * kDim * 2 + (size_t)cap * 37 * 4 + 256 * 16;
  CK(cudaStreamSynchronize(h->stream));
  if (c->work) cudaFree(c->work);
  c->work = nullptr;
  c->cap = 0;
  if (cudaMalloc(&c->work, bytes) != cudaSuccess)
    return h->fail(VX_E_NOMEM, "codec work buffers for %d frames (%.2f GB)", cap, bytes / 1e9);
  uint8_t* cur = (uint8_t*)c->work;
  c->cur = (float*)carve(cur, R * kDim * 4);
  c->y = (float*)carve(cur, R * 2 * kHidden * 4);
  c->ws = (float*)carve(cur, ws_floats * 4);
  c->ws_floats = ws_floats;
  c->concat = (float*)carve(cur, (size_t)cap * kInCh * 4);
  c->audio = (float*)carve(cur, R * kPatch * 4);
  c->hi = (__half*)carve(cur, R * kOutTaps * kDim * 2);
  c->lo = (__half*)carve(cur, R * kOutTaps * kDim * 2);
  c->sem = (uint32_t*)carve(cur, (size_t)cap * 4);
  c->ac = (uint32_t*)carve(cur, (size_t)cap * 36 * 4);
  int rc;
  for (int i = 0; i < 5; ++i) {
    const int K = kCodecKs[i];
    if ((rc = encode_f16_2d(h, &c->xhi[i], c->hi, K, (long long)R, (long long)K * 2, tc::kBK, kCodecBN))) return rc;
    if ((rc = encode_f16_2d(h, &c->xlo[i], c->lo, K, (long long)R, (long long)K * 2, tc::kBK, kCodecBN))) return rc;
  }
  c->cap = cap;
  return VX_OK;
}

int codec_gemm(vx_handle* h, const CUtensorMap& w, int K, float* y, long long ldy, int M, int N) {
  CodecState* c = h->codec;
  const int ki = codec_kidx(K);
  if (ki < 0) return h->fail(VX_E_INVALID, "codec GEMM K %d", K);
  return run_tc_gemm_ws<kCodecBN>(h, w, c->xhi[ki], c->xlo[ki], y, ldy, M, N, K, 0, c->ws, c->ws_floats);
}

int codec_row(vx_handle* h, int n, const float* y, long long ldy, const __half* scale, const float* fscale, int residual,
              int out, const __half* norm_w, const float* op_scale) {
  CodecState* c = h->codec;
  codec::RowParams p{};
  p.y = y; p.ldy = ldy; p.scale = scale; p.fscale = fscale; p.residual = residual; p.cur = c->cur; p.n_rows = n;
  p.out = out; p.norm_w = norm_w; p.op_scale = op_scale; p.hi = c->hi; p.lo = c->lo;
  CK(launch(h, codec::k_codec_row, dim3(n), dim3(256), 0, p));
  return VX_OK;
}

// Copies `n` floats of a device buffer into the debug output at *off (if any).
int codec_dump(vx_handle* h, float* out, size_t& off, const float* src, size_t n) {
  if (!out) return VX_OK;
  CK(cudaMemcpyAsync(out + off, src, n * 4, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  off += n;
  return VX_OK;
}

int codec_run(vx_handle* h, const uint32_t* sem, const uint32_t* ac, int T, float* audio, float* dbg) {
  using namespace codec;
  CodecState* c = h->codec;
  int rc;
  if ((rc = codec_work(h, T))) return rc;
  CK(cudaMemcpyAsync(c->sem, sem, (size_t)T * 4, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(c->ac, ac, (size_t)T * 36 * 4, cudaMemcpyHostToDevice, h->stream));
  size_t off = 0;
  const long long nin = (long long)T * kInTaps * kInChPad;
  CK(launch(h, k_codec_embed, dim3((unsigned)std::min<long long>((nin + 255) / 256, 8L * h->num_sms)), dim3(256), 0,
            (const uint32_t*)c->sem, (const uint32_t*)c->ac, (const __half*)c->cb, T, c->concat, c->hi, c->lo));
  if ((rc = codec_gemm(h, c->m_in, kInTaps * kInChPad, c->y, kDim, kDim, T))) return rc;
  if ((rc = codec_row(h, T, c->y, kDim, nullptr, c->in_scale, 0, kOpNorm, c->layers[0].attn_norm, nullptr))) return rc;
  if ((rc = codec_dump(h, dbg, off, c->concat, (size_t)T * kInCh))) return rc;
  if ((rc = codec_dump(h, dbg, off, c->cur, (size_t)T * kDim))) return rc;
  for (int s = 0; s < 4; ++s) {
    const int N = T << s, W = 2 << s;
    for (int l = 0; l < 2; ++l) {
      const CodecLayer& L = c->layers[2 * s + l];
      if ((rc = codec_gemm(h, L.m_wqkv, kDim, c->y, 3 * kDim, 3 * kDim, N))) return rc;
      CK(launch(h, k_codec_qknorm, dim3((unsigned)(N * 2)), dim3(256), 0, c->y, N, (const __half*)L.q_norm,
                (const __half*)L.k_norm));
      CK(launch(h, k_codec_attn, dim3((unsigned)N), dim3(256), 0, (const float*)c->y, N, W, c->hi, c->lo));
      if ((rc = codec_gemm(h, L.m_wo, kDim, c->y, kDim, kDim, N))) return rc;
      if ((rc = codec_row(h, N, c->y, kDim, L.attn_scale, nullptr, 1, kOpNorm, L.ffn_norm, nullptr))) return rc;
      if ((rc = codec_gemm(h, L.m_w13, kDim, c->y, 2 * kHidden, 2 * kHidden, N))) return rc;
      const long long ng = (long long)N * kHidden;
      CK(launch(h, tc::k_tb_swiglu_split, dim3((unsigned)std::min<long long>((ng + 255) / 256, 8L * h->num_sms)),
                dim3(256), 0, (const float*)c->y, N, kHidden, c->hi, c->lo));
      if ((rc = codec_gemm(h, L.m_w2, kHidden, c->y, kDim, kDim, N))) return rc;
      if (l == 0)
        rc = codec_row(h, N, c->y, kDim, L.ffn_scale, nullptr, 1, kOpNorm, c->layers[2 * s + 1].attn_norm, nullptr);
      else if (s < 3)
        rc = codec_row(h, N, c->y, kDim, L.ffn_scale, nullptr, 1, kOpConvT, nullptr, c->up_scale[s]);
      else
        rc = codec_row(h, N, c->y, kDim, L.ffn_scale, nullptr, 1, kOpOutConv, nullptr, nullptr);
      if (rc) return rc;
    }
    if ((rc = codec_dump(h, dbg, off, c->cur, (size_t)N * kDim))) return rc;
    if (s < 3) {
      for (int par = 0; par < 2; ++par)
        if ((rc = codec_gemm(h, c->m_up[s][par], 2 * kDim, c->y + par * kDim, 2 * kDim, kDim, N))) return rc;
      if ((rc = codec_dump(h, dbg, off, c->y, (size_t)2 * N * kDim))) return rc;
      if ((rc = codec_row(h, 2 * N, c->y, kDim, nullptr, nullptr, 0, kOpNorm, c->layers[2 * s + 2].attn_norm,
                          nullptr)))
        return rc;
    }
  }
  const int NO = 8 * T;
  if ((rc = codec_gemm(h, c->m_out, kOutTaps * kDim, c->y, kPatch, kPatch, NO))) return rc;
  const long long na = (long long)NO * kPatch;
  CK(launch(h, k_codec_audio, dim3((unsigned)std::min<long long>((na + 255) / 256, 8L * h->num_sms)), dim3(256), 0,
            (const float*)c->y, (long long)kPatch, (const float*)c->out_scale, NO, c->audio));
  if ((rc = codec_dump(h, dbg, off, c->audio, (size_t)na))) return rc;
  if (audio) CK(cudaMemcpyAsync(audio, c->audio, (size_t)na * 4, cudaMemcpyDeviceToHost, h->stream));
  return finish(h);
}

void codec_destroy(vx_handle* h) {
  if (!h->codec) return;
  if (h->codec->work) cudaFree(h->codec->work);
  if (h->codec->arena) cudaFree(h->codec->arena);
  delete h->codec;
  h->codec = nullptr;
}

}  // namespace

extern "C" {

int vx_codec_decode(vx_handle* h, const uint32_t* sem, const uint32_t* ac, int32_t n_frames, float* audio) {
  if (!h || !sem || !ac || !audio) return VX_E_INVALID;
  if (!h->codec) return h->fail(VX_E_STATE, "engine created without the codec decoder");
  if (!h->codec->prepared) return h->fail(VX_E_STATE, "Engine not initialized. Call init() and loadWeights() first.");
  if (n_frames < 1 || n_frames > kCodecMaxFrames)
    return h->fail(VX_E_RANGE, "%d frames outside [1, %d]", n_frames, kCodecMaxFrames);
  CK(cudaSetDevice(h->dev));
  return codec_run(h, sem, ac, n_frames, audio, nullptr);
}

size_t vx_codec_debug_size(int32_t n_frames) {
  return n_frames < 1 ? 0 : (size_t)n_frames * (codec::kInCh + 30 * codec::kDim + 8 * codec::kPatch);
}

int vx_codec_debug(vx_handle* h, const uint32_t* sem, const uint32_t* ac, int32_t n_frames, float* out, size_t n_out) {
  if (!h || !sem || !ac || !out) return VX_E_INVALID;
  if (!h->codec) return h->fail(VX_E_STATE, "engine created without the codec decoder");
  if (!h->codec->prepared) return h->fail(VX_E_STATE, "Engine not initialized. Call init() and loadWeights() first.");
  if (n_frames < 1 || n_frames > kCodecMaxFrames)
    return h->fail(VX_E_RANGE, "%d frames outside [1, %d]", n_frames, kCodecMaxFrames);
  if (n_out != vx_codec_debug_size(n_frames))
    return h->fail(VX_E_INVALID, "debug buffer holds %zu floats, %zu needed", n_out, vx_codec_debug_size(n_frames));
  CK(cudaSetDevice(h->dev));
  return codec_run(h, sem, ac, n_frames, nullptr, out);
}

}  // extern "C"
