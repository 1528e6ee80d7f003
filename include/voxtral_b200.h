/* voxtral_b200.h — C ABI of the B200-native Voxtral decode path.
 *
 * This is the boundary a host binding (Node N-API / FFI, Python ctypes, C, C++)
 * loads in place of the reference's WebGPU engine internals.  The reference's
 * public TypeScript class VoxtralEngine (svenflow/webgpu-voxtral, src/engine.ts:291)
 * keeps its signatures; its methods call these functions.  Each declaration cites
 * the reference interface it replaces (file:line in the reference tree).
 *
 * Conventions (mirroring src/engine.ts):
 *  - Ownership: the library owns all device memory.  Caller arrays are copied in
 *    during the call; output arrays are caller-allocated host memory filled before
 *    the call returns (src/engine.ts:2436-2451 copies caller arrays likewise).
 *  - Errors: every int-returning function returns VX_OK (0) or a negative VX_E_*
 *    code, and vx_last_error() describes the last failure of that handle (the
 *    reference throws `new Error(...)`, e.g. src/engine.ts:314-320, 666, 2425).
 *    No C++ exception crosses this boundary.
 *  - Threading: one handle per host thread; calls on one handle are serialised by
 *    the caller (the reference engine is single-threaded, src/engine.ts:299).
 *  - Values: weights are IEEE binary16 bit patterns, activations f32, token ids
 *    int32, codes uint32 (semantic 0..8193, acoustic 2..22).
 */
#ifndef VOXTRAL_B200_H
#define VOXTRAL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VX_OK 0
#define VX_E_INVALID (-1) /* bad argument (null pointer, size, name)           */
#define VX_E_CUDA (-2)    /* a CUDA runtime / driver call failed                 */
#define VX_E_STATE (-3)   /* not ready: weights not loaded, slot not prefilled   */
#define VX_E_RANGE (-4)   /* token / code / position / slot out of range         */
#define VX_E_NOMEM (-5)   /* device allocation failed                            */
#define VX_E_NCCL (-6)    /* NCCL missing or a collective failed                 */
#define VX_E_DEVICE (-7)  /* a kernel reported a device-side error (bounded wait
                             expired, index out of range); the handle stays usable */

typedef struct vx_handle vx_handle;

/* VoxtralConfig (src/types.ts:10-37, defaultConfig :70-97) + EngineOptions
 * (src/engine.ts:213-219) + the B200 engine's own options. */
typedef struct vx_config {
  /* backbone (BackboneConfig) */
  int32_t dim, n_layers, head_dim, hidden_dim, n_heads, n_kv_heads, vocab_size;
  float rope_theta, norm_eps;
  /* acoustic (flow-matching) transformer (FMTransformerConfig) */
  int32_t fm_n_layers, fm_nfe;
  float fm_cfg_alpha;
  int32_t fm_n_acoustic, fm_semantic_vocab, acoustic_levels;
  int32_t audio_vocab; /* rows of audio_codebook_embeddings (9088) */
  /* engine */
  int32_t max_seq_len; /* EngineOptions.maxSeqLen (default 4096) */
  int32_t max_slots;   /* utterance slots that can decode concurrently */
  int32_t max_frames;  /* capacity of each slot's on-device code ring */
  int32_t max_voice_rows;
  int32_t enable_fm;   /* allocate the acoustic transformer */
  int32_t device;      /* CUDA device ordinal */
  int32_t tp_size, tp_rank; /* tensor parallelism (1 = off) */
  int32_t enable_codec;     /* allocate the codec decoder (CodecConfig, src/types.ts:39-62) */
} vx_config;

/* defaultConfig (src/types.ts:70-122) with maxSeqLen 4096, 1 slot. */
void vx_default_config(vx_config* cfg);

/* new VoxtralEngine(options) + init() (src/engine.ts:301-344): selects the
 * device, allocates weights, KV cache and work buffers. */
int vx_create(const vx_config* cfg, vx_handle** out);

/* destroy() (src/engine.ts:2621-2633). */
void vx_destroy(vx_handle* h);

/* Message of the last failure on this handle ("" if none). */
const char* vx_last_error(const vx_handle* h);

/* Replaces loadWeights()/loadWeightsFromHF() (src/engine.ts:539-586) for the
 * benchmark: fills every tensor with the synthetic values of vx_rng.h
 * (matrices N(0,0.02) in f16 from stream fnv1a(name) of `seed`, norm gains 1). */
int vx_init_random_weights(vx_handle* h, uint64_t seed);

/* One tensor of organizeWeights (src/engine.ts:659-743) by its checkpoint name
 * (e.g. "layers.3.attention.wk.weight"), row-major f16 bits, full (unsharded)
 * shape; the library keeps the shard of its tp_rank.  Returns VX_E_INVALID for an
 * unknown name or a wrong element count. */
int vx_load_tensor(vx_handle* h, const char* name, const uint16_t* f16, size_t n_elems);

/* The checkpoint tensor names the engine holds (the keys organizeWeights expects,
 * src/engine.ts:659-743), sorted and newline-separated into buf (NUL-terminated, cut at
 * len).  Returns the bytes needed, terminator included. */
size_t vx_tensor_names(const vx_handle* h, char* buf, size_t len);

/* One checkpoint tensor in its stored dtype (0 F16, 1 BF16, 2 F32, little endian, full
 * tensor as in vx_load_tensor), converted to F16 on the GPU with the reference loader's
 * bit rules: convertBF16toF16 (src/weights.ts:94-138) and float32ToFloat16
 * (src/weights.ts:222-232).  The first call allocates a 64 MB staging buffer.  Replaces
 * loadTensorFromSafetensors / loadFromSafetensors (src/weights.ts:182-215, :491-669). */
int vx_load_tensor_typed(vx_handle* h, const char* name, const void* data, int32_t dtype, size_t n_elems);

/* Completion of loadWeights() after the vx_load_tensor calls: builds the derived
 * frame-independent tables (time_projection of the 7 Euler times). */
int vx_mark_weights_loaded(vx_handle* h);

/* Element count of a named tensor (0 if unknown). */
size_t vx_tensor_numel(const vx_handle* h, const char* name);

/* Copy a named tensor back (f16 bits) — used to verify loaded/synthetic weights. */
int vx_read_tensor(vx_handle* h, const char* name, uint16_t* out, size_t n_elems);

/* reset() (src/engine.ts:2323-2327): position 0, frame 0 for one slot. */
int vx_reset(vx_handle* h, int32_t slot);

int vx_get_position(vx_handle* h, int32_t slot, int32_t* pos);

/* Token-by-token prefill of generate() (src/engine.ts:2457-2472): prompt
 * positions [audio_start, audio_start+audio_count) take the rows of `voice`
 * ([audio_count][dim] f32, REPLACING the token embedding, :843-854); every other
 * position embeds tokens[i].  Starts at the slot's current position. */
int vx_prefill(vx_handle* h, int32_t slot, const int32_t* tokens, int32_t n_tokens, int32_t audio_start,
               int32_t audio_count, const float* voice);

/* backboneStep (src/engine.ts:814-1042) as exposed by backboneStepAndRead /
 * debugBackboneStepFull (:2333-2358): one token through the backbone at the
 * slot's position; embed = tok_embeddings[token] (or audio_embeddings[token] if
 * use_audio_embedding), or the caller's row `embed` [dim] if non-null.
 * normed_out [dim] (nullable) receives the final-norm output that feeds the FM.
 * argmax_out (nullable) runs the tied LM head + argmax (:1017-1041). */
int vx_backbone_step(vx_handle* h, int32_t slot, int32_t token, int32_t use_audio_embedding, const float* embed,
                     float* normed_out, int32_t* argmax_out);

/* The frame-loop backbone step of generate() (src/engine.ts:2499-2541): the
 * input is multiCodebookEmbed(semantic, acoustic[36]) (src/shaders.ts:1878-1917). */
int vx_backbone_step_codes(vx_handle* h, int32_t slot, uint32_t semantic_code, const uint32_t* acoustic_codes,
                           float* normed_out);

/* fmForward (src/engine.ts:1240-1380) on the slot's current normed state, as
 * exposed by debugFMStep(noise) / fmStepAndRead (:2363-2398).  noise [36]
 * (nullable: the slot's seeded stream).  Outputs (all nullable): semantic logits
 * [semantic_vocab], the semantic code chosen from them (index 0 and >= 8194 masked,
 * :2559-2563; masked argmax, or top-p sampling when vx_set_sampling enabled it), acoustic
 * codes [36], x_final [36]. */
int vx_fm_step(vx_handle* h, int32_t slot, const float* noise, float* semantic_logits, uint32_t* semantic_code,
               uint32_t* acoustic_codes, float* x_final);

/* debugBackboneLayerByLayer (src/engine.ts:2106-2287) at the slot's position for
 * tok_embeddings[token]: out [(4*n_layers+3)][dim] = embed, per layer {attn_norm,
 * attn_out (hidden after the attention residual), ffn_norm, ffn_out}, final_norm,
 * hidden.  Advances the position like the reference.  The step runs in the persistent
 * decode kernel that vx_decode runs (option persistent_decode, on by default), which
 * records these tensors as it goes; with that option off, in the per-op kernels. */
int vx_debug_layers(vx_handle* h, int32_t slot, int32_t token, float* out);

/* Device-resident frame loop of generate() (src/engine.ts:2498-2585) with the
 * host round trips removed: n_frames frames starting at the slot's current frame,
 * each one CUDA graph.  with_fm = 1: frame f > 0 embeds frame f-1's codes, runs the
 * backbone, then fmForward with the slot's noise stream and the slot's semantic
 * selection (masked argmax or top-p, vx_set_sampling; frame 0 runs the FM on the state
 * left by the AUDIO kick).  with_fm = 0 (backbone-only):
 * frame 0 is the AUDIO kick (token 24, text embedding, :2481-2487) and frame f > 0
 * embeds the synthetic codes of frame f-1.  Asynchronous: returns after enqueueing;
 * read results with vx_read_codes / vx_read_normed after vx_synchronize. */
int vx_decode(vx_handle* h, int32_t slot, int32_t n_frames, int32_t with_fm);

/* vx_decode(slot, n_frames, 0) that also records the per-layer tensors of frame
 * record_frame of this call, in the layout of vx_debug_layers, into out
 * [(4*n_layers+3)][dim] (debugBackboneLayerByLayer, src/engine.ts:2106-2287, taken inside
 * the benchmarked frame loop instead of as a separate step).  Synchronous. */
int vx_decode_record(vx_handle* h, int32_t slot, int32_t n_frames, int32_t record_frame, float* out);

/* Batched backbone-only decode: n_frames frames of slots [slot0, slot0 + n_slots) in
 * lockstep, each slot at its own position with its own synthetic feedback codes
 * (vx_set_streams), exactly as vx_decode(slot, n_frames, 0) would produce them one slot
 * at a time (frame 0 of a slot is the AUDIO kick).  The reference decodes one utterance
 * per engine (generate() frame loop, src/engine.ts:2498-2585); here every projection of
 * a step is one tensor-core GEMM over the n_slots rows, so the weights stream once per
 * step for all slots.  Needs tp_size 1; n_slots <= 512. */
int vx_decode_batch(vx_handle* h, int32_t slot0, int32_t n_slots, int32_t n_frames);

/* Synthetic long context (long-context benchmark configuration): K/V of positions
 * [0, n_positions) of every layer of the slot = f16(N(0,1)) from the counter-based
 * generator (stream (seed, 2*layer + kv), counter pos*1024 + head*128 + d), then the
 * slot's position = n_positions and frame = 0, as if a prompt of that length had been
 * prefilled.  No counterpart in the reference (its prefill is the only way to fill
 * the cache, src/engine.ts:2457-2472); the CPU oracle's orc_fill_kv draws the same
 * values in f32. */
int vx_fill_kv(vx_handle* h, int32_t slot, int32_t n_positions, uint64_t seed);

/* Seeds of the slot's synthetic streams (FM noise, backbone-only feedback codes);
 * `utt` selects the utterance stream of vx_rng.h. */
int vx_set_streams(vx_handle* h, int32_t slot, uint64_t noise_seed, uint64_t codes_seed, int32_t utt);

/* Semantic code selection of the slot's FM frames.  mode 0 (default): masked argmax
 * (index 0 and >= 8194 masked, ties to the lowest index).  mode 1: the reference's
 * temperature + top-p sampling, sampleTopP(semLogits, 0.9, 0.8) of generate()
 * (src/engine.ts:247-289, called at :2565 on the logits masked at :2559-2563), run on
 * the device inside the FM graph; the uniform draw of frame f is counter f of the
 * stream (seed, "sample") of vx_rng.h in place of Math.random.  Every TP rank must
 * be given the same seed. */
int vx_set_sampling(vx_handle* h, int32_t slot, int32_t mode, double top_p, double temperature, uint64_t seed);

/* Codes of frames [frame0, frame0+n): out [n][37] = semantic, 36 acoustic. */
int vx_read_codes(vx_handle* h, int32_t slot, int32_t frame0, int32_t n, uint32_t* out);
/* Final-norm state of frames [frame0, frame0+n): out [n][dim]. */
int vx_read_normed(vx_handle* h, int32_t slot, int32_t frame0, int32_t n, float* out);

/* Save / restore a slot's decode state (position, frame, codes, normed state):
 * a checkpoint taken after prefill lets a benchmark replay the same decode. */
int vx_checkpoint(vx_handle* h, int32_t slot);
int vx_rewind(vx_handle* h, int32_t slot);

/* Use the caller's CUDA stream (cudaStream_t as void*, e.g. torch's current
 * stream) for all later work; NULL restores the handle's own stream. */
int vx_set_stream(vx_handle* h, void* stream);
int vx_synchronize(vx_handle* h);

/* Engine options.  Returns VX_E_INVALID for an unknown name or value, VX_E_STATE /
 * VX_E_RANGE when the handle cannot take the value.  No counterpart in the reference
 * (EngineOptions, src/engine.ts:213-219, has none of these).
 *   "persistent_decode"  1 (default where cooperative launch exists and tp_size <= 4):
 *                        vx_decode, token-by-token vx_prefill and vx_debug_layers run
 *                        the persistent decode kernel; 0: one CUDA graph of per-op kernels
 *                        per step (always at tp_size 8, where 1 returns VX_E_STATE).
 *   "batched_prefill"    1 (default, tp_size 1): vx_prefill runs the prompt through
 *                        tensor-core GEMMs in batches of up to 512 positions; 0: token
 *                        by token, as the reference (src/engine.ts:2457-2472).
 *   "residual_handoff"   1 (default): the persistent kernel's o_proj / down epilogues hand
 *                        the residual stream to the next phase as tagged 8-byte words
 *                        that the next phase polls (a one-rank form of its tensor-parallel
 *                        all-reduce), so that phase starts without a grid barrier; 0: the
 *                        epilogues add into the residual and the next phase waits at a
 *                        grid barrier (tp_size 1 only).
 *   "l2_prefetch_tiles"  0-32 (default 2): weight tiles the persistent kernel prefetches
 *                        into L2 ahead of its shared-memory ring.
 *   "early_kv_pair"      1 (default): the persistent kernel copies each CTA's first pair
 *                        of K/V pages into shared memory while the QKV phase runs (the
 *                        current position's row is patched in afterwards); 0: the copy
 *                        starts after the barrier that ends the QKV phase.
 *   "wait_limit"        polls before a wait of the persistent kernel on a grid barrier
 *                        or on a tensor-parallel peer's all-reduce words gives up and the
 *                        call returns VX_E_DEVICE (0, default: 2^27 / 2^24 polls, seconds).
 *   "tp_loopback"        1 (test support, tp_size > 1, one process): every peer receive
 *                        buffer is this handle's own, so the other ranks' all-reduce words
 *                        never arrive; a decode then ends in VX_E_DEVICE once wait_limit
 *                        expires, which exercises the failure path of a lost rank without
 *                        a second GPU. */
int vx_set_option(vx_handle* h, const char* name, int64_t value);

/* Kernel launches enqueued by this handle since creation (graph launches count
 * the kernels they contain). */
int64_t vx_launch_count(const vx_handle* h);

/* Measurement: captures three variants of one backbone step of the slot as CUDA
 * graphs — the full step, only its weight-streaming GEMVs, only its attention
 * kernels — and times `reps` back-to-back launches of each with CUDA events on the
 * handle's stream.  out_ms[3] = ms per step of {full, GEMV chain, attention chain};
 * out_bytes[1] = algorithmic bytes the GEMVs of one step move.  The slot's state is
 * restored afterwards.  No counterpart in the reference (its benchmark times whole
 * submits with the CPU clock, src/benchmark.ts:288-292). */
int vx_profile_step(vx_handle* h, int32_t slot, int32_t reps, float* out_ms, double* out_bytes);

/* Phase tracing of the persistent decode kernel (the reference records stage
 * wall-clock times only, src/engine.ts:2428-2601).  mode 1 arms tracing for the next
 * persistent launch on this handle; mode 0 copies the trace out, indexed
 * [cta][step < 2][phase][8]: %globaltimer stamps (ns) {0: consumers released, 1:
 * consumers done, 2: epilogue arrival, 3: consumers' prologue done}, then SM cycles spent
 * waiting {4: consumer warp 0 on weight stages, 5: consumer warp 0 on reduction slots,
 * 6: epilogue warp on reduction results}, 7 unused; mode 2 only reports the dimensions.
 * dims (nullable) receives {ctas, steps, phases, 8}. */
int vx_trace(vx_handle* h, int32_t mode, uint64_t* out, size_t n_elems, int32_t* dims);

/* Test support for the tensor-core GEMM of the batched paths (tcgen05 / TMEM,
 * k_gemm.cuh), which replaces matvecF16 (src/shaders.ts:21-71) when a batch of
 * tokens shares a layer (batched prefill; the reference prefills token by token,
 * src/engine.ts:2457-2472).  No counterpart in the reference.  Computes Y = X W^T,
 * then Y += X W^T, for seeded random W f16 [M,K] ~ N(0, 0.02) and X f32 [N,K] ~ N(0,1),
 * with tile width bn (16, 64, 128 or 256) and at most max_splits K splits, and compares
 * each pass with an f32 CUDA-core product of the same operands:
 * out_rel_err[2] = max|Y - Yref| / max|Yref| of the two passes. */
int vx_selftest_gemm(vx_handle* h, int32_t M, int32_t N, int32_t K, int32_t bn, int32_t max_splits, uint64_t seed,
                     double* out_rel_err);

/* Codec decoder, codecDecode(semanticCodes, acousticCodes) (src/engine.ts:1402-1713):
 * sem[n_frames] semantic codes and ac[n_frames * 36] acoustic codes (as generate()
 * produces them) -> audio[n_frames * 1920] f32 samples at 24 kHz.  VQ lookup (the
 * raw semantic code indexes the 8192-entry codebook; codes >= 8192 give a zero row)
 * + FSQ dequantisation, the causal input convolution, 4 stages of 2 transformer
 * layers (windowed ALiBi attention, windows 2/4/8/16) with a stride-2 transposed
 * convolution after stages 0-2, and the 7-tap output convolution.  1 <= n_frames <=
 * 8192.  Needs enable_codec and loaded weights. */
int vx_codec_decode(vx_handle* h, const uint32_t* sem, const uint32_t* ac, int32_t n_frames, float* audio);

/* debugCodecDecode (src/engine.ts:1719-1975): the same decode with its intermediates,
 * concatenated in this order into out[vx_codec_debug_size(n_frames)] (T = n_frames):
 *   concat [T][292] (vq_embed | fsq_dequant), after_input_conv [T][1024],
 *   after_stage0_transformer [T][1024], after_stage0_conv_up [2T][1024],
 *   after_stage1_transformer [2T][1024], after_stage1_conv_up [4T][1024],
 *   after_stage2_transformer [4T][1024], after_stage2_conv_up [8T][1024],
 *   after_stage3_transformer [8T][1024], audio [8T][240]. */
size_t vx_codec_debug_size(int32_t n_frames);
int vx_codec_debug(vx_handle* h, const uint32_t* sem, const uint32_t* ac, int32_t n_frames, float* out, size_t n_out);

/* Test support for the device top-p sampler (sampleTopP, src/engine.ts:247-289): the
 * logits[n] (n <= 16384) with indices outside [valid_lo, valid_hi) masked to -Inf, one
 * sample per uniform draw u[i] in [0, 1) (the reference's Math.random()), out[i] = index. */
int vx_selftest_top_p(vx_handle* h, const float* logits, int32_t n, int32_t valid_lo, int32_t valid_hi, double top_p,
                      double temperature, const double* u, int32_t n_draws, int32_t* out);

/* Tensor parallelism over NCCL (batch-1 latency, heads and FFN columns
 * sharded): the unique id comes from vx_nccl_unique_id on rank 0 and is shared by
 * the host (e.g. torch.distributed).  nccl_lib: path of libnccl.so.2 (NULL: the
 * default search path). */
int vx_nccl_unique_id(const char* nccl_lib, uint8_t out[128]);
int vx_tp_init(vx_handle* h, const char* nccl_lib, const uint8_t id[128]);

/* Tensor parallelism inside the persistent decode kernel (vx_decode / vx_prefill with
 * tp_size > 1): the o_proj and down all-reduces of every layer run inside the kernel over
 * peer memory (NVLink), instead of as NCCL calls between kernels.  Each rank exports the
 * CUDA IPC handle (64 bytes) of its receive buffer with vx_tp_p2p_handle, the host
 * gathers the tp_size handles in rank order (e.g. torch.distributed), and every rank
 * passes them to vx_tp_p2p_open, then all ranks meet at a host barrier before their
 * first decode.  All ranks must issue the same sequence of decode/prefill calls.  The
 * reference runs on one device (src/engine.ts:814-1042); this is its step split over
 * tp_size GPUs.  The persistent kernel serves tp_size 2 and 4; at tp_size 8 the handle
 * keeps the per-op kernels with NCCL all-reduces. */
int vx_tp_p2p_handle(vx_handle* h, uint8_t out[64]);
int vx_tp_p2p_open(vx_handle* h, const uint8_t* handles /* [tp_size][64] */);

/* LM-head argmax for callers that cannot allocate device memory.  No counterpart in
 * the reference.  Callers that cannot call cudaMalloc (a real-time audio callback, where
 * cudaMalloc may synchronise the device and block; a host framework that owns all
 * device memory through its own arena) cannot create a vx_handle, but can pass their
 * own device buffers here.  Computes *out_index = argmax_r (W[r,:] . x) (maximum value,
 * lowest index on ties) and *out_value = that maximum (nullable), the same greedy
 * choice as vx_backbone_step's argmax_out, in one kernel that allocates nothing.
 * A NaN product never wins; if every product is NaN, *out_index = -1 and *out_value
 * = NaN.
 * weight: device f16 bits [rows][dim], 16-byte aligned; x: device f32 [dim];
 * out_index / out_value: device; stream: cudaStream_t (NULL = default stream);
 * err (nullable): receives a message.  Limits: rows <= 2,097,152, dim a multiple of 8
 * and <= 16,384 (VX_E_RANGE beyond them).  Its scratch is a 65,792-byte static device
 * array that every GPU loading the library holds until the process exits; the first
 * call on a device looks up that array's address (call it once before any stream
 * capture) and later calls reuse it, so the entry point must not be called on a device
 * after cudaDeviceReset of that device.  All calls on a device share the array, so calls
 * that overlap on the GPU race; calls ordered on one stream do not. */
int vx_lm_head_argmax_noalloc(const uint16_t* weight, const float* x, int32_t rows, int32_t dim, int32_t* out_index,
                              float* out_value, void* stream, char* err, size_t err_len);

#ifdef __cplusplus
}
#endif
#endif /* VOXTRAL_B200_H */
