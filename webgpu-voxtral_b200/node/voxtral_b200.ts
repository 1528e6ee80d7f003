// voxtral_b200.ts — Node binding of libvoxtral_b200.so (include/voxtral_b200.h) for the
// reference's TypeScript engine.
//
// The reference's VoxtralEngine (src/engine.ts:291) keeps its public signatures; with
// `options.backend === 'b200'` its GPU internals (backboneStep :814-1042,
// fmTransformerPass :1057-1225, fmForward :1240-1380, codecDecode :1402-1713) call this
// module instead of WebGPU.  It uses koffi (a pure FFI, no native build step); an N-API
// addon wrapping the same C calls works the same way.
//
// UNTESTED in this repository's build container: Node, npm and tsc are not installed
// there.  The Python binding (engine.py) binds the same symbols and is what the tests run.
import koffi from 'koffi';

const lib = koffi.load(process.env.VOXTRAL_B200_LIB ?? 'libvoxtral_b200.so');

export const VX_OK = 0;
export const VX_E_DEVICE = -7;

const vx_config = koffi.struct('vx_config', {
  dim: 'int32', n_layers: 'int32', head_dim: 'int32', hidden_dim: 'int32', n_heads: 'int32',
  n_kv_heads: 'int32', vocab_size: 'int32', rope_theta: 'float', norm_eps: 'float',
  fm_n_layers: 'int32', fm_nfe: 'int32', fm_cfg_alpha: 'float', fm_n_acoustic: 'int32',
  fm_semantic_vocab: 'int32', acoustic_levels: 'int32', audio_vocab: 'int32',
  max_seq_len: 'int32', max_slots: 'int32', max_frames: 'int32', max_voice_rows: 'int32',
  enable_fm: 'int32', device: 'int32', tp_size: 'int32', tp_rank: 'int32', enable_codec: 'int32',
});
koffi.opaque('vx_handle');

// One entry per declaration of include/voxtral_b200.h.
export const vx = {
  default_config: lib.func('void vx_default_config(_Out_ vx_config *cfg)'),
  create: lib.func('int vx_create(const vx_config *cfg, _Out_ vx_handle **out)'),
  destroy: lib.func('void vx_destroy(vx_handle *h)'),
  last_error: lib.func('const char *vx_last_error(const vx_handle *h)'),
  init_random_weights: lib.func('int vx_init_random_weights(vx_handle *h, uint64_t seed)'),
  load_tensor: lib.func('int vx_load_tensor(vx_handle *h, const char *name, const uint16_t *f16, size_t n)'),
  tensor_names: lib.func('size_t vx_tensor_names(const vx_handle *h, _Out_ char *buf, size_t len)'),
  load_tensor_typed: lib.func('int vx_load_tensor_typed(vx_handle *h, const char *name, const void *data, int32_t dtype, size_t n)'),
  mark_weights_loaded: lib.func('int vx_mark_weights_loaded(vx_handle *h)'),
  tensor_numel: lib.func('size_t vx_tensor_numel(const vx_handle *h, const char *name)'),
  read_tensor: lib.func('int vx_read_tensor(vx_handle *h, const char *name, _Out_ uint16_t *out, size_t n)'),
  reset: lib.func('int vx_reset(vx_handle *h, int32_t slot)'),
  get_position: lib.func('int vx_get_position(vx_handle *h, int32_t slot, _Out_ int32_t *pos)'),
  prefill: lib.func('int vx_prefill(vx_handle *h, int32_t slot, const int32_t *tok, int32_t n, int32_t a0, int32_t na, const float *voice)'),
  backbone_step: lib.func('int vx_backbone_step(vx_handle *h, int32_t slot, int32_t tok, int32_t useAudio, const float *emb, _Out_ float *normed, _Out_ int32_t *argmax)'),
  backbone_step_codes: lib.func('int vx_backbone_step_codes(vx_handle *h, int32_t slot, uint32_t sem, const uint32_t *ac, _Out_ float *normed)'),
  fm_step: lib.func('int vx_fm_step(vx_handle *h, int32_t slot, const float *noise, _Out_ float *logits, _Out_ uint32_t *sem, _Out_ uint32_t *ac, _Out_ float *xf)'),
  debug_layers: lib.func('int vx_debug_layers(vx_handle *h, int32_t slot, int32_t tok, _Out_ float *out)'),
  decode: lib.func('int vx_decode(vx_handle *h, int32_t slot, int32_t n, int32_t withFm)'),
  decode_record: lib.func('int vx_decode_record(vx_handle *h, int32_t slot, int32_t n, int32_t recordFrame, _Out_ float *out)'),
  decode_batch: lib.func('int vx_decode_batch(vx_handle *h, int32_t slot0, int32_t nSlots, int32_t n)'),
  fill_kv: lib.func('int vx_fill_kv(vx_handle *h, int32_t slot, int32_t nPos, uint64_t seed)'),
  set_streams: lib.func('int vx_set_streams(vx_handle *h, int32_t slot, uint64_t noiseSeed, uint64_t codesSeed, int32_t utt)'),
  set_sampling: lib.func('int vx_set_sampling(vx_handle *h, int32_t slot, int32_t mode, double topP, double temperature, uint64_t seed)'),
  read_codes: lib.func('int vx_read_codes(vx_handle *h, int32_t slot, int32_t f0, int32_t n, _Out_ uint32_t *out)'),
  read_normed: lib.func('int vx_read_normed(vx_handle *h, int32_t slot, int32_t f0, int32_t n, _Out_ float *out)'),
  checkpoint: lib.func('int vx_checkpoint(vx_handle *h, int32_t slot)'),
  rewind: lib.func('int vx_rewind(vx_handle *h, int32_t slot)'),
  set_stream: lib.func('int vx_set_stream(vx_handle *h, void *stream)'),
  synchronize: lib.func('int vx_synchronize(vx_handle *h)'),
  set_option: lib.func('int vx_set_option(vx_handle *h, const char *name, int64_t value)'),
  launch_count: lib.func('int64_t vx_launch_count(const vx_handle *h)'),
  codec_decode: lib.func('int vx_codec_decode(vx_handle *h, const uint32_t *sem, const uint32_t *ac, int32_t T, _Out_ float *audio)'),
  codec_debug_size: lib.func('size_t vx_codec_debug_size(int32_t T)'),
  codec_debug: lib.func('int vx_codec_debug(vx_handle *h, const uint32_t *sem, const uint32_t *ac, int32_t T, _Out_ float *out, size_t n)'),
  nccl_unique_id: lib.func('int vx_nccl_unique_id(const char *ncclLib, _Out_ uint8_t *out)'),
  tp_init: lib.func('int vx_tp_init(vx_handle *h, const char *ncclLib, const uint8_t *id)'),
  tp_p2p_handle: lib.func('int vx_tp_p2p_handle(vx_handle *h, _Out_ uint8_t *out)'),
  tp_p2p_open: lib.func('int vx_tp_p2p_open(vx_handle *h, const uint8_t *handles)'),
  profile_step: lib.func('int vx_profile_step(vx_handle *h, int32_t slot, int32_t reps, _Out_ float *ms, _Out_ double *bytes)'),
  trace: lib.func('int vx_trace(vx_handle *h, int32_t mode, _Out_ uint64_t *out, size_t n, _Out_ int32_t *dims)'),
  selftest_gemm: lib.func('int vx_selftest_gemm(vx_handle *h, int32_t M, int32_t N, int32_t K, int32_t bn, int32_t maxSplits, uint64_t seed, _Out_ double *err)'),
  selftest_top_p: lib.func('int vx_selftest_top_p(vx_handle *h, const float *logits, int32_t n, int32_t lo, int32_t hi, double topP, double temperature, const double *u, int32_t nDraws, _Out_ int32_t *out)'),
  lm_head_argmax_noalloc: lib.func('int vx_lm_head_argmax_noalloc(const uint16_t *w, const float *x, int32_t rows, int32_t dim, int32_t *outIndex, float *outValue, void *stream, _Out_ char *err, size_t errLen)'),
};

const DIM = 3072;

// The reference throws Error (src/engine.ts:314-320, 666, 2425); so does this binding.
export class VoxtralB200Error extends Error {
  constructor(public code: number, message: string) { super(`${message} [${code}]`); }
}

export interface TTSCodes { semanticCodes: number[]; acousticCodes: number[][]; }

// The GPU half of VoxtralEngine for one device (tp_size 1).  generate() keeps the
// reference's host logic (prompt, onFrame / onStage, EOS, TTSResult) and calls these.
export class B200Engine {
  private h: unknown = null;

  constructor(opts: { maxSeqLen?: number; maxFrames?: number; device?: number; nLayers?: number } = {}) {
    const cfg: Record<string, number> = {};
    vx.default_config(cfg);
    cfg.max_seq_len = opts.maxSeqLen ?? 4096;
    cfg.max_frames = opts.maxFrames ?? 2048;
    cfg.device = opts.device ?? 0;
    if (opts.nLayers) cfg.n_layers = opts.nLayers;
    const out = [null];
    const rc = vx.create(cfg, out);
    this.h = out[0];
    this.check(rc);
  }

  private check(rc: number) {
    if (rc !== VX_OK) throw new VoxtralB200Error(rc, this.h ? vx.last_error(this.h) : 'vx_create failed');
  }

  // loadWeights(): one call per checkpoint tensor (f16 bits, or dtype 1 = BF16, 2 = F32).
  loadTensor(name: string, data: Uint16Array | Float32Array, dtype = 0) {
    this.check(vx.load_tensor_typed(this.h, name, data, dtype, data.length));
  }
  finishLoading() { this.check(vx.mark_weights_loaded(this.h)); }
  loadRandomWeights(seed = 0) { this.check(vx.init_random_weights(this.h, BigInt(seed))); }

  reset() { this.check(vx.reset(this.h, 0)); }

  // generate() (src/engine.ts:2416-2616) minus its host-only parts.
  generate(tokens: number[], audioTokenStart: number, audioTokenCount: number,
           voiceEmbeddings: Float32Array | null, maxFrames = 500,
           onFrame?: (f: number, sem: number, ac: number[]) => boolean | void,
           sampling: { topP: number; temperature: number; seed: bigint } | null = { topP: 0.9, temperature: 0.8, seed: BigInt(Date.now()) }): TTSCodes {
    this.reset();
    if (sampling) this.check(vx.set_sampling(this.h, 0, 1, sampling.topP, sampling.temperature, sampling.seed));
    this.check(vx.prefill(this.h, 0, Int32Array.from(tokens), tokens.length, audioTokenStart, audioTokenCount,
                          voiceEmbeddings));
    this.check(vx.backbone_step(this.h, 0, 24, 0, null, null, null));   // AUDIO kick (:2481-2487)
    const semanticCodes: number[] = [];
    const acousticCodes: number[][] = [];
    const CHUNK = 16;                                                 // frames per device round trip
    for (let f = 0; f < maxFrames; f += CHUNK) {
      const n = Math.min(CHUNK, maxFrames - f);
      this.check(vx.decode(this.h, 0, n, 1));
      const codes = new Uint32Array(n * 37);
      this.check(vx.read_codes(this.h, 0, f, n, codes));
      for (let i = 0; i < n; ++i) {
        const sem = codes[i * 37];
        if (sem <= 1) return { semanticCodes, acousticCodes };         // EOS (:2567-2570)
        const ac = Array.from(codes.subarray(i * 37 + 1, i * 37 + 37));
        semanticCodes.push(sem);
        acousticCodes.push(ac);
        if (onFrame && onFrame(f + i, sem, ac) === false) return { semanticCodes, acousticCodes };
      }
    }
    return { semanticCodes, acousticCodes };
  }

  // codecDecode (src/engine.ts:1402-1713): T x 1920 samples at 24 kHz.
  codecDecode(sem: number[], ac: number[][]): Float32Array {
    const audio = new Float32Array(sem.length * 1920);
    this.check(vx.codec_decode(this.h, Uint32Array.from(sem), Uint32Array.from(ac.flat()), sem.length, audio));
    return audio;
  }

  // backboneStepAndRead (src/engine.ts:2333): greedy LM-head token.
  backboneStepAndRead(tokenId: number, useAudioEmbedding = false): number {
    const am = new Int32Array(1);
    this.check(vx.backbone_step(this.h, 0, tokenId, useAudioEmbedding ? 1 : 0, null, null, am));
    return am[0];
  }

  // debugFMStep(noise) (src/engine.ts:2363).
  debugFMStep(noise: Float32Array | null) {
    const logits = new Float32Array(8320), sem = new Uint32Array(1), ac = new Uint32Array(36), xf = new Float32Array(36);
    this.check(vx.fm_step(this.h, 0, noise, logits, sem, ac, xf));
    return { semanticLogits: logits, semanticCode: sem[0], acousticCodes: ac, xFinal: xf };
  }

  // debugBackboneLayerByLayer (src/engine.ts:2106): rows embed, 4 per layer, final_norm, hidden.
  debugBackboneLayerByLayer(tokenId: number, nLayers = 26): Float32Array {
    const out = new Float32Array((4 * nLayers + 3) * DIM);
    this.check(vx.debug_layers(this.h, 0, tokenId, out));
    return out;
  }

  destroy() { if (this.h) { vx.destroy(this.h); this.h = null; } }
}
