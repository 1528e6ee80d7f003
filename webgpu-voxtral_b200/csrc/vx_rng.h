// vx_rng.h — counter-based synthetic-input generator shared by the CUDA engine,
// the CPU oracle and the numpy checker.
//
// The reference (svenflow/webgpu-voxtral) loads real checkpoint weights
// (src/weights.ts:497-669) and draws FM noise from Math.random
// (src/engine.ts:1265-1274).  Neither is reproducible, so every synthetic input
// of this project (weights, prompt ids, voice rows, FM noise, feedback codes)
// comes from this header instead.  It uses integer arithmetic plus ONE IEEE f32
// multiply and ONE f32->f16 round-to-nearest-even, so the GPU, the C oracle and
// numpy produce bit-identical tensors.
//
//   key            = stream_key(seed, stream)            (stream = FNV-1a of a
//                                                          tensor name, or an
//                                                          utterance index)
//   normal(key, i) = (2*sum_{j<12} u16_j - 12*65535) / 2^17
//                    with the twelve 16-bit uniforms u16_j taken from
//                    splitmix64(key ^ (3i+t)*C) for t = 0,1,2.
// normal() is the Irwin-Hall sum of 12 uniforms: mean 0, variance 1 - 2^-32,
// bounded at +-6 — the classical approximation of N(0,1).
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define VX_HD __host__ __device__ __forceinline__
#else
#define VX_HD static inline
#endif

VX_HD uint64_t vx_splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Key of one independent stream (a tensor, or one utterance's prompt / noise).
VX_HD uint64_t vx_stream_key(uint64_t seed, uint64_t stream) {
  return vx_splitmix64(vx_splitmix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}

// 64 uniform bits for counter i of a stream.
VX_HD uint64_t vx_bits(uint64_t key, uint64_t i) {
  return vx_splitmix64(key ^ (i * 0x9FB21C651E98DF25ull));
}

// Approximately standard-normal f32, exact in integer arithmetic.
VX_HD float vx_normal(uint64_t key, uint64_t i) {
  int64_t s = 0;
  for (uint64_t t = 0; t < 3; ++t) {
    uint64_t h = vx_bits(key, 3 * i + t);
    s += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) +
         (int64_t)((h >> 32) & 0xFFFF) + (int64_t)(h >> 48);
  }
  int64_t c = 2 * s - 12 * 65535;           // |c| <= 786420 < 2^24: exact in f32
  return (float)c * (1.0f / 131072.0f);     // power-of-two scale: exact
}

// Uniform double in [0, 1) from the top 53 bits of counter i (the sampler's draw).
VX_HD double vx_uniform01(uint64_t key, uint64_t i) {
  return (double)(vx_bits(key, i) >> 11) * (1.0 / 9007199254740992.0);
}

// Uniform integer in [lo, hi) (modulo bias < 2^-40 for the ranges used here).
VX_HD uint32_t vx_uniform_int(uint64_t key, uint64_t i, uint32_t lo, uint32_t hi) {
  return lo + (uint32_t)(vx_bits(key, i) % (uint64_t)(hi - lo));
}

// FNV-1a 64 of a NUL-terminated tensor name: the stream id of that tensor.
VX_HD uint64_t vx_fnv1a(const char* s) {
  uint64_t h = 0xCBF29CE484222325ull;
  while (*s) { h ^= (uint8_t)(*s++); h *= 0x100000001B3ull; }
  return h;
}

// Host-side IEEE binary16 round-to-nearest-even (the device uses
// __float2half_rn, which rounds identically).  Handles subnormals, inf, nan.
static inline uint16_t vx_f32_to_f16_bits(float f) {
  union { float f; uint32_t u; } v; v.f = f;
  uint32_t x = v.u;
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ex = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (ex == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
  int32_t e = (int32_t)ex - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {                                   // subnormal or zero in f16
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);          // 14..24
    uint32_t half = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1u);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) half++;
    return (uint16_t)(sign | half);
  }
  uint32_t half = ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;  // may carry into exponent: correct
  return (uint16_t)(sign | half);
}

static inline float vx_f16_bits_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t ex = ((uint32_t)h >> 10) & 0x1Fu;
  uint32_t man = (uint32_t)h & 0x3FFu;
  uint32_t u;
  if (ex == 0) {
    if (man == 0) { u = sign; }
    else {                                        // normalise the subnormal
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400u));
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (ex == 0x1F) {
    u = sign | 0x7F800000u | (man << 13);
  } else {
    u = sign | ((ex - 15 + 127) << 23) | (man << 13);
  }
  union { uint32_t u; float f; } v; v.u = u;
  return v.f;
}

// Seeds and streams of the synthetic workload (one place, used everywhere).
#define VX_SEED_WEIGHTS 0ull
#define VX_SEED_PROMPT 1ull
#define VX_SEED_VOICE 2ull
#define VX_SEED_FM_NOISE 3ull
#define VX_SEED_CODES 4ull
#define VX_WEIGHT_SIGMA 0.02f
