// tn_common.cuh -- shared definitions of the B200 stage engine.
//
// Error plumbing for the C ABI, exact fp16 conversions (the activation hop
// codec of web/inference-worker.js:68-88 and IEEE round-to-nearest-even for
// the synthetic pack writer), and the counter-based weight generator used on
// both host and device.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstring>

#include "../../include/tabnet_stage.h"

namespace tn {

// ---------------------------------------------------------------- errors
void set_error(const char* fmt, ...);
void clear_error();

// A failing runtime call also leaves its error in the runtime's last-error
// slot; it is read back here so that the next TN_CHECK_LAUNCH (which asks
// cudaGetLastError) does not report this call's error as its own.
#define TN_CHECK_CUDA(expr)                                                              \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess) {                                                             \
      (void)cudaGetLastError();                                                          \
      ::tn::set_error("%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__); \
      return TN_ECUDA;                                                                   \
    }                                                                                    \
  } while (0)

#define TN_REQUIRE(cond, code, ...)   \
  do {                                \
    if (!(cond)) {                    \
      ::tn::set_error(__VA_ARGS__);   \
      return (code);                  \
    }                                 \
  } while (0)

// a launch's own error (configuration errors surface here, not at sync)
#define TN_CHECK_LAUNCH() TN_CHECK_CUDA(cudaGetLastError())

// ---------------------------------------------------------------- bit casts
__host__ __device__ __forceinline__ uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
#endif
}
__host__ __device__ __forceinline__ float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  std::memcpy(&f, &u, 4);
  return f;
#endif
}

// IEEE single ops that must not be contracted into FMAs (the generator must
// give identical bits on host and device).
__host__ __device__ __forceinline__ float fmul_rn(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  volatile float r = a * b;
  return r;
#endif
}
__host__ __device__ __forceinline__ float fadd_rn(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fadd_rn(a, b);
#else
  volatile float r = a + b;
  return r;
#endif
}
__host__ __device__ __forceinline__ float fdiv_rn(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fdiv_rn(a, b);
#else
  volatile float r = a / b;
  return r;
#endif
}

// ---------------------------------------------------------------- fp16
// fp16 bits -> f32, exact (f16ToF32, web/inference-worker.js:68-73; NaN
// canonicalised as a Float32Array store of NaN does).
__host__ __device__ __forceinline__ float f16_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  const uint32_t m = h & 0x3ffu;
  if (e == 0) {
    if (m == 0) return u2f(s);
    // subnormal: m * 2^-24, exact in float
    const float v = (float)m * 5.9604644775390625e-8f;
    return s ? -v : v;
  }
  if (e == 31) return m ? u2f(0x7fc00000u) : u2f(s | 0x7f800000u);
  return u2f(s | ((e + 112u) << 23) | (m << 13));
}

// f32 -> fp16 with the reference's rounding (f32ToF16, web/inference-worker.js:74-88):
// the magnitude rounds half UP (Math.round), a carry to m == 1024 bumps the
// exponent, exponents above 15 give infinity, NaN gives 0x7e00 with no sign,
// and in the subnormal branch the rounded mantissa is masked with 0x3ff, so a
// value that rounds up to 2^-14 becomes a signed zero.
__host__ __device__ __forceinline__ uint16_t hop_encode(float f) {
  const uint32_t x = f2u(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return 0x7e00u;
  if (ax == 0x7f800000u) return (uint16_t)(sign | 0x7c00u);
  const int E = (int)(ax >> 23);
  if (E == 0) return (uint16_t)sign;  // zero, or an f32 subnormal: round(v * 2^24) == 0
  const int e = E - 127;              // floor(log2 v), exact for normal floats
  if (e >= 16) return (uint16_t)(sign | 0x7c00u);
  const uint32_t mant = ax & 0x7fffffu;
  if (e >= -14) {
    uint32_t m = (mant >> 13) + ((mant >> 12) & 1u);  // half up
    int ee = e;
    if (m == 1024u) {
      ee += 1;
      m = 0;
    }
    if (ee > 15) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)(ee + 15) << 10) | m);
  }
  const int sh = -1 - e;  // v * 2^24 = m24 * 2^-sh, sh >= 14
  if (sh >= 25) return (uint16_t)sign;
  const uint32_t m24 = mant | 0x800000u;
  const uint32_t m = (m24 >> sh) + ((m24 >> (sh - 1)) & 1u);
  return (uint16_t)(sign | (m & 0x3ffu));
}

// f32 -> fp16, IEEE round to nearest even (used only by the pack writer).
__host__ __device__ __forceinline__ uint16_t f32_to_f16_rne(float f) {
  const uint32_t x = f2u(f);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // >= 65520 rounds to inf
  if (ax < 0x38800000u) {                                    // below 2^-14
    const uint32_t e = ax >> 23;
    if (e < 102u) return (uint16_t)sign;
    const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;  // 14..24
    uint32_t m = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (m & 1u))) m++;
    return (uint16_t)(sign | m);
  }
  uint32_t r = (((ax >> 23) - 112u) << 10) | ((ax >> 13) & 0x3ffu);
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
  return (uint16_t)(sign | r);
}

// ---------------------------------------------------------------- generator
// Counter-based synthetic weights: value(seed, tag, i) is an Irwin-Hall(4)
// approximation of N(0, 0.02) built from a splitmix64-style hash of the
// element index -- integer arithmetic plus one IEEE multiply, so host and
// device produce identical bits.
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xBF58476D1CE4E5B9ull;
  z ^= z >> 27;
  z *= 0x94D049BB133111EBull;
  z ^= z >> 31;
  return z;
}
__host__ __device__ __forceinline__ uint64_t synth_key(uint64_t seed, uint32_t tag) {
  return mix64(seed * 0x9E3779B97F4A7C15ull + (uint64_t)tag * 0xD1B54A32D192ED03ull + 1ull);
}
// 0.02 / sqrt(4 * (65536^2 - 1) / 12) as a float
#define TN_SYNTH_SCALE_BITS 0x350de3bdu
__host__ __device__ __forceinline__ float synth_value(uint64_t key, uint64_t i) {
  const uint64_t h = mix64(key + (i + 1ull) * 0x9E3779B97F4A7C15ull);
  const int32_t s = (int32_t)(h & 0xffffu) + (int32_t)((h >> 16) & 0xffffu) +
                    (int32_t)((h >> 32) & 0xffffu) + (int32_t)(h >> 48);
  return fmul_rn((float)(s - 131070), u2f(TN_SYNTH_SCALE_BITS));
}

// tag of tensor t (layerLayout order) of absolute layer l
__host__ __device__ __forceinline__ uint32_t layer_tag(int layer, int t) {
  return (uint32_t)(layer + 1) * 16u + (uint32_t)t;
}

// Quantise one 32-element block of synthetic values starting at element b*32
// of a tensor with `count` elements into `out` (18 or 34 bytes, byte stores).
//   q8_0: d = amax/127, q = round(x/d)
//   q4_0: d = m/-8 (m the value of largest magnitude), q = clamp(round(x/d)+8, 0, 15)
__host__ __device__ inline void synth_quant_block(uint64_t key, uint64_t count, uint64_t b, int quant,
                                                  uint8_t* out) {
  float x[32];
  float amax = 0.f, m = 0.f;
  for (int j = 0; j < 32; j++) {
    const uint64_t i = b * 32ull + (uint64_t)j;
    x[j] = (i < count) ? synth_value(key, i) : 0.f;
    const float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      m = x[j];
    }
  }
  if (quant == TN_QUANT_Q8_0) {
    const float d = fdiv_rn(amax, 127.0f);
    const uint16_t dh = f32_to_f16_rne(d);
    out[0] = (uint8_t)(dh & 0xff);
    out[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 32; j++) {
      int q = 0;
      if (d != 0.f) {
        q = (int)roundf(fdiv_rn(x[j], d));
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
      }
      out[2 + j] = (uint8_t)(int8_t)q;
    }
  } else {
    const float d = fdiv_rn(m, -8.0f);
    const uint16_t dh = f32_to_f16_rne(d);
    out[0] = (uint8_t)(dh & 0xff);
    out[1] = (uint8_t)(dh >> 8);
    int q[32];
    for (int j = 0; j < 32; j++) {
      int v = 8;
      if (d != 0.f) v = (int)roundf(fdiv_rn(x[j], d)) + 8;
      q[j] = v < 0 ? 0 : (v > 15 ? 15 : v);
    }
    for (int j = 0; j < 16; j++) out[2 + j] = (uint8_t)(q[2 * j] | (q[2 * j + 1] << 4));
  }
}

// ---------------------------------------------------------------- layout
// web/inference-worker.js:142-163 (layerLayout, roundFfn) and quantBytesFor :130-137
__host__ __device__ inline uint64_t quant_bytes(uint64_t count, int quant) {
  if (quant == TN_QUANT_F32) return count * 4ull;
  if (quant == TN_QUANT_F16) return count * 2ull;
  const uint64_t nb = (count + 31ull) / 32ull;
  if (quant == TN_QUANT_Q8_0) return nb * 34ull;
  if (quant == TN_QUANT_Q4_0) return nb * 18ull;
  return 0;
}
inline int round_ffn(int H) {
  const int x = (int)((8ll * H) / 3);
  return ((x + 255) / 256) * 256;
}
struct LayerLayout {
  int H, nH, nKV, hd, qDim, kvDim, ffn;
  uint64_t off[9], count[9], total;
};
inline bool layer_layout(int H, int nH, int nKV, int ffn_dim, int quant, LayerLayout* L) {
  if (H <= 0 || nH <= 0 || nKV <= 0) return false;
  if (quant_bytes(1, quant) == 0) return false;
  L->H = H;
  L->nH = nH;
  L->nKV = nKV;
  L->hd = H / nH;
  L->qDim = nH * L->hd;
  L->kvDim = nKV * L->hd;
  L->ffn = ffn_dim ? ffn_dim : round_ffn(H);
  const uint64_t h = (uint64_t)H;
  const uint64_t c[9] = {h,
                         h * (uint64_t)L->qDim,
                         h * (uint64_t)L->kvDim,
                         h * (uint64_t)L->kvDim,
                         (uint64_t)L->qDim * h,
                         h,
                         h * (uint64_t)L->ffn,
                         h * (uint64_t)L->ffn,
                         (uint64_t)L->ffn * h};
  uint64_t off = 0;
  for (int t = 0; t < 9; t++) {
    const int eff = (t == 0 || t == 5) ? TN_QUANT_F16 : quant;
    L->off[t] = off;
    L->count[t] = c[t];
    off += quant_bytes(c[t], eff);
  }
  L->total = off;
  return true;
}

}  // namespace tn
