// The sweep's counter-based generator, shared by the device fill (fill.cu)
// and its host twin (fill_host.cpp): plain C++ so that both nvcc and the host
// compiler read it.
//
// Generator: SplitMix64 finalizer over (seed, stream, k) -> two 24-bit
// uniforms (u1, u2).  Normals come in Box-Muller pairs: elements 2k and
// 2k + 1 are r cos(2 pi u2) and r sin(2 pi u2) with r = sqrt(-2 ln u1).
#pragma once

#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define PHEW_HD __host__ __device__ __forceinline__
#else
#define PHEW_HD inline
#endif

namespace phew {

PHEW_HD uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

PHEW_HD uint64_t draw(uint64_t seed, uint64_t stream, uint64_t i) {
  return mix64(mix64(mix64(seed) ^ stream) ^ i);
}

// (0, 1] uniform with 24 bits
PHEW_HD float u24(uint64_t bits) {
  return (static_cast<float>(bits & 0xFFFFFFull) + 1.0f) * (1.0f / 16777216.0f);
}

// fp32 -> 16-bit storage, round to nearest even (NaN kept quiet).
inline uint16_t host_bf16_bits(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

inline uint16_t host_f16_bits(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return static_cast<uint16_t>(sign | 0x7e00u);  // NaN
  if (a >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);  // rounds to inf
  if (a < 0x38800000u) {
    // half subnormal (or zero): value / 2^-24, rounded to nearest even; the
    // scaled value is below 2^10, so adding 1.5 * 2^23 rounds it to an integer
    float f;
    memcpy(&f, &a, 4);
    const float scaled = f * 16777216.0f;  // exact: power-of-two scale
    const float r = (scaled + 12582912.0f) - 12582912.0f;
    return static_cast<uint16_t>(sign | static_cast<uint32_t>(r));
  }
  // normal: rebias the exponent, round the 13 dropped mantissa bits
  uint32_t m = a + 0xc8000000u;  // exponent 127 -> 15 (subtract 112 << 23)
  m += 0xfffu + ((m >> 13) & 1u);
  return static_cast<uint16_t>(sign | (m >> 13));
}

// Normal draws of elements [2 * k0, min(2 * k1, n)) of (seed, stream), times
// `scale`, stored as `dtype` (PHEW_F32 / PHEW_F16 / PHEW_BF16) at their
// element index in `out`.  Vectorised for the host's widest SIMD unit
// (fill_host.cpp); values within a few fp32 ulps of the exact transform.
void host_normals(void* out, int dtype, int64_t k0, int64_t k1, int64_t n, uint64_t seed,
                  uint64_t stream, float scale);

// The same draws scaled into bf16's subnormal range (|scale| < 2^-129, so
// that every value, at most 5.78 |scale|, is below 2^-126): the fp32 radius
// times `scale` is formed in double and rounded straight to bf16's subnormal
// grid (an fp32 product with a subnormal result takes a microcode assist on
// x86, about a hundred cycles each).
void host_normals_tiny_bf16(uint16_t* out, int64_t k0, int64_t k1, int64_t n, uint64_t seed,
                            uint64_t stream, float scale);

}  // namespace phew
