// Host twin of the sweep's normal draws (phew_fill_host), written for the
// host compiler's auto-vectoriser: each block of pairs goes through short
// loops over arrays (draws, radius, angle, store), and the clones of the entry
// points for AVX-512 and AVX2 hosts run them 16 / 8 lanes wide.  libm's logf
// and sincosf are scalar calls, which made the host generator, not the copy
// or the GPU, the bound of the sweep's end-to-end leg.
//
// The transforms are written here from their series, not taken from a math
// library:
//   ln u      u = 2^e * m with m in [sqrt(1/2), sqrt(2)); ln m = 2 atanh(s),
//             s = (m - 1) / (m + 1), by its Maclaurin series
//             2 (s + s^3/3 + s^5/5 + s^7/7 + s^9/9) (|s| <= 0.172, the next
//             term below 2^-27 relative);
//   cos, sin  of 2 pi u2: x = 4 u2 is exact, k = round(x), the angle
//             (x - k) * pi/2 lies in [-pi/4, pi/4] and goes through the
//             Taylor series of sin (to x^9) and cos (to x^10); k mod 4 picks
//             the quadrant.
// Each is within a few fp32 ulps of the exact value, as the device's logf /
// sincospif are, so host and device draws agree to that order.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../../include/phew_b200.h"
#include "fill_host.h"

namespace phew {
namespace {

constexpr int kBlock = 256;  // pairs per block of the array loops

#define PHEW_INLINE inline __attribute__((always_inline))

PHEW_INLINE float bits_float(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
PHEW_INLINE uint32_t float_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

// sqrt(-2 ln u) for u in [2^-24, 1]
PHEW_INLINE float radius(float u) {
  const uint32_t b = float_bits(u);
  int e = static_cast<int>(b >> 23) - 127;
  float m = bits_float((b & 0x7fffffu) | 0x3f800000u);  // [1, 2)
  const bool big = m > 1.41421356f;
  m = big ? m * 0.5f : m;
  e = big ? e + 1 : e;
  const float s = (m - 1.0f) / (m + 1.0f);
  const float z = s * s;
  float p = 1.0f / 9.0f;
  p = p * z + 1.0f / 7.0f;
  p = p * z + 1.0f / 5.0f;
  p = p * z + 1.0f / 3.0f;
  p = p * z + 1.0f;
  const float ln = static_cast<float>(e) * 0.693147181f + 2.0f * s * p;
  return sqrtf(-2.0f * ln);
}

// cos and sin of 2 pi u for u in (0, 1]
PHEW_INLINE void turn(float u, float* c, float* s) {
  const float x = 4.0f * u;
  const float k = (x + 12582912.0f) - 12582912.0f;  // round to nearest even
  const float t = (x - k) * 1.57079633f;            // [-pi/4, pi/4]
  const float t2 = t * t;
  float ps = 1.0f / 362880.0f;
  ps = ps * t2 - 1.0f / 5040.0f;
  ps = ps * t2 + 1.0f / 120.0f;
  ps = ps * t2 - 1.0f / 6.0f;
  const float sn = t + t * t2 * ps;
  float pc = -1.0f / 3628800.0f;
  pc = pc * t2 + 1.0f / 40320.0f;
  pc = pc * t2 - 1.0f / 720.0f;
  pc = pc * t2 + 1.0f / 24.0f;
  pc = pc * t2 - 0.5f;
  const float cs = 1.0f + t2 * pc;
  const int q = static_cast<int>(k) & 3;
  const float sv = (q & 1) ? cs : sn;
  const float cv = (q & 1) ? sn : cs;
  *s = (q & 2) ? -sv : sv;
  *c = ((q + 1) & 2) ? -cv : cv;
}

// Radius and (cos, sin) of pairs k0 .. k0 + cnt - 1
PHEW_INLINE void block_draws(uint64_t seed, uint64_t stream, int64_t k0, int cnt, float* r,
                             float* c, float* s) {
  const uint64_t base = mix64(mix64(seed) ^ stream);
  float u1[kBlock], u2[kBlock];
  // u24 of both halves (values below 2^24 convert exactly through int32)
  for (int j = 0; j < cnt; ++j) {
    const uint64_t b = mix64(base ^ static_cast<uint64_t>(k0 + j));
    u1[j] = (static_cast<float>(static_cast<int32_t>(b & 0xFFFFFFu)) + 1.0f) * (1.0f / 16777216.0f);
    u2[j] = (static_cast<float>(static_cast<int32_t>((b >> 32) & 0xFFFFFFu)) + 1.0f) *
            (1.0f / 16777216.0f);
  }
  for (int j = 0; j < cnt; ++j) r[j] = radius(u1[j]);
  for (int j = 0; j < cnt; ++j) turn(u2[j], &c[j], &s[j]);
}

template <typename Cvt, typename T>
PHEW_INLINE void normals_as(T* o, int64_t k0, int64_t k1, int64_t n, uint64_t seed,
                            uint64_t stream, float scale, Cvt cvt) {
  float r[kBlock], c[kBlock], s[kBlock];
  for (int64_t kb = k0; kb < k1; kb += kBlock) {
    const int cnt = static_cast<int>(k1 - kb < kBlock ? k1 - kb : kBlock);
    block_draws(seed, stream, kb, cnt, r, c, s);
    // a pair whose second element is past the end is the last one: store it apart
    const int full = (2 * (kb + cnt) <= n) ? cnt : cnt - 1;
    T* p = o + 2 * kb;
    for (int j = 0; j < full; ++j) {
      const float rs = r[j] * scale;
      p[2 * j] = cvt(rs * c[j]);
      p[2 * j + 1] = cvt(rs * s[j]);
    }
    if (full < cnt) p[2 * full] = cvt(r[full] * scale * c[full]);
  }
}

}  // namespace

#define PHEW_CLONES __attribute__((target_clones("arch=x86-64-v4", "arch=x86-64-v3", "default")))

PHEW_CLONES void host_normals(void* out, int dtype, int64_t k0, int64_t k1, int64_t n,
                              uint64_t seed, uint64_t stream, float scale) {
  if (dtype == PHEW_F32) {
    normals_as(static_cast<float*>(out), k0, k1, n, seed, stream, scale, [](float v) { return v; });
  } else if (dtype == PHEW_BF16) {
    normals_as(static_cast<uint16_t*>(out), k0, k1, n, seed, stream, scale,
               [](float v) { return host_bf16_bits(v); });
  } else {
    normals_as(static_cast<uint16_t*>(out), k0, k1, n, seed, stream, scale,
               [](float v) { return host_f16_bits(v); });
  }
}

PHEW_CLONES void host_normals_tiny_bf16(uint16_t* out, int64_t k0, int64_t k1, int64_t n,
                                        uint64_t seed, uint64_t stream, float scale) {
  const double sc = static_cast<double>(scale);
  // |v| <= 5.78 |scale| < 2^-126: the bf16 subnormal m * 2^-133 (m <= 128),
  // m rounded to nearest even by the 1.5 * 2^52 addition
  auto tiny = [](double v) -> uint16_t {
    uint64_t vb;
    memcpy(&vb, &v, 8);
    const uint32_t sign = static_cast<uint32_t>(vb >> 48) & 0x8000u;
    const double a = v < 0 ? -v : v;
    const double m = (a * 0x1p133 + 6755399441055744.0) - 6755399441055744.0;
    return static_cast<uint16_t>(sign | static_cast<uint32_t>(static_cast<int32_t>(m)));
  };
  float r[kBlock], c[kBlock], s[kBlock];
  for (int64_t kb = k0; kb < k1; kb += kBlock) {
    const int cnt = static_cast<int>(k1 - kb < kBlock ? k1 - kb : kBlock);
    block_draws(seed, stream, kb, cnt, r, c, s);
    const int full = (2 * (kb + cnt) <= n) ? cnt : cnt - 1;
    uint16_t* p = out + 2 * kb;
    for (int j = 0; j < full; ++j) {
      const double rs = static_cast<double>(r[j]) * sc;
      p[2 * j] = tiny(rs * c[j]);
      p[2 * j + 1] = tiny(rs * s[j]);
    }
    if (full < cnt) p[2 * full] = tiny(static_cast<double>(r[full]) * sc * c[full]);
  }
}

}  // namespace phew
