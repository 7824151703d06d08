// Shared helpers for the phew_b200 native library: status handling, dtype
// conversions and small warp/block reductions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/phew_b200.h"

namespace phew {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);

inline int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PHEW_OK;
  return set_error(PHEW_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define PHEW_CHECK_CUDA(expr)                                  \
  do {                                                         \
    int _st = ::phew::cuda_status((expr), #expr);              \
    if (_st != PHEW_OK) return _st;                            \
  } while (0)

#define PHEW_REQUIRE(cond, msg)                                \
  do {                                                         \
    if (!(cond)) return ::phew::set_error(PHEW_ERR_INVALID, msg); \
  } while (0)

// Count of kernels this library launched (phew_launch_count).
void count_launch();
unsigned long long launch_counter();

// Launch-error check used right after every <<<>>> launch; counts the launch.
inline int launch_status(const char* what) {
  const int s = cuda_status(cudaGetLastError(), what);
  if (s == PHEW_OK) count_launch();
  return s;
}

inline int dtype_bytes(int dtype) {
  switch (dtype) {
    case PHEW_F32: return 4;
    case PHEW_F16: return 2;
    case PHEW_BF16: return 2;
    default: return 0;
  }
}

int sm_count_current();

// ---------------------------------------------------------------------------
// Device-side conversions.  16-bit floats are stored as raw uint16_t so that
// no CUDA half headers are needed; conversions use round-to-nearest-even.
// ---------------------------------------------------------------------------
struct f16 { uint16_t bits; };
struct bf16 { uint16_t bits; };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(f16 v) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(v.bits));
  return f;
}
__device__ __forceinline__ float to_f32(bf16 v) {
  return __uint_as_float(static_cast<uint32_t>(v.bits) << 16);
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ f16 from_f32<f16>(float v) {
  f16 r;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r.bits) : "f"(v));
  return r;
}
template <> __device__ __forceinline__ bf16 from_f32<bf16>(float v) {
  bf16 r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r.bits) : "f"(v));
  return r;
}

// Rounds an fp32 value to the precision of T and back.
template <typename T> __device__ __forceinline__ float round_to(float v) {
  return to_f32(from_f32<T>(v));
}

// ---------------------------------------------------------------------------
// Reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace phew
