// Rotary position embedding over the last axis.
//
// Stands in for mx.fast.rope(x, dims, traditional=, base=, scale=, offset=)
// (phew emit/codegen.py:413-419, node FastRoPE ir/ops.py:172-179, matched by
// rules/primitive_subst.py:339-407).
//
// x is [rows, D] row-major with rows = (leading dims) x L, the position of a
// row being offset + (row % L) (L = the second-to-last extent).  For pair i
// of the first `dims` features (i < dims/2):
//   inv_i = fp32(base ^ (-2i / dims))            (double pow, rounded once)
//   a     = fp32(fp32(position * scale) * inv_i)
//   (u, v) = (x[i], x[i + dims/2])   or, traditional, (x[2i], x[2i+1])
//   out_u = T(u cos a - v sin a),  out_v = T(u sin a + v cos a)
// with every product and sum rounded to fp32 (no contraction) and cosf /
// sinf for the trigonometry; features at and beyond `dims` are copied.
// HBM-bound: one read and one write of x.
#include <math.h>

#include "common.cuh"

namespace phew {
namespace {

template <typename T>
__global__ void rope_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int64_t D,
                            int64_t L, int dims, int traditional, float base, float scale,
                            int64_t offset) {
  extern __shared__ float inv_freq[];  // [dims / 2]
  const int half = dims / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x)
    inv_freq[i] = static_cast<float>(pow(static_cast<double>(base), -2.0 * i / static_cast<double>(dims)));
  __syncthreads();
  const int64_t per_row = half + (D - 2 * half);  // rotated pairs + copied tail
  const int64_t total = rows * per_row;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = t / per_row;
    const int64_t k = t % per_row;
    const T* xr = x + row * D;
    T* yr = y + row * D;
    if (k < half) {
      const int i = static_cast<int>(k);
      const float pos = static_cast<float>(offset + row % L);
      const float a = __fmul_rn(__fmul_rn(pos, scale), inv_freq[i]);
      const float c = cosf(a), s = sinf(a);
      const int64_t iu = traditional ? 2 * i : i;
      const int64_t iv = traditional ? 2 * i + 1 : i + half;
      const float u = to_f32(xr[iu]), v = to_f32(xr[iv]);
      yr[iu] = from_f32<T>(__fsub_rn(__fmul_rn(u, c), __fmul_rn(v, s)));
      yr[iv] = from_f32<T>(__fadd_rn(__fmul_rn(u, s), __fmul_rn(v, c)));
    } else {
      const int64_t col = 2 * half + (k - half);
      yr[col] = xr[col];
    }
  }
}

template <typename T>
int rope_typed(const void* x, void* y, int64_t rows, int64_t D, int64_t L, int dims, int traditional,
               float base, float scale, int64_t offset, cudaStream_t st) {
  const int64_t per_row = dims / 2 + (D - 2 * (dims / 2));
  const int64_t total = rows * per_row;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total + 255) / 256;
  const unsigned grid = static_cast<unsigned>(want < 16LL * sms ? (want > 0 ? want : 1) : 16LL * sms);
  const size_t smem = sizeof(float) * static_cast<size_t>(dims / 2 > 0 ? dims / 2 : 1);
  rope_kernel<T><<<grid, 256, smem, st>>>(static_cast<const T*>(x), static_cast<T*>(y), rows, D, L, dims,
                                          traditional, base, scale, offset);
  return launch_status("rope_kernel");
}

}  // namespace
}  // namespace phew

using namespace phew;

extern "C" int phew_rope(const void* x, void* y, int64_t rows, int64_t D, int64_t L, int dims,
                         int traditional, float base, float scale, int64_t offset, int dtype,
                         void* stream) {
  PHEW_REQUIRE(x && y, "phew_rope: null pointer");
  PHEW_REQUIRE(rows >= 0 && D > 0 && L > 0 && (L == 1 || rows % L == 0), "phew_rope: bad shape");
  PHEW_REQUIRE(dims >= 0 && dims <= D && dims % 2 == 0, "phew_rope: dims must be even and <= D");
  PHEW_REQUIRE(dims / 2 <= 12288, "phew_rope: dims too large");
  PHEW_REQUIRE(base > 0.0f, "phew_rope: base must be positive");
  if (rows == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PHEW_F32: return rope_typed<float>(x, y, rows, D, L, dims, traditional, base, scale, offset, st);
    case PHEW_F16: return rope_typed<f16>(x, y, rows, D, L, dims, traditional, base, scale, offset, st);
    case PHEW_BF16: return rope_typed<bf16>(x, y, rows, D, L, dims, traditional, base, scale, offset, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_rope: bad dtype");
  }
}
