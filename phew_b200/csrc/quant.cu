// Affine group-wise dequantisation of packed low-bit weights.
//
// Stands in for the weight side of mx.quantized_matmul /
// mx.fast.quantized_scaled_dot_product_attention (phew emit/codegen.py:428-449,
// nodes QuantizedMatMul ir/ops.py:209-218 and
// FastQuantizedScaledDotProductAttention ir/ops.py:191-200, produced by
// rules/quantization.py:37-71 and traced at ir/importer.py:1255-1280).
//
// Format (MLX's affine layout): w is [rows, cols] quantised along cols in
// groups of `group_size`; the codes are packed 32 / bits per uint32 word,
// code j of a word in bits [j * bits, (j + 1) * bits); scales and biases are
// [rows, cols / group_size] in the output dtype.
//   out[r, c] = T(scale[r, c / g] * q[r, c] + bias[r, c / g])   (fp32 fma)
// One thread per packed word (8 codes at 4 bits): reads 4 bytes of codes
// and writes 16 bytes of output; HBM-bound.
#include "common.cuh"

namespace phew {
namespace {

template <typename T>
__global__ void dequant_kernel(const uint32_t* __restrict__ wq, const T* __restrict__ scales,
                               const T* __restrict__ biases, T* __restrict__ out, int64_t rows,
                               int64_t cols, int group_size, int bits) {
  const int per = 32 / bits;
  const uint32_t mask = (bits == 32) ? 0xffffffffu : ((1u << bits) - 1u);
  const int64_t words_per_row = cols / per;
  const int64_t total = rows * words_per_row;
  const int64_t groups_per_row = cols / group_size;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < total;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = w / words_per_row;
    const int64_t c0 = (w % words_per_row) * per;
    const uint32_t word = wq[w];
    T* o = out + r * cols + c0;
    for (int j = 0; j < per; ++j) {
      const int64_t g = r * groups_per_row + (c0 + j) / group_size;
      const float q = static_cast<float>((word >> (j * bits)) & mask);
      o[j] = from_f32<T>(fmaf(to_f32(scales[g]), q, to_f32(biases[g])));
    }
  }
}

template <typename T>
int dequant_typed(const void* wq, const void* s, const void* b, void* out, int64_t rows, int64_t cols,
                  int group_size, int bits, cudaStream_t st) {
  const int64_t total = rows * (cols / (32 / bits));
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count_current()) * 32;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  dequant_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const uint32_t*>(wq), static_cast<const T*>(s), static_cast<const T*>(b), static_cast<T*>(out),
      rows, cols, group_size, bits);
  return launch_status("dequant_kernel");
}

}  // namespace
}  // namespace phew

using namespace phew;

extern "C" int phew_dequantize(const void* wq, const void* scales, const void* biases, void* out,
                               int64_t rows, int64_t cols, int group_size, int bits, int dtype,
                               void* stream) {
  PHEW_REQUIRE(wq && scales && biases && out, "phew_dequantize: null pointer");
  PHEW_REQUIRE(bits == 2 || bits == 4 || bits == 8, "phew_dequantize: bits must be 2, 4 or 8");
  PHEW_REQUIRE(group_size > 0 && rows >= 0 && cols > 0 && cols % group_size == 0 &&
                   cols % (32 / bits) == 0,
               "phew_dequantize: cols must be a multiple of group_size and of 32 / bits");
  if (rows == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PHEW_F32: return dequant_typed<float>(wq, scales, biases, out, rows, cols, group_size, bits, st);
    case PHEW_F16: return dequant_typed<f16>(wq, scales, biases, out, rows, cols, group_size, bits, st);
    case PHEW_BF16: return dequant_typed<bf16>(wq, scales, biases, out, rows, cols, group_size, bits, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_dequantize: bad dtype");
  }
}
