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

// ---------------------------------------------------------------------------
// Affine group-wise quantisation (the producer of the layout above), for
// mx.quantize (phew rules/quantization.py:37-71 quantises weights ahead of
// QuantizedMatMul).  Per group of `group_size` values along a row:
//   scale = T(max((max - min) / (2^bits - 1), 1e-8)),  bias = T(min),
//   q = clamp(rint((w - bias) / scale), 0, 2^bits - 1)   (fp32, IEEE divide)
// packed 32 / bits codes per uint32 word, code j in bits [j*bits, (j+1)*bits).
// One thread per group (a group is 32..128 values); HBM-bound.
// ---------------------------------------------------------------------------
namespace phew {
namespace {

template <typename T>
__global__ void quant_kernel(const T* __restrict__ w, uint32_t* __restrict__ wq, T* __restrict__ scales,
                             T* __restrict__ biases, int64_t rows, int64_t cols, int group_size,
                             int bits) {
  const int per = 32 / bits;
  const int n_bins = (1 << bits) - 1;
  const int64_t groups_per_row = cols / group_size;
  const int64_t total = rows * groups_per_row;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = g / groups_per_row;
    const int64_t c0 = (g % groups_per_row) * group_size;
    const T* src = w + r * cols + c0;
    float lo = to_f32(src[0]), hi = lo;
    for (int j = 1; j < group_size; ++j) {
      const float v = to_f32(src[j]);
      lo = fminf(lo, v);
      hi = fmaxf(hi, v);
    }
    const float sc = round_to<T>(fmaxf(__fdiv_rn(hi - lo, static_cast<float>(n_bins)), 1e-8f));
    const float bi = round_to<T>(lo);
    scales[g] = from_f32<T>(sc);
    biases[g] = from_f32<T>(bi);
    uint32_t* dst = wq + (r * cols + c0) / per;
    for (int k = 0; k < group_size / per; ++k) {
      uint32_t word = 0;
      for (int j = 0; j < per; ++j) {
        float q = rintf(__fdiv_rn(to_f32(src[k * per + j]) - bi, sc));
        q = fminf(fmaxf(q, 0.0f), static_cast<float>(n_bins));
        word |= static_cast<uint32_t>(q) << (j * bits);
      }
      dst[k] = word;
    }
  }
}

template <typename T>
int quant_typed(const void* w, void* wq, void* s, void* b, int64_t rows, int64_t cols, int group_size,
                int bits, cudaStream_t st) {
  const int64_t total = rows * (cols / group_size);
  int64_t blocks = (total + 127) / 128;
  const int64_t cap = static_cast<int64_t>(sm_count_current()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  quant_kernel<T><<<static_cast<unsigned>(blocks), 128, 0, st>>>(
      static_cast<const T*>(w), static_cast<uint32_t*>(wq), static_cast<T*>(s), static_cast<T*>(b), rows,
      cols, group_size, bits);
  return launch_status("quant_kernel");
}

}  // namespace
}  // namespace phew

extern "C" int phew_quantize(const void* w, void* wq, void* scales, void* biases, int64_t rows,
                             int64_t cols, int group_size, int bits, int dtype, void* stream) {
  PHEW_REQUIRE(w && wq && scales && biases, "phew_quantize: null pointer");
  PHEW_REQUIRE(bits == 2 || bits == 4 || bits == 8, "phew_quantize: bits must be 2, 4 or 8");
  PHEW_REQUIRE(group_size > 0 && rows >= 0 && cols > 0 && cols % group_size == 0 &&
                   group_size % (32 / bits) == 0,
               "phew_quantize: cols must be a multiple of group_size, and group_size of 32 / bits");
  if (rows == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PHEW_F32: return quant_typed<float>(w, wq, scales, biases, rows, cols, group_size, bits, st);
    case PHEW_F16: return quant_typed<f16>(w, wq, scales, biases, rows, cols, group_size, bits, st);
    case PHEW_BF16: return quant_typed<bf16>(w, wq, scales, biases, rows, cols, group_size, bits, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_quantize: bad dtype");
  }
}
