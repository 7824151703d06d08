// Seeded device-side input generation for the verification sweep.
//
// The sweep evaluates every candidate on inputs derived from (seed, variant,
// argument index); drawing them on the host would dominate a sweep over
// decoder-block sizes (hundreds of millions of values per seed and size), so
// they are drawn here from a counter-based generator: element i of stream
// (seed, stream_id) is a pure function of those three numbers, independent
// of the grid, the GPU and the number of GPUs in the sweep.
//
// Generator: SplitMix64 finalizer over (seed, stream, i) -> two 24-bit
// uniforms -> Box-Muller for normals.
#include <math.h>

#include "common.cuh"

namespace phew {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t draw(uint64_t seed, uint64_t stream, uint64_t i) {
  return mix64(mix64(mix64(seed) ^ stream) ^ i);
}

// (0, 1] uniform with 24 bits
__device__ __forceinline__ float u24(uint64_t bits) {
  return (static_cast<float>(bits & 0xFFFFFFull) + 1.0f) * (1.0f / 16777216.0f);
}

template <typename T>
__global__ void fill_kernel(T* out, int64_t n, int64_t cols, int kind, uint64_t seed,
                            uint64_t stream, float scale) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += step) {
    float v;
    switch (kind) {
      case PHEW_FILL_NORMAL: {
        const uint64_t b = draw(seed, stream, static_cast<uint64_t>(i));
        const float r = sqrtf(-2.0f * logf(u24(b)));
        v = r * cospif(2.0f * u24(b >> 32)) * scale;
        break;
      }
      case PHEW_FILL_UNIFORM: {
        const uint64_t b = draw(seed, stream, static_cast<uint64_t>(i));
        v = (2.0f * u24(b) - 1.0f) * scale;
        break;
      }
      case PHEW_FILL_ONE_HOT_ROWS: {
        const int64_t row = i / cols, col = i % cols;
        const int64_t hot = static_cast<int64_t>(draw(seed, stream, static_cast<uint64_t>(row)) %
                                                 static_cast<uint64_t>(cols));
        v = col == hot ? scale : 0.0f;
        break;
      }
      default:
        v = scale;
    }
    out[i] = from_f32<T>(v);
  }
}

}  // namespace
}  // namespace phew

using namespace phew;

extern "C" int phew_fill(void* out, int64_t n, int64_t cols, int dtype, int kind, uint64_t seed,
                         uint64_t stream_id, float scale, void* stream) {
  PHEW_REQUIRE(out != nullptr || n == 0, "phew_fill: null output");
  PHEW_REQUIRE(n >= 0 && cols > 0, "phew_fill: bad extent");
  PHEW_REQUIRE(kind >= PHEW_FILL_NORMAL && kind <= PHEW_FILL_CONSTANT, "phew_fill: bad kind");
  if (n == 0) return PHEW_OK;
  int64_t blocks = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count_current()) * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>(blocks);
  switch (dtype) {
    case PHEW_F32: fill_kernel<float><<<g, 256, 0, st>>>(static_cast<float*>(out), n, cols, kind, seed, stream_id, scale); break;
    case PHEW_F16: fill_kernel<f16><<<g, 256, 0, st>>>(static_cast<f16*>(out), n, cols, kind, seed, stream_id, scale); break;
    case PHEW_BF16: fill_kernel<bf16><<<g, 256, 0, st>>>(static_cast<bf16*>(out), n, cols, kind, seed, stream_id, scale); break;
    default: return set_error(PHEW_ERR_INVALID, "phew_fill: bad dtype");
  }
  return launch_status("fill_kernel");
}
