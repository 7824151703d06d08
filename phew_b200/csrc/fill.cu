// Seeded device-side input generation for the verification sweep.
//
// The sweep evaluates every candidate on inputs derived from (seed, variant,
// argument index); drawing them on the host would dominate a sweep over
// decoder-block sizes (hundreds of millions of values per seed and size), so
// they are drawn here from a counter-based generator: element i of stream
// (seed, stream_id) is a pure function of those three numbers, independent
// of the grid, the GPU and the number of GPUs in the sweep.
//
// Generator (fill_host.h): SplitMix64 finalizer over (seed, stream, k) ->
// two 24-bit uniforms; normals in Box-Muller pairs (elements 2k and 2k + 1
// share draw k), uniforms from the draw of their own index, one-hot rows from
// the draw of the row index.
//
// phew_fill_host runs the same generator on host threads, for callers whose
// inputs start in host memory (the sweep's end-to-end leg copies them in):
// the same bits feed the same transforms, so host and device draws agree
// except in the last places of the fp32 value, where the host's vectorised
// series (fill_host.cpp) and the device's logf / sincospif(2u) round apart.
#include <math.h>
#include <string.h>

#include <cmath>

#include <algorithm>
#include <thread>
#include <vector>

#include "common.cuh"
#include "fill_host.h"

namespace phew {
namespace {

template <typename T>
__global__ void fill_kernel(T* out, int64_t n, int64_t cols, int kind, uint64_t seed,
                            uint64_t stream, float scale) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (kind == PHEW_FILL_NORMAL) {
    // one Box-Muller pair (elements 2k, 2k + 1) per iteration
    const int64_t pairs = (n + 1) / 2;
    for (int64_t k = first; k < pairs; k += step) {
      const uint64_t b = draw(seed, stream, static_cast<uint64_t>(k));
      const float r = sqrtf(-2.0f * logf(u24(b))) * scale;
      float sn, cs;
      sincospif(2.0f * u24(b >> 32), &sn, &cs);
      out[2 * k] = from_f32<T>(r * cs);
      if (2 * k + 1 < n) out[2 * k + 1] = from_f32<T>(r * sn);
    }
    return;
  }
  for (int64_t i = first; i < n; i += step) {
    float v;
    switch (kind) {
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

// ---- host twin ------------------------------------------------------------

inline float host_value(int kind, int64_t i, int64_t cols, uint64_t seed, uint64_t stream,
                        float scale) {
  switch (kind) {
    case PHEW_FILL_UNIFORM: {
      const uint64_t b = draw(seed, stream, static_cast<uint64_t>(i));
      return (2.0f * u24(b) - 1.0f) * scale;
    }
    case PHEW_FILL_ONE_HOT_ROWS: {
      const int64_t row = i / cols, col = i % cols;
      const int64_t hot = static_cast<int64_t>(draw(seed, stream, static_cast<uint64_t>(row)) %
                                               static_cast<uint64_t>(cols));
      return col == hot ? scale : 0.0f;
    }
    default:
      return scale;
  }
}

template <typename Store>
void host_fill_typed(Store store, int64_t lo, int64_t hi, int64_t cols, int kind, uint64_t seed,
                     uint64_t stream, float scale) {
  for (int64_t i = lo; i < hi; ++i) store(i, host_value(kind, i, cols, seed, stream, scale));
}

void host_fill_range(void* out, int64_t lo, int64_t hi, int64_t n, int64_t cols, int dtype,
                     int kind, uint64_t seed, uint64_t stream, float scale) {
  if (kind == PHEW_FILL_NORMAL) {
    // [lo, hi) starts on an even index (ranges are split on pair boundaries)
    if (dtype == PHEW_BF16 && std::fabs(scale) < 0x1p-129f)
      host_normals_tiny_bf16(static_cast<uint16_t*>(out), lo / 2, (hi + 1) / 2, n, seed, stream, scale);
    else
      host_normals(out, dtype, lo / 2, (hi + 1) / 2, n, seed, stream, scale);
    return;
  }
  if (dtype == PHEW_F32) {
    float* o = static_cast<float*>(out);
    host_fill_typed([o](int64_t i, float v) { o[i] = v; }, lo, hi, cols, kind, seed, stream, scale);
  } else if (dtype == PHEW_BF16) {
    uint16_t* o = static_cast<uint16_t*>(out);
    host_fill_typed([o](int64_t i, float v) { o[i] = host_bf16_bits(v); }, lo, hi, cols, kind, seed,
                    stream, scale);
  } else {
    uint16_t* o = static_cast<uint16_t*>(out);
    host_fill_typed([o](int64_t i, float v) { o[i] = host_f16_bits(v); }, lo, hi, cols, kind, seed,
                    stream, scale);
  }
}

}  // namespace
}  // namespace phew

using namespace phew;

extern "C" int phew_fill_host(void* out, int64_t n, int64_t cols, int dtype, int kind,
                              uint64_t seed, uint64_t stream_id, float scale, int threads) {
  PHEW_REQUIRE(out != nullptr || n == 0, "phew_fill_host: null output");
  PHEW_REQUIRE(n >= 0 && cols > 0, "phew_fill_host: bad extent");
  PHEW_REQUIRE(kind >= PHEW_FILL_NORMAL && kind <= PHEW_FILL_CONSTANT, "phew_fill_host: bad kind");
  PHEW_REQUIRE(dtype == PHEW_F32 || dtype == PHEW_F16 || dtype == PHEW_BF16,
               "phew_fill_host: bad dtype");
  if (n == 0) return PHEW_OK;
  if (threads <= 0) threads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  // at least 1 Mi elements per thread: thread start-up is not free
  const int64_t max_threads = std::max<int64_t>(1, n >> 20);
  const int nt = static_cast<int>(std::min<int64_t>(threads, max_threads));
  if (nt == 1) {
    host_fill_range(out, 0, n, n, cols, dtype, kind, seed, stream_id, scale);
    return PHEW_OK;
  }
  std::vector<std::thread> pool;
  pool.reserve(nt);
  // even chunk lengths: a normal pair never straddles two threads
  const int64_t per = ((n + nt - 1) / nt + 1) & ~int64_t(1);
  for (int t = 0; t < nt; ++t) {
    const int64_t lo = t * per, hi = std::min(n, lo + per);
    if (lo >= hi) break;
    pool.emplace_back(host_fill_range, out, lo, hi, n, cols, dtype, kind, seed, stream_id, scale);
  }
  for (auto& th : pool) th.join();
  return PHEW_OK;
}

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
