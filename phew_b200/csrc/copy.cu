// Strided copies: view materialisation (Transpose / non-contiguous views) and
// writes into strided destinations (concatenate, pad, slice_update, ...).
//
// Element (i0..in) of `shape` moves from src + sum(ik * src_strides[k]) to
// dst + sum(ik * dst_strides[k]) (a contiguous dst for phew_copy_strided).
// When both innermost strides are 1 and the inner extent and every other
// stride are multiples of 16 bytes, each thread moves 16-byte vectors;
// otherwise single elements.
#include "common.cuh"

namespace phew {
namespace {

constexpr int kMaxDims = 8;

struct Geometry {
  int ndim;
  bool dst_contig;
  int64_t shape[kMaxDims];
  int64_t stride[kMaxDims];      // source, in units of the moved word
  int64_t dst_stride[kMaxDims];  // destination (unused when dst_contig)
};

template <typename W>
__global__ void copy_kernel(const W* __restrict__ src, W* __restrict__ dst, Geometry g,
                            int64_t total) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += step) {
    int64_t rem = i, off = 0, doff = 0;
#pragma unroll
    for (int k = kMaxDims - 1; k >= 0; --k) {
      if (k < g.ndim) {
        const int64_t c = rem % g.shape[k];
        rem /= g.shape[k];
        off += c * g.stride[k];
        doff += c * g.dst_stride[k];
      }
    }
    dst[g.dst_contig ? i : doff] = src[off];
  }
}

template <typename W>
int launch_copy(const void* src, void* dst, const Geometry& g, int64_t total, cudaStream_t st) {
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count_current()) * 32;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  copy_kernel<W><<<static_cast<unsigned>(blocks), 256, 0, st>>>(static_cast<const W*>(src),
                                                               static_cast<W*>(dst), g, total);
  return launch_status("copy_kernel");
}

}  // namespace
}  // namespace phew

using namespace phew;

extern "C" int phew_copy_strided_to(const void* src, void* dst, int ndim, const int64_t* shape,
                                    const int64_t* src_strides, const int64_t* dst_strides,
                                    int elem_bytes, void* stream) {
  PHEW_REQUIRE(src && dst && shape && src_strides, "phew_copy_strided: null argument");
  PHEW_REQUIRE(ndim >= 1 && ndim <= kMaxDims, "phew_copy_strided: ndim must be 1..8");
  PHEW_REQUIRE(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4 || elem_bytes == 8,
               "phew_copy_strided: element size must be 1, 2, 4 or 8 bytes");
  int64_t total = 1;
  for (int k = 0; k < ndim; ++k) {
    PHEW_REQUIRE(shape[k] >= 0, "phew_copy_strided: negative extent");
    total *= shape[k];
  }
  if (total == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Geometry g;
  g.ndim = ndim;
  g.dst_contig = dst_strides == nullptr;
  int64_t contig[kMaxDims];
  {
    int64_t s = 1;
    for (int k = ndim - 1; k >= 0; --k) {
      contig[k] = s;
      s *= shape[k];
    }
  }
  const int64_t* ds = dst_strides ? dst_strides : contig;
  for (int k = 0; k < ndim; ++k) {
    g.shape[k] = shape[k];
    g.stride[k] = src_strides[k];
    g.dst_stride[k] = ds[k];
  }
  // Vectorise along the innermost axis when it is contiguous on both sides.
  const int64_t inner_bytes = shape[ndim - 1] * elem_bytes;
  const bool aligned = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0;
  bool vec = aligned && src_strides[ndim - 1] == 1 && ds[ndim - 1] == 1 && inner_bytes % 16 == 0;
  for (int k = 0; vec && k < ndim - 1; ++k)
    if ((src_strides[k] * elem_bytes) % 16 != 0 || (ds[k] * elem_bytes) % 16 != 0) vec = false;
  if (vec) {
    const int per = 16 / elem_bytes;
    g.shape[ndim - 1] = shape[ndim - 1] / per;
    for (int k = 0; k < ndim - 1; ++k) {
      g.stride[k] = src_strides[k] / per;
      g.dst_stride[k] = ds[k] / per;
    }
    g.stride[ndim - 1] = 1;
    g.dst_stride[ndim - 1] = 1;
    return launch_copy<uint4>(src, dst, g, total / per, st);
  }
  switch (elem_bytes) {
    case 1: return launch_copy<uint8_t>(src, dst, g, total, st);
    case 2: return launch_copy<uint16_t>(src, dst, g, total, st);
    case 4: return launch_copy<uint32_t>(src, dst, g, total, st);
    default: return launch_copy<uint64_t>(src, dst, g, total, st);
  }
}

extern "C" int phew_copy_strided(const void* src, void* dst, int ndim, const int64_t* shape,
                                 const int64_t* src_strides, int elem_bytes, void* stream) {
  return phew_copy_strided_to(src, dst, ndim, shape, src_strides, nullptr, elem_bytes, stream);
}
