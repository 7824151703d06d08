// Row-wise primitives: rms_norm, layer_norm, softmax and axis reductions.
//
// Layout: the reduced axis is the innermost, contiguous one ([rows, cols],
// row-major) except for phew_reduce's strided form ([outer, red, inner]).
// Each CTA row group keeps its row in registers (up to 8 16-byte vectors per
// thread), so a row is read from HBM once and written once: these kernels are
// HBM-bound at 2 * rows * cols * sizeof(T) bytes.
#include <math.h>

#include "common.cuh"

namespace phew {
namespace {

constexpr int kMaxVPT = 8;    // 16-byte vectors held per thread
constexpr int kMaxTPR = 512;  // threads per row (keeps VPT=8 kernels within the register file)

template <typename T> struct Vec {
  static constexpr int E = 16 / sizeof(T);  // elements per 16-byte vector
};

// Loads 16 bytes at p (E elements of T) into fp32 registers.
template <typename T>
__device__ __forceinline__ void load_vec(const T* p, float* out) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::E; ++i) out[i] = to_f32(e[i]);
}

template <typename T>
__device__ __forceinline__ void store_vec(T* p, const float* in) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int i = 0; i < Vec<T>::E; ++i) e[i] = from_f32<T>(in[i]);
  *reinterpret_cast<uint4*>(p) = raw;
}

// Block-wide reduction of one value per row group.  Threads of a row are
// threadIdx.x in [0, blockDim.x); rows of the block are threadIdx.y.
template <bool IS_MAX>
__device__ __forceinline__ float row_allreduce(float v, float* smem) {
  v = IS_MAX ? warp_max(v) : warp_sum(v);
  const int warps_per_row = blockDim.x / 32;
  if (warps_per_row == 1) return v;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* row_smem = smem + threadIdx.y * 32;
  __syncthreads();
  if (lane == 0) row_smem[warp] = v;
  __syncthreads();
  float r = lane < warps_per_row ? row_smem[lane] : (IS_MAX ? -INFINITY : 0.f);
  r = IS_MAX ? warp_max(r) : warp_sum(r);
  return r;
}

// ---------------------------------------------------------------------------
// rms_norm: y = w * T(x * rsqrt(mean(x^2) + eps))
// ---------------------------------------------------------------------------
//
// EXACT: blockDim.x * VPT vectors cover the row exactly, so no load needs a
// guard: the threads of a row past the end (the last CTA's spare rows) read
// the last row instead and store nothing.  Without guards the body is
// straight-line code that keeps all of a thread's loads in flight together;
// with them (even the row's own `active` test alone) the compiler issued the
// loads group by group (0.71 vs 0.96 of the HBM copy rate on 8192-wide bf16
// rows).
template <typename T, int VPT, bool EXACT>
__global__ void __launch_bounds__(512) rms_norm_vec_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                    T* __restrict__ y, int64_t rows, int64_t cols, float eps) {
  __shared__ float smem[32 * 32];
  constexpr int E = Vec<T>::E;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  const int64_t nvec = cols / E;
  const T* xr = x + (EXACT && !active ? rows - 1 : row) * cols;
  float v[VPT][E];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    if (EXACT || (active && vi < nvec)) {
      load_vec<T>(xr + vi * E, v[j]);
#pragma unroll
      for (int i = 0; i < E; ++i) ss = fmaf(v[j][i], v[j][i], ss);
    }
  }
  const float total = row_allreduce<false>(ss, smem);
  const float r = 1.0f / sqrtf(total / static_cast<float>(cols) + eps);
  if (!active) return;
  T* yr = y + row * cols;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    if (EXACT || vi < nvec) {
      float o[E];
      if (w != nullptr) {
        float wv[E];
        load_vec<T>(w + vi * E, wv);
#pragma unroll
        for (int i = 0; i < E; ++i) o[i] = __fmul_rn(wv[i], round_to<T>(__fmul_rn(v[j][i], r)));
      } else {
#pragma unroll
        for (int i = 0; i < E; ++i) o[i] = __fmul_rn(v[j][i], r);
      }
      store_vec<T>(yr + vi * E, o);
    }
  }
}

// Scalar two-pass form for unaligned rows or rows too long for registers.
template <typename T>
__global__ void rms_norm_loop_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                     T* __restrict__ y, int64_t rows, int64_t cols, float eps) {
  __shared__ float smem[32 * 32];
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  const T* xr = x + row * cols;
  float ss = 0.f;
  if (active)
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float a = to_f32(xr[c]);
      ss = fmaf(a, a, ss);
    }
  const float total = row_allreduce<false>(ss, smem);
  const float r = 1.0f / sqrtf(total / static_cast<float>(cols) + eps);
  if (!active) return;
  T* yr = y + row * cols;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float n = __fmul_rn(to_f32(xr[c]), r);
    yr[c] = from_f32<T>(w != nullptr ? __fmul_rn(to_f32(w[c]), round_to<T>(n)) : n);
  }
}

// ---------------------------------------------------------------------------
// layer_norm: n = T((x - mean) * rsqrt(var + eps)), y = T(w * n + b)
// (mean and the biased variance in fp32 over the row; w, b optional)
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float ln_out(float n, const T* w, const T* b, int64_t c) {
  float y = round_to<T>(n);
  if (w != nullptr) y = __fmul_rn(to_f32(w[c]), y);
  if (b != nullptr) y = __fadd_rn(y, to_f32(b[c]));
  return y;
}

// EXACT: as for rms_norm_vec_kernel.
template <typename T, int VPT, bool EXACT>
__global__ void __launch_bounds__(512) layer_norm_vec_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                             const T* __restrict__ b, T* __restrict__ y,
                                                             int64_t rows, int64_t cols, float eps) {
  __shared__ float smem[32 * 32];
  constexpr int E = Vec<T>::E;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  const int64_t nvec = cols / E;
  const T* xr = x + (EXACT && !active ? rows - 1 : row) * cols;
  float v[VPT][E];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    if (EXACT || (active && vi < nvec)) {
      load_vec<T>(xr + vi * E, v[j]);
#pragma unroll
      for (int i = 0; i < E; ++i) sum += v[j][i];
    }
  }
  const float mean = row_allreduce<false>(sum, smem) / static_cast<float>(cols);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    if (EXACT || (active && vi < nvec)) {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        v[j][i] = __fsub_rn(v[j][i], mean);
        ss = fmaf(v[j][i], v[j][i], ss);
      }
    }
  }
  const float var = row_allreduce<false>(ss, smem) / static_cast<float>(cols);
  const float r = 1.0f / sqrtf(var + eps);
  if (!active) return;
  T* yr = y + row * cols;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
    if (EXACT || vi < nvec) {
      float o[E];
#pragma unroll
      for (int i = 0; i < E; ++i) o[i] = ln_out<T>(__fmul_rn(v[j][i], r), w, b, vi * E + i);
      store_vec<T>(yr + vi * E, o);
    }
  }
}

template <typename T>
__global__ void layer_norm_loop_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                       const T* __restrict__ b, T* __restrict__ y, int64_t rows,
                                       int64_t cols, float eps) {
  __shared__ float smem[32 * 32];
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  const T* xr = x + row * cols;
  float sum = 0.f;
  if (active)
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) sum += to_f32(xr[c]);
  const float mean = row_allreduce<false>(sum, smem) / static_cast<float>(cols);
  float ss = 0.f;
  if (active)
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
      const float d = __fsub_rn(to_f32(xr[c]), mean);
      ss = fmaf(d, d, ss);
    }
  const float var = row_allreduce<false>(ss, smem) / static_cast<float>(cols);
  const float r = 1.0f / sqrtf(var + eps);
  if (!active) return;
  T* yr = y + row * cols;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
    yr[c] = from_f32<T>(ln_out<T>(__fmul_rn(__fsub_rn(to_f32(xr[c]), mean), r), w, b, c));
}

// ---------------------------------------------------------------------------
// softmax over the last axis: y = exp(x - max) / sum(exp(x - max))
// ---------------------------------------------------------------------------
// For 16-bit rows the exponential is the hardware 2^x of (x - max) * log2(e)
// and the division a multiply by the row's reciprocal sum: both err by a few
// fp32 ulps, far below half an ulp of the 16-bit result, and they keep the
// kernel at the HBM rate instead of the cost of the IEEE exp and division
// (which fp32 rows keep).
template <typename T>
__device__ __forceinline__ float softmax_exp(float d) {
  if (sizeof(T) == 4) return expf(d);
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d * 1.44269504088896341f));
  return y;
}

// Persistent row groups: CTA b handles row groups b, b + gridDim.x, ...; the
// raw 16-byte vectors of its next row group are loaded into registers before
// the current one's reductions, so loads stay in flight across them (a CTA
// per row left the loads idle for the two block reductions and the store).
// Per-element arithmetic and reduction order are those of one row per CTA.
template <typename T, int VPT>
__global__ void __launch_bounds__(512) softmax_vec_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                   int64_t cols) {
  __shared__ float smem[32 * 32];
  constexpr int E = Vec<T>::E;
  const int64_t nvec = cols / E;
  const int64_t groups = (rows + blockDim.y - 1) / blockDim.y;
  uint4 cur[VPT], nxt[VPT];
  auto load_group = [&](int64_t g, uint4* buf) {
    const int64_t row = g * blockDim.y + threadIdx.y;
    const T* xr = x + row * cols;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
      if (row < rows && vi < nvec) buf[j] = __ldg(reinterpret_cast<const uint4*>(xr + vi * E));
    }
  };
  int64_t g = blockIdx.x;
  if (g < groups) load_group(g, cur);
  for (; g < groups; g += gridDim.x) {
    const int64_t gn = g + gridDim.x;
    if (gn < groups) load_group(gn, nxt);
    const int64_t row = g * blockDim.y + threadIdx.y;
    const bool active = row < rows;
    float v[VPT][E];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
      if (active && vi < nvec) {
        const T* e = reinterpret_cast<const T*>(&cur[j]);
#pragma unroll
        for (int i = 0; i < E; ++i) {
          v[j][i] = to_f32(e[i]);
          m = fmaxf(m, v[j][i]);
        }
      }
    }
    m = row_allreduce<true>(m, smem);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
      if (active && vi < nvec) {
#pragma unroll
        for (int i = 0; i < E; ++i) {
          v[j][i] = softmax_exp<T>(v[j][i] - m);
          s += v[j][i];
        }
      }
    }
    s = row_allreduce<false>(s, smem);
    if (active) {
      T* yr = y + row * cols;
      const float inv = 1.0f / s;
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int64_t vi = threadIdx.x + static_cast<int64_t>(j) * blockDim.x;
        if (vi < nvec) {
          float o[E];
#pragma unroll
          for (int i = 0; i < E; ++i) o[i] = sizeof(T) == 4 ? __fdiv_rn(v[j][i], s) : v[j][i] * inv;
          store_vec<T>(yr + vi * E, o);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < VPT; ++j) cur[j] = nxt[j];
  }
}

// One row group per CTA, the vectors covering each row exactly (EXACT of
// rms_norm_vec_kernel: a spare row reads the last row and stores nothing).
// Per-element arithmetic and reduction order are those of softmax_vec_kernel
// (and of the fused softmax mx.compile emits), so the bits are the same.
template <typename T, int VPT>
__global__ void __launch_bounds__(512) softmax_row_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                          int64_t rows, int64_t cols) {
  __shared__ float smem[32 * 32];
  constexpr int E = Vec<T>::E;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  if (blockDim.y == 1 && !active) return;  // the whole CTA
  const int stride = blockDim.x * E;  // elements between a thread's vectors
  const T* xt = x + (active ? row : rows - 1) * cols + threadIdx.x * E;
  float v[VPT][E];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    load_vec<T>(xt + j * stride, v[j]);
#pragma unroll
    for (int i = 0; i < E; ++i) m = fmaxf(m, v[j][i]);
  }
  m = row_allreduce<true>(m, smem);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j)
#pragma unroll
    for (int i = 0; i < E; ++i) {
      v[j][i] = softmax_exp<T>(v[j][i] - m);
      s += v[j][i];
    }
  s = row_allreduce<false>(s, smem);
  if (!active) return;
  T* yt = y + row * cols + threadIdx.x * E;
  const float inv = 1.0f / s;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    float o[E];
#pragma unroll
    for (int i = 0; i < E; ++i) o[i] = sizeof(T) == 4 ? __fdiv_rn(v[j][i], s) : v[j][i] * inv;
    store_vec<T>(yt + j * stride, o);
  }
}

template <typename T>
__global__ void softmax_loop_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                    int64_t cols) {
  __shared__ float smem[32 * 32];
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  const T* xr = x + row * cols;
  float m = -INFINITY;
  if (active)
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, to_f32(xr[c]));
  m = row_allreduce<true>(m, smem);
  float s = 0.f;
  if (active)
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) s += softmax_exp<T>(to_f32(xr[c]) - m);
  s = row_allreduce<false>(s, smem);
  if (!active) return;
  T* yr = y + row * cols;
  const float inv = 1.0f / s;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float e = softmax_exp<T>(to_f32(xr[c]) - m);
    yr[c] = from_f32<T>(sizeof(T) == 4 ? __fdiv_rn(e, s) : e * inv);
  }
}

// ---------------------------------------------------------------------------
// Reductions over the middle axis of [outer, red, inner]
// ---------------------------------------------------------------------------
__device__ __forceinline__ float combine(int op, float a, float b) {
  switch (op) {
    case PHEW_REDUCE_MAX: return (b > a || isnan(b)) && !isnan(a) ? b : a;
    case PHEW_REDUCE_MIN: return (b < a || isnan(b)) && !isnan(a) ? b : a;
    case PHEW_REDUCE_PROD: return a * b;
    default: return a + b;
  }
}
__device__ __forceinline__ float identity(int op) {
  switch (op) {
    case PHEW_REDUCE_MAX: return -INFINITY;
    case PHEW_REDUCE_MIN: return INFINITY;
    case PHEW_REDUCE_PROD: return 1.f;
    default: return 0.f;
  }
}

// inner == 1: one row group per reduced row.
template <typename T>
__global__ void reduce_rows_kernel(int op, const T* __restrict__ x, T* __restrict__ y,
                                   int64_t rows, int64_t red) {
  __shared__ float smem[32 * 32];
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  const T* xr = x + row * red;
  float acc = identity(op);
  if (active)
    for (int64_t c = threadIdx.x; c < red; c += blockDim.x) acc = combine(op, acc, to_f32(xr[c]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = combine(op, acc, __shfl_xor_sync(0xffffffffu, acc, o));
  const int warps_per_row = blockDim.x / 32;
  if (warps_per_row > 1) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* row_smem = smem + threadIdx.y * 32;
    __syncthreads();
    if (lane == 0) row_smem[warp] = acc;
    __syncthreads();
    acc = lane < warps_per_row ? row_smem[lane] : identity(op);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = combine(op, acc, __shfl_xor_sync(0xffffffffu, acc, o));
  }
  if (active && threadIdx.x == 0) {
    if (op == PHEW_REDUCE_MEAN) acc = __fdiv_rn(acc, static_cast<float>(red));
    y[row] = from_f32<T>(acc);
  }
}

// inner > 1: one thread per (outer, inner) output, coalesced along inner.
template <typename T>
__global__ void reduce_cols_kernel(int op, const T* __restrict__ x, T* __restrict__ y,
                                   int64_t outer, int64_t red, int64_t inner) {
  const int64_t total = outer * inner;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t o = idx / inner, i = idx % inner;
    const T* p = x + o * red * inner + i;
    float acc = identity(op);
    for (int64_t r = 0; r < red; ++r) acc = combine(op, acc, to_f32(p[r * inner]));
    if (op == PHEW_REDUCE_MEAN) acc = __fdiv_rn(acc, static_cast<float>(red));
    y[idx] = from_f32<T>(acc);
  }
}

// Chooses threads-per-row (multiple of 32) and rows-per-block for a row of
// `nvec` vectors so that each thread holds about 4 vectors.
struct RowLaunch {
  int tpr, rpb, vpt;
};
RowLaunch plan_rows(int64_t nvec) {
  int tpr = static_cast<int>(((nvec + 3) / 4 + 31) / 32 * 32);
  if (tpr < 32) tpr = 32;
  if (tpr > kMaxTPR) tpr = kMaxTPR;
  int vpt = static_cast<int>((nvec + tpr - 1) / tpr);
  int rpb = tpr >= 128 ? 1 : 128 / tpr;
  return {tpr, rpb, vpt};
}

template <typename T>
int rms_norm_typed(const void* x, const void* w, void* y, int64_t rows, int64_t cols, float eps,
                   cudaStream_t st) {
  constexpr int E = Vec<T>::E;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(w)) & 15) == 0;
  const int64_t nvec = cols / E;
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(w);
  T* yp = static_cast<T*>(y);
  if (aligned && cols % E == 0 && nvec <= static_cast<int64_t>(kMaxTPR) * kMaxVPT) {
    RowLaunch L = plan_rows(nvec);
    dim3 block(L.tpr, L.rpb), grid(static_cast<unsigned>((rows + L.rpb - 1) / L.rpb));
    const bool exact = static_cast<int64_t>(L.tpr) * L.vpt == nvec;
    switch (L.vpt) {
#define PHEW_CASE(N) \
  case N:                                                                                          \
    if (exact) rms_norm_vec_kernel<T, N, true><<<grid, block, 0, st>>>(xp, wp, yp, rows, cols, eps); \
    else rms_norm_vec_kernel<T, N, false><<<grid, block, 0, st>>>(xp, wp, yp, rows, cols, eps);      \
    break;
      PHEW_CASE(1) PHEW_CASE(2) PHEW_CASE(3) PHEW_CASE(4)
      PHEW_CASE(5) PHEW_CASE(6) PHEW_CASE(7) PHEW_CASE(8)
#undef PHEW_CASE
      default: return set_error(PHEW_ERR_INVALID, "rms_norm: bad plan");
    }
    return launch_status("rms_norm_vec_kernel");
  }
  const int tpr = cols >= 1024 ? 256 : 32;
  const int rpb = tpr == 32 ? 4 : 1;
  dim3 block(tpr, rpb), grid(static_cast<unsigned>((rows + rpb - 1) / rpb));
  rms_norm_loop_kernel<T><<<grid, block, 0, st>>>(xp, wp, yp, rows, cols, eps);
  return launch_status("rms_norm_loop_kernel");
}

template <typename T>
int layer_norm_typed(const void* x, const void* w, const void* b, void* y, int64_t rows, int64_t cols,
                     float eps, cudaStream_t st) {
  constexpr int E = Vec<T>::E;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const int64_t nvec = cols / E;
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(w);
  const T* bp = static_cast<const T*>(b);
  T* yp = static_cast<T*>(y);
  if (aligned && cols % E == 0 && nvec <= static_cast<int64_t>(kMaxTPR) * kMaxVPT) {
    RowLaunch L = plan_rows(nvec);
    dim3 block(L.tpr, L.rpb), grid(static_cast<unsigned>((rows + L.rpb - 1) / L.rpb));
    const bool exact = static_cast<int64_t>(L.tpr) * L.vpt == nvec;
    switch (L.vpt) {
#define PHEW_CASE(N) \
  case N:                                                                                                  \
    if (exact) layer_norm_vec_kernel<T, N, true><<<grid, block, 0, st>>>(xp, wp, bp, yp, rows, cols, eps); \
    else layer_norm_vec_kernel<T, N, false><<<grid, block, 0, st>>>(xp, wp, bp, yp, rows, cols, eps);      \
    break;
      PHEW_CASE(1) PHEW_CASE(2) PHEW_CASE(3) PHEW_CASE(4)
      PHEW_CASE(5) PHEW_CASE(6) PHEW_CASE(7) PHEW_CASE(8)
#undef PHEW_CASE
      default: return set_error(PHEW_ERR_INVALID, "layer_norm: bad plan");
    }
    return launch_status("layer_norm_vec_kernel");
  }
  const int tpr = cols >= 1024 ? 256 : 32;
  const int rpb = tpr == 32 ? 4 : 1;
  dim3 block(tpr, rpb), grid(static_cast<unsigned>((rows + rpb - 1) / rpb));
  layer_norm_loop_kernel<T><<<grid, block, 0, st>>>(xp, wp, bp, yp, rows, cols, eps);
  return launch_status("layer_norm_loop_kernel");
}

template <typename T>
int softmax_typed(const void* x, void* y, int64_t rows, int64_t cols, cudaStream_t st) {
  constexpr int E = Vec<T>::E;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const int64_t nvec = cols / E;
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  if (aligned && cols % E == 0 && nvec <= static_cast<int64_t>(kMaxTPR) * kMaxVPT) {
    RowLaunch L = plan_rows(nvec);  // the mapping the emitted fused softmax follows too
    const int64_t groups = (rows + L.rpb - 1) / L.rpb;
    dim3 block(L.tpr, L.rpb);
    if (static_cast<int64_t>(L.tpr) * L.vpt == nvec && groups <= 0x7fffffff) {
      const dim3 grid(static_cast<unsigned>(groups));
      switch (L.vpt) {
#define PHEW_CASE(N) \
  case N: softmax_row_kernel<T, N><<<grid, block, 0, st>>>(xp, yp, rows, cols); break;
        PHEW_CASE(1) PHEW_CASE(2) PHEW_CASE(3) PHEW_CASE(4)
        PHEW_CASE(5) PHEW_CASE(6) PHEW_CASE(7) PHEW_CASE(8)
#undef PHEW_CASE
        default: return set_error(PHEW_ERR_INVALID, "softmax: bad plan");
      }
      return launch_status("softmax_row_kernel");
    }
    // persistent: as many CTAs as fit on the GPU at once (or one per group)
    auto grid_for = [&](const void* fn) {
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, L.tpr * L.rpb, 0) != cudaSuccess ||
          per_sm < 1)
        per_sm = 1;
      const int64_t cap = static_cast<int64_t>(sm_count_current()) * per_sm;
      return dim3(static_cast<unsigned>(groups < cap ? groups : cap));
    };
    switch (L.vpt) {
#define PHEW_CASE(N) \
  case N: softmax_vec_kernel<T, N><<<grid_for(reinterpret_cast<const void*>(softmax_vec_kernel<T, N>)), block, 0, st>>>(xp, yp, rows, cols); break;
      PHEW_CASE(1) PHEW_CASE(2) PHEW_CASE(3) PHEW_CASE(4)
      PHEW_CASE(5) PHEW_CASE(6) PHEW_CASE(7) PHEW_CASE(8)
#undef PHEW_CASE
      default: return set_error(PHEW_ERR_INVALID, "softmax: bad plan");
    }
    return launch_status("softmax_vec_kernel");
  }
  const int tpr = cols >= 1024 ? 256 : 32;
  const int rpb = tpr == 32 ? 4 : 1;
  dim3 block(tpr, rpb), grid(static_cast<unsigned>((rows + rpb - 1) / rpb));
  softmax_loop_kernel<T><<<grid, block, 0, st>>>(xp, yp, rows, cols);
  return launch_status("softmax_loop_kernel");
}

// Variance over the middle axis: fp32 mean, then the fp32 sum of squared
// deviations divided by (red - ddof), rounded once to T.
template <typename T>
__global__ void var_rows_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int64_t red,
                                float denom) {
  __shared__ float smem[32 * 32];
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.y + threadIdx.y;
  const bool active = row < rows;
  const T* xr = x + row * red;
  float sum = 0.f;
  if (active)
    for (int64_t c = threadIdx.x; c < red; c += blockDim.x) sum += to_f32(xr[c]);
  const float mean = row_allreduce<false>(sum, smem) / static_cast<float>(red);
  float ss = 0.f;
  if (active)
    for (int64_t c = threadIdx.x; c < red; c += blockDim.x) {
      const float d = __fsub_rn(to_f32(xr[c]), mean);
      ss = fmaf(d, d, ss);
    }
  ss = row_allreduce<false>(ss, smem);
  if (active && threadIdx.x == 0) y[row] = from_f32<T>(__fdiv_rn(ss, denom));
}

template <typename T>
__global__ void var_cols_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t outer, int64_t red,
                                int64_t inner, float denom) {
  const int64_t total = outer * inner;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t o = idx / inner, i = idx % inner;
    const T* p = x + o * red * inner + i;
    float sum = 0.f;
    for (int64_t r = 0; r < red; ++r) sum += to_f32(p[r * inner]);
    const float mean = sum / static_cast<float>(red);
    float ss = 0.f;
    for (int64_t r = 0; r < red; ++r) {
      const float d = __fsub_rn(to_f32(p[r * inner]), mean);
      ss = fmaf(d, d, ss);
    }
    y[idx] = from_f32<T>(__fdiv_rn(ss, denom));
  }
}

template <typename T>
int var_typed(const void* x, void* y, int64_t outer, int64_t red, int64_t inner, float denom,
              cudaStream_t st) {
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  if (inner == 1) {
    const int tpr = red >= 1024 ? 256 : 32;
    const int rpb = tpr == 32 ? 4 : 1;
    dim3 block(tpr, rpb), grid(static_cast<unsigned>((outer + rpb - 1) / rpb));
    var_rows_kernel<T><<<grid, block, 0, st>>>(xp, yp, outer, red, denom);
    return launch_status("var_rows_kernel");
  }
  const int64_t total = outer * inner;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count_current()) * 16;
  if (blocks > cap) blocks = cap;
  var_cols_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(xp, yp, outer, red, inner, denom);
  return launch_status("var_cols_kernel");
}

template <typename T>
int reduce_typed(int op, const void* x, void* y, int64_t outer, int64_t red, int64_t inner,
                 cudaStream_t st) {
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  if (inner == 1) {
    const int tpr = red >= 1024 ? 256 : 32;
    const int rpb = tpr == 32 ? 4 : 1;
    dim3 block(tpr, rpb), grid(static_cast<unsigned>((outer + rpb - 1) / rpb));
    reduce_rows_kernel<T><<<grid, block, 0, st>>>(op, xp, yp, outer, red);
    return launch_status("reduce_rows_kernel");
  }
  const int64_t total = outer * inner;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count_current()) * 16;
  if (blocks > cap) blocks = cap;
  reduce_cols_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(op, xp, yp, outer, red, inner);
  return launch_status("reduce_cols_kernel");
}

}  // namespace
}  // namespace phew

using namespace phew;

extern "C" int phew_rms_norm(const void* x, const void* w, void* y, int64_t rows, int64_t cols,
                             float eps, int dtype, void* stream) {
  PHEW_REQUIRE(x && y, "phew_rms_norm: null pointer");
  PHEW_REQUIRE(rows >= 0 && cols > 0, "phew_rms_norm: bad shape");
  PHEW_REQUIRE(rows < (1LL << 31) * 1024, "phew_rms_norm: too many rows");
  if (rows == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PHEW_F32: return rms_norm_typed<float>(x, w, y, rows, cols, eps, st);
    case PHEW_F16: return rms_norm_typed<f16>(x, w, y, rows, cols, eps, st);
    case PHEW_BF16: return rms_norm_typed<bf16>(x, w, y, rows, cols, eps, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_rms_norm: bad dtype");
  }
}

extern "C" int phew_layer_norm(const void* x, const void* w, const void* b, void* y, int64_t rows,
                               int64_t cols, float eps, int dtype, void* stream) {
  PHEW_REQUIRE(x && y, "phew_layer_norm: null pointer");
  PHEW_REQUIRE(rows >= 0 && cols > 0, "phew_layer_norm: bad shape");
  PHEW_REQUIRE(rows < (1LL << 31) * 1024, "phew_layer_norm: too many rows");
  if (rows == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PHEW_F32: return layer_norm_typed<float>(x, w, b, y, rows, cols, eps, st);
    case PHEW_F16: return layer_norm_typed<f16>(x, w, b, y, rows, cols, eps, st);
    case PHEW_BF16: return layer_norm_typed<bf16>(x, w, b, y, rows, cols, eps, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_layer_norm: bad dtype");
  }
}

extern "C" int phew_softmax(const void* x, void* y, int64_t rows, int64_t cols, int dtype,
                            void* stream) {
  PHEW_REQUIRE(x && y, "phew_softmax: null pointer");
  PHEW_REQUIRE(rows >= 0 && cols > 0, "phew_softmax: bad shape");
  if (rows == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PHEW_F32: return softmax_typed<float>(x, y, rows, cols, st);
    case PHEW_F16: return softmax_typed<f16>(x, y, rows, cols, st);
    case PHEW_BF16: return softmax_typed<bf16>(x, y, rows, cols, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_softmax: bad dtype");
  }
}

extern "C" int phew_reduce_var(const void* x, void* y, int64_t outer, int64_t red, int64_t inner,
                               int ddof, int dtype, void* stream) {
  PHEW_REQUIRE(x && y, "phew_reduce_var: null pointer");
  PHEW_REQUIRE(outer >= 0 && red > 0 && inner > 0, "phew_reduce_var: bad shape");
  if (outer == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float denom = static_cast<float>(red - ddof);
  switch (dtype) {
    case PHEW_F32: return var_typed<float>(x, y, outer, red, inner, denom, st);
    case PHEW_F16: return var_typed<f16>(x, y, outer, red, inner, denom, st);
    case PHEW_BF16: return var_typed<bf16>(x, y, outer, red, inner, denom, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_reduce_var: bad dtype");
  }
}

extern "C" int phew_reduce(int op, const void* x, void* y, int64_t outer, int64_t red,
                           int64_t inner, int dtype, void* stream) {
  PHEW_REQUIRE(x && y, "phew_reduce: null pointer");
  PHEW_REQUIRE(outer >= 0 && red > 0 && inner > 0, "phew_reduce: bad shape");
  PHEW_REQUIRE(op >= PHEW_REDUCE_SUM && op <= PHEW_REDUCE_PROD, "phew_reduce: bad op");
  if (outer == 0) return PHEW_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PHEW_F32: return reduce_typed<float>(op, x, y, outer, red, inner, st);
    case PHEW_F16: return reduce_typed<f16>(op, x, y, outer, red, inner, st);
    case PHEW_BF16: return reduce_typed<bf16>(op, x, y, outer, red, inner, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_reduce: bad dtype");
  }
}
