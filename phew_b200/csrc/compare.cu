// Device-side equivalence comparison: the numpy comparison of the reference's
// EquivalenceChecker (verify/checker.py:144-209, _allclose :220-233) done in
// HBM, so a verification unit reads each output once instead of copying it to
// the host.
//
// Three launches, all with a grid that depends only on n (so the result bits
// do not depend on which GPU ran them):
//   1. stats:   per block, sum |b| (fp64) and the count of non-finite b
//   2. compare: every block derives the tolerance from the stats partials in a
//               fixed order, then counts allclose failures, NaNs and max |b-c|
//   3. final:   one block sums the compare partials and writes the record
// Scratch (caller-owned): kMaxBlocks stats partials + kMaxBlocks compare
// partials.
#include <math.h>

#include "common.cuh"

namespace phew {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 1024;

struct StatsPartial {
  double sum_abs;
  long long nonfinite;
};
struct ComparePartial {
  double max_diff;
  long long mismatch;
  long long nan_any;
  long long pad;
};

int blocks_for(int64_t n) {
  int64_t b = (n + 65535) / 65536;
  if (b < 1) b = 1;
  if (b > kMaxBlocks) b = kMaxBlocks;
  return static_cast<int>(b);
}

template <typename T> __device__ __forceinline__ T load_elem(const T* p, int64_t i) { return p[i]; }

// Fixed-order block sum of a double and a count: per-thread values are reduced
// by a shuffle tree and then across warps in warp order.
__device__ void block_sum2(double& d, long long& k) {
  __shared__ double sd[kThreads / 32];
  __shared__ long long sk[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    d += __shfl_xor_sync(0xffffffffu, d, o);
    k += __shfl_xor_sync(0xffffffffu, k, o);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sd[warp] = d;
    sk[warp] = k;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    d = 0.0;
    k = 0;
    for (int w = 0; w < kThreads / 32; ++w) {
      d += sd[w];
      k += sk[w];
    }
  }
  __syncthreads();
}

template <typename T>
__global__ void stats_kernel(const T* __restrict__ b, int64_t n, StatsPartial* part) {
  double s = 0.0;
  long long nf = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = to_f32(b[i]);
    if (isfinite(v)) {
      s += fabs(static_cast<double>(v));
    } else {
      ++nf;
      s += fabs(static_cast<double>(v));  // mean|b| is only used when all are finite
    }
  }
  block_sum2(s, nf);
  if (threadIdx.x == 0) {
    part[blockIdx.x].sum_abs = s;
    part[blockIdx.x].nonfinite = nf;
  }
}

struct Tol {
  int skipped;
  double mean_abs;
  double atol, rtol;
  double sum_abs;
  long long nonfinite;
};

// Every block computes the same tolerance from the stats partials.
__device__ Tol derive_tolerance(const StatsPartial* part, int nblocks, int64_t n, int dtype,
                                double atol, double rtol) {
  __shared__ Tol tol;
  if (threadIdx.x < 32) {
    double s = 0.0;
    long long nf = 0;
    for (int i = threadIdx.x; i < nblocks; i += 32) {
      s += part[i].sum_abs;
      nf += part[i].nonfinite;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s += __shfl_xor_sync(0xffffffffu, s, o);
      nf += __shfl_xor_sync(0xffffffffu, nf, o);
    }
    if (threadIdx.x == 0) {
      Tol t;
      t.sum_abs = s;
      t.nonfinite = nf;
      t.mean_abs = n > 0 ? s / static_cast<double>(n) : 0.0;
      t.skipped = 0;
      t.atol = atol;
      t.rtol = rtol;
      if (nf > 0) {
        t.skipped = 1;  // baseline numerically undefined (checker.py:155-156)
      } else if (dtype == PHEW_BF16) {
        if (t.mean_abs > 1e10) {
          t.skipped = 1;  // extreme-scale bf16 output (checker.py:163-164)
        } else {
          const double f = t.mean_abs > 1e6 ? 0.30 : 0.05;  // checker.py:174-190
          t.atol = fmax(atol, t.mean_abs * f);
          t.rtol = fmax(rtol, f);
        }
      }
      tol = t;
    }
  }
  __syncthreads();
  return tol;
}

// numpy isclose(x, y) = (|x - y| <= atol + rtol * |y|) & isfinite(y) | (x == y)
// in the arithmetic of the compared arrays.
__device__ __forceinline__ bool close_f32(float x, float y, float atol, float rtol) {
  const float d = fabsf(__fsub_rn(x, y));
  const float lim = __fadd_rn(atol, __fmul_rn(rtol, fabsf(y)));
  return (d <= lim && isfinite(y)) || x == y;
}
__device__ __forceinline__ float r16(float v) { return round_to<f16>(v); }
__device__ __forceinline__ bool close_f16(float x, float y, float atol16, float rtol16) {
  const float d = fabsf(r16(__fsub_rn(x, y)));
  const float lim = r16(__fadd_rn(atol16, r16(__fmul_rn(rtol16, fabsf(y)))));
  return (d <= lim && isfinite(y)) || x == y;
}

template <typename T>
__global__ void compare_kernel(const T* __restrict__ b, const T* __restrict__ c, int64_t n,
                               int dtype, double atol, double rtol, const StatsPartial* stats,
                               int nblocks, ComparePartial* part) {
  const Tol t = derive_tolerance(stats, nblocks, n, dtype, atol, rtol);
  double mx = 0.0;
  long long mism = 0, nans = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const bool half = dtype == PHEW_F16;
  const float a32 = half ? r16(static_cast<float>(t.atol)) : static_cast<float>(t.atol);
  const float r32 = half ? r16(static_cast<float>(t.rtol)) : static_cast<float>(t.rtol);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float x = to_f32(b[i]);
    const float y = to_f32(c[i]);
    const bool xn = isnan(x), yn = isnan(y);
    if (xn || yn) ++nans;
    const double d = fabs(static_cast<double>(x) - static_cast<double>(y));
    if (!isnan(d)) mx = fmax(mx, d);
    if (!t.skipped) {
      const float x0 = xn ? 0.f : x, y0 = yn ? 0.f : y;
      const bool cl = half ? close_f16(x0, y0, a32, r32) : close_f32(x0, y0, a32, r32);
      const bool ok = (xn == yn) && (xn || cl);
      if (!ok) ++mism;
    }
  }
  // max is order-independent; counts are exact.
  __shared__ double smx[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) smx[threadIdx.x >> 5] = mx;
  double dummy = 0.0;
  block_sum2(dummy, mism);
  double dummy2 = 0.0;
  block_sum2(dummy2, nans);
  if (threadIdx.x == 0) {
    double m = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) m = fmax(m, smx[w]);
    part[blockIdx.x].max_diff = m;
    part[blockIdx.x].mismatch = mism;
    part[blockIdx.x].nan_any = nans;
  }
}

__global__ void final_kernel(const StatsPartial* stats, const ComparePartial* part, int nblocks,
                             int64_t n, int dtype, double atol, double rtol,
                             phew_compare_stats* out) {
  const Tol t = derive_tolerance(stats, nblocks, n, dtype, atol, rtol);
  // the warp reads the partials together (one thread walking 1024 of them
  // took ~120 us); the max is order-independent and the counts are exact
  double mx = 0.0;
  long long mism = 0, nans = 0;
#pragma unroll 4
  for (int i = threadIdx.x; i < nblocks; i += 32) {
    mx = fmax(mx, part[i].max_diff);
    mism += part[i].mismatch;
    nans += part[i].nan_any;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mism += __shfl_xor_sync(0xffffffffu, mism, o);
    nans += __shfl_xor_sync(0xffffffffu, nans, o);
  }
  if (threadIdx.x != 0) return;
  out->sum_abs_base = t.sum_abs;
  out->mean_abs_base = t.mean_abs;
  out->max_abs_diff = mx;
  out->atol_used = t.atol;
  out->rtol_used = t.rtol;
  out->n = n;
  out->n_nonfinite_base = t.nonfinite;
  out->n_mismatch = t.skipped ? 0 : mism;
  out->n_nan_any = nans;
  out->skipped = t.skipped;
  out->passed = t.skipped ? 1 : (mism == 0 ? 1 : 0);
}

template <typename T>
int compare_typed(const void* b, const void* c, int64_t n, int dtype, double atol, double rtol,
                  void* scratch, phew_compare_stats* out, cudaStream_t st) {
  const int nb = blocks_for(n);
  StatsPartial* sp = static_cast<StatsPartial*>(scratch);
  ComparePartial* cp = reinterpret_cast<ComparePartial*>(
      static_cast<char*>(scratch) + sizeof(StatsPartial) * kMaxBlocks);
  const T* bp = static_cast<const T*>(b);
  const T* cpp = static_cast<const T*>(c);
  stats_kernel<T><<<nb, kThreads, 0, st>>>(bp, n, sp);
  int s = launch_status("compare stats_kernel");
  if (s) return s;
  compare_kernel<T><<<nb, kThreads, 0, st>>>(bp, cpp, n, dtype, atol, rtol, sp, nb, cp);
  s = launch_status("compare_kernel");
  if (s) return s;
  final_kernel<<<1, 32, 0, st>>>(sp, cp, nb, n, dtype, atol, rtol, out);
  return launch_status("compare final_kernel");
}

}  // namespace
}  // namespace phew

using namespace phew;

extern "C" size_t phew_compare_scratch_bytes(int64_t n) {
  (void)n;
  return sizeof(StatsPartial) * kMaxBlocks + sizeof(ComparePartial) * kMaxBlocks;
}

extern "C" int phew_compare(const void* b, const void* c, int64_t n, int dtype, double atol,
                            double rtol, void* scratch, size_t scratch_bytes,
                            phew_compare_stats* out, void* stream) {
  PHEW_REQUIRE(out != nullptr && scratch != nullptr, "phew_compare: null output or scratch");
  PHEW_REQUIRE(n == 0 || (b != nullptr && c != nullptr), "phew_compare: null input");
  PHEW_REQUIRE(n >= 0, "phew_compare: negative n");
  PHEW_REQUIRE(scratch_bytes >= phew_compare_scratch_bytes(n), "phew_compare: scratch too small");
  PHEW_REQUIRE((reinterpret_cast<uintptr_t>(scratch) & 15) == 0, "phew_compare: scratch not 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PHEW_F32: return compare_typed<float>(b, c, n, dtype, atol, rtol, scratch, out, st);
    case PHEW_F16: return compare_typed<f16>(b, c, n, dtype, atol, rtol, scratch, out, st);
    case PHEW_BF16: return compare_typed<bf16>(b, c, n, dtype, atol, rtol, scratch, out, st);
    default: return set_error(PHEW_ERR_INVALID, "phew_compare: bad dtype");
  }
}

// ---------------------------------------------------------------------------
// phew_compare_static: the same comparison without any allocation.
//
// Some callers cannot allocate device memory at the moment they need a
// verdict: code running while a CUDA graph is being captured (cudaMalloc is
// not capturable), code inside a host runtime whose allocator owns the whole
// device (an inference server's pool, where a stray cudaMalloc can fail or
// fragment it), or a watchdog that checks outputs from a context that must
// not synchronise the device (cudaMalloc / cudaFree can).  For them the
// per-block partial results live in one array in this library's own device
// memory instead of a caller-provided scratch buffer.
// ---------------------------------------------------------------------------
#include <cuda.h>

#include <mutex>

namespace phew {
namespace {
// Partials of at most kMaxBlocks blocks: 48 KiB.  Every GPU that loads this
// library holds the array until the process exits.
constexpr size_t kStaticScratchBytes =
    sizeof(StatsPartial) * kMaxBlocks + sizeof(ComparePartial) * kMaxBlocks;
constexpr int kMaxStaticDevices = 256;
std::mutex g_static_mu;
// Per device: the array's address and the id of the context it was looked
// up in.  A device reset (cudaDeviceReset, or a primary context that was
// released and re-created) reloads the module at a new address in a new
// context, so an address is reused only while the context id is the same.
void* g_static_scratch[kMaxStaticDevices] = {};
unsigned long long g_static_ctx[kMaxStaticDevices] = {};

// Unique id of the calling thread's current context (0 when the driver
// offers no way to read it; the cache is then kept per device only).
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* a = nullptr;
    void* b = nullptr;
    cudaDriverEntryPointQueryResult qa, qb;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &qa) == cudaSuccess &&
        qa == cudaDriverEntryPointSuccess &&
        cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &qb) == cudaSuccess &&
        qb == cudaDriverEntryPointSuccess) {
      get_current = reinterpret_cast<GetCurrent>(a);
      get_id = reinterpret_cast<GetId>(b);
    }
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}
}  // namespace
}  // namespace phew

static __device__ __align__(256) unsigned char g_compare_static_scratch[phew::kStaticScratchBytes];

extern "C" int phew_compare_static(const void* b, const void* c, int64_t n, int dtype,
                                   double atol, double rtol, phew_compare_stats* out,
                                   void* stream) {
  int dev = 0;
  PHEW_CHECK_CUDA(cudaGetDevice(&dev));
  PHEW_REQUIRE(dev >= 0 && dev < kMaxStaticDevices, "phew_compare_static: device index out of range");
  const size_t need = phew_compare_scratch_bytes(n);
  if (need > kStaticScratchBytes)
    return set_error(PHEW_ERR_INVALID,
                     "phew_compare_static: this comparison needs " + std::to_string(need) +
                         " bytes of scratch but the static array holds " +
                         std::to_string(kStaticScratchBytes) + "; use phew_compare");
  void* scratch = nullptr;
  {
    // First call on each device (and first call after a device reset):
    // translate the array's symbol into this device's address (with the
    // device current).  A host-side reference to g_compare_static_scratch is
    // only a stand-in, never a device address.
    std::lock_guard<std::mutex> lk(g_static_mu);
    // The context is made current here (runtime calls initialise it), so
    // its id is read after a runtime call.
    const unsigned long long ctx = current_context_id();
    if (g_static_scratch[dev] == nullptr || g_static_ctx[dev] != ctx) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_compare_static_scratch);
      if (e != cudaSuccess || p == nullptr)
        return set_error(PHEW_ERR_CUDA, std::string("phew_compare_static: cudaGetSymbolAddress: ") +
                                            cudaGetErrorString(e));
      g_static_scratch[dev] = p;
      g_static_ctx[dev] = current_context_id();
    }
    scratch = g_static_scratch[dev];
  }
  // Nothing in the array needs clearing: each call writes every partial it
  // later reads.
  return phew_compare(b, c, n, dtype, atol, rtol, scratch, kStaticScratchBytes, out, stream);
}
