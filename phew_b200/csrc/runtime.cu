// Library core: error reporting, device setup, the NVRTC compile cache that
// stands in for MLX's metal_kernel JIT, kernel launch and the L2 flush.
#include <nvrtc.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "tc_common.cuh"

namespace phew {

static thread_local std::string g_last_error;
static thread_local std::string g_last_compile_log;  // NVRTC log of this thread's last compilation

namespace tc {
namespace {
thread_local TestStall g_test_stall{-1, 0};
}  // namespace

TestStall take_test_stall() {
  TestStall t = g_test_stall;
  g_test_stall = TestStall{-1, 0};
  if (t.wait_ns == 0) t.wait_ns = kWaitLimitNs;
  return t;
}
}  // namespace tc

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

namespace {
std::atomic<unsigned long long> g_launches{0};
}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
unsigned long long launch_counter() { return g_launches.load(std::memory_order_relaxed); }

int sm_count_current() {
  static thread_local int cached_dev = -1;
  static thread_local int cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != cached_dev) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      sms = 148;
    cached_dev = dev;
    cached_sms = sms;
  }
  return cached_sms;
}

namespace {

struct CompiledKernel {
  cudaLibrary_t library = nullptr;
  cudaKernel_t kernel = nullptr;
  // per device: the largest dynamic shared memory size already allowed
  // (the attribute is set on the current device; read and written under
  // g_cache_mu)
  std::unordered_map<int, size_t> smem_attr_set;
};

std::mutex g_cache_mu;
std::unordered_map<uint64_t, CompiledKernel> g_cache;

uint64_t fnv1a(const char* s, uint64_t h = 1469598103934665603ull) {
  for (; *s; ++s) {
    h ^= static_cast<unsigned char>(*s);
    h *= 1099511628211ull;
  }
  return h;
}

std::string nvrtc_log(nvrtcProgram prog) {
  size_t n = 0;
  if (nvrtcGetProgramLogSize(prog, &n) != NVRTC_SUCCESS || n == 0) return std::string();
  std::string log(n, '\0');
  nvrtcGetProgramLog(prog, &log[0]);
  return log;
}

}  // namespace
}  // namespace phew

using namespace phew;

extern "C" {

int phew_abi_version(void) { return 1; }

int phew_last_error(char* buf, size_t len) {
  const std::string& m = g_last_error;
  if (buf && len > 0) {
    size_t k = m.size() < len - 1 ? m.size() : len - 1;
    std::memcpy(buf, m.data(), k);
    buf[k] = '\0';
  }
  return static_cast<int>(m.size());
}

int phew_init(int device) {
  PHEW_REQUIRE(device >= 0, "phew_init: negative device index");
  PHEW_CHECK_CUDA(cudaSetDevice(device));
  // Touch the primary context so later launches do not pay for it.
  PHEW_CHECK_CUDA(cudaFree(nullptr));
  (void)sm_count_current();
  return PHEW_OK;
}

int phew_device_query(int device, phew_device_info* out) {
  PHEW_REQUIRE(out != nullptr, "phew_device_query: null output");
  cudaDeviceProp p;
  PHEW_CHECK_CUDA(cudaGetDeviceProperties(&p, device));
  out->sm_count = p.multiProcessorCount;
  out->cc_major = p.major;
  out->cc_minor = p.minor;
  out->max_smem_per_block_optin = static_cast<int>(p.sharedMemPerBlockOptin);
  out->l2_bytes = p.l2CacheSize;
  out->hbm_bytes = static_cast<int64_t>(p.totalGlobalMem);
  std::strncpy(out->name, p.name, sizeof(out->name) - 1);
  out->name[sizeof(out->name) - 1] = '\0';
  return PHEW_OK;
}

int phew_compile(const char* source, const char* kernel_name, uint64_t* handle) {
  PHEW_REQUIRE(source && kernel_name && handle, "phew_compile: null argument");
  const uint64_t key = fnv1a(kernel_name, fnv1a(source)) ^ 0x9e3779b97f4a7c15ull;
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    if (g_cache.count(key)) {
      *handle = key;
      return PHEW_OK;
    }
  }
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, source, "phew_kernel.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return set_error(PHEW_ERR_COMPILE, "nvrtcCreateProgram failed");
  const char* opts[] = {
      "--gpu-architecture=sm_100a",
      "--std=c++17",
      "-default-device",
      "--generate-line-info",
  };
  nvrtcResult rc = nvrtcCompileProgram(prog, sizeof(opts) / sizeof(opts[0]), opts);
  phew::g_last_compile_log = nvrtc_log(prog);
  if (rc != NVRTC_SUCCESS) {
    std::string log = phew::g_last_compile_log;
    nvrtcDestroyProgram(&prog);
    return set_error(PHEW_ERR_COMPILE, std::string("NVRTC: ") + nvrtcGetErrorString(rc) + "\n" + log);
  }
  size_t n = 0;
  if (nvrtcGetCUBINSize(prog, &n) != NVRTC_SUCCESS || n == 0) {
    nvrtcDestroyProgram(&prog);
    return set_error(PHEW_ERR_COMPILE, "nvrtcGetCUBINSize failed");
  }
  std::vector<char> image(n);
  nvrtcGetCUBIN(prog, image.data());
  nvrtcDestroyProgram(&prog);

  CompiledKernel ck;
  PHEW_CHECK_CUDA(cudaLibraryLoadData(&ck.library, image.data(), nullptr, nullptr, 0,
                                      nullptr, nullptr, 0));
  cudaError_t e = cudaLibraryGetKernel(&ck.kernel, ck.library, kernel_name);
  if (e != cudaSuccess) {
    cudaLibraryUnload(ck.library);
    return set_error(PHEW_ERR_NOT_FOUND, std::string("kernel symbol not found: ") + kernel_name);
  }
  std::lock_guard<std::mutex> lk(g_cache_mu);
  auto it = g_cache.find(key);
  if (it != g_cache.end()) {  // another thread won the race
    cudaLibraryUnload(ck.library);
  } else {
    g_cache.emplace(key, ck);
  }
  *handle = key;
  return PHEW_OK;
}

int phew_compile_log(char* buf, size_t len) {
  const std::string& m = phew::g_last_compile_log;
  if (buf && len > 0) {
    size_t k = m.size() < len - 1 ? m.size() : len - 1;
    std::memcpy(buf, m.data(), k);
    buf[k] = '\0';
  }
  return static_cast<int>(m.size());
}

int phew_stream_create(void** stream) {
  PHEW_REQUIRE(stream != nullptr, "phew_stream_create: null output");
  cudaStream_t s = nullptr;
  PHEW_CHECK_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = s;
  return PHEW_OK;
}

int phew_stream_destroy(void* stream) {
  PHEW_REQUIRE(stream != nullptr, "phew_stream_destroy: null stream");
  PHEW_CHECK_CUDA(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
  return PHEW_OK;
}

int phew_event_create(void** event) {
  PHEW_REQUIRE(event != nullptr, "phew_event_create: null output");
  cudaEvent_t e = nullptr;
  PHEW_CHECK_CUDA(cudaEventCreate(&e));
  *event = e;
  return PHEW_OK;
}

int phew_event_record(void* event, void* stream) {
  PHEW_REQUIRE(event != nullptr, "phew_event_record: null event");
  PHEW_CHECK_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
  return PHEW_OK;
}

int phew_event_elapsed_ms(void* start, void* stop, float* ms) {
  PHEW_REQUIRE(start && stop && ms, "phew_event_elapsed_ms: null argument");
  PHEW_CHECK_CUDA(cudaEventSynchronize(static_cast<cudaEvent_t>(stop)));
  PHEW_CHECK_CUDA(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(stop)));
  return PHEW_OK;
}

int phew_event_destroy(void* event) {
  PHEW_REQUIRE(event != nullptr, "phew_event_destroy: null event");
  PHEW_CHECK_CUDA(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
  return PHEW_OK;
}

int phew_compile_cache_size(void) {
  std::lock_guard<std::mutex> lk(g_cache_mu);
  return static_cast<int>(g_cache.size());
}

int phew_launch(uint64_t handle, void** args, int nargs, unsigned grid_x, unsigned grid_y,
                unsigned grid_z, unsigned block_x, unsigned block_y, unsigned block_z,
                size_t dynamic_smem, void* stream) {
  PHEW_REQUIRE(nargs == 0 || args != nullptr, "phew_launch: null args");
  PHEW_REQUIRE(grid_x > 0 && grid_y > 0 && grid_z > 0, "phew_launch: empty grid");
  PHEW_REQUIRE(block_x > 0 && block_y > 0 && block_z > 0 &&
                   block_x * block_y * block_z <= 1024,
               "phew_launch: block must have 1..1024 threads");
  const void* fn = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = g_cache.find(handle);
    if (it == g_cache.end()) return set_error(PHEW_ERR_NOT_FOUND, "phew_launch: unknown handle");
    CompiledKernel& ck = it->second;
    fn = reinterpret_cast<const void*>(ck.kernel);
    if (dynamic_smem > 48 * 1024) {
      int dev = 0;
      PHEW_CHECK_CUDA(cudaGetDevice(&dev));
      size_t& allowed = ck.smem_attr_set[dev];
      if (dynamic_smem > allowed) {
        PHEW_CHECK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(dynamic_smem)));
        allowed = dynamic_smem;
      }
    }
  }
  PHEW_CHECK_CUDA(cudaLaunchKernel(fn, dim3(grid_x, grid_y, grid_z),
                                   dim3(block_x, block_y, block_z), args, dynamic_smem,
                                   static_cast<cudaStream_t>(stream)));
  phew::count_launch();
  return PHEW_OK;
}

int phew_launch_count(uint64_t* out) {
  PHEW_REQUIRE(out != nullptr, "phew_launch_count: null output");
  *out = phew::launch_counter();
  return PHEW_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// L2 flush: a streaming write over a buffer larger than the L2.
// ---------------------------------------------------------------------------
namespace phew {
__global__ void l2_flush_kernel(uint4* buf, size_t n_vec, uint32_t salt) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const uint4 v = make_uint4(salt, salt + 1, salt + 2, salt + 3);
  for (; i < n_vec; i += stride) buf[i] = v;
}
}  // namespace phew

extern "C" int phew_l2_flush(void* buf, size_t bytes, void* stream) {
  PHEW_REQUIRE(buf != nullptr, "phew_l2_flush: null buffer");
  PHEW_REQUIRE((reinterpret_cast<uintptr_t>(buf) & 15) == 0, "phew_l2_flush: buffer not 16-byte aligned");
  const size_t n_vec = bytes / 16;
  if (n_vec == 0) return PHEW_OK;
  static uint32_t salt = 1;
  const int blocks = sm_count_current() * 8;
  l2_flush_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(buf), n_vec, salt++);
  return launch_status("l2_flush_kernel");
}

extern "C" int phew_test_inject_stall(int stage, uint64_t wait_limit_ns) {
  PHEW_REQUIRE(stage >= 0, "phew_test_inject_stall: stage must be >= 0");
  PHEW_REQUIRE(wait_limit_ns > 0 && wait_limit_ns <= phew::tc::kWaitLimitNs,
               "phew_test_inject_stall: wait limit must be in (0, 1 s]");
  phew::tc::g_test_stall = phew::tc::TestStall{stage, static_cast<unsigned long long>(wait_limit_ns)};
  return PHEW_OK;
}
