// Library-wide device status word and ABI bookkeeping entry points.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include "common.cuh"

namespace {
__device__ unsigned int g_rk_device_status = 0;
constexpr int kMaxDevices = 64;
unsigned int* g_status_ptr[kMaxDevices] = {nullptr};
}  // namespace

std::atomic<unsigned long long> g_launches{0};

namespace rk_host {
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("REVK_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// The address is looked up once per device (with that device current) and cached.
unsigned int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_rk_device_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<unsigned int*>(p);
  }
  return g_status_ptr[dev];
}

int ensure_smem_attr(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, std::unordered_map<int, int>> done;  // kernel -> device -> bytes set
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RK_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(mu);
  auto& per_dev = done[kernel];
  auto it = per_dev.find(dev);
  if (it != per_dev.end() && it->second >= bytes) return RK_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    cudaGetLastError();  // reported through the return value, not left for the next launch check
    return RK_ERR_LAUNCH;
  }
  per_dev[dev] = bytes;
  return RK_OK;
}
}  // namespace rk_host

extern "C" int rk_abi_version(void) { return 1; }

extern "C" unsigned long long rk_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" const char* rk_status_string(int status) {
  switch (status) {
    case RK_OK: return "ok";
    case RK_ERR_ARG: return "invalid argument (null pointer, negative or inconsistent size)";
    case RK_ERR_ALIGN: return "alignment rule broken (pointer or leading dimension)";
    case RK_ERR_DTYPE: return "unsupported dtype combination";
    case RK_ERR_LAUNCH: return "CUDA launch or driver call failed";
    case RK_ERR_UNSUPPORTED: return "shape outside what the kernel implements";
    case RK_ERR_WORKSPACE: return "workspace too small";
    case RK_ERR_DEVICE: return "device status word set: a bounded device-side wait gave up";
    case RK_ERR_SCRATCH: return "request exceeds the static scratch of an allocation-free entry point";
    default: return "unknown status";
  }
}

extern "C" int rk_device_status_read(unsigned int* out, void* stream) {
  if (!out) return RK_ERR_ARG;
  unsigned int* p = rk_host::device_status_ptr();
  if (!p) return RK_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int v = 0;
  if (cudaMemcpyAsync(&v, p, sizeof(v), cudaMemcpyDeviceToHost, s) != cudaSuccess) return RK_ERR_LAUNCH;
  if (cudaMemsetAsync(p, 0, sizeof(v), s) != cudaSuccess) return RK_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return RK_ERR_LAUNCH;
  *out = v;
  return RK_OK;
}
