// Library-level entry points: error string, version, device check.
#include <atomic>

#include "common.cuh"

namespace cgym {

char* error_buffer() {
  static thread_local char buffer[512] = {0};
  return buffer;
}

int fail(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(error_buffer(), 512, fmt, args);
  va_end(args);
  return 1;
}

std::atomic<long long> g_kernel_launches{0};
thread_local int g_pdl_enabled = 0;

int check_launch(const char* what, int kernels) {
  const cudaError_t rc = cudaGetLastError();
  if (rc == cudaSuccess) {
    g_kernel_launches.fetch_add(kernels, std::memory_order_relaxed);
    return 0;
  }
  return fail("%s: CUDA launch failed: %s", what, cudaGetErrorString(rc));
}

}  // namespace cgym

extern "C" const char* cgym_last_error(void) { return cgym::error_buffer(); }

extern "C" int cgym_version(void) { return 1; }

extern "C" int cgym_set_pdl(int enabled) {
  const int previous = cgym::g_pdl_enabled;
  cgym::g_pdl_enabled = enabled ? 1 : 0;
  return previous;
}

extern "C" long long cgym_launch_count(void) {
  return cgym::g_kernel_launches.load(std::memory_order_relaxed);
}

extern "C" int cgym_device_supported(void) {
  int device = 0, major = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return 0;
  return major == 10 ? 1 : 0;
}
