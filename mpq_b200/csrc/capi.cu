// Library-level C-ABI entry points: version and the last error message.
#include <stdarg.h>
#include <stdio.h>
#include <map>
#include <mutex>
#include <utility>
#include "common.cuh"

namespace mpq {
static thread_local char g_last_error[512] = {0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}
}  // namespace mpq

namespace mpq {
// The dynamic shared-memory limit is an attribute of the kernel in one device's context, so it is raised once per
// (device, kernel) and again only when a launch asks for more; a mutex makes the check safe across host threads.
int smem_opt_in(const void* kernel, size_t bytes, const char* what) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> raised;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_error("%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
    return (int)e;
  }
  std::lock_guard<std::mutex> lock(mu);
  size_t& have = raised[std::make_pair(dev, kernel)];
  if (have >= bytes) return MPQ_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) {
    set_last_error("%s: raising the shared-memory limit to %zu bytes: %s", what, bytes, cudaGetErrorString(e));
    return (int)e;
  }
  have = bytes;
  return MPQ_OK;
}
}  // namespace mpq

MPQ_API const char* mpq_last_error(void) { return mpq::g_last_error; }

MPQ_API int mpq_abi_version(void) { return 1; }
