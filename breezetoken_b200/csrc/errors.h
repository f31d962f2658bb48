// Host-side error reporting shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <utility>

namespace bt {

// Kernels this library has launched (or recorded into a CUDA graph being
// captured) in this process; read by bt_launch_count().
inline std::atomic<long long> g_launch_count{0};
inline void note_launch() { g_launch_count.fetch_add(1, std::memory_order_relaxed); }
// cudaLaunchKernelEx, counted.
template <typename... Exp, typename... Act>
cudaError_t launch_ex(const cudaLaunchConfig_t* cfg, void (*kernel)(Exp...), Act&&... args) {
  note_launch();
  return cudaLaunchKernelEx(cfg, kernel, std::forward<Act>(args)...);
}

// Record a formatted message as the thread's last error and return `code`.
int fail(int code, const char* fmt, ...);
// Record a CUDA runtime failure of `what` and return BT_ERR_CUDA.
int fail_cuda(cudaError_t err, const char* what);
// SM count of the current device (cached per device).
int sm_count();

}  // namespace bt
