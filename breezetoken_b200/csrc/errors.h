// Host-side error reporting shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>

namespace bt {

// Record a formatted message as the thread's last error and return `code`.
int fail(int code, const char* fmt, ...);
// Record a CUDA runtime failure of `what` and return BT_ERR_CUDA.
int fail_cuda(cudaError_t err, const char* what);
// SM count of the current device (cached per device).
int sm_count();

}  // namespace bt
