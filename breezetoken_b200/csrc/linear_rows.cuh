// Dense projection by bf16 / f32 weight rows (see linear_rows.cu).
#pragma once

#include "common.cuh"

namespace bt {

int bf16_planes(const float* x, void* planes, int64_t t, int64_t k, cudaStream_t stream);

int linear_rows(const void* w, int w_dtype, const void* x_planes, float* y, int64_t n, int64_t k, int64_t t,
                cudaStream_t stream);

// Bounded waits of the tensor-core path that gave up since the last call
// (synchronous; resets the count; -1 if the device could not be read).
int linear_rows_timeouts();

}  // namespace bt
