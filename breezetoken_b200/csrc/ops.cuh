// Host launchers of the stand-alone operations in ops.cu.
#pragma once

#include <algorithm>

#include "common.cuh"

namespace bt {

int repack_q8_0(const void* src, void* dst, int64_t rows, int64_t k, int64_t dst_row0, int64_t dst_row_step,
                cudaStream_t stream);
int dequant_q8_rows(const void* w, float* out, int64_t rows, int64_t k, cudaStream_t stream);
int dequant_iq3_s(const void* raw, float* out, int64_t rows, int64_t cols, cudaStream_t stream);
int linear_kn(const void* w, int w_dtype, const float* x, float* y, int64_t k, int64_t n, cudaStream_t stream);
// h/b may be null: plain RMSNorm.  With b: h = a + b, y = rmsnorm(h).
int rms_norm(const float* a, const float* b, const float* w, float* h, float* y, int64_t rows, int64_t n, float eps,
             cudaStream_t stream);
int silu_mul(const float* g, const float* u, float* y, int64_t n, cudaStream_t stream);
int rope(const float* x, const float* cos_t, const float* sin_t, const int32_t* pos, float* y, int64_t rows,
         int64_t dim, int64_t rope_dim, int64_t cap, cudaStream_t stream);
int argmax(const float* x, int64_t rows, int64_t n, int32_t* out, void* workspace, cudaStream_t stream);
int conv_silu(const float* entry, float* state, const float* w, float* out, int64_t steps, int64_t batch,
              int64_t channels, int64_t taps, cudaStream_t stream);

}  // namespace bt
