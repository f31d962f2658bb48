// Fused per-layer kernels of the Qwen3.6-MoE decode step (see qwen36_layer.cu).
#pragma once

#include "common.cuh"

namespace bt {

constexpr int kGdnStepThreads = 256;

struct GdnStepParams {
  // Token j of sequence b is row j * batch + b of mixed, ba, z and planes
  // (steps == 1: the decode step, row b).
  const float* mixed;  // (steps*batch, 2*heads_k*dim + heads_v*dim): q | k | v, row stride mixed_bs
  int64_t mixed_bs;
  const float* ba;  // (steps*batch, 2*heads_v): beta logits | alpha logits, row stride ba_bs
  int64_t ba_bs;
  const float* a_log;    // (heads_v,) = -exp(A_log)
  const float* dt_bias;  // (heads_v,)
  float* state;          // (batch, heads_v, dim, dim) f32, in place
  const float* z;        // (steps*batch, heads_v*dim), row stride z_bs
  int64_t z_bs;
  const float* norm_w;  // (dim,)
  void* planes;         // (steps*batch, 3, heads_v*dim) bf16 out
  int32_t steps, batch, heads_k, heads_v, dim;
  float scale, l2_eps, norm_eps;
};

int gdn_gated_step_launch(const GdnStepParams& p, cudaStream_t stream);
int add_rms_norm_planes(const float* a, const float* b, const float* w, float* h, float* y, void* planes,
                        int64_t rows, int64_t n, float eps, cudaStream_t stream);

}  // namespace bt
