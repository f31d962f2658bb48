// The GDN layer's in-projection, causal conv, gated-delta recurrence and
// gated RMSNorm as one kernel (see gdn_fused.cu).
#pragma once

#include "gemv_q8.cuh"

namespace bt {

struct GdnFusedParams {
  // in-projection (q8 rows [q | k | v | z | alpha | beta], K = hidden) with its
  // residual/embedding RMSNorm prologue and the conv / decay operands
  GemvQ8Params g;
  int32_t heads;      // value heads (= key heads)
  int32_t dim;        // head dim (key = value)
  float* state;       // (batch, heads, dim, dim) f32, in place
  float scale;        // q scale (1/sqrt(dim))
  float l2_eps;       // q/k L2-norm epsilon
  const float* norm_w;  // gated-norm weight (dim)
  float norm_eps;
  float* out;         // gated output (batch, heads*dim) at batch stride out_bs
  int64_t out_bs;
};

// Whether the fused kernel serves these shapes (else the caller runs the
// in-projection GEMV, gdn_decode and a gated-norm out-projection).
bool gdn_fused_supported(int64_t hidden, int heads_k, int heads_v, int dim, int batch);

// Host: plan the in-projection tiling inside `p.g` and launch.
int gdn_fused_launch(GdnFusedParams& p, cudaStream_t stream, bool pdl);

}  // namespace bt
