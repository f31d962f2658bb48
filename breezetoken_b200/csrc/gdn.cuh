// Parameters of the GDN recurrent decode step (see gdn.cu).
#pragma once

#include "common.cuh"

namespace bt {

struct GdnParams {
  const void* q;  // (batch, heads_k, dim) at batch stride q_bs elements
  const void* k;  // (batch, heads_k, dim) at batch stride k_bs
  const void* v;  // (batch, heads_v, dim) at batch stride v_bs
  int32_t in_dtype;  // BT_F32 or BT_BF16 for q/k/v
  int64_t q_bs, k_bs, v_bs;
  const float* g;     // log decay (batch, heads_v) at batch stride g_bs
  const float* beta;  // beta logits (batch, heads_v) at batch stride beta_bs
  int64_t g_bs, beta_bs;
  float* state;  // (batch, heads_v, dim, dim) f32, in place
  float* out;    // (batch, heads_v, dim) at batch stride out_bs
  int64_t out_bs;
  int32_t batch, heads_k, heads_v, dim;
  float scale, eps;
  int32_t* status;
  TraceRec* trace;  // optional launch timeline record (null = off)
};

int gdn_decode_launch(const GdnParams& p, cudaStream_t stream, bool pdl);

// Token strides (elements) of the multi-token prefill scan over `len` tokens.
struct GdnScan {
  int32_t len;
  int64_t tok_q, tok_k, tok_v, tok_g, tok_beta, tok_out;
};
int gdn_prefill_launch(const GdnParams& p, const GdnScan& sc, cudaStream_t stream);

}  // namespace bt
