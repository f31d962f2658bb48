// Parameters of the split-KV GQA decode attention (see attention.cu).
#pragma once

#include "common.cuh"

namespace bt {

struct AttnParams {
  // queries: head h of sequence b at q[b*q_bs + h*q_hs]
  const float* q;
  int64_t q_bs;
  int32_t q_hs;
  // keys / values: (batch, cap, kv_heads, dim) in kv_dtype
  const void* k;
  const void* v;
  int32_t kv_dtype;
  int64_t kv_bs;  // elements per sequence = cap * kv_heads * dim
  int32_t kv_ts;  // elements per position = kv_heads * dim
  const int32_t* lens;  // op mode: attended length per sequence
  // output: head h of sequence b at out[b*out_bs + h*dim]
  float* out;
  int64_t out_bs;
  int32_t batch, heads, kv_heads, dim, cap, splits;
  int32_t cluster;  // 1: the splits of a (sequence, group) form a cluster and merge in DSMEM
  float scale;
  // model mode (Qwen3.5 full-attention layer, model/layers.py:55-82):
  // q/k RMSNorm, partial RoPE at pos, KV-cache write at pos, sigmoid gate.
  int32_t model;
  const int32_t* pos;    // (batch,) position of the new token; length = pos + 1
  const float* q_norm;   // (dim,)
  const float* k_norm;   // (dim,)
  const float* k_new;    // k of group g at k_new[b*q_bs + g*dim]
  const float* v_new;    // v of group g at v_new[b*q_bs + g*dim]
  const float* gate;     // gate of head h at gate[b*q_bs + h*q_hs]
  const float* rope_cos; // (cap, rope_dim)
  const float* rope_sin;
  int32_t rope_dim;
  float eps;
  // workspace (zero between calls): partials and per-(b, g) counters
  float* part;
  uint32_t* counters;
  int32_t* status;
  TraceRec* trace;  // optional launch timeline record (null = off)
};

// More than kMergeGroup splits merge in two levels: the last CTA of each
// group of kMergeGroup splits merges the group, the last group merger the
// groups.
constexpr int kMergeGroup = 16;
__host__ __device__ inline int64_t attn_groups(int64_t splits) {
  return splits > kMergeGroup ? (splits + kMergeGroup - 1) / kMergeGroup : 0;
}

// Workspace floats for the split (and group) partial records...
inline int64_t attn_part_floats(int64_t batch, int64_t kv_heads, int64_t heads, int64_t dim,
                                int64_t splits) {
  const int64_t gs = heads / kv_heads;
  return batch * kv_heads * (splits + attn_groups(splits)) * gs * (dim + 2);
}
// ... then the u32 arrival counters: one per (b, g), then one per group.
inline int64_t attn_counters(int64_t batch, int64_t kv_heads, int64_t splits) {
  return batch * kv_heads * (1 + attn_groups(splits));
}

int attention_launch(const AttnParams& p, cudaStream_t stream, bool pdl);

}  // namespace bt
