// Routed-expert (MoE) decode on IQ3_S experts (see moe.cu).
#pragma once

#include "common.cuh"

namespace bt {

// Device IQ3_S layout: rows in tiles of 16; each 16-row x 256-weight tile
// (16 GGUF blocks of 110 bytes) is a 2176-byte chunk of 4-bit signed weight
// codes and per-row scale records arranged for the m16n8k16 MMA's A
// fragments (moe.cu), i.e. 136 bytes per row and block.
constexpr int kIq3sBlockBytes = 136;

inline int64_t iq3s_row_bytes(int64_t k) { return k / 256 * kIq3sBlockBytes; }

int repack_iq3_s(const void* src, void* dst, int64_t rows, int64_t k, cudaStream_t stream);

int moe_route(const float* logits, int64_t t, int64_t n_experts, int top_k, int32_t* ids, float* weights,
              cudaStream_t stream);

// The layer's shared expert: bf16 (out, in) rows, f32 gate vector.
struct MoeShared {
  const void* gate;      // (ffn, hidden)
  const void* up;        // (ffn, hidden)
  const void* down;      // (hidden, ffn)
  const float* gate_inp; // (hidden,)
  int64_t ffn;
};

int64_t moe_workspace_bytes(int64_t t, int64_t hidden, int64_t ffn, int64_t shared_ffn, int64_t n_experts, int top_k);

// The residual add + RMSNorm + bf16 planes that follow a MoE layer in the
// decoder: h_out = h + out, y = rms_norm(h_out) * w, planes of y
// (add_rms_norm_planes); fused into the combine for batches (out is then
// not written).
struct MoeNorm {
  const float* h;
  const float* w;
  float* h_out;
  float* y;
  void* planes;
  float eps;
};

// The layer's prep kernel in parts: kPrepAll everything (the layer alone:
// the pairs' sort, the tokens' fp16 planes, the shared expert's gate/up);
// kPrepX all but the sort; kPrepNone: a layer call after
// moe_route_sort_iq3s, which routed, sorted and encoded into its workspace.
constexpr int kPrepAll = 0, kPrepX = 1, kPrepNone = 2;

// shared may be null (routed experts only); norm may be null (out only).
int moe_layer_iq3s(const void* gate, const void* up, const void* down, const MoeShared* shared, const float* x,
                   int64_t t, int64_t hidden, int64_t ffn, int64_t n_experts, const int32_t* ids, const float* weights,
                   int top_k, float* out, void* workspace, cudaStream_t stream, const MoeNorm* norm = nullptr,
                   int prep_part = kPrepAll);

// moe_route (the same ids and weights) plus the prep kernel's pair sort and
// token encoding of a layer call into `workspace` (the last routing block
// sorts), for a following moe_layer_iq3s(..., kPrepNone) with the same x.
int moe_route_sort_iq3s(const float* logits, const float* x, int64_t t, int64_t hidden, int64_t ffn,
                        int64_t n_experts, int top_k, int64_t shared_ffn, int32_t* ids, float* weights,
                        void* workspace, cudaStream_t stream);

}  // namespace bt
