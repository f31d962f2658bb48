// Q8_0 GEMV for batch-1..8 decode: y[v][n] = sum_k x[v][k] * d[n][k/32] * q[n][k].
//
// Replaces the reference's split-K tilelang GEMV + torch split reduction
// (breezetoken/kernels/cuda/gemv.py:19-40, backends.py:304-333) and the
// torch GEMV of the f32 oracle (backends.py:182-184).  Weights stay Q8_0 in
// HBM (1.0625 B/weight) in "q8 rows": [fp16 scales padded to 16 B][int8 K].
//
// Design (sm_100a):
//  * one CTA per SM; CTA b owns a contiguous range of rows, so its weights
//    are one contiguous byte range;
//  * warp 8 is the producer: one lane streams the CTA's rows into a ring of
//    shared-memory stages with cp.async.bulk (TMA engine), L2 evict-first,
//    completing on per-stage mbarriers.  It starts BEFORE griddepcontrol.wait,
//    so under programmatic dependent launch the weight stream of this kernel
//    overlaps the tail of the previous kernel;
//  * warps 0-7 consume stages round-robin (warp w takes stages w, w+8, ...),
//    build the activation vector(s) in shared memory in a lane-major layout
//    (conflict-free LDS.128) after griddepcontrol.wait, convert int8 with a
//    PRMT/FADD trick instead of I2F, accumulate in f32 and reduce with warp
//    shuffles (a 4-row reduce-scatter: 6 shuffles per 4 rows);
//  * fused prologues (residual add + RMSNorm, embedding gather + RMSNorm,
//    per-head RMSNorm * silu(z)) and epilogues (GDN conv window + SiLU,
//    softplus decay, SiLU-gate of interleaved gate/up rows, argmax).
#pragma once

#include "common.cuh"

namespace bt {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumerThreads + 32;
constexpr int kMaxStages = 32;
constexpr int kMaxVec = 8;

enum GemvPrologue : int {
  PRO_LOAD = 0,        // x = src
  PRO_RESID_NORM = 1,  // h = h_in + delta -> h_out (CTA 0); x = rmsnorm(h) * w
  PRO_EMBED_NORM = 2,  // h = dequant(embed[token]) -> h_out (CTA 0); x = rmsnorm(h) * w
  PRO_GATED_NORM = 3,  // x = rmsnorm_per_group(o) * w[k % group] * silu_z
};

enum GemvEpilogue : int {
  EPI_STORE = 0,      // y = acc
  EPI_GDN_IN = 1,     // qkv conv window + SiLU | silu(z) | softplus decay | beta logits
  EPI_SILU_PAIR = 2,  // rows (2j, 2j+1) = (gate_j, up_j): y[j] = silu(gate) * up
  EPI_ARGMAX = 3,     // optional logits store + argmax -> token, history, pos += 1
};

struct GemvQ8Params {
  const uint8_t* w;
  int64_t n_rows;
  int32_t k, row_bytes, sb;  // K, bytes per row, scale bytes per row
  int32_t group_rows;        // rows per consumer task (1 or 4)
  int32_t stage_rows;        // rows per stage (multiple of group_rows)
  int32_t stages;            // ring depth per consumer warp (each warp owns its slots)
  int32_t n_vec;             // activation vectors (batch)
  int32_t xs_stride;         // floats per vector in the smem x layout
  // prologue
  int32_t prologue;
  const float* x;   // LOAD: x; RESID: h_in; GATED: o        ([v][k])
  const float* x2;  // RESID: delta; GATED: silu(z)          ([v][k])
  int64_t x_bs, x2_bs;  // per-vector strides of x / x2 (elements); 0 = k
  const float* norm_w;
  float* h_out;
  const uint8_t* embed;  // EMBED: q8 rows (embed_rows x k)
  int64_t embed_rows;
  const int32_t* tokens;  // EMBED: [v]
  int32_t group;          // GATED: normalisation group (head dim)
  float eps;
  // epilogue
  int32_t epilogue;
  float* y;
  int64_t y_stride;  // per vector
  // EPI_GDN_IN
  float* conv_state;         // [v][n_conv][conv_k-1]
  const float* conv_w;       // [n_conv][conv_k]
  const float* a_log;        // [n_gh]
  const float* dt_bias;      // [n_gh]
  int32_t n_conv, n_z, n_gh, conv_k;
  // EPI_ARGMAX
  unsigned long long* best;  // [v] packed (ordered value, ~index), 0 between steps
  uint32_t* counter;         // CTA arrival counter, 0 between steps
  int32_t* token_out;        // [v]
  int32_t* pos;              // [v] incremented by the last CTA
  int32_t* history;          // [v][history_stride] or null
  int32_t history_stride;
  int32_t* status;
};

// ------------------------------------------------------------ smem layout
// [full mbar x stages][empty mbar x stages][scratch 64 floats][argmax 8 u64]
// [x: n_vec * xs_stride floats][stages * stage_rows * row_bytes]
struct GemvSmem {
  static constexpr int kHeader = 2 * kMaxStages * 8 + 64 * 4 + kConsumerWarps * kMaxVec * 8;
};

__host__ __device__ inline int64_t gemv_x_stride(int k) {
  // J = ceil(k / 512) lane-major float4 slots of 16 elements per lane
  return ((k + 511) / 512) * 512;
}

// Index of element k of a vector in the lane-major x layout: chunk c = k/16
// is owned by lane c % 32 at slot j = c / 32; element e = k % 16 sits in
// float4 number e / 4 of that chunk.
__device__ __forceinline__ int x_perm(int k) {
  const int c = k >> 4, e = k & 15;
  return ((((c >> 5) * 4 + (e >> 2)) * 32 + (c & 31)) << 2) + (e & 3);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(idx));
}

// 16 products of one 16-byte chunk of int8 quants with 16 f32 activations.
__device__ __forceinline__ float dot16(const uint4 q, const float4 x0, const float4 x1,
                                       const float4 x2, const float4 x3) {
  const uint32_t u0 = q.x ^ 0x80808080u, u1 = q.y ^ 0x80808080u;
  const uint32_t u2 = q.z ^ 0x80808080u, u3 = q.w ^ 0x80808080u;
  float s = biased_byte_to_f32<0>(u0) * x0.x;
  s = fmaf(biased_byte_to_f32<1>(u0), x0.y, s);
  s = fmaf(biased_byte_to_f32<2>(u0), x0.z, s);
  s = fmaf(biased_byte_to_f32<3>(u0), x0.w, s);
  s = fmaf(biased_byte_to_f32<0>(u1), x1.x, s);
  s = fmaf(biased_byte_to_f32<1>(u1), x1.y, s);
  s = fmaf(biased_byte_to_f32<2>(u1), x1.z, s);
  s = fmaf(biased_byte_to_f32<3>(u1), x1.w, s);
  s = fmaf(biased_byte_to_f32<0>(u2), x2.x, s);
  s = fmaf(biased_byte_to_f32<1>(u2), x2.y, s);
  s = fmaf(biased_byte_to_f32<2>(u2), x2.z, s);
  s = fmaf(biased_byte_to_f32<3>(u2), x2.w, s);
  s = fmaf(biased_byte_to_f32<0>(u3), x3.x, s);
  s = fmaf(biased_byte_to_f32<1>(u3), x3.y, s);
  s = fmaf(biased_byte_to_f32<2>(u3), x3.z, s);
  s = fmaf(biased_byte_to_f32<3>(u3), x3.w, s);
  return s;
}

struct GemvQ8Launch {
  int grid;
  int threads;
  size_t smem;
};

// Host: fill the tiling fields of `p` for `sm_count` SMs and return the launch shape.
int gemv_q8_plan(GemvQ8Params& p, int sm_count, GemvQ8Launch& launch);
// Host: launch (optionally with programmatic stream serialization).
int gemv_q8_launch(const GemvQ8Params& p, const GemvQ8Launch& launch, cudaStream_t stream,
                   bool pdl);

}  // namespace bt
