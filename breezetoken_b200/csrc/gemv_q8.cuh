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
//  * the 8 warps stream row groups (4 rows for K <= 1024, else 1) straight
//    from HBM with 128-bit non-allocating loads, double-buffered in
//    registers.  Before griddepcontrol.wait -- i.e. while the previous kernel
//    still runs under programmatic dependent launch -- each CTA prefetches
//    the head of its weight slice into L2 (cp.async.bulk.prefetch) and loads
//    its first groups into registers; weights never depend on earlier work;
//  * after the wait the activation vector(s) are built in shared memory,
//    encoded per 32-element block as three int8 digits of a 22-bit
//    fixed-point value, so the int8 weights multiply by dp4a without any
//    int->float conversion (12 dp4a per 16 weights); per-block sums are
//    scaled and accumulated in f32 and reduced with warp shuffles (a 4-row
//    reduce-scatter: 6 shuffles per 4 rows);
//  * fused prologues (residual add + RMSNorm, embedding gather + RMSNorm,
//    per-head RMSNorm * silu(z)) and epilogues (GDN conv window + SiLU,
//    softplus decay, SiLU-gate of interleaved gate/up rows, argmax).
#pragma once

#include "common.cuh"

namespace bt {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumerThreads;
constexpr int kMaxVec = 8;

enum GemvPrologue : int {
  PRO_LOAD = 0,        // x = src
  PRO_RESID_NORM = 1,  // h = h_in + delta -> h_out (CTA 0); x = rmsnorm(h) * w
  PRO_EMBED_NORM = 2,  // h = dequant(embed[token]) -> h_out (CTA 0); x = rmsnorm(h) * w
  PRO_GATED_NORM = 3,  // x = rmsnorm_per_group(o) * w[k % group] * silu_z
  PRO_SILU_PAIR = 4,   // src = (gate_0, up_0, gate_1, up_1, ...): x[j] = silu(gate_j) * up_j
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
  int64_t prefetch_bytes;    // weight bytes per CTA prefetched into L2 before the wait
  int32_t n_vec;             // activation vectors (batch)
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
  TraceRec* trace;  // optional launch timeline record (null = off)
};

// ------------------------------------------------------------ smem layout
// [scratch 64 floats][argmax 8 x 8 u64][activations: gemv_x_layout(k, n_vec)]
struct GemvSmem {
  static constexpr int kHeader = 64 * 4 + kConsumerWarps * kMaxVec * 8;
};

// Activation vectors in shared memory.  The prologue builds each vector in
// f32 registers, then encodes every block of 32 elements in fixed point:
// X = rint(x / sx) with sx the power of two for which max|x_block| / sx lies
// in [2^21, 2^22), so |X| <= 2^22, stored as three signed base-256 digits
// (X = d2*2^16 + d1*2^8 + d0, each in [-128, 127]).  A chunk of 16 int8
// weights q then dots with x as sx * (2^16 * dp4a(q, d2) + 2^8 * dp4a(q, d1)
// + dp4a(q, d0)): the integer sums are exact and the scaling by sx is exact,
// so the only rounding beyond f32 accumulation is x itself, represented to
// at most 2^-22 of its block maximum.  Digits are stored lane-major:
// chunk c = lane + 32*j keeps its 16 d2, d1, d0 bytes in uint4 slots
// ((3*j + t) * 32 + lane), so each lane's LDS.128 is bank-conflict free.
struct XLayout {
  int64_t xd, sx, total;  // byte offsets of the digits and scales, total size
};

__host__ __device__ inline XLayout gemv_x_layout(int k, int nv) {
  const int64_t J = (k + 511) / 512;
  XLayout l;
  l.xd = 0;
  l.sx = static_cast<int64_t>(nv) * J * 1536;
  l.total = l.sx + ((static_cast<int64_t>(nv) * (k / 32) * 4 + 127) / 128) * 128;
  return l;
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int64_t idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) |
         static_cast<unsigned long long>(0xFFFFFFFFu - static_cast<uint32_t>(idx));
}

// sum_{i<16} q_i * X_i for one chunk of 16 int8 weights and the digits of X,
// returned as f32 (exact integer sums, one rounding).
__device__ __forceinline__ float dot16_digits(const uint4 q, const uint4 d2, const uint4 d1, const uint4 d0) {
  int s2 = __dp4a(static_cast<int>(q.x), static_cast<int>(d2.x), 0);
  int s1 = __dp4a(static_cast<int>(q.x), static_cast<int>(d1.x), 0);
  int s0 = __dp4a(static_cast<int>(q.x), static_cast<int>(d0.x), 0);
  s2 = __dp4a(static_cast<int>(q.y), static_cast<int>(d2.y), s2);
  s1 = __dp4a(static_cast<int>(q.y), static_cast<int>(d1.y), s1);
  s0 = __dp4a(static_cast<int>(q.y), static_cast<int>(d0.y), s0);
  s2 = __dp4a(static_cast<int>(q.z), static_cast<int>(d2.z), s2);
  s1 = __dp4a(static_cast<int>(q.z), static_cast<int>(d1.z), s1);
  s0 = __dp4a(static_cast<int>(q.z), static_cast<int>(d0.z), s0);
  s2 = __dp4a(static_cast<int>(q.w), static_cast<int>(d2.w), s2);
  s1 = __dp4a(static_cast<int>(q.w), static_cast<int>(d1.w), s1);
  s0 = __dp4a(static_cast<int>(q.w), static_cast<int>(d0.w), s0);
  const int t = s1 * 256 + s0;  // |t| < 2^26
  return fmaf(static_cast<float>(s2), 65536.0f, static_cast<float>(t));
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
