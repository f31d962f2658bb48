// Routed experts of a Qwen3.6-MoE layer at decode, on IQ3_S expert weights.
//
// Follows the reference's ExpertPool.forward (breezetoken/model/moe.py:205-233)
// and route() (:33-39): softmax over the router logits, top-k, renormalise by
// the clamped sum; per selected expert act = silu(gate x) * up x, then
// out = sum_k w_k * down_k act_k.  The reference stages the selected experts'
// bytes to the device and dequantises them to f32 before a matmul; here the
// IQ3_S bytes are decoded inside the GEMV and never materialised.
//
// A decode batch of T tokens selects P = T * top_k (token, expert) pairs.
// `moe_group_kernel` sorts the pairs by expert (ascending id, stable), so each
// selected expert's weights are read once for all the tokens that chose it
// (U unique experts: bytes = U * 1,351,680 at the 35B shape).  The gate/up
// kernel gives each expert 32 CTAs of 16 gate + 16 matching up rows and
// writes act for every pair; the down kernel gives each expert 32 CTAs of
// 64 rows; the pairs of a token are summed in routing order.
//
// IQ3_S GEMV: a warp lane decodes one 32-weight sub-block at a time -- eight
// loads from the sign-applied codebook (8192 entries, in shared memory) --
// into signed int8 words, and dots them with the activation
// encoded as three int8 digits of a 22-bit fixed-point value per 32-element
// block (the q8 GEMV's encoding), 24 dp4a per sub-block: the integer sums are
// exact, so the only roundings are the activation's encoding and the f32
// accumulation over sub-blocks.
#include <cuda_fp16.h>

#include <algorithm>

#include "errors.h"
#include "gemv_q8.cuh"
#include "moe.cuh"

namespace bt {

namespace {

// The IQ3_S codebook with the 4 sign bits of a group applied: entry
// idx9 | (signs4 << 9) holds the group's 4 signed int8 weights (before the
// sub-block scale), so decoding a group is one table load.
constexpr uint32_t kGrid[512] = {
#include "iq3s_grid.inc"
};

struct SignedGrid {
  uint32_t v[8192];
};

constexpr SignedGrid make_signed_grid() {
  SignedGrid t{};
  for (int i = 0; i < 8192; ++i) {
    const uint32_t g = kGrid[i & 511], sb4 = static_cast<uint32_t>(i) >> 9;
    // bit j of sb4 -> 0xFF in byte j; then per-byte two's-complement negation
    const uint32_t mask = ((sb4 * 0x00204081u) & 0x01010101u) * 0xFFu;
    t.v[i] = (g ^ mask) + (mask & 0x01010101u);
  }
  return t;
}

__device__ const SignedGrid g_signed = make_signed_grid();

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kGateRowsPerCta = 16;   // + the 16 matching up rows
constexpr int kDownRowsPerCta = 64;
constexpr float kWeightSumMin = 6.103515625e-5f;  // moe.py:24
// Workspace header words [kTicketBase, kTicketBase + hidden / 64): the
// one-token combine's arrival counters (zero between calls).
constexpr int kTicketBase = 16;
constexpr int kHeaderBytes = 512;

// ------------------------------------------------------------------ repack
// GGUF IQ3_S block (110 B: d[2] qs[64] qh[8] signs[32] scales[4]) -> the
// aligned 112-byte block. One thread per block.
__global__ void repack_iq3s_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t n_blocks) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_blocks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* s = src + i * 110;
    uint8_t* d = dst + i * kIq3sBlockBytes;
    for (int j = 0; j < 64; ++j) d[j] = s[2 + j];        // qs
    for (int j = 0; j < 32; ++j) d[64 + j] = s[74 + j];  // signs
    for (int j = 0; j < 8; ++j) d[96 + j] = s[66 + j];   // qh
    for (int j = 0; j < 4; ++j) d[104 + j] = s[106 + j]; // scales
    d[108] = s[0];
    d[109] = s[1];
    d[110] = 0;
    d[111] = 0;
  }
}

// ------------------------------------------------------------------ route
// One warp per token: softmax over the expert logits (f32), top-k by
// repeated warp argmax (ties -> lower id), renormalised weights.
__global__ void moe_route_kernel(const float* __restrict__ logits, int64_t t, int n_experts, int top_k,
                                 int32_t* __restrict__ ids, float* __restrict__ weights) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tok = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + warp;
  if (tok >= t) return;
  const float* lg = logits + tok * n_experts;
  float m = -INFINITY;
  for (int e = lane; e < n_experts; e += 32) m = fmaxf(m, lg[e]);
  m = warp_max(m);
  float s = 0.f;
  for (int e = lane; e < n_experts; e += 32) s += expf(lg[e] - m);
  s = warp_sum(s);
  // selection state: bit set = taken (n_experts <= 32 * 32)
  uint32_t taken = 0;
  float sel[16];
  int sid[16];
  float wsum = 0.f;
  for (int k = 0; k < top_k && k < 16; ++k) {
    float best = -INFINITY;
    int bid = 0x7fffffff;
    for (int e = lane, i = 0; e < n_experts; e += 32, ++i) {
      if ((taken >> i) & 1u) continue;
      const float v = lg[e];
      if (v > best || (v == best && e < bid)) {
        best = v;
        bid = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bid, o);
      if (ob > best || (ob == best && oi < bid)) {
        best = ob;
        bid = oi;
      }
    }
    if ((bid & 31) == lane) taken |= 1u << (bid >> 5);
    const float p = expf(best - m) / s;  // softmax probability of the pick
    sel[k] = p;
    sid[k] = bid;
    wsum += p;
  }
  const float denom = fmaxf(wsum, kWeightSumMin);
  if (lane == 0)
    for (int k = 0; k < top_k && k < 16; ++k) {
      ids[tok * top_k + k] = sid[k];
      weights[tok * top_k + k] = sel[k] / denom;
    }
}

// ------------------------------------------------------------------ group
// Workspace header: [n_unique, bad ids] then per slot u < P: expert, first
// pair, pair count; then the pair list sorted by (expert, pair).
struct MoeWs {
  int32_t* hdr;
  int32_t* slot_expert;
  int32_t* slot_start;
  int32_t* slot_count;
  int32_t* pairs;
  float* act;  // (P, ffn)
  float* dn;   // (P, hidden)
};

__host__ __device__ inline int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

__host__ __device__ inline MoeWs moe_ws(void* base, int64_t p, int64_t hidden, int64_t ffn) {
  uint8_t* b = static_cast<uint8_t*>(base);
  MoeWs w;
  int64_t o = 0;
  w.hdr = reinterpret_cast<int32_t*>(b + o);
  o += kHeaderBytes;
  w.slot_expert = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.slot_start = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.slot_count = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.pairs = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.act = reinterpret_cast<float*>(b + o);
  o += align256(4 * p * ffn);
  w.dn = reinterpret_cast<float*>(b + o);
  return w;
}

inline int64_t moe_ws_bytes(int64_t p, int64_t hidden, int64_t ffn) {
  return kHeaderBytes + 4 * align256(4 * p) + align256(4 * p * ffn) + align256(4 * p * hidden);
}

// One CTA: counting sort of the P pairs by expert id (stable).
__global__ void moe_group_kernel(const int32_t* __restrict__ ids, int p_total, int n_experts, MoeWs ws) {
  extern __shared__ int32_t sm[];
  int32_t* cnt = sm;               // [n_experts]
  int32_t* off = sm + n_experts;   // [n_experts] exclusive prefix of counts
  int32_t* sid = off + n_experts;  // [p_total] the ids
  __shared__ int32_t s_bad;
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
  for (int q = threadIdx.x; q < p_total; q += blockDim.x) sid[q] = ids[q];
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int q = threadIdx.x; q < p_total; q += blockDim.x) {
    const int e = sid[q];
    if (e >= 0 && e < n_experts)
      atomicAdd(&cnt[e], 1);
    else
      atomicAdd(&s_bad, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0, u = 0;
    for (int e = 0; e < n_experts; ++e) {
      off[e] = o;
      if (cnt[e]) {
        ws.slot_expert[u] = e;
        ws.slot_start[u] = o;
        ws.slot_count[u] = cnt[e];
        ++u;
      }
      o += cnt[e];
    }
    ws.hdr[0] = u;
    ws.hdr[1] = s_bad;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < p_total; q += blockDim.x) {
    const int e = sid[q];
    if (e < 0 || e >= n_experts) continue;
    int rank = 0;
    for (int q2 = 0; q2 < q; ++q2) rank += sid[q2] == e;
    ws.pairs[off[e] + rank] = q;
  }
}

// ------------------------------------------------------------------ GEMV core
// Activation vectors in shared memory, per vector v: three digit planes x two
// halves of each 32-element sub-block, SBR sub-blocks (uint4 each), then the
// per-sub-block scales.
template <int SBR>
struct XSmem {
  static constexpr int kPlaneBytes = SBR * 16;
  static constexpr int kVecBytes = 6 * kPlaneBytes + SBR * 4;
};

// Encode `n` f32 values at src (16-byte aligned) into vector slot v.
template <int SBR>
__device__ __forceinline__ void encode_vec(const float* __restrict__ src, uint8_t* xs, int v) {
  constexpr int K = SBR * 32, NF4 = K / 4;
  uint8_t* base = xs + v * XSmem<SBR>::kVecBytes;
  float* sx = reinterpret_cast<float*>(base + 6 * XSmem<SBR>::kPlaneBytes);
  for (int f = threadIdx.x; f < ((NF4 + kThreads - 1) / kThreads) * kThreads; f += kThreads) {
    const int fc = min(f, NF4 - 1);
    float4 h = reinterpret_cast<const float4*>(src)[fc];
    if (f >= NF4) h = make_float4(0.f, 0.f, 0.f, 0.f);
    float m = fmaxf(fmaxf(fabsf(h.x), fabsf(h.y)), fmaxf(fabsf(h.z), fabsf(h.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    const uint32_t be = (__float_as_uint(m) >> 23) & 255u;
    const bool ok = be >= 22u;
    const float inv = ok ? __uint_as_float((275u - be) << 23) : 0.f;
    const float scale = ok ? __uint_as_float((be - 21u) << 23) : 0.f;
    int a[4], b[4], c[4];
    const float e4[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int X = __float2int_rn(e4[i] * inv);
      c[i] = ((X + 128) & 255) - 128;
      const int x1 = (X - c[i]) >> 8;
      b[i] = ((x1 + 128) & 255) - 128;
      a[i] = (x1 - b[i]) >> 8;
    }
    if (f < NF4) {
      const int sb = f >> 3, w = f & 7;
      const int h2 = w >> 2, comp = w & 3;
      auto pk = [](const int (&d)[4]) {
        return (static_cast<uint32_t>(d[0]) & 255u) | ((static_cast<uint32_t>(d[1]) & 255u) << 8) |
               ((static_cast<uint32_t>(d[2]) & 255u) << 16) | ((static_cast<uint32_t>(d[3]) & 255u) << 24);
      };
      reinterpret_cast<uint32_t*>(base + (0 * 2 + h2) * XSmem<SBR>::kPlaneBytes + sb * 16)[comp] = pk(a);
      reinterpret_cast<uint32_t*>(base + (1 * 2 + h2) * XSmem<SBR>::kPlaneBytes + sb * 16)[comp] = pk(b);
      reinterpret_cast<uint32_t*>(base + (2 * 2 + h2) * XSmem<SBR>::kPlaneBytes + sb * 16)[comp] = pk(c);
      if (w == 0) sx[sb] = scale;
    }
  }
}

// One 32-weight sub-block of a repacked IQ3_S row as 8 signed int8x4 words
// plus its scale d * (1 + 2 * nibble) (quant/dequant.py:164-185).
struct SubBlock {
  uint32_t q[8];
  float db;
};

__device__ __forceinline__ void load_sub_block(const uint8_t* row, int sb, const uint32_t* lut, SubBlock& o) {
  // `row` is a shared-memory copy; all loads are naturally aligned (blocks
  // are 112 = 7 x 16 bytes)
  const int b = sb >> 3, p = (sb & 7) >> 1, s = sb & 1;
  const uint8_t* blk = row + b * kIq3sBlockBytes;
  const uint64_t qs = *reinterpret_cast<const uint64_t*>(blk + 16 * p + 8 * s);
  const uint32_t signs = *reinterpret_cast<const uint32_t*>(blk + 64 + 8 * p + 4 * s);
  const uint64_t qh8 = *reinterpret_cast<const uint64_t*>(blk + 96);   // qh[0..7]
  const uint64_t tail = *reinterpret_cast<const uint64_t*>(blk + 104); // scales[0..3], d, pad
  const uint32_t qh = static_cast<uint32_t>(qh8 >> (8 * (2 * p + s))) & 255u;
  const uint32_t nib = static_cast<uint32_t>(tail >> (8 * p + 4 * s)) & 15u;
  o.db = __half2float(__ushort_as_half(static_cast<unsigned short>((tail >> 32) & 0xFFFFu))) *
         static_cast<float>(1 + 2 * static_cast<int>(nib));
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t idx = static_cast<uint32_t>((qs >> (8 * w)) & 255u) | (((qh >> w) & 1u) << 8) |
                         (((signs >> (4 * w)) & 15u) << 9);
    o.q[w] = lut[idx];
  }
}

// q . X for vector slot v, sub-block sb (exact integer sums, one rounding)
template <int SBR>
__device__ __forceinline__ float sub_block_dot(const SubBlock& w, const uint8_t* xs, int v, int sb) {
  const uint8_t* base = xs + v * XSmem<SBR>::kVecBytes;
  const uint4 a0 = *reinterpret_cast<const uint4*>(base + 0 * XSmem<SBR>::kPlaneBytes + sb * 16);
  const uint4 a1 = *reinterpret_cast<const uint4*>(base + 1 * XSmem<SBR>::kPlaneBytes + sb * 16);
  const uint4 b0 = *reinterpret_cast<const uint4*>(base + 2 * XSmem<SBR>::kPlaneBytes + sb * 16);
  const uint4 b1 = *reinterpret_cast<const uint4*>(base + 3 * XSmem<SBR>::kPlaneBytes + sb * 16);
  const uint4 c0 = *reinterpret_cast<const uint4*>(base + 4 * XSmem<SBR>::kPlaneBytes + sb * 16);
  const uint4 c1 = *reinterpret_cast<const uint4*>(base + 5 * XSmem<SBR>::kPlaneBytes + sb * 16);
  const uint32_t d2[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  const uint32_t d1[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  const uint32_t d0[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  int s2 = 0, s1 = 0, s0 = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s2 = __dp4a(static_cast<int>(w.q[i]), static_cast<int>(d2[i]), s2);
    s1 = __dp4a(static_cast<int>(w.q[i]), static_cast<int>(d1[i]), s1);
    s0 = __dp4a(static_cast<int>(w.q[i]), static_cast<int>(d0[i]), s0);
  }
  const int t = s1 * 256 + s0;
  return fmaf(static_cast<float>(s2), 65536.0f, static_cast<float>(t));
}

// Dot of RW rows (row pointers) with the NV vectors in xs, mc of them live.
// Lanes: LPR lanes per row (all 32 when the row has >= 32 sub-blocks).
// Returns, in every lane, the totals of the lane's row group.
template <int SBR, int NV, int RW>
__device__ __forceinline__ void rows_dot(const uint8_t* const (&rows)[RW], const uint8_t* xs, const uint32_t* lut,
                                         int mc, float (&res)[RW][NV]) {
  static_assert(SBR >= 16, "rows of at least 512 weights");
  constexpr int LPR = SBR >= 32 ? 32 : SBR;
  constexpr int RPP = 32 / LPR;  // rows per pass
  constexpr int SPL = SBR / LPR; // sub-blocks per lane per row
  const int lane = threadIdx.x & 31;
  const int rin = lane / LPR, lr = lane % LPR;
#pragma unroll
  for (int r0 = 0; r0 < RW; r0 += RPP) {
    float acc[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) acc[v] = 0.f;
    const uint8_t* row = rows[r0];
    if (RPP > 1 && rin == 1 && r0 + 1 < RW) row = rows[r0 + 1];
#pragma unroll
    for (int i = 0; i < SPL; ++i) {
      const int sb = lr + LPR * i;
      SubBlock w;
      load_sub_block(row, sb, lut, w);
      const uint8_t* base = xs;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        if (v < mc) {
          const float sxv = reinterpret_cast<const float*>(base + v * XSmem<SBR>::kVecBytes +
                                                           6 * XSmem<SBR>::kPlaneBytes)[sb];
          acc[v] = fmaf(w.db * sxv, sub_block_dot<SBR>(w, xs, v, sb), acc[v]);
        }
      }
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) acc[v] += __shfl_xor_sync(0xffffffffu, acc[v], o);
    }
    // lanes of pass row j (j < RPP) now hold that row's totals; gather all
#pragma unroll
    for (int j = 0; j < RPP; ++j)
      if (r0 + j < RW)
#pragma unroll
        for (int v = 0; v < NV; ++v) res[r0 + j][v] = __shfl_sync(0xffffffffu, acc[v], j * LPR);
  }
}

// ------------------------------------------------------------------ staging
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Copy `bytes` (a multiple of 16) from global to shared memory, all threads.
__device__ __forceinline__ void stage(uint8_t* dst, const uint8_t* src, int64_t bytes) {
  for (int64_t i = threadIdx.x; i < bytes / 16; i += kThreads) cp_async16(dst + 16 * i, src + 16 * i);
}

// The expert slot a CTA serves: from the grouping kernel, or (one token,
// whose top-k experts are distinct) straight from the routing ids.
struct Slot {
  int expert, start, count;
};

__device__ __forceinline__ bool slot_of(int u, bool direct, const int32_t* ids, int n_experts, const MoeWs& ws,
                                        Slot& s) {
  if (direct) {
    s.expert = ids[u];
    s.start = u;
    s.count = 1;
    return s.expert >= 0 && s.expert < n_experts;
  }
  if (u >= ws.hdr[0]) return false;
  s.expert = ws.slot_expert[u];
  s.start = ws.slot_start[u];
  s.count = ws.slot_count[u];
  return true;
}

__device__ __forceinline__ int pair_of(bool direct, const MoeWs& ws, int i) { return direct ? i : ws.pairs[i]; }

// ------------------------------------------------------------------ gate/up
// CTA (u, c): expert slot u, outputs [16c, 16c + 16); warp w: outputs
// 16c + 2w + [0, 2) (its 2 gate rows and 2 up rows).  The CTA's 32 rows are
// copied into shared memory first (cp.async, all in flight at once); in
// direct mode that copy starts before the dependency wait.  Pairs of the
// slot in chunks of NV.
template <int SBR, int NV>
__global__ void __launch_bounds__(kThreads) moe_gate_up_kernel(const uint8_t* __restrict__ gate,
                                                               const uint8_t* __restrict__ up,
                                                               const float* __restrict__ x, const int32_t* ids,
                                                               int n_experts, int direct, int top_k, int ffn,
                                                               MoeWs ws) {
  constexpr int K = SBR * 32;
  constexpr int RB = K / 256 * kIq3sBlockBytes;
  constexpr int WBYTES = 2 * kGateRowsPerCta * RB;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* wsm = smem;                 // [gate rows 32][up rows 32]
  uint8_t* xs = smem + WBYTES;         // encoded vectors
  __shared__ __align__(16) uint32_t lut[8192];
  const int u = blockIdx.x, c = blockIdx.y;
  stage(reinterpret_cast<uint8_t*>(lut), reinterpret_cast<const uint8_t*>(g_signed.v), sizeof(lut));
  cp_async_commit();
  // The op's inputs (ids, x) come from whatever ran before: read them only
  // after the wait, and let the down kernel start only then, so that it may
  // read them before its own wait.
  pdl_wait();
  pdl_launch_dependents();
  Slot sl{};
  if (!slot_of(u, direct != 0, ids, n_experts, ws, sl)) return;
  stage(wsm, gate + (static_cast<int64_t>(sl.expert) * ffn + c * kGateRowsPerCta) * RB, kGateRowsPerCta * RB);
  stage(wsm + kGateRowsPerCta * RB, up + (static_cast<int64_t>(sl.expert) * ffn + c * kGateRowsPerCta) * RB,
        kGateRowsPerCta * RB);
  cp_async_commit();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int OPW = kGateRowsPerCta / kWarps;  // outputs per warp
  const int o0 = c * kGateRowsPerCta + warp * OPW;
  const uint8_t* rows[2 * OPW];
#pragma unroll
  for (int i = 0; i < OPW; ++i) {
    rows[i] = wsm + (warp * OPW + i) * RB;
    rows[OPW + i] = wsm + (kGateRowsPerCta + warp * OPW + i) * RB;
  }
  for (int c0 = 0; c0 < sl.count; c0 += NV) {
    const int mc = min(NV, sl.count - c0);
    __syncthreads();  // (previous chunk's readers done)
    for (int v = 0; v < mc; ++v)
      encode_vec<SBR>(x + static_cast<int64_t>(pair_of(direct != 0, ws, sl.start + c0 + v) / top_k) * K, xs, v);
    cp_async_wait_all();
    __syncthreads();
    float res[2 * OPW][NV];
    rows_dot<SBR, NV, 2 * OPW>(rows, xs, lut, mc, res);
    if (lane < OPW) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        if (v < mc) {
          // lane i writes output o0 + i (model/moe.py:229: act = silu(g) * u)
          float g = 0.f, uu = 0.f;
#pragma unroll
          for (int i = 0; i < OPW; ++i)
            if (i == lane) {
              g = res[i][v];
              uu = res[OPW + i][v];
            }
          ws.act[static_cast<int64_t>(pair_of(direct != 0, ws, sl.start + c0 + v)) * ffn + o0 + lane] = silu_f(g) * uu;
        }
      }
    }
  }
}

// ------------------------------------------------------------------ down
// CTA (u, c): expert slot u, rows [64c, 64c + 64) staged into shared
// memory before the dependency wait: the gate/up kernel lets this kernel
// start only after its own wait, so the routing ids and the grouping
// kernel's slots are complete by then; warp w: 8 rows.
template <int SBR, int NV>
__global__ void __launch_bounds__(kThreads) moe_down_kernel(const uint8_t* __restrict__ down, const int32_t* ids,
                                                            const float* __restrict__ weights, float* out,
                                                            int n_experts, int direct, int hidden, MoeWs ws,
                                                            int ffn) {
  constexpr int K = SBR * 32;
  constexpr int RB = K / 256 * kIq3sBlockBytes;
  constexpr int WBYTES = kDownRowsPerCta * RB;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* wsm = smem;
  uint8_t* xs = smem + WBYTES;
  __shared__ __align__(16) uint32_t lut[8192];
  const int u = blockIdx.x, c = blockIdx.y;
  stage(reinterpret_cast<uint8_t*>(lut), reinterpret_cast<const uint8_t*>(g_signed.v), sizeof(lut));
  cp_async_commit();
  Slot sl{};
  const bool live = slot_of(u, direct != 0, ids, n_experts, ws, sl);
  if (live) {
    stage(wsm, down + (static_cast<int64_t>(sl.expert) * hidden + c * kDownRowsPerCta) * RB, WBYTES);
    cp_async_commit();
  }
  pdl_launch_dependents();
  pdl_wait();
  if (!live && !direct) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int RW = kDownRowsPerCta / kWarps;
  const int h0 = c * kDownRowsPerCta + warp * RW;
  const uint8_t* rows[RW];
#pragma unroll
  for (int i = 0; i < RW; ++i) rows[i] = wsm + (warp * RW + i) * RB;
  for (int c0 = 0; live && c0 < sl.count; c0 += NV) {
    const int mc = min(NV, sl.count - c0);
    __syncthreads();
    for (int v = 0; v < mc; ++v)
      encode_vec<SBR>(ws.act + static_cast<int64_t>(pair_of(direct != 0, ws, sl.start + c0 + v)) * ffn, xs, v);
    cp_async_wait_all();
    __syncthreads();
    float res[RW][NV];
    rows_dot<SBR, NV, RW>(rows, xs, lut, mc, res);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      if (v < mc) {
        float* dst = ws.dn + static_cast<int64_t>(pair_of(direct != 0, ws, sl.start + c0 + v)) * hidden + h0;
#pragma unroll
        for (int i = 0; i < RW; ++i)
          if (lane == i) dst[i] = res[i][v];
      }
    }
  }
  if (!direct) return;
  // one token: the last of the top_k CTAs of this row chunk sums the experts'
  // rows in routing order (atomic ticket, re-armed for the next call)
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(ws.hdr + kTicketBase + c, 1) == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int r = threadIdx.x; r < kDownRowsPerCta; r += kThreads) {
    const int hh = c * kDownRowsPerCta + r;
    float acc = 0.f;
    for (int k = 0; k < static_cast<int>(gridDim.x); ++k) {
      const int e = ids[k];
      if (e < 0 || e >= n_experts) continue;
      acc = __fadd_rn(acc, __fmul_rn(__ldcg(ws.dn + static_cast<int64_t>(k) * hidden + hh), weights[k]));
    }
    out[hh] = acc;
  }
  if (threadIdx.x == 0) atomicExch(ws.hdr + kTicketBase + c, 0);
}

// ------------------------------------------------------------------ combine
// out[t] = sum_k w[t, k] * down_k(act) in routing order, each product rounded
// before the add like the reference's (out * w).sum(0) in f32.
__global__ void moe_combine_kernel(const float* __restrict__ weights, const int32_t* __restrict__ ids, int64_t t,
                                   int top_k, int hidden, int n_experts, MoeWs ws, float* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = t * hidden;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i / hidden;
    const int hh = static_cast<int>(i % hidden);
    float acc = 0.f;
    for (int k = 0; k < top_k; ++k) {
      const int e = ids[tok * top_k + k];
      if (e < 0 || e >= n_experts) continue;
      acc = __fadd_rn(acc, __fmul_rn(ws.dn[(tok * top_k + k) * hidden + hh], weights[tok * top_k + k]));
    }
    out[i] = acc;
  }
}

template <int SBR>
constexpr int xs_bytes(int nv) {
  return nv * XSmem<SBR>::kVecBytes;
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <int SBR_GU, int SBR_D, int NV>
int launch_all(const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* x, int64_t t, int hidden,
               int ffn, int n_experts, const int32_t* ids, const float* weights, int top_k, float* out, MoeWs ws,
               cudaStream_t stream) {
  const int p = static_cast<int>(t * top_k);
  // one token selects top_k distinct experts: no grouping needed
  const int direct = t == 1 ? 1 : 0;
  const int slots = direct ? top_k : (p < n_experts ? p : n_experts);
  if (!direct) moe_group_kernel<<<1, 512, (2 * n_experts + p) * sizeof(int32_t), stream>>>(ids, p, n_experts, ws);
  constexpr int gu_w = 2 * kGateRowsPerCta * (SBR_GU * 32 / 256) * kIq3sBlockBytes;
  constexpr int d_w = kDownRowsPerCta * (SBR_D * 32 / 256) * kIq3sBlockBytes;
  const size_t gu_smem = gu_w + xs_bytes<SBR_GU>(NV), d_smem = d_w + xs_bytes<SBR_D>(NV);
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(moe_gate_up_kernel<SBR_GU, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(gu_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_down_kernel<SBR_D, NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(d_smem));
    if (e != cudaSuccess) return fail_cuda(e, "moe set smem");
    configured_device = dev;
  }
  cudaError_t e = launch_pdl(moe_gate_up_kernel<SBR_GU, NV>, dim3(slots, ffn / kGateRowsPerCta), gu_smem, stream, gate,
                             up, x, ids, n_experts, direct, top_k, ffn, ws);
  if (e == cudaSuccess)
    e = launch_pdl(moe_down_kernel<SBR_D, NV>, dim3(slots, hidden / kDownRowsPerCta), d_smem, stream, down, ids,
                   weights, out, n_experts, direct, hidden, ws, ffn);
  const int64_t total = t * hidden;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  if (e == cudaSuccess && !direct)
    e = launch_pdl(moe_combine_kernel, dim3(blocks), 0, stream, weights, ids, t, top_k, hidden, n_experts, ws, out);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "moe experts launch");
  return BT_OK;
}

template <int SBR_GU, int SBR_D>
int launch_nv(const uint8_t* gate, const uint8_t* up, const uint8_t* down, const float* x, int64_t t, int hidden,
              int ffn, int n_experts, const int32_t* ids, const float* weights, int top_k, float* out, MoeWs ws,
              cudaStream_t stream) {
  // one token selects each expert once: a single vector per expert
  if (t == 1)
    return launch_all<SBR_GU, SBR_D, 1>(gate, up, down, x, t, hidden, ffn, n_experts, ids, weights, top_k, out, ws,
                                        stream);
  return launch_all<SBR_GU, SBR_D, 4>(gate, up, down, x, t, hidden, ffn, n_experts, ids, weights, top_k, out, ws,
                                      stream);
}

}  // namespace

int repack_iq3_s(const void* src, void* dst, int64_t rows, int64_t k, cudaStream_t stream) {
  if (!src || !dst || rows < 0 || k <= 0 || k % 256) return fail(BT_ERR_INVALID, "repack_iq3_s: K must be a multiple of 256");
  if (reinterpret_cast<uintptr_t>(dst) & 15) return fail(BT_ERR_INVALID, "repack_iq3_s: dst must be 16-byte aligned");
  const int64_t nb = rows * (k / 256);
  if (nb == 0) return BT_OK;
  const int blocks = static_cast<int>(std::min<int64_t>((nb + 255) / 256, 65535));
  repack_iq3s_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), nb);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "repack_iq3_s launch");
  return BT_OK;
}

int moe_route(const float* logits, int64_t t, int64_t n_experts, int top_k, int32_t* ids, float* weights,
              cudaStream_t stream) {
  if (!logits || !ids || !weights || t < 0) return fail(BT_ERR_INVALID, "moe_route: null pointer or negative T");
  if (n_experts < 1 || n_experts > 1024 || top_k < 1 || top_k > 16 || top_k > n_experts)
    return fail(BT_ERR_UNSUPPORTED, "moe_route serves <= 1024 experts and top-k <= 16 (got %lld, %d)",
                static_cast<long long>(n_experts), top_k);
  if (t == 0) return BT_OK;
  const int blocks = static_cast<int>((t + 7) / 8);
  moe_route_kernel<<<blocks, 256, 0, stream>>>(logits, t, static_cast<int>(n_experts), top_k, ids, weights);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "moe_route launch");
  return BT_OK;
}

int64_t moe_workspace_bytes(int64_t t, int64_t hidden, int64_t ffn, int64_t n_experts, int top_k) {
  (void)n_experts;
  if (t < 1 || top_k < 1) return 0;
  return moe_ws_bytes(t * top_k, hidden, ffn);
}

int moe_experts_iq3s(const void* gate, const void* up, const void* down, const float* x, int64_t t, int64_t hidden,
                     int64_t ffn, int64_t n_experts, const int32_t* ids, const float* weights, int top_k, float* out,
                     void* workspace, cudaStream_t stream) {
  if (!gate || !up || !down || !x || !ids || !weights || !out || !workspace)
    return fail(BT_ERR_INVALID, "moe_experts_iq3s: null pointer");
  if (t < 1 || t * top_k > 4096 || top_k < 1 || n_experts < 1 || n_experts > 4096)
    return fail(BT_ERR_UNSUPPORTED, "moe_experts_iq3s serves T * top_k <= 4096 pairs over <= 4096 experts");
  if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(down) |
       reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(workspace)) & 15)
    return fail(BT_ERR_INVALID, "moe_experts_iq3s: weights, x and workspace must be 16-byte aligned");
  if (ffn % kGateRowsPerCta || hidden % kDownRowsPerCta || hidden / kDownRowsPerCta > kHeaderBytes / 4 - kTicketBase)
    return fail(BT_ERR_UNSUPPORTED, "moe_experts_iq3s: ffn must be a multiple of 16 and hidden of 64 (<= 7168)");
  const MoeWs ws = moe_ws(workspace, t * top_k, hidden, ffn);
  const uint8_t* g = static_cast<const uint8_t*>(gate);
  const uint8_t* u = static_cast<const uint8_t*>(up);
  const uint8_t* d = static_cast<const uint8_t*>(down);
  const int h = static_cast<int>(hidden), f = static_cast<int>(ffn), ne = static_cast<int>(n_experts);
  if (hidden == 2048 && ffn == 512) return launch_nv<64, 16>(g, u, d, x, t, h, f, ne, ids, weights, top_k, out, ws, stream);
  if (hidden == 2048 && ffn == 768) return fail(BT_ERR_UNSUPPORTED, "moe_experts_iq3s: ffn must be a multiple of 256");
  if (hidden == 1024 && ffn == 512) return launch_nv<32, 16>(g, u, d, x, t, h, f, ne, ids, weights, top_k, out, ws, stream);
  if (hidden == 4096 && ffn == 1024) return launch_nv<128, 32>(g, u, d, x, t, h, f, ne, ids, weights, top_k, out, ws, stream);
  if (hidden == 2048 && ffn == 1024) return launch_nv<64, 32>(g, u, d, x, t, h, f, ne, ids, weights, top_k, out, ws, stream);
  return fail(BT_ERR_UNSUPPORTED, "moe_experts_iq3s serves (hidden, ffn) in {(1024,512), (2048,512), (2048,1024), (4096,1024)}");
}

}  // namespace bt
