// Routed experts of a Qwen3.6-MoE layer at decode, on IQ3_S expert weights.
//
// Follows the reference's ExpertPool.forward (breezetoken/model/moe.py:205-233)
// and route() (:33-39): softmax over the router logits, top-k, renormalise by
// the clamped sum; per selected expert act = silu(gate x) * up x, then
// out = sum_k w_k * down_k act_k.  The reference stages the selected experts'
// bytes to the device and dequantises them to f32 before a matmul; here the
// IQ3_S bytes are decoded in registers and fed to the tensor cores.
//
// A decode batch of T tokens selects P = T * top_k (token, expert) pairs.
// `moe_prep_kernel` sorts the pairs by expert (ascending id, stable), so each
// selected expert's weights are read once for all the tokens that chose it
// (U unique experts: bytes = U * 1,351,680 at the 35B shape), and encodes
// each token's activation once.  The gate/up and down kernels are persistent
// (two 8-warp CTAs per SM, each taking a contiguous range of (expert, row
// chunk) items, balanced by token passes); every warp decodes two 16-row
// tiles of one 256-weight column block per item and loads the next item's
// tiles while it computes.  Above 16 tokens the items are whole passes of up
// to 4 tokens pulled from a counter; at prefill sizes (>= 8 pairs per expert)
// wide passes of up to 16 tokens let each decoded tile serve four 4-token
// groups (moe_gate_up_wide_kernel, moe_down_pulled_kernel<KB, 4>).
//
// Weights: every IQ3_S weight is d * (1 + 2 * scale nibble) * v with v a
// signed codebook value, odd and in [-15, 15] (quant/dequant.py:164-185), so
// v = 2c - 15 for a 4-bit code c.  `bt_repack_iq3_s` re-encodes the GGUF
// blocks losslessly as these codes (the codebook index, its high bit and the
// signs become one nibble per weight) and stores each 16-row x 256-weight
// tile (16 GGUF blocks) as one 2176-byte chunk laid out for the m16n8k16
// MMA: lane (g, t) loads, with four 16-byte and two 8-byte coalesced loads,
// the codes of rows g and g+8 for weights 8t..8t+7 of all 8 sub-blocks, one
// 32-bit word per (row, sub-block), so a word is four of the MMA's
// A-fragment registers (the k order inside a sub-block is permuted
// identically on both operands).  A register is two fp16 weights made with
// one mask-and-or (the codes land in an fp16 mantissa under the exponent of
// 1024) and one f16x2 add or fma (exact: the results are small integers):
// no codebook lookups and no sign arithmetic.  The layout costs 136 bytes
// per 256 weights against the format's 110.
//
// Activations: each vector x is scaled by a power of two (max |x| in
// [2^13, 2^14)) and split into fp16 hi + lo planes (hi = fp16(x), lo =
// fp16(x - hi): ~22 significant bits); B columns 2j and 2j+1 are token j's
// hi and lo planes, so one MMA pair serves 4 tokens and a lane's C fragment
// holds both planes of its token.  Products are exact and accumulate in f32;
// per sub-block the rows' scales d * (1 + 2 * nibble) multiply the sums.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "errors.h"
#include "moe.cuh"
#include "norm_planes.cuh"
#include "qwen36_layer.cuh"

namespace bt {

namespace {

// The IQ3_S codebook (quant/_tables.py:1042): 512 entries of 4 unsigned
// weights, byte j = weight j of the group.
constexpr uint32_t kGrid[512] = {
#include "iq3s_grid.inc"
};

constexpr bool grid_values_small() {
  for (int i = 0; i < 512; ++i)
    for (int j = 0; j < 4; ++j)
      if (((kGrid[i] >> (8 * j)) & 255u) > 15u) return false;
  return true;
}
static_assert(grid_values_small(), "IQ3_S codebook values must be <= 15 (exact fp16 operands)");

constexpr bool grid_values_odd() {
  for (int i = 0; i < 512; ++i)
    for (int j = 0; j < 4; ++j)
      if ((((kGrid[i] >> (8 * j)) & 255u) & 1u) == 0u) return false;
  return true;
}
static_assert(grid_values_odd(), "IQ3_S codebook values must be odd: v = 2c - 15 for a 4-bit code c");

// The codebook for the repack kernel.
__device__ const uint32_t g_grid[512] = {
#include "iq3s_grid.inc"
};

constexpr int kThreads = 256;  // 8 warps; the expert kernels run two CTAs per SM
constexpr int kWarps = kThreads / 32;
constexpr float kWeightSumMin = 6.103515625e-5f;  // moe.py:24
// Workspace header words [kTicketBase, kTicketBase + hidden / rows per item):
// the one-token combine's arrival counters (zero between calls).
constexpr int kTicketBase = 16;
// Header words 2 and 3: the next gate/up and down item of the pulled-item
// kernels (T > 1), reset by the prep kernel of every call.
constexpr int kWorkGateUp = 2, kWorkDown = 3;
// Header word 4: the number of passes (T > 1).
constexpr int kPassCount = 4;
// Header word 5: arrivals of the routing blocks of moe_route_sort_kernel
// (zero between calls).
constexpr int kRouteTicket = 5;
constexpr int kHeaderBytes = 512;
// Item ranges of the expert kernels' CTAs (T > 1): gate/up at [0, 2G), down
// at [kRangeDown, kRangeDown + 2G), G <= kMaxGrid.
constexpr int kMaxGrid = 512;
constexpr int kRangeDown = 2 * kMaxGrid;
constexpr int kRangeBytes = 4 * 2 * kRangeDown;

// Tile chunk: 16 rows x 256 weights.  Sections (lane L = 4 g + t):
//   [0, 2048)     codes: part j (sub-blocks 2j, 2j+1) at 512 j, lane L's 16
//                 bytes at 512 j + 16 L = the words of (row g, sub-block 2j),
//                 (row g+8, 2j), (row g, 2j+1), (row g+8, 2j+1); a word holds
//                 the codes c_i of weights 8t + i (i = 0..7) of its
//                 sub-block, code c_i at bits (kCodeBit[i] + b) mod 32, b =
//                 0..3 (see decode_word)
//   [2048, 2176)  per row: scales[4], d (fp16), 2 zero bytes
constexpr int kChunkBytes = 16 * kIq3sBlockBytes;
constexpr int kCodes = 0, kScales = 2048;
static_assert(kChunkBytes == 2176, "tile chunk");
__host__ __device__ constexpr int code_bit(int i) {
  // codes 0, 2, 4, 6 (the low halves' weights) at bits 1, 5, 9, 13; codes 1,
  // 3, 5, 7 at bits 17, 21, 25, 29 (code 7's top bit wraps to bit 0)
  return (i & 1) * 16 + 1 + 4 * (i >> 1);
}

constexpr int kTokensPerPass = 4;              // 8 MMA columns: hi and lo per token
// Wide passes (prefill-sized batches, >= kWideMinPairs pairs per expert on
// average): up to kWideGroups groups of kTokensPerPass tokens share each
// decoded weight tile.  The `pulled` word of the prep: 0 static items, 1
// pulled passes of kTokensPerPass tokens, kPulledWide pulled wide passes.
constexpr int kWideGroups = 4;
constexpr int kWideTokensPerPass = kWideGroups * kTokensPerPass;
constexpr int kWideMinPairs = 8;
constexpr int kPulledWide = 2;
// 4 partial sums per lane; two buffers, so that a pass may write its sums
// while the previous pass's epilogue still reads the other buffer
constexpr int kRedFloats = kWarps * 32 * 4;
constexpr int kRedBytes = 2 * kRedFloats * 4;
// token scales [0, 16), block maxima [16, 32) (two buffers of 8), the staged
// tokens' pair ids (ints) [32, 32 + kWideTokensPerPass)
constexpr int kMiscBytes = 256;
constexpr int kMiscPair = 32;

// fp16 planes of one vector of K elements in shared memory: hi at 0, lo at
// plane_stride (== 64 mod 128 bytes, so a quarter warp's hi and lo reads
// fall on disjoint banks), vectors token_stride apart.
__host__ __device__ constexpr int plane_stride(int k) { return 2 * k + 64; }
__host__ __device__ constexpr int token_stride(int k) { return 2 * plane_stride(k); }

// ------------------------------------------------------------------ repack
// GGUF IQ3_S rows (110-byte blocks: d[2] qs[64] qh[8] signs[32] scales[4])
// -> tile chunks.  One thread per (chunk, lane): weight 8t + i of sub-block s
// is weight j = i % 4 of group q = 8s + 2t + i / 4, whose codebook entry is
// qs[q] | qh bit q << 8 and whose sign is bit 8t + i of signs[4s .. 4s+3].
__global__ void repack_iq3s_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t n_chunks,
                                   int kb_per_row) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_chunks * 32;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t chunk = i >> 5;
    const int lane = static_cast<int>(i & 31), g = lane >> 2, t = lane & 3;
    const int64_t tile = chunk / kb_per_row;
    const int kb = static_cast<int>(chunk % kb_per_row);
    uint8_t* d = dst + chunk * kChunkBytes;
    for (int r = 0; r < 2; ++r) {
      const uint8_t* blk = src + ((tile * 16 + g + 8 * r) * kb_per_row + kb) * 110;
      for (int sb = 0; sb < 8; ++sb) {
        const uint32_t signs = blk[74 + 4 * sb + t];
        uint32_t word = 0;
        for (int w = 0; w < 8; ++w) {
          const int q = 8 * sb + 2 * t + (w >> 2);
          const uint32_t idx = blk[2 + q] | (((static_cast<uint32_t>(blk[66 + sb]) >> (2 * t + (w >> 2))) & 1u) << 8);
          const int mag = static_cast<int>((g_grid[idx] >> (8 * (w & 3))) & 255u);
          const int v = ((signs >> w) & 1u) ? -mag : mag;
          const uint32_t code = static_cast<uint32_t>((v + 15) >> 1);
          for (int b = 0; b < 4; ++b) word |= ((code >> b) & 1u) << ((code_bit(w) + b) & 31);
        }
        *reinterpret_cast<uint32_t*>(d + kCodes + 512 * (sb >> 1) + 16 * lane + 4 * (2 * (sb & 1) + r)) = word;
      }
    }
    if (lane < 16) {
      const uint8_t* blk = src + ((tile * 16 + lane) * kb_per_row + kb) * 110;
      uint8_t* rec = d + kScales + 8 * lane;
      for (int j = 0; j < 4; ++j) rec[j] = blk[106 + j];
      rec[4] = blk[0];
      rec[5] = blk[1];
      rec[6] = 0;
      rec[7] = 0;
    }
  }
}

// ------------------------------------------------------------------ route
// One warp per token: softmax over the expert logits (f32), top-k by
// repeated warp argmax (ties -> lower id), renormalised weights.
// One warp per token; lane l holds the logits of experts l, l + 32, ... in
// registers (PL of them), so the max, the softmax sum and the top-k rounds
// read global memory once.
template <int PL>
__device__ __forceinline__ void route_token(const float* __restrict__ logits, int64_t tok, int n_experts, int top_k,
                                            int32_t* ids, float* weights) {
  const int lane = threadIdx.x & 31;
  const float* lg = logits + tok * n_experts;
  float v[PL];
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < n_experts ? lg[e] : -INFINITY;
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PL; ++i) m = fmaxf(m, v[i]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PL; ++i)
    if (lane + 32 * i < n_experts) s += expf(v[i] - m);
  s = warp_sum(s);
  // selection state: bit i set = expert lane + 32 i taken; pick k is kept
  // by lane k
  uint32_t taken = 0;
  float my_p = 0.f;
  int my_id = 0;
  float wsum = 0.f;
  for (int k = 0; k < top_k && k < 16; ++k) {
    float best = -INFINITY;
    int bid = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int e = lane + 32 * i;
      if (e >= n_experts || ((taken >> i) & 1u)) continue;
      if (v[i] > best || (v[i] == best && e < bid)) {
        best = v[i];
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
    if (lane == k) {
      my_p = p;
      my_id = bid;
    }
    wsum += p;
  }
  const float denom = fmaxf(wsum, kWeightSumMin);
  if (lane < top_k && lane < 16) {
    ids[tok * top_k + lane] = my_id;
    weights[tok * top_k + lane] = my_p / denom;
  }
}

template <int PL>
__global__ void moe_route_kernel(const float* __restrict__ logits, int64_t t, int n_experts, int top_k,
                                 int32_t* __restrict__ ids, float* __restrict__ weights) {
  const int64_t tok = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_launch_dependents();
  pdl_wait();  // the logits come from the previous kernel
  if (tok < t) route_token<PL>(logits, tok, n_experts, top_k, ids, weights);
}

// ------------------------------------------------------------------ workspace
// Header: [n_unique, bad ids, ..., tickets]; per slot u < P: expert, first
// pair, pair count; the pair list sorted by (expert, pair); every token's
// fp16 planes and scale; every pair's act and down output (f32).
struct MoeWs {
  int32_t* hdr;
  int32_t* ranges;  // per CTA [first item, end item)
  int32_t* slot_expert;
  int32_t* slot_start;
  int32_t* slot_count;
  int32_t* pairs;
  // passes (T > 1): the slots' pair ranges cut into runs of kTokensPerPass,
  // in slot order; header word kPassCount holds their number
  int32_t* pass_expert;
  int32_t* pass_start;
  int32_t* pass_count;
  uint8_t* xenc;  // (T, 4 * hidden): hi plane, lo plane
  float* xscale;  // (T): x = (hi + lo) * xscale
  float* act;     // (P, ffn)
  float* dn;      // (P, hidden)
  // shared expert (model/qwen36_moe.py:634-642), when the layer has one
  uint16_t* ab;   // (T, 3, shared ffn) bf16 planes of the shared act
  float* sgate;   // (T): sigmoid(x . gate_inp)
  float* sout;    // (T, hidden): shared down output
};

__host__ __device__ inline int64_t align256(int64_t b) { return (b + 255) / 256 * 256; }

__host__ __device__ inline MoeWs moe_ws(void* base, int64_t t, int64_t p, int64_t hidden, int64_t ffn,
                                        int64_t sffn) {
  uint8_t* b = static_cast<uint8_t*>(base);
  MoeWs w;
  int64_t o = 0;
  w.hdr = reinterpret_cast<int32_t*>(b + o);
  o += kHeaderBytes;
  w.ranges = reinterpret_cast<int32_t*>(b + o);
  o += kRangeBytes;
  w.slot_expert = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.slot_start = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.slot_count = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.pairs = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.pass_expert = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.pass_start = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.pass_count = reinterpret_cast<int32_t*>(b + o);
  o += align256(4 * p);
  w.xenc = b + o;
  o += align256(4 * t * hidden);
  w.xscale = reinterpret_cast<float*>(b + o);
  o += align256(4 * t);
  w.act = reinterpret_cast<float*>(b + o);
  o += align256(4 * p * ffn);
  w.dn = reinterpret_cast<float*>(b + o);
  o += align256(4 * p * hidden);
  w.ab = reinterpret_cast<uint16_t*>(b + o);
  o += align256(6 * t * sffn);
  w.sgate = reinterpret_cast<float*>(b + o);
  o += align256(4 * t * (sffn > 0));
  w.sout = reinterpret_cast<float*>(b + o);
  return w;
}

inline int64_t moe_ws_bytes(int64_t t, int64_t p, int64_t hidden, int64_t ffn, int64_t sffn) {
  const int64_t shared = sffn > 0 ? align256(6 * t * sffn) + align256(4 * t) + align256(4 * t * hidden) : 0;
  return kHeaderBytes + kRangeBytes + 7 * align256(4 * p) + align256(4 * t * hidden) + align256(4 * t) +
         align256(4 * p * ffn) + align256(4 * p * hidden) + shared;
}

// ------------------------------------------------------------------ encode
// Power-of-two scale of a vector with max |x| = m: inv = 2^e with m * inv in
// [2^13, 2^14) (fp16 holds it with room), sx = 1 / inv.  Vectors with
// m < 2^-113 (all-zero ones included) encode as zero.
__device__ __forceinline__ void vector_scale(float m, float& inv, float& sx) {
  const uint32_t be = (__float_as_uint(m) >> 23) & 255u;  // biased exponent; m >= 0
  const bool ok = be >= 14u;
  inv = ok ? __uint_as_float((267u - be) << 23) : 0.f;
  sx = ok ? __uint_as_float((be - 13u) << 23) : 0.f;
}

// hi = fp16(x * inv), lo = fp16(x * inv - hi): hi + lo = x * inv to ~22 bits.
__device__ __forceinline__ void split_half(float x, float inv, __half& hi, __half& lo) {
  const float v = x * inv;  // exact (power of two)
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

__device__ __forceinline__ void store_planes(const float4& h, float inv, uint8_t* hi_dst, uint8_t* lo_dst) {
  __half a[4], b[4];
  split_half(h.x, inv, a[0], b[0]);
  split_half(h.y, inv, a[1], b[1]);
  split_half(h.z, inv, a[2], b[2]);
  split_half(h.w, inv, a[3], b[3]);
  *reinterpret_cast<uint2*>(hi_dst) = make_uint2(__half_as_ushort(a[0]) | (__half_as_ushort(a[1]) << 16),
                                                 __half_as_ushort(a[2]) | (__half_as_ushort(a[3]) << 16));
  *reinterpret_cast<uint2*>(lo_dst) = make_uint2(__half_as_ushort(b[0]) | (__half_as_ushort(b[1]) << 16),
                                                 __half_as_ushort(b[2]) | (__half_as_ushort(b[3]) << 16));
}

// x = hi + mid + lo in bf16: each remainder is exact in f32, so the three
// planes hold x to its 24 bits.
__device__ __forceinline__ void split3_bf16(float x, uint16_t& hi, uint16_t& mid, uint16_t& lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(h);
  const __nv_bfloat16 m = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(m);
  hi = __bfloat16_as_ushort(h);
  mid = __bfloat16_as_ushort(m);
  lo = __bfloat16_as_ushort(__float2bfloat16_rn(r2));
}

// Max over the CTA (all threads call it; `red` holds kWarps floats).
__device__ __forceinline__ float cta_max(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_max(v);
  __syncthreads();  // earlier readers of red are done
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return warp_max(lane < kWarps ? red[lane] : 0.f);
}

// ------------------------------------------------------------------ shared expert
// model/qwen36_moe.py:634-642: shared = down(silu(gate x) * up x), scaled by
// sigmoid(x . gate_inp) and added to the routed output.  bf16 weight rows
// (GGUF (out, in) orientation) are the A fragments of m16n8k16 bf16 MMAs
// as loaded (16 bytes per lane: weights 8t .. 8t+7 of a 32-column step, the
// k order permuted identically on both operands); x (and act) are three
// bf16 planes whose MMAs accumulate into the same f32 sums, so the products
// carry x to 24 bits.  8 tokens per pass (MMA columns).
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// c += rows (ra: row g, rb: row g+8; 8 bf16 each) x the 3 planes of the
// lane's B column (8 bf16 each): 32 columns of K.
__device__ __forceinline__ void bf16_step(float (&c)[4], const uint4& ra, const uint4& rb, const uint4 (&b)[3]) {
#pragma unroll
  for (int p = 0; p < 3; ++p) {
    mma_bf16(c, ra.x, rb.x, ra.y, rb.y, b[p].x, b[p].y);
    mma_bf16(c, ra.z, rb.z, ra.w, rb.w, b[p].z, b[p].w);
  }
}

// Planes of token `tok` (< t, else zeros) at column `col` of a K-row.
__device__ __forceinline__ void load_planes(const uint16_t* planes, int64_t tok, int t_total, int k, int col,
                                            uint4 (&b)[3]) {
#pragma unroll
  for (int p = 0; p < 3; ++p)
    b[p] = tok < t_total ? __ldcg(reinterpret_cast<const uint4*>(planes + (tok * 3 + p) * k + col))
                         : make_uint4(0u, 0u, 0u, 0u);
}

// The same from f32 values: x[col .. col + 8) of token `tok`, split here.
__device__ __forceinline__ void split_planes(const float* x, int64_t tok, int t_total, int k, int col,
                                             uint4 (&b)[3]) {
  float v[8];
  if (tok < t_total) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(x + tok * k + col));
    const float4 c = __ldcg(reinterpret_cast<const float4*>(x + tok * k + col + 4));
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = c.x, v[5] = c.y, v[6] = c.z, v[7] = c.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
  uint32_t w[3][4];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    uint16_t h0, m0, l0, h1, m1, l1;
    split3_bf16(v[i], h0, m0, l0);
    split3_bf16(v[i + 1], h1, m1, l1);
    w[0][i / 2] = h0 | (static_cast<uint32_t>(h1) << 16);
    w[1][i / 2] = m0 | (static_cast<uint32_t>(m1) << 16);
    w[2][i / 2] = l0 | (static_cast<uint32_t>(l1) << 16);
  }
#pragma unroll
  for (int p = 0; p < 3; ++p) b[p] = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
}

constexpr int kSharedPass = 8;  // tokens per shared-expert pass (MMA columns)

// Bulk prefetch of [p, p + bytes) into L2 (p 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__host__ __device__ inline int shared_passes(int64_t t) { return static_cast<int>((t + kSharedPass - 1) / kSharedPass); }

// Shared gate/up block b (run as extra blocks of the prep kernel): pass
// b / (ffn/16 + 1), row tile i = b % (ffn/16 + 1).  i < ffn/16: gate and up
// rows [16 i, 16 i + 16), warp w over columns [w K/8, (w+1) K/8); act =
// silu(g) * u (model/qwen36_moe.py:640) stored as bf16 planes.  i == ffn/16:
// sigmoid(x . gate_inp) for the pass's tokens.
__device__ void shared_gu_block(int b, const MoeShared& sh, const float* __restrict__ x, int t_total, int hidden,
                                const MoeWs& ws) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int sffn = static_cast<int>(sh.ffn), tiles = sffn / 16;
  const int i = b % (tiles + 1), c0 = (b / (tiles + 1)) * kSharedPass;
  const int span = hidden / kWarps;
  if (i < tiles) {  // the warp's 32 row slices (16 gate + 16 up rows x span columns) into L2 at once
    const uint16_t* m = lane < 16 ? static_cast<const uint16_t*>(sh.gate) : static_cast<const uint16_t*>(sh.up);
    prefetch_l2(m + static_cast<int64_t>(16 * i + (lane & 15)) * hidden + warp * span, 2 * span);
  }
  pdl_wait();  // x comes from earlier kernels; the weights do not
  if (i == tiles) {
    static_assert(kSharedPass == kWarps, "one token of the pass per warp");
    const int tok = c0 + warp;
    if (tok < t_total) {
      const float4* gv = reinterpret_cast<const float4*>(sh.gate_inp);
      const float4* xv = reinterpret_cast<const float4*>(x + static_cast<int64_t>(tok) * hidden);
      float a = 0.f;
#pragma unroll 8  // independent loads: eight in flight per lane
      for (int f = lane; f < hidden / 4; f += 32) {
        const float4 u = __ldg(gv + f), v = __ldcg(xv + f);
        a = fmaf(u.x, v.x, fmaf(u.y, v.y, fmaf(u.z, v.z, fmaf(u.w, v.w, a))));
      }
      a = warp_sum(a);
      if (lane == 0) ws.sgate[tok] = sigmoid_f(a);
    }
    return;
  }
  __shared__ float4 red[kWarps][32][2];
  const uint16_t* ga = static_cast<const uint16_t*>(sh.gate) + static_cast<int64_t>(16 * i + g) * hidden;
  const uint16_t* ua = static_cast<const uint16_t*>(sh.up) + static_cast<int64_t>(16 * i + g) * hidden;
  float cg[4] = {0.f, 0.f, 0.f, 0.f}, cu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4  // span / 32 is a multiple of 4: four steps' loads in flight
  for (int k0 = warp * span; k0 < (warp + 1) * span; k0 += 32) {
    const int col = k0 + 8 * t;
    const uint4 g0 = __ldg(reinterpret_cast<const uint4*>(ga + col));
    const uint4 g1 = __ldg(reinterpret_cast<const uint4*>(ga + 8 * hidden + col));
    const uint4 u0 = __ldg(reinterpret_cast<const uint4*>(ua + col));
    const uint4 u1 = __ldg(reinterpret_cast<const uint4*>(ua + 8 * hidden + col));
    uint4 bp[3];
    split_planes(x, c0 + g, t_total, hidden, col, bp);
    bf16_step(cg, g0, g1, bp);
    bf16_step(cu, u0, u1, bp);
  }
  red[warp][lane][0] = make_float4(cg[0], cg[1], cg[2], cg[3]);
  red[warp][lane][1] = make_float4(cu[0], cu[1], cu[2], cu[3]);
  __syncthreads();
  if (threadIdx.x < 16 * kSharedPass) {  // (row r, token v) of the pass
    const int r = threadIdx.x & 15, v = threadIdx.x >> 4;
    const int src = (r & 7) * 4 + (v >> 1), reg = (r >> 3) * 2 + (v & 1);
    float gs = 0.f, us = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      gs += reinterpret_cast<const float*>(&red[w][src][0])[reg];
      us += reinterpret_cast<const float*>(&red[w][src][1])[reg];
    }
    if (c0 + v < t_total) {
      uint16_t a, bb, c;
      split3_bf16(silu_f(gs) * us, a, bb, c);
      uint16_t* dst = ws.ab + static_cast<int64_t>(c0 + v) * 3 * sffn + 16 * i + r;
      dst[0] = a;
      dst[sffn] = bb;
      dst[2 * sffn] = c;
    }
  }
}

// Shared down block b (run as the first blocks of the routed gate/up
// kernel, after its dependency wait): pass b / (hidden/64), rows [64 i,
// 64 i + 64) (4 tiles), i = b % (hidden/64); warp w: tile w & 3 over
// columns [(w >> 2) K/2, ...).
__device__ void shared_down_block(int b, const MoeShared& sh, int t_total, int hidden, const MoeWs& ws) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int sffn = static_cast<int>(sh.ffn), groups = hidden / 64;
  const int i = b % groups, c0 = (b / groups) * kSharedPass;
  __shared__ float4 red[kWarps][32];
  const int tile = 4 * i + (warp & 3), half = warp >> 2, span = sffn / 2;
  const uint16_t* da = static_cast<const uint16_t*>(sh.down) + static_cast<int64_t>(16 * tile + g) * sffn;
  if (lane < 16)  // the warp's 16 row slices into L2 at once
    prefetch_l2(static_cast<const uint16_t*>(sh.down) + static_cast<int64_t>(16 * tile + lane) * sffn + half * span,
                2 * span);
  pdl_wait();  // act comes from the prep kernel; the weights do not
  pdl_launch_dependents();
  float cc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4  // span / 32 is a multiple of 4: four steps' loads in flight
  for (int k0 = half * span; k0 < (half + 1) * span; k0 += 32) {
    const int col = k0 + 8 * t;
    const uint4 d0 = __ldg(reinterpret_cast<const uint4*>(da + col));
    const uint4 d1 = __ldg(reinterpret_cast<const uint4*>(da + 8 * sffn + col));
    uint4 bp[3];
    load_planes(ws.ab, c0 + g, t_total, sffn, col, bp);
    bf16_step(cc, d0, d1, bp);
  }
  red[warp][lane] = make_float4(cc[0], cc[1], cc[2], cc[3]);
  __syncthreads();
  for (int o = threadIdx.x; o < 64 * kSharedPass; o += kThreads) {  // (row, token v) of the pass
    const int row = o & 63, v = o >> 6, tl = row >> 4, r = row & 15;
    const int src = (r & 7) * 4 + (v >> 1), reg = (r >> 3) * 2 + (v & 1);
    const float sum = reinterpret_cast<const float*>(&red[tl][src])[reg] +
                      reinterpret_cast<const float*>(&red[4 + tl][src])[reg];
    if (c0 + v < t_total) ws.sout[static_cast<int64_t>(c0 + v) * hidden + 64 * i + row] = sum;
  }
}

// ------------------------------------------------------------------ prep
// The first item of a CTA whose share of the work starts at cost w: items
// (u, c) of slot u cost passes(u) = cum[u + 1] - cum[u] each and are
// ordered by (u, c); an item belongs to the CTA its start cost falls in.
// CTA b of a static grid of G takes items [item_at(w_b), item_at(w_b+1)) with
// w_b = b W / G over the W = cum[n_slots] * chunks units of work (a pass's
// chunk is one unit; a slot's items are its chunks), where item_at(w) for w
// in slot u's units [cum[u] chunks, cum[u+1] chunks) is
// u chunks + ceil((w - cum[u] chunks) / (cum[u+1] - cum[u])).  Each slot's
// thread writes the boundaries that fall in its units (the first b there is
// ceil(cum[u] chunks G / W)), so no boundary needs a search.  32-bit: W <=
// 4096 passes x 64 chunks, G <= kMaxGrid.
__device__ __forceinline__ void static_ranges(const int32_t* cum, int n_slots, int chunks, int grid,
                                              int32_t* ranges) {
  const int w_total = cum[n_slots] * chunks;
  auto put = [&](int b, int item) {  // boundary b: the end of CTA b - 1 and the start of CTA b
    if (b > 0) ranges[2 * b - 1] = item;
    if (b < grid) ranges[2 * b] = item;
  };
  if (w_total == 0) {
    for (int b = threadIdx.x; b <= grid; b += blockDim.x) put(b, 0);
    return;
  }
  if (threadIdx.x == 0) put(grid, n_slots * chunks);
  for (int u = threadIdx.x; u < n_slots; u += blockDim.x) {
    const int w0 = cum[u] * chunks, w1 = cum[u + 1] * chunks, pu = cum[u + 1] - cum[u];
    for (int b = static_cast<int>((static_cast<int64_t>(w0) * grid + w_total - 1) / w_total); b < grid; ++b) {
      const int w = static_cast<int>(static_cast<int64_t>(b) * w_total / grid);
      if (w >= w1) break;
      put(b, u * chunks + (w - w0 + pu - 1) / pu);
    }
  }
}

// Exclusive prefix sum of v over the threads of a kThreads block, in thread
// order; *total gets the sum over all threads.  Every thread calls it.
// (v: packed fields whose sums do not carry)
__device__ __forceinline__ uint64_t block_exscan64(uint64_t v, uint64_t* wsum, uint64_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  uint64_t base = 0;
  total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint64_t sw = wsum[w];
    if (w < warp) base += sw;
    total += sw;
  }
  __syncthreads();
  return base + inc - v;
}

// Token `tok`'s fp16 hi / lo planes and scale for the expert kernels.
__device__ void encode_token(int tok, const float* __restrict__ x, int hidden, const MoeWs& ws) {
  __shared__ float red[kWarps];
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<int64_t>(tok) * hidden);
  float m = 0.f;
  for (int f = threadIdx.x; f < hidden / 4; f += kThreads) {
    const float4 h = src[f];
    m = fmaxf(m, fmaxf(fmaxf(fabsf(h.x), fabsf(h.y)), fmaxf(fabsf(h.z), fabsf(h.w))));
  }
  m = cta_max(m, red);
  float inv, sx;
  vector_scale(m, inv, sx);
  uint8_t* dst = ws.xenc + static_cast<int64_t>(tok) * 4 * hidden;
  for (int f = threadIdx.x; f < hidden / 4; f += kThreads)
    store_planes(src[f], inv, dst + 8 * f, dst + 2 * hidden + 8 * f);
  if (threadIdx.x == 0) ws.xscale[tok] = sx;
}

// The pairs' sort: block 0 of the prep kernel, or the last block of the
// routing kernel (moe_route_sort_kernel), whose other blocks wrote the ids
// (read through L2).  Dynamic shared memory: (3 n_experts + 1 + P) int32.
__device__ void prep_sort(const int32_t* ids, int p_total, int n_experts, const MoeWs& ws, int gu_grid, int gu_chunks,
                          int d_grid, int d_chunks, int pulled) {
  extern __shared__ int32_t sm[];
  int32_t* cnt = sm;               // [n_experts]
  int32_t* off = sm + n_experts;   // [n_experts] exclusive prefix of counts
  int32_t* cum = off + n_experts;  // [n_experts + 1] prefix of the slots' passes
  int32_t* sid = cum + n_experts + 1;  // [p_total] the ids
  __shared__ int32_t s_bad;
  __shared__ uint64_t s_wsum64[kWarps];
  const int tpp = pulled == kPulledWide ? kWideTokensPerPass : kTokensPerPass;  // tokens per pass
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
  for (int q = threadIdx.x; q < p_total; q += blockDim.x) sid[q] = __ldcg(ids + q);
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
  // Slots = the experts with pairs, in id order.  Thread j owns a contiguous
  // range of expert ids; one block scan of the three counts packed into 21-bit
  // fields (each total <= 4096) gives each range its first pair offset,
  // first slot and first pass (the same values a serial walk over the ids
  // would give).
  int n_slots;
  {
    const int per = (n_experts + kThreads - 1) / kThreads;
    const int e0 = min(n_experts, static_cast<int>(threadIdx.x) * per), e1 = min(n_experts, e0 + per);
    int c_sum = 0, s_sum = 0, p_sum = 0;
    for (int e = e0; e < e1; ++e) {
      const int c = cnt[e];
      c_sum += c;
      s_sum += c > 0;
      p_sum += (c + tpp - 1) / tpp;
    }
    constexpr uint64_t kField = (1ull << 21) - 1;
    uint64_t tot;
    const uint64_t ex = block_exscan64(static_cast<uint64_t>(c_sum) | (static_cast<uint64_t>(s_sum) << 21) |
                                           (static_cast<uint64_t>(p_sum) << 42),
                                       s_wsum64, tot);
    int o = static_cast<int>(ex & kField), u = static_cast<int>((ex >> 21) & kField);
    int pc = static_cast<int>(ex >> 42);
    const int s_tot = static_cast<int>((tot >> 21) & kField), p_tot = static_cast<int>(tot >> 42);
    n_slots = s_tot;
    if (threadIdx.x == 0) {
      cum[0] = 0;
      ws.hdr[0] = s_tot;
      ws.hdr[1] = s_bad;
      ws.hdr[kWorkGateUp] = 0;
      ws.hdr[kWorkDown] = 0;
      ws.hdr[kPassCount] = p_tot;
    }
    for (int e = e0; e < e1; ++e) {
      const int c = cnt[e];
      off[e] = o;
      if (c) {
        ws.slot_expert[u] = e;
        ws.slot_start[u] = o;
        ws.slot_count[u] = c;
        for (int c0 = 0; c0 < c; c0 += tpp, ++pc) {
          ws.pass_expert[pc] = e;
          ws.pass_start[pc] = o + c0;
          ws.pass_count[pc] = min(tpp, c - c0);
        }
        cum[u + 1] = pc;
        ++u;
      }
      o += c;
    }
  }
  __syncthreads();  // cum and off complete
  // A token's expert output does not depend on its place in the expert's
  // pair list (each pass column is one token's own): place the pairs with a
  // per-expert cursor (one shared-memory atomic each).
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int q = threadIdx.x; q < p_total; q += blockDim.x) {
    const int e = sid[q];
    if (e >= 0 && e < n_experts) ws.pairs[off[e] + atomicAdd(&cnt[e], 1)] = q;
  }
  if (pulled) return;  // pulled items need no static ranges
  static_ranges(cum, n_slots, gu_chunks, gu_grid, ws.ranges);
  static_ranges(cum, n_slots, d_chunks, d_grid, ws.ranges + kRangeDown);
}

// Block 0 (T > 1): counting sort of the P pairs by expert id (stable) into
// slots, and each expert-kernel CTA's contiguous item range, balanced by
// token passes.  The next T blocks: encode token (block - 1) (T == 1: block
// 0, token 0).  The rest: the shared expert's gate/up blocks.
// part (moe.cuh): kPrepAll runs every block; kPrepX only the blocks that
// read x alone (encode + shared gate/up, launched ahead of the routing).
__global__ void __launch_bounds__(kThreads) moe_prep_kernel(const int32_t* __restrict__ ids, int p_total,
                                                            int n_experts, int direct, const float* __restrict__ x,
                                                            int t_total, int hidden, MoeWs ws, int gu_grid,
                                                            int gu_chunks, int d_grid, int d_chunks, MoeShared sh,
                                                            int pulled, int part) {
  pdl_launch_dependents();
  const int enc0 = direct ? 0 : 1;
  // the block's role in the full layout
  const int bx = static_cast<int>(blockIdx.x) + (part == kPrepX ? enc0 : 0);
  if (bx >= enc0 + t_total) {
    shared_gu_block(bx - enc0 - t_total, sh, x, t_total, hidden, ws);  // waits after its L2 prefetch
    return;
  }
  pdl_wait();
  if (direct || bx > 0) {
    encode_token(bx - (direct ? 0 : 1), x, hidden, ws);
    return;
  }
  prep_sort(ids, p_total, n_experts, ws, gu_grid, gu_chunks, d_grid, d_chunks, pulled);
}


// bt_moe_route_sort_iq3s, the prep kernel's work folded into the routing
// launch: blocks [0, n_route) route (moe_route_kernel's warps), and the last
// of them to finish (an arrival ticket in header word kRouteTicket, re-armed
// by that block) sorts the pairs; blocks [n_route, n_route + T) encode the
// tokens (n_enc = T, or 0 for one token, whose layer call encodes).
template <int PL>
__global__ void __launch_bounds__(kThreads) moe_route_sort_kernel(const float* __restrict__ logits, int64_t t,
                                                                  int n_experts, int top_k, int32_t* ids,
                                                                  float* weights, MoeWs ws, int gu_grid,
                                                                  int gu_chunks, int d_grid, int d_chunks,
                                                                  int pulled, const float* __restrict__ x,
                                                                  int hidden, int n_route) {
  pdl_launch_dependents();
  pdl_wait();  // the logits and x come from earlier kernels
  if (static_cast<int>(blockIdx.x) >= n_route) {
    encode_token(blockIdx.x - n_route, x, hidden, ws);
    return;
  }
  const int64_t tok = blockIdx.x * static_cast<int64_t>(kWarps) + (threadIdx.x >> 5);
  if (tok < t) route_token<PL>(logits, tok, n_experts, top_k, ids, weights);
  if (t == 1) return;
  if (n_route == 1) {  // one routing block: its own ids, visible after a block barrier
    __syncthreads();
    prep_sort(ids, static_cast<int>(t * top_k), n_experts, ws, gu_grid, gu_chunks, d_grid, d_chunks, pulled);
    return;
  }
  __shared__ int s_last;
  __threadfence();  // this block's ids before its arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    s_last = atomicAdd(ws.hdr + kRouteTicket, 1) == n_route - 1;
    if (s_last) atomicExch(ws.hdr + kRouteTicket, 0);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // every block's ids are visible past its arrival
  prep_sort(ids, static_cast<int>(t * top_k), n_experts, ws, gu_grid, gu_chunks, d_grid, d_chunks, pulled);
}

// ------------------------------------------------------------------ MMA core
__device__ __forceinline__ uint4 ld_stream16(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// A lane's share of one tile chunk (rows g and g+8): the code words of all
// 8 sub-blocks (part[j] = sub-blocks 2j, 2j+1) and the two rows' scale
// records.
struct Tile {
  uint4 part[4];
  uint2 ra, rb;
};

__device__ __forceinline__ void load_tile(const uint8_t* chunk, int lane, Tile& T) {
#pragma unroll
  for (int j = 0; j < 4; ++j) T.part[j] = ld_stream16(chunk + kCodes + 512 * j + 16 * lane);
  const int g = lane >> 2;
  T.ra = __ldg(reinterpret_cast<const uint2*>(chunk + kScales) + g);
  T.rb = __ldg(reinterpret_cast<const uint2*>(chunk + kScales) + g + 8);
}

__device__ __forceinline__ uint32_t f16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t f16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// The fp16 pairs (w0, w1), (w2, w3), (w4, w5), (w6, w7) of a code word.  A
// code c at mantissa bits [k, k+4) of an fp16 with the exponent of 1024 (bit
// pattern 0x6400) makes 1024 + 2^k c; then v = 2c - 15 is one exact f16x2
// add (k = 1: minus 1039) or fma (k = 5: times 1/16, minus 79).  Codes 4/5
// reach bits 1-4 of each half by a shift of 8, codes 6/7 by a rotation by 12.
__device__ __forceinline__ void decode_word(uint32_t w, uint32_t& p01, uint32_t& p23, uint32_t& p45,
                                            uint32_t& p67) {
  constexpr uint32_t kMagic = 0x64006400u;       // fp16 1024 | 1024
  constexpr uint32_t kMinus1039 = 0xE40FE40Fu;   // fp16 -1039 | -1039
  constexpr uint32_t kSixteenth = 0x2C002C00u;   // fp16 1/16 | 1/16
  constexpr uint32_t kMinus79 = 0xD4F0D4F0u;     // fp16 -79 | -79
  p01 = f16x2_add((w & 0x001E001Eu) | kMagic, kMinus1039);
  p23 = f16x2_fma((w & 0x01E001E0u) | kMagic, kSixteenth, kMinus79);
  p45 = f16x2_add(((w >> 8) & 0x001E001Eu) | kMagic, kMinus1039);
  p67 = f16x2_add((__funnelshift_r(w, w, 12) & 0x001E001Eu) | kMagic, kMinus1039);
}

// d * (1 + 2 * nibble of sub-block sb) (quant/dequant.py:164-185), as one
// fma: the float with bits 0x4B000000 | (2n + 1) is 2^23 + 2n + 1, so m * d -
// 2^23 d is (2n + 1) d exactly (an 11-bit by 5-bit product), rounded once:
// the same value as the f32 product.
__device__ __forceinline__ float sub_scale(uint32_t nibbles, int sb, float d, float dneg) {
  const uint32_t two_n = (sb == 0 ? (nibbles << 1) : (nibbles >> (4 * sb - 1))) & 0x1Eu;
  return fmaf(__uint_as_float(0x4B000001u | two_n), d, dneg);
}

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// acc[r] += scale(row) * (hi + lo sums of one sub-block) for rows g (r = 0)
// and g+8, token column pair t.  wg / wg8: the sub-block's code words of
// rows g and g+8; `b`: elements 8t..8t+7 of the sub-block of this lane's B
// column (token g/2, plane g%2).
__device__ __forceinline__ void tile_step(uint32_t wg, uint32_t wg8, float sg, float sg8, const uint4& b,
                                          float (&acc)[2]) {
  uint32_t a01, a23, a45, a67, c01, c23, c45, c67;
  decode_word(wg, a01, a23, a45, a67);
  decode_word(wg8, c01, c23, c45, c67);
  float cc[4] = {0.f, 0.f, 0.f, 0.f};
  mma_f16(cc, a01, c01, a23, c23, b.x, b.y);  // weights 8t .. 8t+3
  mma_f16(cc, a45, c45, a67, c67, b.z, b.w);  // weights 8t+4 .. 8t+7
  acc[0] = fmaf(sg, cc[0] + cc[1], acc[0]);
  acc[1] = fmaf(sg8, cc[2] + cc[3], acc[1]);
}

__device__ __forceinline__ float half_lo(uint32_t v) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu)));
}

// All 8 sub-blocks of K-block `kb` for two tiles sharing the B operands,
// in sub-block order.  Each part of a tile's registers is refilled with the
// same part of the next chunk (na / nb; null: none) as soon as it has been
// read, so one tile's registers carry the current block and the next one's
// loads in flight.  `xl`: this lane's B column base (token g/2, plane g%2,
// element 8t).
__device__ __forceinline__ void block_steps(Tile& ta, Tile& tb, const uint8_t* na, const uint8_t* nb, int lane,
                                            const uint8_t* xl, int kb, float (&acc)[2][2]) {
  // the 4 lanes of a quad share rows g and g+8: lane t computes the scales of
  // sub-blocks 2t and 2t+1, the others read them with a shuffle
  const int g = lane >> 2, tq = lane & 3, q0 = lane & ~3;
  float s_a0e, s_a0o, s_a1e, s_a1o, s_b0e, s_b0o, s_b1e, s_b1o;
  {
    const float da0 = half_lo(ta.ra.y), da1 = half_lo(ta.rb.y), db0 = half_lo(tb.ra.y), db1 = half_lo(tb.rb.y);
    s_a0e = sub_scale(ta.ra.x, 2 * tq, da0, -8388608.0f * da0);
    s_a0o = sub_scale(ta.ra.x, 2 * tq + 1, da0, -8388608.0f * da0);
    s_a1e = sub_scale(ta.rb.x, 2 * tq, da1, -8388608.0f * da1);
    s_a1o = sub_scale(ta.rb.x, 2 * tq + 1, da1, -8388608.0f * da1);
    s_b0e = sub_scale(tb.ra.x, 2 * tq, db0, -8388608.0f * db0);
    s_b0o = sub_scale(tb.ra.x, 2 * tq + 1, db0, -8388608.0f * db0);
    s_b1e = sub_scale(tb.rb.x, 2 * tq, db1, -8388608.0f * db1);
    s_b1o = sub_scale(tb.rb.x, 2 * tq + 1, db1, -8388608.0f * db1);
  }
  if (na) {
    ta.ra = __ldg(reinterpret_cast<const uint2*>(na + kScales) + g);
    ta.rb = __ldg(reinterpret_cast<const uint2*>(na + kScales) + g + 8);
  }
  if (nb) {
    tb.ra = __ldg(reinterpret_cast<const uint2*>(nb + kScales) + g);
    tb.rb = __ldg(reinterpret_cast<const uint2*>(nb + kScales) + g + 8);
  }
  const uint8_t* xq = xl + kb * 512;  // 8 sub-blocks x 32 fp16
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint4 b0 = *reinterpret_cast<const uint4*>(xq + 128 * p);
    const uint4 b1 = *reinterpret_cast<const uint4*>(xq + 128 * p + 64);
    const uint4 &pa = ta.part[p], &pb = tb.part[p];
    const int src = q0 | p;
    tile_step(pa.x, pa.y, __shfl_sync(0xffffffffu, s_a0e, src), __shfl_sync(0xffffffffu, s_a1e, src), b0, acc[0]);
    tile_step(pb.x, pb.y, __shfl_sync(0xffffffffu, s_b0e, src), __shfl_sync(0xffffffffu, s_b1e, src), b0, acc[1]);
    tile_step(pa.z, pa.w, __shfl_sync(0xffffffffu, s_a0o, src), __shfl_sync(0xffffffffu, s_a1o, src), b1, acc[0]);
    tile_step(pb.z, pb.w, __shfl_sync(0xffffffffu, s_b0o, src), __shfl_sync(0xffffffffu, s_b1o, src), b1, acc[1]);
    if (na) ta.part[p] = ld_stream16(na + kCodes + 512 * p + 16 * lane);
    if (nb) tb.part[p] = ld_stream16(nb + kCodes + 512 * p + 16 * lane);
  }
}

// tile_step on code words decoded beforehand: a[0..3] row g, a[4..7] row g+8.
__device__ __forceinline__ void mma_sub(const uint32_t (&a)[8], float sg, float sg8, const uint4& b,
                                        float (&acc)[2]) {
  float cc[4] = {0.f, 0.f, 0.f, 0.f};
  mma_f16(cc, a[0], a[4], a[1], a[5], b.x, b.y);
  mma_f16(cc, a[2], a[6], a[3], a[7], b.z, b.w);
  acc[0] = fmaf(sg, cc[0] + cc[1], acc[0]);
  acc[1] = fmaf(sg8, cc[2] + cc[3], acc[1]);
}

// block_steps for a wide pass: each code word is decoded once and multiplied
// with the planes of every 4-token group s < ng (group s's planes `gstride`
// bytes after group 0's) into acc[s].  Per token the MMAs, the sub-block
// order and the f32 adds are block_steps', so the sums are the same bits.
template <int NG>
__device__ __forceinline__ void block_steps_wide(Tile& ta, Tile& tb, const uint8_t* na, const uint8_t* nb, int lane,
                                                 const uint8_t* xl, int gstride, int kb, int ng,
                                                 float (&acc)[NG][2][2]) {
  const int g = lane >> 2, tq = lane & 3, q0 = lane & ~3;
  float s_a0[2], s_a1[2], s_b0[2], s_b1[2];  // [even, odd] sub-block of the lane's pair
  {
    const float da0 = half_lo(ta.ra.y), da1 = half_lo(ta.rb.y), db0 = half_lo(tb.ra.y), db1 = half_lo(tb.rb.y);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      s_a0[h] = sub_scale(ta.ra.x, 2 * tq + h, da0, -8388608.0f * da0);
      s_a1[h] = sub_scale(ta.rb.x, 2 * tq + h, da1, -8388608.0f * da1);
      s_b0[h] = sub_scale(tb.ra.x, 2 * tq + h, db0, -8388608.0f * db0);
      s_b1[h] = sub_scale(tb.rb.x, 2 * tq + h, db1, -8388608.0f * db1);
    }
  }
  if (na) {
    ta.ra = __ldg(reinterpret_cast<const uint2*>(na + kScales) + g);
    ta.rb = __ldg(reinterpret_cast<const uint2*>(na + kScales) + g + 8);
  }
  if (nb) {
    tb.ra = __ldg(reinterpret_cast<const uint2*>(nb + kScales) + g);
    tb.rb = __ldg(reinterpret_cast<const uint2*>(nb + kScales) + g + 8);
  }
  const uint8_t* xq = xl + kb * 512;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint4 &pa = ta.part[p], &pb = tb.part[p];
    const int src = q0 | p;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t da[8], db[8];
      decode_word(h ? pa.z : pa.x, da[0], da[1], da[2], da[3]);
      decode_word(h ? pa.w : pa.y, da[4], da[5], da[6], da[7]);
      decode_word(h ? pb.z : pb.x, db[0], db[1], db[2], db[3]);
      decode_word(h ? pb.w : pb.y, db[4], db[5], db[6], db[7]);
      const float sa0 = __shfl_sync(0xffffffffu, s_a0[h], src), sa1 = __shfl_sync(0xffffffffu, s_a1[h], src);
      const float sb0 = __shfl_sync(0xffffffffu, s_b0[h], src), sb1 = __shfl_sync(0xffffffffu, s_b1[h], src);
#pragma unroll
      for (int s = 0; s < NG; ++s) {
        if (s < ng) {
          const uint4 b = *reinterpret_cast<const uint4*>(xq + s * gstride + 128 * p + 64 * h);
          mma_sub(da, sa0, sa1, b, acc[s][0]);
          mma_sub(db, sb0, sb1, b, acc[s][1]);
        }
      }
    }
    if (na) ta.part[p] = ld_stream16(na + kCodes + 512 * p + 16 * lane);
    if (nb) tb.part[p] = ld_stream16(nb + kCodes + 512 * p + 16 * lane);
  }
}

// ------------------------------------------------------------------ staging
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// The expert slot an item serves: from the prep kernel's sort, or (one
// token, whose top-k experts are distinct) straight from the routing ids.
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
  s.expert = ws.slot_expert[u];
  s.start = ws.slot_start[u];
  s.count = ws.slot_count[u];
  return true;
}

__device__ __forceinline__ int pair_of(bool direct, const MoeWs& ws, int i) { return direct ? i : ws.pairs[i]; }

// The slot records of a CTA's item range, read once into shared memory so
// that looking up the next item (to load its tiles ahead) costs no global
// round trip.  A CTA's contiguous range spans a few slots; one past the
// cache falls back to global memory.
constexpr int kSlotCache = 16;
struct SlotCache {
  int first, n;
  int expert[kSlotCache], start[kSlotCache], count[kSlotCache], live[kSlotCache];
};

__device__ __forceinline__ void fill_slots(SlotCache& sc, int i0, int i1, int chunks, bool direct, const int32_t* ids,
                                           int n_experts, const MoeWs& ws) {
  const int first = i0 / chunks;
  const int n = i1 > i0 ? min(kSlotCache, (i1 - 1) / chunks - first + 1) : 0;
  if (threadIdx.x < n) {
    Slot s{};
    sc.live[threadIdx.x] = slot_of(first + threadIdx.x, direct, ids, n_experts, ws, s) ? 1 : 0;
    sc.expert[threadIdx.x] = s.expert;
    sc.start[threadIdx.x] = s.start;
    sc.count[threadIdx.x] = s.count;
  }
  if (threadIdx.x == 0) {
    sc.first = first;
    sc.n = n;
  }
  __syncthreads();
}

__device__ __forceinline__ bool cached_slot(const SlotCache& sc, int u, bool direct, const int32_t* ids,
                                            int n_experts, const MoeWs& ws, Slot& s) {
  const int i = u - sc.first;
  if (i < 0 || i >= sc.n) return slot_of(u, direct, ids, n_experts, ws, s);
  s.expert = sc.expert[i];
  s.start = sc.start[i];
  s.count = sc.count[i];
  return sc.live[i] != 0;
}

// sum_k w[k] * dn[k * stride] over a token's top_k pairs in routing order,
// each product rounded before the add like the reference's (out * w).sum(0)
// in f32; pairs with an invalid id contribute nothing.  Eight pairs' loads
// are in flight at a time.
__device__ __forceinline__ float routed_sum(const int32_t* ids, const float* w, const float* dn, int64_t stride,
                                            int top_k, int n_experts) {
  float a = 0.f;
  for (int k0 = 0; k0 < top_k; k0 += 8) {
    float v[8], wk[8];
    bool ok[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j;
      const int e = k < top_k ? ids[k] : -1;
      ok[j] = e >= 0 && e < n_experts;
      v[j] = ok[j] ? __ldcg(dn + k * stride) : 0.f;
      wk[j] = ok[j] ? w[k] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (ok[j]) a = __fadd_rn(a, __fmul_rn(v[j], wk[j]));
  }
  return a;
}

// ------------------------------------------------------------------ gate/up
// Items (slot u, chunk c): gate/up rows [OUT c, OUT c + OUT) of the slot's
// expert, OUT = 16 * TP, TP = 8 / KB tile pairs.  Warp w: tile pair
// tp = w % TP (gate rows + the same up rows) over K-block kb = w / TP.  The
// K-blocks meet in shared memory; act = silu(g) * u (model/moe.py:229).
template <int KB>
__global__ void __launch_bounds__(kThreads, 2)
    moe_gate_up_kernel(const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up, const int32_t* ids,
                       int n_experts, int direct, int top_k, int ffn, MoeWs ws, int gu_grid, MoeShared sh,
                       int s_blocks, int t_total, int hidden, const float* __restrict__ x, int sgu_blocks) {
  constexpr int K = KB * 256, TP = kWarps / KB, OUT = 16 * TP;
  static_assert(kWarps % KB == 0, "K blocks per item");
  extern __shared__ __align__(16) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem);
  float* xsc = reinterpret_cast<float*>(smem + kRedBytes);
  int* spair = reinterpret_cast<int*>(xsc) + kMiscPair;
  uint8_t* xs = smem + kRedBytes + kMiscBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (static_cast<int>(blockIdx.x) < s_blocks) {  // the shared expert's down rows
    shared_down_block(blockIdx.x, sh, t_total, hidden, ws);
    return;
  }
  if (static_cast<int>(blockIdx.x) < s_blocks + sgu_blocks) {  // or its gate/up rows
    shared_gu_block(blockIdx.x - s_blocks, sh, x, t_total, hidden, ws);
    return;
  }
  const int rb = blockIdx.x - s_blocks - sgu_blocks;  // routed CTA
  // The op's inputs (ids, x) come from whatever ran before: read them only
  // after the wait, and let the down kernel start only then, so that it may
  // read the slots before its own wait.
  pdl_wait();
  pdl_launch_dependents();
  const int chunks = ffn / OUT;
  const int i0 = direct ? rb * top_k * chunks / gu_grid : ws.ranges[2 * rb];
  const int i1 = direct ? (rb + 1) * top_k * chunks / gu_grid : ws.ranges[2 * rb + 1];
  const int tp = warp % TP, kb = warp / TP;
  const uint8_t* xl = xs + (g >> 1) * token_stride(K) + (g & 1) * plane_stride(K) + 16 * t;
  __shared__ SlotCache sc;
  fill_slots(sc, i0, i1, chunks, direct != 0, ids, n_experts, ws);
  // this warp's chunk offset of item `it` (-1: a slot with an invalid expert)
  auto item_off = [&](int it) -> int64_t {
    const int u = it / chunks, c = it - u * chunks;
    Slot s;
    if (!cached_slot(sc, u, direct != 0, ids, n_experts, ws, s)) return -1;
    return ((static_cast<int64_t>(s.expert) * (ffn / 16) + c * TP + tp) * KB + kb) * kChunkBytes;
  };
  Tile tg{}, tu{};
  int64_t cur = i0 < i1 ? item_off(i0) : -1;
  if (cur >= 0) {
    load_tile(gate + cur, lane, tg);
    load_tile(up + cur, lane, tu);
  }
  int staged = -1;  // (slot, first pair) whose tokens are in xs
  int npass = 0;    // passes so far: the reduction buffer of a pass is npass & 1
  for (int it = i0; it < i1; ++it) {
    const int u = it / chunks, c = it - u * chunks;
    Slot s;
    const bool live = cached_slot(sc, u, direct != 0, ids, n_experts, ws, s);
    const int64_t nxt = it + 1 < i1 ? item_off(it + 1) : -1;
    if (!live && nxt >= 0) {  // nothing computed here: load the next item's tiles now
      load_tile(gate + nxt, lane, tg);
      load_tile(up + nxt, lane, tu);
    }
    for (int c0 = 0; live && c0 < s.count; c0 += kTokensPerPass) {
      const int mc = min(kTokensPerPass, s.count - c0);
      // the tiles to load during this pass: this item's again for a later
      // pass, else the next item's
      const int64_t load = c0 + kTokensPerPass < s.count ? cur : nxt;
      if (u * 4096 + c0 != staged) {
        __syncthreads();  // readers of xs are done
        for (int i = threadIdx.x; i < mc * (K / 4); i += kThreads) {  // 16-byte pieces, K/8 per plane
          const int v = i / (K / 4), j = i - v * (K / 4), plane = j / (K / 8), piece = j - plane * (K / 8);
          const int tok = pair_of(direct != 0, ws, s.start + c0 + v) / top_k;
          cp_async16(xs + v * token_stride(K) + plane * plane_stride(K) + 16 * piece,
                     ws.xenc + static_cast<int64_t>(tok) * 4 * K + plane * 2 * K + 16 * piece);
        }
        cp_async_commit();
        if (threadIdx.x < mc) {
          const int pair = pair_of(direct != 0, ws, s.start + c0 + threadIdx.x);
          spair[threadIdx.x] = pair;
          xsc[threadIdx.x] = ws.xscale[pair / top_k];
        }
        cp_async_wait_all();
        __syncthreads();
        staged = u * 4096 + c0;
      }
      float acc[2][2] = {};
      block_steps(tg, tu, load >= 0 ? gate + load : nullptr, load >= 0 ? up + load : nullptr, lane, xl, kb, acc);
      float* rb = red + (npass++ & 1) * kRedFloats;
      reinterpret_cast<float4*>(rb)[warp * 32 + lane] = make_float4(acc[0][0], acc[0][1], acc[1][0], acc[1][1]);
      __syncthreads();
      // (no barrier after the epilogue: the next pass writes the other
      // buffer, and a restaging of xs/xsc/spair starts with a barrier)
      for (int i = threadIdx.x; i < OUT * mc; i += kThreads) {
        const int v = i / OUT, o = i - v * OUT;
        const int otp = o >> 4, r = o & 15, src = (r & 7) * 4 + v, reg = r >> 3;
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int k = 0; k < KB; ++k) {
          const float* rr = rb + ((k * TP + otp) * 32 + src) * 4;
          gs += rr[reg];
          us += rr[2 + reg];
        }
        gs *= xsc[v];
        us *= xsc[v];
        ws.act[static_cast<int64_t>(spair[v]) * ffn + c * OUT + o] = silu_f(gs) * us;
      }
    }
    cur = nxt;
  }
}

// ------------------------------------------------------------------ down
// Items (slot u, chunk c): rows [ROWS c, ROWS c + ROWS) of the slot's
// expert, ROWS = 32 * TP, TP = 8 / KB tile pairs.  Warp w: tiles 2tp and
// 2tp+1 (tp = w % TP) over K-block kb = w / TP.  The slots come from the
// prep kernel, which completed before the gate/up kernel released this one,
// so the first item's tiles are loaded before the dependency wait.  Each
// pass encodes its pairs' act (f32, from the gate/up kernel) into fp16
// planes in shared memory.
template <int KB>
__global__ void __launch_bounds__(kThreads, 2)
    moe_down_kernel(const uint8_t* __restrict__ down, const int32_t* ids, const float* __restrict__ weights,
                    float* out, int n_experts, int direct, int top_k, int hidden, MoeWs ws, int shared, MoeShared sh,
                    int sd_blocks, int t_total) {
  constexpr int K = KB * 256, TP = kWarps / KB, ROWS = 32 * TP;
  static_assert(kWarps % KB == 0, "K blocks per item");
  extern __shared__ __align__(16) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem);
  float* xsc = reinterpret_cast<float*>(smem + kRedBytes);
  float* wmax = xsc + 16;
  int* spair = reinterpret_cast<int*>(xsc) + kMiscPair;
  uint8_t* xs = smem + kRedBytes + kMiscBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (static_cast<int>(blockIdx.x) < sd_blocks) {  // the shared expert's down rows (T > 1)
    shared_down_block(blockIdx.x, sh, t_total, hidden, ws);
    return;
  }
  const int rb = blockIdx.x - sd_blocks, nrb = gridDim.x - sd_blocks;  // routed CTA
  const int chunks = hidden / ROWS;
  const int i0 = direct ? rb * top_k * chunks / nrb : ws.ranges[kRangeDown + 2 * rb];
  const int i1 = direct ? (rb + 1) * top_k * chunks / nrb : ws.ranges[kRangeDown + 2 * rb + 1];
  const int tp = warp % TP, kb = warp / TP;
  const uint8_t* xl = xs + (g >> 1) * token_stride(K) + (g & 1) * plane_stride(K) + 16 * t;
  __shared__ SlotCache sc;
  fill_slots(sc, i0, i1, chunks, direct != 0, ids, n_experts, ws);
  // the offset of this warp's first chunk of item `it` (the second follows
  // KB chunks later; -1: a slot with an invalid expert)
  auto item_off = [&](int it) -> int64_t {
    const int u = it / chunks, c = it - u * chunks;
    Slot s;
    if (!cached_slot(sc, u, direct != 0, ids, n_experts, ws, s)) return -1;
    const int64_t tile = static_cast<int64_t>(s.expert) * (hidden / 16) + c * 2 * TP + 2 * tp;
    return (tile * KB + kb) * kChunkBytes;
  };
  constexpr int64_t kNextTile = static_cast<int64_t>(KB) * kChunkBytes;
  Tile ta{}, tb{};
  int64_t cur = i0 < i1 ? item_off(i0) : -1;
  if (cur >= 0) {
    load_tile(down + cur, lane, ta);
    load_tile(down + cur + kNextTile, lane, tb);
  }
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int s_last;
  int staged = -1;
  int npass = 0;  // the reduction buffer of a pass is npass & 1
  for (int it = i0; it < i1; ++it) {
    const int u = it / chunks, c = it - u * chunks;
    Slot s;
    const bool live = cached_slot(sc, u, direct != 0, ids, n_experts, ws, s);
    const int64_t nxt = it + 1 < i1 ? item_off(it + 1) : -1;
    if (!live && nxt >= 0) {  // nothing computed here: load the next item's tiles now
      load_tile(down + nxt, lane, ta);
      load_tile(down + nxt + kNextTile, lane, tb);
    }
    for (int c0 = 0; live && c0 < s.count; c0 += kTokensPerPass) {
      const int mc = min(kTokensPerPass, s.count - c0);
      const int64_t load = c0 + kTokensPerPass < s.count ? cur : nxt;  // as in the gate/up kernel
      if (u * 4096 + c0 != staged) {
        // act of pair slot v: threads [64 v, 64 v + 64) (warps 2v, 2v+1) -> fp16 planes
        const int v = threadIdx.x >> 6, j = threadIdx.x & 63;
        constexpr int F4 = K / 4 / 64;  // float4 per thread
        float4 h[F4];
        float m = 0.f;
        const float4* src = nullptr;
        const int pair = v < mc ? pair_of(direct != 0, ws, s.start + c0 + v) : 0;
        if (v < mc) src = reinterpret_cast<const float4*>(ws.act + static_cast<int64_t>(pair) * K);
#pragma unroll
        for (int i = 0; i < F4; ++i) {
          h[i] = v < mc ? __ldcg(src + j + 64 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
          m = fmaxf(m, fmaxf(fmaxf(fabsf(h[i].x), fabsf(h[i].y)), fmaxf(fabsf(h[i].z), fabsf(h[i].w))));
        }
        m = warp_max(m);
        __syncthreads();  // readers of xs, xsc and wmax are done
        if (lane == 0) wmax[warp] = m;
        __syncthreads();
        m = fmaxf(wmax[2 * v], wmax[2 * v + 1]);
        float inv, sx;
        vector_scale(m, inv, sx);
        if (v < mc) {
          uint8_t* dst = xs + v * token_stride(K);
#pragma unroll
          for (int i = 0; i < F4; ++i)
            store_planes(h[i], inv, dst + 8 * (j + 64 * i), dst + plane_stride(K) + 8 * (j + 64 * i));
          if (j == 0) {
            xsc[v] = sx;
            spair[v] = pair;
          }
        }
        __syncthreads();
        staged = u * 4096 + c0;
      }
      float acc[2][2] = {};
      block_steps(ta, tb, load >= 0 ? down + load : nullptr, load >= 0 ? down + load + kNextTile : nullptr, lane,
                  xl, kb, acc);
      float* rb = red + (npass++ & 1) * kRedFloats;
      reinterpret_cast<float4*>(rb)[warp * 32 + lane] = make_float4(acc[0][0], acc[0][1], acc[1][0], acc[1][1]);
      __syncthreads();
      for (int i = threadIdx.x; i < ROWS * mc; i += kThreads) {
        const int v = i / ROWS, o = i - v * ROWS;
        const int otp = o >> 5, jt = (o >> 4) & 1, r = o & 15;
        const int src = (r & 7) * 4 + v, reg = jt * 2 + (r >> 3);
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < KB; ++k) sum += rb[((k * TP + otp) * 32 + src) * 4 + reg];
        ws.dn[static_cast<int64_t>(spair[v]) * hidden + c * ROWS + o] = sum * xsc[v];
      }
      // one token: every dn store of the block precedes thread 0's ticket;
      // more tokens: the next pass writes the other buffer, and a restaging
      // starts with a barrier
      if (direct) __syncthreads();
    }
    if (direct) {
      // one token: the last of the top_k items of this row chunk sums the
      // experts' rows in routing order (atomic ticket, re-armed after)
      if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(ws.hdr + kTicketBase + c, 1) == top_k - 1;
      }
      __syncthreads();
      if (s_last) {
        __threadfence();
        for (int r = threadIdx.x; r < ROWS; r += kThreads) {
          const int hh = c * ROWS + r;
          float a = routed_sum(ids, weights, ws.dn + hh, hidden, top_k, n_experts);
          if (shared) a = __fadd_rn(a, __fmul_rn(__ldcg(ws.sgate), __ldcg(ws.sout + hh)));  // routed + gate * shared
          out[hh] = a;
        }
        if (threadIdx.x == 0) atomicExch(ws.hdr + kTicketBase + c, 0);
      }
      __syncthreads();  // s_last readers done
    }
    cur = nxt;
  }
}

// ------------------------------------------------- pulled items (T > 1)
// The batched form of the two expert kernels.  An item is (slot u, row
// chunk c) of a whole CTA: each warp owns its own 16-row tile pair (gate/up)
// or two 16-row tiles (down) over ALL K-blocks, accumulating in registers,
// so no partial sums meet across warps and the only barriers are the
// restaging of the item's token planes; CTAs pull items from a counter
// (header word kWorkGateUp / kWorkDown, reset by the prep kernel), so the
// ones that finish early take the remaining work.  The next K-block's tiles
// (and at an item's last K-block the next item's first ones) load while the
// current block computes.

// K splits of a pulled gate/up item.  With the 4-bit code layout an
// undivided K (128-row items: 8 tile pairs over the full K, no partial sums
// to add through shared memory) is the faster choice: 64 tokens 162 -> 154 us
// per layer; 2 gave 64-row items (4 tile pairs x 2 K halves).
constexpr int kGuSplits = 1;
// Batches of up to this many tokens keep the static, K-split items (few
// selected experts: finer items fill the GPU better; on B200 at the 35B
// shape 12 tokens take 71 us static vs 87 us pulled, 16 tokens 79 vs 89,
// 24 tokens break even).
constexpr int64_t kStaticMaxTokens = 16;

// Items are published two ahead: at the start of iteration i thread 0 pulls
// the item of iteration i + 2 into s_next[(i + 2) % 3], so the item of
// iteration i + 1 (published before the previous closing barrier) can be
// read during iteration i, to load its first tiles early; the slot a pull
// overwrites was last read before the previous closing barrier.
__device__ __forceinline__ int pull_item(int32_t* counter) { return atomicAdd(counter, 1); }

// Gate/up: item = (slot u, chunk c) of OUT = 16 TP rows, TP = 8 / KS tile
// pairs; warp w owns tile pair w % TP over the KB / KS K-blocks of split
// w / TP.  KS > 1 adds the splits' partial sums through shared memory.
template <int KB, int KS>
__global__ void __launch_bounds__(kThreads, 2)
    moe_gate_up_pulled_kernel(const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up, int top_k,
                              int ffn, MoeWs ws, MoeShared sh, int s_blocks, int t_total, int hidden,
                              const float* __restrict__ x, int sgu_blocks) {
  constexpr int K = KB * 256, TP = kWarps / KS, OUT = 16 * TP, KPW = KB / KS;
  static_assert(kWarps % KS == 0 && KB % KS == 0, "K splits");
  extern __shared__ __align__(16) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem);
  float* xsc = reinterpret_cast<float*>(smem + kRedBytes);
  int* spair = reinterpret_cast<int*>(xsc) + kMiscPair;
  uint8_t* xs = smem + kRedBytes + kMiscBytes;
  __shared__ int s_next[3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (static_cast<int>(blockIdx.x) < s_blocks) {  // the shared expert's down rows
    shared_down_block(blockIdx.x, sh, t_total, hidden, ws);
    return;
  }
  if (static_cast<int>(blockIdx.x) < s_blocks + sgu_blocks) {  // or its gate/up rows
    shared_gu_block(blockIdx.x - s_blocks, sh, x, t_total, hidden, ws);
    return;
  }
  pdl_wait();
  pdl_launch_dependents();
  const int chunks = ffn / OUT;
  const int n_items = __ldcg(ws.hdr + kPassCount) * chunks;
  const int tp = warp % TP, kb0 = (warp / TP) * KPW;
  const uint8_t* xl = xs + (g >> 1) * token_stride(K) + (g & 1) * plane_stride(K) + 16 * t;
  // offset of K-block 0 of this warp's tile pair in item `item` (-1: none)
  auto item_base = [&](int item) -> int64_t {
    if (item >= n_items) return -1;
    const int q = item / chunks, c = item - q * chunks;
    const int e = __ldcg(ws.pass_expert + q);
    return (static_cast<int64_t>(e) * (ffn / 16) + c * TP + tp) * KB * kChunkBytes;
  };
  if (threadIdx.x == 0) {
    s_next[0] = pull_item(ws.hdr + kWorkGateUp);
    s_next[1] = pull_item(ws.hdr + kWorkGateUp);
  }
  __syncthreads();
  int it = s_next[0];
  Tile tg{}, tu{};
  int64_t base = item_base(it);
  if (base >= 0) {
    load_tile(gate + base + kb0 * kChunkBytes, lane, tg);
    load_tile(up + base + kb0 * kChunkBytes, lane, tu);
  }
  int staged = -1;
  int npass = 0;  // the reduction buffer of a pass is npass & 1
  for (int iter = 0; it < n_items; ++iter) {
    if (threadIdx.x == 0) s_next[(iter + 2) % 3] = pull_item(ws.hdr + kWorkGateUp);
    const int next = s_next[(iter + 1) % 3];
    // the next item's tiles: its expert read now, long before they load
    const int64_t nbase = item_base(next);
    const int q = it / chunks, c = it - q * chunks;  // one pass of <= kTokensPerPass tokens
    const int start = __ldcg(ws.pass_start + q), mc = __ldcg(ws.pass_count + q);
    if (q != staged) {
      for (int i = threadIdx.x; i < mc * (K / 4); i += kThreads) {  // 16-byte pieces, K/8 per plane
        const int v = i / (K / 4), j = i - v * (K / 4), plane = j / (K / 8), piece = j - plane * (K / 8);
        const int tok = __ldcg(ws.pairs + start + v) / top_k;
        cp_async16(xs + v * token_stride(K) + plane * plane_stride(K) + 16 * piece,
                   ws.xenc + static_cast<int64_t>(tok) * 4 * K + plane * 2 * K + 16 * piece);
      }
      cp_async_commit();
      if (threadIdx.x < mc) {
        const int pair = __ldcg(ws.pairs + start + threadIdx.x);
        spair[threadIdx.x] = pair;
        xsc[threadIdx.x] = __ldcg(ws.xscale + pair / top_k);
      }
      cp_async_wait_all();
      __syncthreads();
      staged = q;
    }
    float acc[2][2] = {};
#pragma unroll 1
    for (int kb = kb0; kb < kb0 + KPW; ++kb) {
      // the tiles to load meanwhile: the next K-block's, or at the last one
      // the next item's first
      const int64_t off = kb + 1 < kb0 + KPW ? base + (kb + 1) * kChunkBytes
                          : nbase >= 0         ? nbase + kb0 * kChunkBytes
                                               : -1;
      block_steps(tg, tu, off >= 0 ? gate + off : nullptr, off >= 0 ? up + off : nullptr, lane, xl, kb, acc);
    }
    if constexpr (KS == 1) {
      // lane (g, t): gate and up rows g, g+8 of this warp's tile pair, token t
      if (t < mc) {
        const float sc = xsc[t];
        float* dst = ws.act + static_cast<int64_t>(spair[t]) * ffn + c * OUT + warp * 16 + g;
        dst[0] = silu_f(acc[0][0] * sc) * (acc[1][0] * sc);
        dst[8] = silu_f(acc[0][1] * sc) * (acc[1][1] * sc);
      }
    } else {
      float* rb = red + (npass++ & 1) * kRedFloats;
      reinterpret_cast<float4*>(rb)[warp * 32 + lane] = make_float4(acc[0][0], acc[0][1], acc[1][0], acc[1][1]);
      __syncthreads();
      for (int i = threadIdx.x; i < OUT * mc; i += kThreads) {
        const int v = i / OUT, o = i - v * OUT;
        const int otp = o >> 4, r = o & 15, src = (r & 7) * 4 + v, reg = r >> 3;
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          const float* rr = rb + ((k * TP + otp) * 32 + src) * 4;
          gs += rr[reg];
          us += rr[2 + reg];
        }
        gs *= xsc[v];
        us *= xsc[v];
        ws.act[static_cast<int64_t>(spair[v]) * ffn + c * OUT + o] = silu_f(gs) * us;
      }
    }
    __syncthreads();  // every warp is done with this item's planes and sums (a restaging follows)
    it = next;
    base = nbase;
  }
}

template <int KB, int NG>
__global__ void __launch_bounds__(kThreads, 2)
    moe_down_pulled_kernel(const uint8_t* __restrict__ down, int top_k, int hidden, MoeWs ws, MoeShared sh,
                           int sd_blocks, int t_total) {
  constexpr int K = KB * 256, ROWS = 32 * kWarps;
  extern __shared__ __align__(16) uint8_t smem[];
  float* xsc = reinterpret_cast<float*>(smem + kRedBytes);
  float* wmax = xsc + 16;
  int* spair = reinterpret_cast<int*>(xsc) + kMiscPair;
  uint8_t* xs = smem + kRedBytes + kMiscBytes;
  __shared__ int s_next[3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (static_cast<int>(blockIdx.x) < sd_blocks) {  // the shared expert's down rows
    shared_down_block(blockIdx.x, sh, t_total, hidden, ws);
    return;
  }
  pdl_launch_dependents();
  pdl_wait();
  const int chunks = hidden / ROWS;
  const int n_items = __ldcg(ws.hdr + kPassCount) * chunks;
  const uint8_t* xl = xs + (g >> 1) * token_stride(K) + (g & 1) * plane_stride(K) + 16 * t;
  // offset of K-block 0 of this warp's first tile in item `item` (-1: none);
  // the second tile follows KB chunks later
  auto item_base = [&](int item) -> int64_t {
    if (item >= n_items) return -1;
    const int q = item / chunks, c = item - q * chunks;
    const int e = __ldcg(ws.pass_expert + q);
    return (static_cast<int64_t>(e) * (hidden / 16) + c * 2 * kWarps + 2 * warp) * KB * kChunkBytes;
  };
  constexpr int64_t kHalf = static_cast<int64_t>(KB) * kChunkBytes;
  if (threadIdx.x == 0) {
    s_next[0] = pull_item(ws.hdr + kWorkDown);
    s_next[1] = pull_item(ws.hdr + kWorkDown);
  }
  __syncthreads();
  int it = s_next[0];
  Tile ta{}, tb{};
  int64_t base = item_base(it);
  if (base >= 0) {
    load_tile(down + base, lane, ta);
    load_tile(down + base + kHalf, lane, tb);
  }
  int staged = -1;
  for (int iter = 0; it < n_items; ++iter) {
    if (threadIdx.x == 0) s_next[(iter + 2) % 3] = pull_item(ws.hdr + kWorkDown);
    const int next = s_next[(iter + 1) % 3];
    const int64_t nbase = item_base(next);  // read now, long before the next item's tiles load
    const int q = it / chunks, c = it - q * chunks;  // one pass of <= kTokensPerPass tokens
    const int start = __ldcg(ws.pass_start + q), mc = __ldcg(ws.pass_count + q);
    if (q != staged) {
      // act of pair slot v = 4 s + i of group s: threads [64 i, 64 i + 64)
      // (warps 2i, 2i+1) -> fp16 planes; the groups' block maxima alternate
      // between two buffers, so one barrier per group suffices
      const int ng = NG == 1 ? 1 : (mc + kTokensPerPass - 1) / kTokensPerPass;
#pragma unroll 1
      for (int s = 0; s < ng; ++s) {
        const int v = kTokensPerPass * s + (threadIdx.x >> 6), j = threadIdx.x & 63;
        float* wm = wmax + 8 * (s & 1);
        constexpr int F4 = K / 4 / 64;  // float4 per thread
        float4 h[F4];
        float m = 0.f;
        const float4* src = nullptr;
        const int pair = v < mc ? __ldcg(ws.pairs + start + v) : 0;
        if (v < mc) src = reinterpret_cast<const float4*>(ws.act + static_cast<int64_t>(pair) * K);
#pragma unroll
        for (int i = 0; i < F4; ++i) {
          h[i] = v < mc ? __ldcg(src + j + 64 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
          m = fmaxf(m, fmaxf(fmaxf(fabsf(h[i].x), fabsf(h[i].y)), fmaxf(fabsf(h[i].z), fabsf(h[i].w))));
        }
        m = warp_max(m);
        if (lane == 0) wm[warp] = m;  // (this buffer's last readers passed a later barrier)
        __syncthreads();
        const int w2 = 2 * (threadIdx.x >> 6);
        m = fmaxf(wm[w2], wm[w2 + 1]);
        float inv, sx;
        vector_scale(m, inv, sx);
        if (v < mc) {
          uint8_t* dst = xs + v * token_stride(K);
#pragma unroll
          for (int i = 0; i < F4; ++i)
            store_planes(h[i], inv, dst + 8 * (j + 64 * i), dst + plane_stride(K) + 8 * (j + 64 * i));
          if (j == 0) {
            xsc[v] = sx;
            spair[v] = pair;
          }
        }
      }
      __syncthreads();
      staged = q;
    }
    if constexpr (NG > 1) {
      const int ng = (mc + kTokensPerPass - 1) / kTokensPerPass;
      float acc[NG][2][2] = {};
#pragma unroll 1
      for (int kb = 0; kb < KB; ++kb) {
        const int64_t off = kb + 1 < KB ? base + (kb + 1) * kChunkBytes : nbase;
        const uint8_t* na = off >= 0 ? down + off : nullptr;
        const uint8_t* nb = off >= 0 ? down + off + kHalf : nullptr;
        block_steps_wide<NG>(ta, tb, na, nb, lane, xl, kTokensPerPass * token_stride(K), kb, ng, acc);
      }
#pragma unroll
      for (int s = 0; s < NG; ++s) {  // lane (g, t): token 4 s + t of the pass
        const int v = kTokensPerPass * s + t;
        if (s < ng && v < mc) {
          const float sc = xsc[v];
          float* dst = ws.dn + static_cast<int64_t>(spair[v]) * hidden + c * ROWS + warp * 32 + g;
          dst[0] = acc[s][0][0] * sc;
          dst[8] = acc[s][0][1] * sc;
          dst[16] = acc[s][1][0] * sc;
          dst[24] = acc[s][1][1] * sc;
        }
      }
      __syncthreads();  // every warp is done with this item's planes
      it = next;
      base = nbase;
      continue;
    }
    float acc[2][2] = {};
#pragma unroll 1
    for (int kb = 0; kb < KB; ++kb) {
      // the tiles to load meanwhile: the next K-block's, or at the last one
      // the next item's first
      const int64_t off = kb + 1 < KB ? base + (kb + 1) * kChunkBytes : nbase;
      const uint8_t* na = off >= 0 ? down + off : nullptr;
      const uint8_t* nb = off >= 0 ? down + off + kHalf : nullptr;
      block_steps(ta, tb, na, nb, lane, xl, kb, acc);
    }
    // lane (g, t): rows g, g+8 of the warp's tiles 2w (acc[0]) and 2w+1 (acc[1]), token t
    if (t < mc) {
      const float sc = xsc[t];
      float* dst = ws.dn + static_cast<int64_t>(spair[t]) * hidden + c * ROWS + warp * 32 + g;
      dst[0] = acc[0][0] * sc;
      dst[8] = acc[0][1] * sc;
      dst[16] = acc[1][0] * sc;
      dst[24] = acc[1][1] * sc;
    }
    __syncthreads();  // every warp is done with this item's planes
    it = next;
    base = nbase;
  }
}

// ------------------------------------------------- wide gate/up, 16 warps
// Gate/up over wide passes with one warp per 16-row tile: warp w decodes tile
// w % 8 of the item's 128 gate rows (w < 8) or up rows (w >= 8) over the full
// K, each code word once for the pass's <= 16 tokens, and the up warps hand
// their sums to the gate warps through shared memory.  Half the registers of
// a tile pair per warp, so 16 warps share the SM (one CTA per SM: the planes
// of 16 tokens take 8 KB each at hidden 2048).  The shared expert's blocks
// run in their own launch ahead of it.
constexpr int kWideThreads = 512;

// block_steps_wide for one tile.
template <int NG>
__device__ __forceinline__ void block_steps_one(Tile& ta, const uint8_t* na, int lane, const uint8_t* xl, int gstride,
                                                int kb, int ng, float (&acc)[NG][2]) {
  const int g = lane >> 2, tq = lane & 3, q0 = lane & ~3;
  float s0[2], s1[2];
  {
    const float d0 = half_lo(ta.ra.y), d1 = half_lo(ta.rb.y);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      s0[h] = sub_scale(ta.ra.x, 2 * tq + h, d0, -8388608.0f * d0);
      s1[h] = sub_scale(ta.rb.x, 2 * tq + h, d1, -8388608.0f * d1);
    }
  }
  if (na) {
    ta.ra = __ldg(reinterpret_cast<const uint2*>(na + kScales) + g);
    ta.rb = __ldg(reinterpret_cast<const uint2*>(na + kScales) + g + 8);
  }
  const uint8_t* xq = xl + kb * 512;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint4& pa = ta.part[p];
    const int src = q0 | p;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t da[8];
      decode_word(h ? pa.z : pa.x, da[0], da[1], da[2], da[3]);
      decode_word(h ? pa.w : pa.y, da[4], da[5], da[6], da[7]);
      const float sa0 = __shfl_sync(0xffffffffu, s0[h], src), sa1 = __shfl_sync(0xffffffffu, s1[h], src);
#pragma unroll
      for (int s = 0; s < NG; ++s)
        if (s < ng) mma_sub(da, sa0, sa1, *reinterpret_cast<const uint4*>(xq + s * gstride + 128 * p + 64 * h), acc[s]);
    }
    if (na) ta.part[p] = ld_stream16(na + kCodes + 512 * p + 16 * lane);
  }
}

template <int KB>
__global__ void __launch_bounds__(kWideThreads, 1)
    moe_gate_up_wide_kernel(const uint8_t* __restrict__ gate, const uint8_t* __restrict__ up, int top_k, int ffn,
                            MoeWs ws) {
  constexpr int K = KB * 256, NG = kWideGroups, OUT = 16 * kWarps;
  extern __shared__ __align__(16) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem);  // [tile][lane][NG][2]: the up warps' sums
  float* xsc = reinterpret_cast<float*>(smem + kRedBytes);
  int* spair = reinterpret_cast<int*>(xsc) + kMiscPair;
  uint8_t* xs = smem + kRedBytes + kMiscBytes;
  static_assert(kWarps * 32 * NG * 2 * 4 <= kRedBytes, "up sums");
  __shared__ int s_next[3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile = warp % kWarps;
  const bool is_up = warp >= kWarps;
  const uint8_t* wm = is_up ? up : gate;
  pdl_wait();
  pdl_launch_dependents();
  const int chunks = ffn / OUT;
  const int n_items = __ldcg(ws.hdr + kPassCount) * chunks;
  const uint8_t* xl = xs + (g >> 1) * token_stride(K) + (g & 1) * plane_stride(K) + 16 * t;
  // offset of K-block 0 of this warp's tile in item `item` (-1: none)
  auto item_base = [&](int item) -> int64_t {
    if (item >= n_items) return -1;
    const int q = item / chunks, c = item - q * chunks;
    const int e = __ldcg(ws.pass_expert + q);
    return (static_cast<int64_t>(e) * (ffn / 16) + c * kWarps + tile) * KB * kChunkBytes;
  };
  if (threadIdx.x == 0) {
    s_next[0] = pull_item(ws.hdr + kWorkGateUp);
    s_next[1] = pull_item(ws.hdr + kWorkGateUp);
  }
  __syncthreads();
  int it = s_next[0];
  Tile tw{};
  int64_t base = item_base(it);
  if (base >= 0) load_tile(wm + base, lane, tw);
  int staged = -1;
  for (int iter = 0; it < n_items; ++iter) {
    if (threadIdx.x == 0) s_next[(iter + 2) % 3] = pull_item(ws.hdr + kWorkGateUp);
    const int next = s_next[(iter + 1) % 3];
    const int64_t nbase = item_base(next);  // read now, long before the next item's tiles load
    const int q = it / chunks, c = it - q * chunks;
    const int start = __ldcg(ws.pass_start + q), mc = __ldcg(ws.pass_count + q);
    if (q != staged) {
      for (int i = threadIdx.x; i < mc * (K / 4); i += kWideThreads) {  // 16-byte pieces, K/8 per plane
        const int v = i / (K / 4), j = i - v * (K / 4), plane = j / (K / 8), piece = j - plane * (K / 8);
        const int tok = __ldcg(ws.pairs + start + v) / top_k;
        cp_async16(xs + v * token_stride(K) + plane * plane_stride(K) + 16 * piece,
                   ws.xenc + static_cast<int64_t>(tok) * 4 * K + plane * 2 * K + 16 * piece);
      }
      cp_async_commit();
      if (threadIdx.x < mc) {
        const int pair = __ldcg(ws.pairs + start + threadIdx.x);
        spair[threadIdx.x] = pair;
        xsc[threadIdx.x] = __ldcg(ws.xscale + pair / top_k);
      }
      cp_async_wait_all();
      __syncthreads();
      staged = q;
    }
    const int ng = (mc + kTokensPerPass - 1) / kTokensPerPass;
    float acc[NG][2] = {};
#pragma unroll 1
    for (int kb = 0; kb < KB; ++kb) {
      // the next K-block's tile, or at the last one the next item's first
      const int64_t off = kb + 1 < KB ? base + (kb + 1) * kChunkBytes : nbase;
      block_steps_one<NG>(tw, off >= 0 ? wm + off : nullptr, lane, xl, kTokensPerPass * token_stride(K), kb, ng, acc);
    }
    float* ru = red + (tile * 32 + lane) * (NG * 2);
    if (is_up) {
#pragma unroll
      for (int s = 0; s < NG; ++s) {
        ru[2 * s] = acc[s][0];
        ru[2 * s + 1] = acc[s][1];
      }
    }
    __syncthreads();  // the up sums are in shared memory
    if (!is_up) {
#pragma unroll
      for (int s = 0; s < NG; ++s) {  // lane (g, t): rows g, g+8 of this tile, token 4 s + t of the pass
        const int v = kTokensPerPass * s + t;
        if (s < ng && v < mc) {
          const float sc = xsc[v];
          float* dst = ws.act + static_cast<int64_t>(spair[v]) * ffn + c * OUT + tile * 16 + g;
          dst[0] = silu_f(acc[s][0] * sc) * (ru[2 * s] * sc);
          dst[8] = silu_f(acc[s][1] * sc) * (ru[2 * s + 1] * sc);
        }
      }
    }
    __syncthreads();  // every warp is done with this item's planes and sums
    it = next;
    base = nbase;
  }
}

// The shared expert's gate/up blocks alone (ahead of moe_gate_up_wide_kernel).
__global__ void __launch_bounds__(kThreads) moe_shared_gu_kernel(MoeShared sh, const float* __restrict__ x,
                                                                 int t_total, int hidden, MoeWs ws) {
  pdl_launch_dependents();
  shared_gu_block(blockIdx.x, sh, x, t_total, hidden, ws);
}

// ------------------------------------------------------------------ combine
// out[t] = sum_k w[t, k] * down_k(act) in routing order, each product rounded
// before the add like the reference's (out * w).sum(0) in f32.
__global__ void moe_combine_kernel(const float* __restrict__ weights, const int32_t* __restrict__ ids, int64_t t,
                                   int top_k, int hidden, int n_experts, MoeWs ws, int shared,
                                   float* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = t * hidden;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i / hidden;
    const int hh = static_cast<int>(i % hidden);
    float acc = routed_sum(ids + tok * top_k, weights + tok * top_k, ws.dn + tok * top_k * hidden + hh, hidden,
                           top_k, n_experts);
    if (shared) acc = __fadd_rn(acc, __fmul_rn(ws.sgate[tok], ws.sout[i]));  // routed + gate * shared
    out[i] = acc;
  }
}

// moe_combine_kernel's sums for 8 consecutive outputs (dn: element i0 of the
// token's first pair row), each in routing order with the same roundings,
// the rows read with 16-byte loads.  Eight pairs' rows are loaded at once and
// without waiting for their ids (every pair has a workspace row; the rows of
// invalid ids are read but not added), so a token costs one round trip.
__device__ __forceinline__ void routed_sum8(const int32_t* ids, const float* w, const float* dn, int64_t stride,
                                            int top_k, int n_experts, float (&a)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = 0.f;
  for (int k0 = 0; k0 < top_k; k0 += 8) {
    float4 v[8][2];
    float wk[8];
    int e[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j;
      e[j] = k < top_k ? ids[k] : -1;
      wk[j] = k < top_k ? w[k] : 0.f;
      const float4* row = reinterpret_cast<const float4*>(dn + static_cast<int64_t>(min(k, top_k - 1)) * stride);
      v[j][0] = __ldcg(row);
      v[j][1] = __ldcg(row + 1);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (e[j] < 0 || e[j] >= n_experts) continue;
      const float vv[8] = {v[j][0].x, v[j][0].y, v[j][0].z, v[j][0].w, v[j][1].x, v[j][1].y, v[j][1].z, v[j][1].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = __fadd_rn(a[i], __fmul_rn(vv[i], wk[j]));
    }
  }
}

// The combine of moe_combine_kernel followed by the decoder's residual add +
// RMSNorm + planes (add_rms_norm_planes_row, the same bits as the separate
// kernels), one 256-thread block per token: the layer's output never goes
// through memory.  hidden <= 2048.
__global__ void __launch_bounds__(kThreads) moe_combine_norm_kernel(const float* __restrict__ weights,
                                                                    const int32_t* __restrict__ ids, int top_k,
                                                                    int hidden, int n_experts, MoeWs ws, int shared,
                                                                    MoeNorm nm) {
  __shared__ float scratch[8];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t tok = blockIdx.x;
  const int32_t* id = ids + tok * top_k;
  const float* wt = weights + tok * top_k;
  const float* dn = ws.dn + tok * top_k * hidden;
  const float sg = shared ? __ldcg(ws.sgate + tok) : 0.f;
  auto b_of = [&](int i0, float (&bb)[8]) {
    routed_sum8(id, wt, dn + i0, hidden, top_k, n_experts, bb);
    if (shared) {
      const float4 s0 = __ldcg(reinterpret_cast<const float4*>(ws.sout + tok * hidden + i0));
      const float4 s1 = __ldcg(reinterpret_cast<const float4*>(ws.sout + tok * hidden + i0) + 1);
      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) bb[j] = __fadd_rn(bb[j], __fmul_rn(sg, sv[j]));  // routed + gate * shared
    }
  };
  add_rms_norm_planes_row(nm.h + tok * hidden, true, b_of, nm.w, nm.h_out + tok * hidden, nm.y + tok * hidden,
                          static_cast<__nv_bfloat16*>(nm.planes) + tok * 3 * hidden, hidden, nm.eps, scratch);
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl_n(Kern kern, dim3 grid, int threads, size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return ::bt::launch_ex(&cfg, kern, args...);
}
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, size_t smem, cudaStream_t stream, Args... args) {
  return launch_pdl_n(kern, grid, kThreads, smem, stream, args...);
}

// Launch geometry of a layer call: the expert kernels' persistent grids and
// item sizes, shared by the layer and bt_moe_route_sort_iq3s.  `chain`: the
// shared expert's gate/up blocks ride ahead of the routed gate/up CTAs and
// its down blocks ahead of the routed down CTAs (kPrepNone, T > 1);
// otherwise its down blocks ride ahead of the routed gate/up CTAs.  Static
// grids leave those blocks their slots, so that every routed CTA starts in
// the first wave.
struct Geometry {
  // pulled: 0 static items, 1 pulled passes, kPulledWide pulled wide passes
  int direct, pulled, gu_grid, gu_chunks, d_grid, d_chunks, sgu_blocks, sd_blocks;
  size_t prep_smem;
};
template <int KBG, int KBD>
Geometry geometry(int64_t t, int hidden, int ffn, int n_experts, int top_k, int64_t shared_ffn, bool chain) {
  constexpr int kGuOut = 16 * (kWarps / KBG), kDnRows = 32 * (kWarps / KBD);
  Geometry g;
  g.direct = t == 1 ? 1 : 0;  // one token selects top_k distinct experts: no grouping needed
  g.pulled = t <= kStaticMaxTokens                                   ? 0
             : t * top_k >= static_cast<int64_t>(kWideMinPairs) * n_experts ? kPulledWide
                                                                            : 1;
  const int passes = shared_ffn > 0 ? shared_passes(t) : 0;
  g.sgu_blocks = shared_ffn > 0 ? (static_cast<int>(shared_ffn) / 16 + 1) * passes : 0;
  g.sd_blocks = shared_ffn > 0 ? hidden / 64 * passes : 0;
  // persistent grids: two CTAs per SM, or one per item when there are fewer
  const int slots_max = std::min(2 * sm_count(), kMaxGrid);
  const bool in_chain = chain && !g.direct;
  const int gu_extra = in_chain ? g.sgu_blocks : g.sd_blocks, d_extra = in_chain ? g.sd_blocks : 0;
  g.gu_chunks = ffn / kGuOut;
  g.d_chunks = hidden / kDnRows;
  g.gu_grid = g.direct                   ? std::min(top_k * g.gu_chunks, slots_max)
              : g.pulled == kPulledWide ? std::min(sm_count(), kMaxGrid)  // one CTA per SM
              : g.pulled                ? slots_max
                                        : std::max(1, slots_max - gu_extra);
  g.d_grid = g.direct   ? std::min(top_k * g.d_chunks, slots_max)
             : g.pulled ? slots_max
                        : std::max(1, slots_max - d_extra);
  g.prep_smem = g.direct ? 0 : (3 * n_experts + 1 + static_cast<size_t>(t * top_k)) * sizeof(int32_t);
  return g;
}

template <int KBG, int KBD>
int launch_all(const uint8_t* gate, const uint8_t* up, const uint8_t* down, const MoeShared* sh, const float* x,
               int64_t t, int hidden, int ffn, int n_experts, const int32_t* ids, const float* weights, int top_k,
               float* out, MoeWs ws, cudaStream_t stream, const MoeNorm* norm, int prep_part) {
  const int shared = sh ? 1 : 0;
  const int p = static_cast<int>(t * top_k);
  // one token selects top_k distinct experts: no grouping needed
  const int direct = t == 1 ? 1 : 0;
  constexpr int kGuOut = 16 * (kWarps / KBG), kDnRows = 32 * (kWarps / KBD);
  static_assert(kWarps % KBG == 0 && kWarps % KBD == 0, "K blocks per item");
  constexpr size_t gu_smem = kRedBytes + kMiscBytes + kTokensPerPass * token_stride(KBG * 256);
  constexpr size_t d_smem = kRedBytes + kMiscBytes + kTokensPerPass * token_stride(KBD * 256);
  constexpr size_t gu_smem_w = kRedBytes + kMiscBytes + kWideTokensPerPass * token_stride(KBG * 256);
  constexpr size_t d_smem_w = kRedBytes + kMiscBytes + kWideTokensPerPass * token_stride(KBD * 256);
  static_assert(gu_smem_w <= 227 * 1024 && d_smem_w <= 227 * 1024, "wide pass planes");
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(moe_gate_up_kernel<KBG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(gu_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_down_kernel<KBD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(d_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_gate_up_pulled_kernel<KBG, kGuSplits>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(gu_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_down_pulled_kernel<KBD, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(d_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_gate_up_wide_kernel<KBG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(gu_smem_w));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(moe_down_pulled_kernel<KBD, kWideGroups>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(d_smem_w));
    if (e != cudaSuccess) return fail_cuda(e, "moe set smem");
    configured_device = dev;
  }
  const Geometry geo = geometry<KBG, KBD>(t, hidden, ffn, n_experts, top_k, sh ? sh->ffn : 0, prep_part == kPrepNone);
  const int gu_chunks = geo.gu_chunks, d_chunks = geo.d_chunks, gu_grid = geo.gu_grid, d_grid = geo.d_grid;
  const size_t prep_smem = geo.prep_smem;
  static_assert(kGuOut > 0 && kDnRows > 0, "item rows");
  if (prep_smem > 48 * 1024) return fail(BT_ERR_UNSUPPORTED, "moe_experts_iq3s: too many experts + pairs");
  // the shared expert rides along: its gate/up blocks after the prep
  // kernel's, its down blocks ahead of the routed gate/up CTAs
  const MoeShared shv = sh ? *sh : MoeShared{};
  const int sgu_blocks = geo.sgu_blocks, sd_blocks = geo.sd_blocks;
  const int prep_blocks = (direct ? 1 : 1 + static_cast<int>(t)) + sgu_blocks;
  const int pulled = geo.pulled;
  // kPrepNone (after moe_route_sort_iq3s routed, sorted and encoded), T > 1:
  // no prep launch; the shared expert's gate/up blocks run ahead of the
  // routed gate/up CTAs and its down blocks ahead of the routed down CTAs,
  // so the whole layer is one chain of early-launched kernels.  Otherwise
  // (and for one token, whose down kernel adds the shared output in place)
  // the prep kernel encodes and runs the shared gate/up (kPrepX: without the
  // sort, which moe_route_sort_iq3s did), and the shared down blocks run
  // ahead of the routed gate/up CTAs.
  const bool chain = prep_part == kPrepNone && !direct;
  const int part = prep_part == kPrepNone ? kPrepX : prep_part;
  const int gu_sd = chain ? 0 : sd_blocks, gu_sgu = chain ? sgu_blocks : 0, dn_sd = chain ? sd_blocks : 0;
  cudaError_t e = cudaSuccess;
  if (!chain)
    e = launch_pdl(moe_prep_kernel, dim3(part == kPrepX ? prep_blocks - (direct ? 0 : 1) : prep_blocks),
                   part == kPrepX ? 0 : prep_smem, stream, ids, p, n_experts, direct, x, static_cast<int>(t), hidden,
                   ws, gu_grid, gu_chunks, d_grid, d_chunks, shv, pulled, part);
  // up to kStaticMaxTokens tokens: static item ranges of K-split items (one
  // token: the last of a row chunk's CTAs combines); more: whole-pass items
  // pulled from a counter, then the combine kernel
  if (!pulled) {
    if (e == cudaSuccess)
      e = launch_pdl(moe_gate_up_kernel<KBG>, dim3(gu_sd + gu_sgu + gu_grid), gu_smem, stream, gate, up, ids,
                     n_experts, direct, top_k, ffn, ws, gu_grid, shv, gu_sd, static_cast<int>(t), hidden, x, gu_sgu);
    if (e == cudaSuccess)
      e = launch_pdl(moe_down_kernel<KBD>, dim3(dn_sd + d_grid), d_smem, stream, down, ids, weights, out, n_experts,
                     direct, top_k, hidden, ws, shared, shv, dn_sd, static_cast<int>(t));
  } else if (pulled != kPulledWide) {
    if (e == cudaSuccess)
      e = launch_pdl(moe_gate_up_pulled_kernel<KBG, kGuSplits>, dim3(gu_sd + gu_sgu + gu_grid), gu_smem, stream,
                     gate, up, top_k, ffn, ws, shv, gu_sd, static_cast<int>(t), hidden, x, gu_sgu);
    if (e == cudaSuccess)
      e = launch_pdl(moe_down_pulled_kernel<KBD, 1>, dim3(dn_sd + d_grid), d_smem, stream, down, top_k, hidden, ws,
                     shv, dn_sd, static_cast<int>(t));
  } else {
    // prefill-sized batches: wide passes, each decoded tile shared by up to
    // 16 tokens; the shared expert's gate/up blocks (when the prep kernel
    // did not run them) in a launch of their own, its down blocks ahead of
    // the routed down CTAs
    if (e == cudaSuccess && gu_sgu)
      e = launch_pdl(moe_shared_gu_kernel, dim3(gu_sgu), 0, stream, shv, x, static_cast<int>(t), hidden, ws);
    if (e == cudaSuccess)
      e = launch_pdl_n(moe_gate_up_wide_kernel<KBG>, dim3(gu_grid), kWideThreads, gu_smem_w, stream, gate, up, top_k,
                       ffn, ws);
    if (e == cudaSuccess)
      e = launch_pdl(moe_down_pulled_kernel<KBD, kWideGroups>, dim3(sd_blocks + d_grid), d_smem_w, stream, down,
                     top_k, hidden, ws, shv, sd_blocks, static_cast<int>(t));
  }
  const int64_t total = t * hidden;
  const int blocks = static_cast<int>(std::min<int64_t>((total + kThreads - 1) / kThreads, 4096));
  const bool fused = norm && !direct && hidden <= 8 * kThreads;
  if (e == cudaSuccess && fused)
    e = launch_pdl(moe_combine_norm_kernel, dim3(static_cast<unsigned>(t)), 0, stream, weights, ids, top_k, hidden,
                   n_experts, ws, shared, *norm);
  else if (e == cudaSuccess && !direct)
    e = launch_pdl(moe_combine_kernel, dim3(blocks), 0, stream, weights, ids, t, top_k, hidden, n_experts, ws, shared,
                   out);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "moe experts launch");
  if (norm && !fused)
    return add_rms_norm_planes(norm->h, out, norm->w, norm->h_out, norm->y, norm->planes, t, hidden, norm->eps,
                               stream);
  return BT_OK;
}

template <int KBG, int KBD>
int route_sort_launch(const float* logits, const float* x, int64_t t, int hidden, int ffn, int n_experts, int top_k,
                      int64_t shared_ffn, int32_t* ids, float* weights, MoeWs ws, cudaStream_t stream) {
  const Geometry geo = geometry<KBG, KBD>(t, hidden, ffn, n_experts, top_k, shared_ffn, true);
  if (geo.prep_smem > 48 * 1024) return fail(BT_ERR_UNSUPPORTED, "moe route + sort: too many experts + pairs");
  const int n_route = static_cast<int>((t + kWarps - 1) / kWarps);
  const dim3 grid(static_cast<unsigned>(n_route + (geo.direct ? 0 : t)));  // one token: the layer encodes
  cudaError_t e;
  if (n_experts <= 64)
    e = launch_pdl(moe_route_sort_kernel<2>, grid, geo.prep_smem, stream, logits, t, n_experts, top_k, ids, weights, ws,
                   geo.gu_grid, geo.gu_chunks, geo.d_grid, geo.d_chunks, geo.pulled, x, hidden, n_route);
  else if (n_experts <= 256)
    e = launch_pdl(moe_route_sort_kernel<8>, grid, geo.prep_smem, stream, logits, t, n_experts, top_k, ids, weights,
                   ws, geo.gu_grid, geo.gu_chunks, geo.d_grid, geo.d_chunks, geo.pulled, x, hidden, n_route);
  else
    e = launch_pdl(moe_route_sort_kernel<32>, grid, geo.prep_smem, stream, logits, t, n_experts, top_k, ids, weights,
                   ws, geo.gu_grid, geo.gu_chunks, geo.d_grid, geo.d_chunks, geo.pulled, x, hidden, n_route);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? BT_OK : fail_cuda(e, "moe route + sort launch");
}

}  // namespace

int repack_iq3_s(const void* src, void* dst, int64_t rows, int64_t k, cudaStream_t stream) {
  if (!src || !dst || rows < 0 || k <= 0 || k % 256)
    return fail(BT_ERR_INVALID, "repack_iq3_s: K must be a multiple of 256");
  if (rows % 16) return fail(BT_ERR_INVALID, "repack_iq3_s: rows must be a multiple of 16 (tiles of 16 rows)");
  if (reinterpret_cast<uintptr_t>(dst) & 15) return fail(BT_ERR_INVALID, "repack_iq3_s: dst must be 16-byte aligned");
  const int64_t chunks = rows / 16 * (k / 256);
  if (chunks == 0) return BT_OK;
  const int blocks = static_cast<int>(std::min<int64_t>((chunks * 32 + 255) / 256, 65535));
  ::bt::note_launch();
  repack_iq3s_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), chunks,
                                                 static_cast<int>(k / 256));
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
  const int ne = static_cast<int>(n_experts);
  cudaError_t e;
  if (ne <= 64)
    e = launch_pdl(moe_route_kernel<2>, dim3(blocks), 0, stream, logits, t, ne, top_k, ids, weights);
  else if (ne <= 256)
    e = launch_pdl(moe_route_kernel<8>, dim3(blocks), 0, stream, logits, t, ne, top_k, ids, weights);
  else
    e = launch_pdl(moe_route_kernel<32>, dim3(blocks), 0, stream, logits, t, ne, top_k, ids, weights);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "moe_route launch");
  return BT_OK;
}

int64_t moe_workspace_bytes(int64_t t, int64_t hidden, int64_t ffn, int64_t shared_ffn, int64_t n_experts, int top_k) {
  (void)n_experts;
  if (t < 1 || top_k < 1 || shared_ffn < 0) return 0;
  return moe_ws_bytes(t, t * top_k, hidden, ffn, shared_ffn);
}

int moe_route_sort_iq3s(const float* logits, const float* x, int64_t t, int64_t hidden, int64_t ffn,
                        int64_t n_experts, int top_k, int64_t shared_ffn, int32_t* ids, float* weights,
                        void* workspace, cudaStream_t stream) {
  if (!logits || !x || !ids || !weights || !workspace) return fail(BT_ERR_INVALID, "moe route + sort: null pointer");
  if (t < 1 || t * top_k > 4096 || top_k < 1 || top_k > 16 || n_experts < 1 || n_experts > 1024 ||
      top_k > n_experts)
    return fail(BT_ERR_UNSUPPORTED, "moe route + sort serves T * top_k <= 4096 pairs, <= 1024 experts, top-k <= 16");
  if ((reinterpret_cast<uintptr_t>(workspace) | reinterpret_cast<uintptr_t>(x)) & 15 || hidden % 8)
    return fail(BT_ERR_INVALID, "moe route + sort: workspace and x must be 16-byte aligned, hidden a multiple of 8");
  if (shared_ffn < 0) return fail(BT_ERR_INVALID, "moe route + sort: negative shared ffn");
  const MoeWs ws = moe_ws(workspace, t, t * top_k, hidden, ffn, shared_ffn);
  const int h = static_cast<int>(hidden), f = static_cast<int>(ffn), ne = static_cast<int>(n_experts);
  if (hidden == 2048 && ffn == 512) return route_sort_launch<8, 2>(logits, x, t, h, f, ne, top_k, shared_ffn, ids, weights, ws, stream);
  if (hidden == 1024 && ffn == 512) return route_sort_launch<4, 2>(logits, x, t, h, f, ne, top_k, shared_ffn, ids, weights, ws, stream);
  if (hidden == 2048 && ffn == 1024) return route_sort_launch<8, 4>(logits, x, t, h, f, ne, top_k, shared_ffn, ids, weights, ws, stream);
  return fail(BT_ERR_UNSUPPORTED, "moe route + sort serves (hidden, ffn) in {(1024,512), (2048,512), (2048,1024)}");
}

int moe_layer_iq3s(const void* gate, const void* up, const void* down, const MoeShared* shared, const float* x,
                   int64_t t, int64_t hidden, int64_t ffn, int64_t n_experts, const int32_t* ids, const float* weights,
                   int top_k, float* out, void* workspace, cudaStream_t stream, const MoeNorm* norm, int prep_part) {
  if (!gate || !up || !down || !x || !ids || !weights || !out || !workspace)
    return fail(BT_ERR_INVALID, "moe_experts_iq3s: null pointer");
  if (norm && (!norm->h || !norm->w || !norm->h_out || !norm->y || !norm->planes || hidden % 8 ||
               ((reinterpret_cast<uintptr_t>(norm->h) | reinterpret_cast<uintptr_t>(norm->w) |
                 reinterpret_cast<uintptr_t>(norm->h_out) | reinterpret_cast<uintptr_t>(norm->y) |
                 reinterpret_cast<uintptr_t>(norm->planes) | reinterpret_cast<uintptr_t>(out)) & 15)))
    return fail(BT_ERR_INVALID, "moe layer + norm: null or misaligned norm buffers");
  if (t < 1 || t * top_k > 4096 || top_k < 1 || top_k > 64 || n_experts < 1 || n_experts > 4096)
    return fail(BT_ERR_UNSUPPORTED, "moe_experts_iq3s serves T * top_k <= 4096 pairs over <= 4096 experts");
  if ((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(down) |
       reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(workspace)) & 15)
    return fail(BT_ERR_INVALID, "moe_experts_iq3s: weights, x and workspace must be 16-byte aligned");
  if (shared) {
    if (!shared->gate || !shared->up || !shared->down || !shared->gate_inp)
      return fail(BT_ERR_INVALID, "moe shared expert: null pointer");
    if (shared->ffn < 256 || shared->ffn % 256 || shared->ffn > 8192 || hidden % 1024)
      return fail(BT_ERR_UNSUPPORTED, "moe shared expert: ffn must be a multiple of 256 and hidden of 1024");
    if ((reinterpret_cast<uintptr_t>(shared->gate) | reinterpret_cast<uintptr_t>(shared->up) |
         reinterpret_cast<uintptr_t>(shared->down)) & 15)
      return fail(BT_ERR_INVALID, "moe shared expert: weights must be 16-byte aligned");
  }
  const MoeWs ws = moe_ws(workspace, t, t * top_k, hidden, ffn, shared ? shared->ffn : 0);
  const uint8_t* g = static_cast<const uint8_t*>(gate);
  const uint8_t* u = static_cast<const uint8_t*>(up);
  const uint8_t* d = static_cast<const uint8_t*>(down);
  const int h = static_cast<int>(hidden), f = static_cast<int>(ffn), ne = static_cast<int>(n_experts);
  const int k = top_k;
  if (hidden == 2048 && ffn == 512)
    return launch_all<8, 2>(g, u, d, shared, x, t, h, f, ne, ids, weights, k, out, ws, stream, norm, prep_part);
  if (hidden == 1024 && ffn == 512)
    return launch_all<4, 2>(g, u, d, shared, x, t, h, f, ne, ids, weights, k, out, ws, stream, norm, prep_part);
  if (hidden == 2048 && ffn == 1024)
    return launch_all<8, 4>(g, u, d, shared, x, t, h, f, ne, ids, weights, k, out, ws, stream, norm, prep_part);
  return fail(BT_ERR_UNSUPPORTED, "moe_experts_iq3s serves (hidden, ffn) in {(1024,512), (2048,512), (2048,1024)}");
}

}  // namespace bt
