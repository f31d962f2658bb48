// Dense projection of T tokens by bf16 or f32 weight rows on the tensor cores:
// y[t][n] = sum_k W[n][k] x[t][k], W (N, K) in the GGUF (out, in)
// orientation, y (T, N) f32 -- the reference's _linear / _linear_b of
// model/qwen36_moe.py:352-358 in its f32 form (weights exact in f32,
// activations f32).
//
// x enters as three bf16 planes (x = hi + mid + lo, each remainder exact in
// f32: 24 bits), split once by bf16_planes_kernel and shared by every
// projection of the same input.  One block per 16-row tile and NP passes of
// 8 tokens; its 8 warps split K, and every pass reuses the weight fragments
// a warp loaded.  Per 32-column step a lane loads weights 8t .. 8t+7 of rows
// g and g+8 (16-byte loads; the k order inside the step is permuted
// identically on both MMA operands) and the same columns of token column g's
// planes.  f32 weights are split into three bf16 planes in registers; the
// plane products that reach 2^-24 of the largest are summed (all 3 for bf16
// weights, 6 of 9 for f32), into one f32 sum per output (m16n8k16 bf16
// MMAs).  Before the dependency wait each warp bulk-prefetches its weight
// slices into L2: the weights never depend on earlier kernels.
//
// More than 8 tokens with bf16 weights (the batched decode of many
// sequences) run as a tiled product instead, where the x planes would
// otherwise be re-read from L2 by every 16-row block: a block owns 64 rows
// and up to 64 tokens, and stages 32-column slices of its weight rows and of
// all its tokens' planes through a 4-deep cp.async pipeline in shared
// memory (rows padded to 80 bytes, so ldmatrix reads are conflict-free);
// 8 warps = 2 row halves x 4 token quarters, MMA operands by ldmatrix.  K is
// split over the CTAs of a thread-block cluster (up to 8), whose partial
// sums meet through distributed shared memory and are added in split order
// (deterministic, no workspace).
//
// With N % 128 == 0 the tiled product runs on the 5th-generation tensor
// cores instead: a CTA owns 128 weight rows (the MMA's M, one TMEM lane per
// row) and up to 64 tokens, whose three planes are the MMA's N = 3 NT
// columns (token-major: column 3 t + plane).  One thread streams 64-column
// stages of both operands with TMA (one tensor copy per operand: rows of 128
// bytes in the 128-byte-swizzled K-major layout the MMA descriptors name;
// rows past T read as zeros), another issues tcgen05.mma
// (kind::f16, bf16 x bf16 -> f32 accumulators in TMEM) as stages arrive and
// releases each buffer with tcgen05.commit; full / empty mbarriers pace the
// two.  The epilogue reads TMEM (tcgen05.ld), adds the planes and joins the
// same split-order cluster reduction.  Every mbarrier wait gives up after
// kWaitLimitNs (counted in g_umma_timeouts, read by bt_linear_rows_timeouts).
#include <cooperative_groups.h>
#include <cuda.h>  // CUtensorMap (the encoder comes through the runtime's driver entry point)
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "errors.h"
#include "linear_rows.cuh"

namespace cg = cooperative_groups;

namespace bt {
namespace {

constexpr int kThreads = 256, kWarps = 8, kPass = 8;

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t bf16_pair(float a, float b) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(a)) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(b))) << 16);
}

// Eight f32 values as three bf16 planes (8 bf16 each): v = hi + mid + lo.
__device__ __forceinline__ void split8(const float (&v)[8], uint4 (&p)[3]) {
  float r1[8], r2[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    r1[i] = v[i] - __bfloat162float(__float2bfloat16_rn(v[i]));
    r2[i] = r1[i] - __bfloat162float(__float2bfloat16_rn(r1[i]));
  }
  p[0] = make_uint4(bf16_pair(v[0], v[1]), bf16_pair(v[2], v[3]), bf16_pair(v[4], v[5]), bf16_pair(v[6], v[7]));
  p[1] = make_uint4(bf16_pair(r1[0], r1[1]), bf16_pair(r1[2], r1[3]), bf16_pair(r1[4], r1[5]),
                    bf16_pair(r1[6], r1[7]));
  p[2] = make_uint4(bf16_pair(r2[0], r2[1]), bf16_pair(r2[2], r2[3]), bf16_pair(r2[4], r2[5]),
                    bf16_pair(r2[6], r2[7]));
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p + 4));
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

// c += (A planes of rows g, g+8) x (B planes): 32 columns.  bf16 weights:
// the weight times the three x planes; f32 weights: the six plane products
// with plane-index sum <= 2 (the others lie below 2^-24 of the largest).
template <int NA>
__device__ __forceinline__ void step(float (&c)[4], const uint4 (&ra)[NA], const uint4 (&rb)[NA], const uint4 (&b)[3]) {
#pragma unroll
  for (int i = 0; i < NA; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      if (i + j > 2) continue;
      mma_bf16(c, ra[i].x, rb[i].x, ra[i].y, rb[i].y, b[j].x, b[j].y);
      mma_bf16(c, ra[i].z, rb[i].z, ra[i].w, rb[i].w, b[j].z, b[j].w);
    }
}

// x (T, K) f32 -> planes (T, 3, K) bf16, 8 values per thread.
__global__ void bf16_planes_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ planes, int64_t t,
                                   int k) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t chunks = t * (k / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < chunks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i / (k / 8);
    const int col = static_cast<int>(i - tok * (k / 8)) * 8;
    float v[8];
    load8(x + tok * k + col, v);
    uint4 p[3];
    split8(v, p);
#pragma unroll
    for (int j = 0; j < 3; ++j) *reinterpret_cast<uint4*>(planes + (tok * 3 + j) * k + col) = p[j];
  }
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// KS > 1: the K range is split over the KS CTAs of a cluster (grid z); each
// CTA reduces its warps' sums, then cluster rank 0 adds the CTAs' sums in
// rank order through distributed shared memory (deterministic, no workspace).
template <bool F32W, int NP, int TW, int KS>
__global__ void __launch_bounds__(kThreads) linear_rows_kernel(const void* __restrict__ w,
                                                               const __nv_bfloat16* __restrict__ xp,
                                                               float* __restrict__ y, int n, int k, int t_total) {
  using Elem = typename std::conditional<F32W, float, __nv_bfloat16>::type;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile0 = blockIdx.x * TW, c0 = blockIdx.y * kPass * NP, span = k / (kWarps * KS);
  const int kbase = static_cast<int>(blockIdx.z % KS) * (k / KS);
  if (lane < 16)
#pragma unroll
    for (int j = 0; j < TW; ++j)
      prefetch_l2(static_cast<const Elem*>(w) + static_cast<int64_t>(16 * (tile0 + j) + lane) * k + kbase +
                      warp * span,
                  static_cast<uint32_t>(span * sizeof(Elem)));
  pdl_wait();  // the planes come from earlier kernels
  pdl_launch_dependents();
  const __nv_bfloat16* xr[NP];
  bool live[NP];
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int tok = c0 + kPass * p + g;
    live[p] = tok < t_total;
    xr[p] = xp + static_cast<int64_t>(live[p] ? tok : 0) * 3 * k;
  }
  float c[TW][NP][4] = {};
#pragma unroll(NP * TW < 4 ? 2 : 1)  // the passes of a step already give the loads to overlap
  for (int k0 = kbase + warp * span; k0 < kbase + (warp + 1) * span; k0 += 32) {
    const int col = k0 + 8 * t;
    constexpr int NA = F32W ? 3 : 1;
    uint4 ra[TW][NA], rb[TW][NA];
#pragma unroll
    for (int j = 0; j < TW; ++j) {
      const Elem* wr = static_cast<const Elem*>(w) + static_cast<int64_t>(16 * (tile0 + j) + g) * k;
      if constexpr (F32W) {
        float va[8], vb[8];
        load8(reinterpret_cast<const float*>(wr) + col, va);
        load8(reinterpret_cast<const float*>(wr) + 8 * static_cast<int64_t>(k) + col, vb);
        split8(va, ra[j]);
        split8(vb, rb[j]);
      } else {
        ra[j][0] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(wr) + col));
        rb[j][0] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(wr) +
                                                        8 * static_cast<int64_t>(k) + col));
      }
    }
#pragma unroll
    for (int p = 0; p < NP; ++p) {  // every pass reuses the weight fragments, every tile the x planes
      uint4 b[3];
#pragma unroll
      for (int q = 0; q < 3; ++q)
        b[q] = live[p] ? __ldcg(reinterpret_cast<const uint4*>(xr[p] + q * k + col)) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int j = 0; j < TW; ++j) step<NA>(c[j][p], ra[j], rb[j], b);
    }
  }
  __shared__ float4 red[kWarps][TW * NP][32];
#pragma unroll
  for (int j = 0; j < TW; ++j)
#pragma unroll
    for (int p = 0; p < NP; ++p)
      red[warp][j * NP + p][lane] = make_float4(c[j][p][0], c[j][p][1], c[j][p][2], c[j][p][3]);
  __syncthreads();
  constexpr int OUTS = TW * 16 * kPass * NP;
  __shared__ float part[KS > 1 ? OUTS : 1];
  for (int i = threadIdx.x; i < OUTS; i += kThreads) {  // (tile j, row r, token v), K slices in order
    const int r = i & 15, v = (i >> 4) % (kPass * NP), j = (i >> 4) / (kPass * NP);
    const int p = v / kPass, vv = v % kPass;
    const int src = (r & 7) * 4 + (vv >> 1), reg = (r >> 3) * 2 + (vv & 1);
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) s += reinterpret_cast<const float*>(&red[q][j * NP + p][src])[reg];
    if constexpr (KS > 1)
      part[i] = s;
    else if (c0 + v < t_total)
      y[static_cast<int64_t>(c0 + v) * n + 16 * (tile0 + j) + r] = s;
  }
  if constexpr (KS > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every CTA's sums are in place
    if (cluster.block_rank() == 0) {
      for (int i = threadIdx.x; i < OUTS; i += kThreads) {
        const int r = i & 15, v = (i >> 4) % (kPass * NP), j = (i >> 4) / (kPass * NP);
        float vals[KS];
#pragma unroll
        for (int q = 0; q < KS; ++q) vals[q] = cluster.map_shared_rank(part, q)[i];
        float s = vals[0];
#pragma unroll
        for (int q = 1; q < KS; ++q) s += vals[q];
        if (c0 + v < t_total) y[static_cast<int64_t>(c0 + v) * n + 16 * (tile0 + j) + r] = s;
      }
    }
    cluster.sync();  // no CTA leaves while rank 0 still reads its shared memory
  }
}

// ------------------------------------------------------------------ tiled path
constexpr int kTileRows = 64;                // weight rows per block
constexpr int kKStage = 32;                  // K columns per pipeline stage
constexpr int kStages = 4;
constexpr int kRowBytes = 2 * kKStage + 16;  // padded shared-memory row: 8 rows of a ldmatrix hit distinct banks
constexpr int kMaxSplits = 8;                // cluster size (portable limit)
constexpr int kF32Splits = 4;                // K splits of the per-tile kernel for matrices under a wave

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// Output e of a block's [token][row] partial sums: the splits' values,
// loaded from every CTA of the cluster before any is added (one round trip),
// added in split order.
__device__ __forceinline__ float split_sum(cg::cluster_group& cluster, float* part, int e, int splits) {
  float v[kMaxSplits];
#pragma unroll
  for (int r = 0; r < kMaxSplits; ++r) v[r] = r < splits ? cluster.map_shared_rank(part, r)[e] : 0.f;
  float s = 0.f;
#pragma unroll
  for (int r = 0; r < kMaxSplits; ++r)
    if (r < splits) s += v[r];
  return s;
}

template <int GW>
constexpr int tiled_stage_bytes() {
  return kTileRows * kRowBytes + 3 * 32 * GW * kRowBytes;
}
template <int GW>
constexpr int tiled_smem_bytes() {
  return kStages * tiled_stage_bytes<GW>();
}

// Block (row block, split, token chunk): rows [64 x, 64 x + 64), K columns
// [K/S * split, K/S * (split + 1)), tokens [NT z, NT z + NT), NT = 32 GW.
// Warp w: rows 32 (w & 1) .. + 32 (two 16-row tiles), token groups
// GW (w >> 1) .. + GW (8 tokens each), all three planes, summed into one
// f32 accumulator per output like the per-tile kernel.  Tokens past T load
// the last token's planes and are not stored.
template <int GW>
__global__ void __launch_bounds__(kThreads, 2)
    linear_rows_tiled_kernel(const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ xp,
                             float* __restrict__ y, int n, int k, int t_total, int splits) {
  constexpr int NT = 32 * GW, XROWS = 3 * NT;
  constexpr int W_BYTES = kTileRows * kRowBytes, STAGE = tiled_stage_bytes<GW>();
  static_assert(NT * kTileRows * 4 <= tiled_smem_bytes<GW>(), "partial sums reuse the stages");
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int wr = warp & 1, wc = warp >> 1;
  const int row0 = blockIdx.x * kTileRows, split = blockIdx.y, tok0 = blockIdx.z * NT;
  const int kspan = k / splits, kbeg = split * kspan, nst = kspan / kKStage;
  if (threadIdx.x < kTileRows)
    prefetch_l2(w + static_cast<int64_t>(row0 + threadIdx.x) * k + kbeg, static_cast<uint32_t>(kspan * 2));
  pdl_wait();  // the planes come from earlier kernels
  pdl_launch_dependents();

  auto load_stage = [&](int st) {
    uint8_t* sw = sm + (st % kStages) * STAGE;
    uint8_t* sx = sw + W_BYTES;
    const int kk = kbeg + st * kKStage;
    {  // weights: 64 rows x 4 pieces of 16 bytes, one per thread
      const int r = threadIdx.x >> 2, c = threadIdx.x & 3;
      cp_async16(sw + r * kRowBytes + 16 * c, w + static_cast<int64_t>(row0 + r) * k + kk + 8 * c);
    }
#pragma unroll
    for (int i = threadIdx.x; i < XROWS * 4; i += kThreads) {  // planes: row q * NT + token
      const int r = i >> 2, c = i & 3, q = r / NT, tok = min(tok0 + r - q * NT, t_total - 1);
      cp_async16(sx + r * kRowBytes + 16 * c, xp + (static_cast<int64_t>(tok) * 3 + q) * k + kk + 8 * c);
    }
  };

  float acc[2][GW][4] = {};
#pragma unroll
  for (int st = 0; st < kStages - 1; ++st) {
    if (st < nst) load_stage(st);
    cp_async_commit();  // (empty groups keep the count uniform)
  }
  for (int st = 0; st < nst; ++st) {
    cp_async_wait<kStages - 2>();  // stage st has landed
    __syncthreads();               // ... for every thread, and stage st - 1 is no longer read
    if (st + kStages - 1 < nst) load_stage(st + kStages - 1);
    cp_async_commit();
    const uint8_t* sw = sm + (st % kStages) * STAGE;
    const uint8_t* sx = sw + W_BYTES;
    // B: per token group and plane, the 8 tokens' 32 columns (4 matrices of 8 columns)
    uint32_t b[GW][3][4];
#pragma unroll
    for (int j = 0; j < GW; ++j)
#pragma unroll
      for (int q = 0; q < 3; ++q)
        ldmatrix_x4(b[j][q], sx + (q * NT + (wc * GW + j) * 8 + (lane & 7)) * kRowBytes + 16 * (lane >> 3));
#pragma unroll
    for (int ks = 0; ks < 2; ++ks)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint32_t a[4];  // rows (2 wr + i) * 16 + (lane & 15), columns 16 ks + 8 (lane >> 4)
        ldmatrix_x4(a, sw + ((wr * 2 + i) * 16 + (lane & 15)) * kRowBytes + 16 * (2 * ks + (lane >> 4)));
#pragma unroll
        for (int j = 0; j < GW; ++j)
#pragma unroll
          for (int q = 0; q < 3; ++q) mma_bf16(acc[i][j], a[0], a[1], a[2], a[3], b[j][q][2 * ks], b[j][q][2 * ks + 1]);
      }
  }
  cp_async_wait<0>();
  __syncthreads();  // every stage consumed: the partial sums reuse the buffers
  float* part = reinterpret_cast<float*>(sm);  // [token][row], NT x 64
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < GW; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int row = (wr * 2 + i) * 16 + g + 8 * (c >> 1), tok = (wc * GW + j) * 8 + 2 * t + (c & 1);
        part[tok * kTileRows + row] = acc[i][j][c];
      }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every split's partial sums are in place
  // split r finishes outputs [r per, (r + 1) per), adding the splits in order
  const int per = NT * kTileRows / splits;
#pragma unroll 2
  for (int e = split * per + threadIdx.x; e < (split + 1) * per; e += kThreads) {
    const float s = split_sum(cluster, part, e, splits);
    const int tok = tok0 + e / kTileRows;
    if (tok < t_total) y[static_cast<int64_t>(tok) * n + row0 + e % kTileRows] = s;
  }
  cluster.sync();  // no CTA leaves while another still reads its shared memory
}

// ------------------------------------------------------------------ tcgen05 path
// bf16 projections of more than this many tokens take a tensor-core path
// (measured at the 35B shapes: 16 tokens on tcgen05 with a 32-token tile
// 8192 x 2048 12.7 us and the head 164 us, against 19.5 and 210 us on the
// per-tile path, which stays ahead at 8 tokens: 9.6 and 137 us).
constexpr int64_t kTensorMinTokens = 8;
constexpr int kUmmaRows = 128;  // weight rows per CTA: the MMA's M, one TMEM lane per row
constexpr int kUmmaKStage = 64;  // K columns per stage (one 128-byte swizzle row): four MMAs of K 16
__device__ int g_umma_timeouts;  // mbarrier waits that gave up

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits until the phase of `parity` has completed; true once it has.  Gives
// up after kWaitLimitNs, counting the timeout; once a wait of this CTA gave
// up (*abort), the others return false at once, so a broken pipeline stops
// issuing work promptly.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(a, parity)) {
    if (*abort) return false;
    if (global_ns() - t0 > kWaitLimitNs) {
      *abort = 1;
      atomicAdd(&g_umma_timeouts, 1);
      return false;
    }
  }
  return true;
}
// The same wait without the early return on *abort: used after an abort to
// let copies and MMAs already issued complete before the CTA reuses its
// shared memory or frees its TMEM.  Still bounded by kWaitLimitNs.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(a, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicAdd(&g_umma_timeouts, 1);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte swizzle (layout type 2 at bits 61-63): rows of 128
// bytes (64 bf16 columns) in 1024-byte atoms of 8 rows, the 16-byte pieces
// of row r XOR-permuted by r % 8 -- what TMA writes with SWIZZLE_128B; 1024
// bytes between 8-row groups (stride byte offset), the leading byte offset
// unused within one atom's width (1); bits 46-48 hold the fixed 0b001.  The
// MMA of K columns [16 s, 16 s + 16) starts 32 s bytes into the rows (the
// swizzle is applied to the computed addresses, so the atom must sit at a
// 1024-byte boundary).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// 2-D tensor copy global -> this CTA's shared memory (no multicast), box at
// (x = column, y = row), completion counted on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B bf16
// (bits 7-9, 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17,
// M >> 4 at bit 24.
template <int N>
constexpr uint32_t umma_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(kUmmaRows >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Columns [c, c + 24) of this warp's 32 TMEM lanes (8 tokens x 3 planes),
// loaded and waited for in one statement so no use of the registers can
// move ahead of the wait.
__device__ __forceinline__ void tmem_ld24(uint32_t taddr, uint32_t (&r)[24]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%24];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [%25];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16, %17, %18, %19, %20, %21, %22, %23}, [%26];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23])
      : "r"(taddr), "r"(taddr + 8), "r"(taddr + 16)
      : "memory");
}

// RB row blocks of 128 per CTA share each stage's token planes (the B
// operand): with RB = 2 a stage carries 32 KB of weights per 24 KB of planes
// instead of 16 per 24.  Each row's accumulation (its K split and the K
// order inside it) is the same for RB = 1 and 2.
template <int RB>
constexpr int umma_stages() {
  return RB == 1 ? 5 : 4;
}
template <int NT, int RB>
constexpr int umma_stage_bytes() {
  return (RB * kUmmaRows + 3 * NT) * kUmmaKStage * 2;
}
template <int NT, int RB>
constexpr int umma_smem_bytes() {  // stages + alignment slack
  return umma_stages<RB>() * umma_stage_bytes<NT, RB>() + 1024;
}

// Block (row block, split, token chunk): rows [128 RB x, 128 RB (x + 1)), K
// columns [K/S split, K/S (split + 1)), tokens [NT z, NT z + NT).  `tmw`
// maps W (N rows x K), `tmx` the planes ((3 T) rows x K, row 3 t + plane);
// both with 64-column boxes, of 128 and 3 NT rows.  Row blocks past N load
// zeros (TMA fill) and store nothing.
template <int NT, int RB>
__global__ void __launch_bounds__(kThreads, 1)
    linear_rows_umma_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                            const __nv_bfloat16* __restrict__ w, float* __restrict__ y, int n, int k, int t_total,
                            int splits) {
  constexpr int NB = 3 * NT;  // B rows (token-major: 3 t + plane) = the MMA's N
  constexpr int S = umma_stages<RB>(), ROWS = RB * kUmmaRows;
  constexpr int W_BYTES = kUmmaRows * kUmmaKStage * 2, A_BYTES = RB * W_BYTES, STAGE = umma_stage_bytes<NT, RB>();
  constexpr uint32_t ACC = NB <= 64 ? 64 : NB <= 128 ? 128 : 256;  // TMEM columns of one accumulator
  constexpr uint32_t COLS = RB * ACC;                             // a power of 2 (RB = 1, 2)
  constexpr uint32_t IDESC = umma_idesc<NB>();
  static_assert(NB % 16 == 0 && NB <= 256, "M = 128 takes N = 16 .. 256 in steps of 16");
  static_assert(RB == 1 || RB == 2, "one or two row blocks per CTA");
  static_assert(NT * ROWS * 4 <= S * STAGE, "partial sums reuse the stages");
  static_assert(W_BYTES % 1024 == 0 && STAGE % 1024 == 0, "swizzle atoms at 1024-byte boundaries");
  extern __shared__ uint8_t sm_raw[];
  __shared__ __align__(8) uint64_t full[S], empty[S], done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * ROWS, split = blockIdx.y, tok0 = blockIdx.z * NT;
  const int kspan = k / splits, kbeg = split * kspan, nst = kspan / kUmmaKStage;
  // stage buffers at a 1024-byte boundary (128-byte swizzle atoms)
  uint8_t* sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {  // TMEM for the accumulators (the whole warp allocates)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
#pragma unroll
    for (int b = 0; b < S; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], 1);
    }
    mbar_init(&done, 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmw)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmx)) : "memory");
  }
  for (int r = static_cast<int>(threadIdx.x) - 64; r >= 0 && r < ROWS; r += kThreads - 64)  // weight slice into L2
    if (row0 + r < n) prefetch_l2(w + static_cast<int64_t>(row0 + r) * k + kbeg, static_cast<uint32_t>(kspan * 2));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  pdl_wait();  // the planes come from earlier kernels
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    // producer: stage st into buffer st % S once the MMAs of stage st - S
    // released it; after a wait gave up nothing new is issued
    int issued = 0;
    for (int st = 0; st < nst; ++st) {
      const int b = st % S;
      if (st >= S && !mbar_wait(&empty[b], ((st / S) - 1) & 1, &s_abort)) break;
      mbar_arrive_expect_tx(&full[b], STAGE);
      const uint32_t sa = sbase + b * STAGE;
      const int kk = kbeg + st * kUmmaKStage;
#pragma unroll
      for (int j = 0; j < RB; ++j) tma_load_2d(sa + j * W_BYTES, &tmw, kk, row0 + j * kUmmaRows, &full[b]);
      tma_load_2d(sa + A_BYTES, &tmx, kk, 3 * tok0, &full[b]);
      issued = st + 1;
    }
    if (s_abort) {
      // each buffer has at most one copy in flight (its last issued stage):
      // let them land before the stages are overwritten below
      for (int st = issued > S ? issued - S : 0; st < issued; ++st) mbar_drain(&full[st % S], (st / S) & 1);
    }
  } else if (threadIdx.x == 32) {
    // MMA issuer: four K-16 steps per stage, then the stage's buffer goes back
    for (int st = 0; st < nst; ++st) {
      const int b = st % S;
      if (!mbar_wait(&full[b], (st / S) & 1, &s_abort)) break;
      tc_fence_after();
      const uint32_t a0 = sbase + b * STAGE, b0 = a0 + A_BYTES;
#pragma unroll
      for (int s4 = 0; s4 < kUmmaKStage / 16; ++s4)
#pragma unroll
        for (int j = 0; j < RB; ++j)
          umma_bf16(tmem + j * ACC, umma_desc(a0 + j * W_BYTES + 32 * s4), umma_desc(b0 + 32 * s4), IDESC,
                    (st > 0 || s4 > 0) ? 1u : 0u);
      umma_commit(&empty[b]);
    }
    umma_commit(&done);  // every MMA issued by this thread, also after an abort
  }
  // every MMA completes before TMEM is read or freed, also after an abort
  mbar_drain(&done, 0);
  tc_fence_after();
  __syncthreads();  // the producer's drained copies have landed before the stages are reused

  // TMEM lane r, accumulator j = weight row row0 + 128 j + r, column
  // 128 j... + 3 t + plane; warp w reads lanes 32 (w % 4) .. + 32 and
  // tokens [NT/2 (w / 4), NT/2 (w / 4 + 1))
  float* part = reinterpret_cast<float*>(sm);  // [token][row], NT x ROWS (every TMA landed, every MMA done)
  const int lq = warp & 3, half = warp >> 2;
  const uint32_t tl = tmem + (static_cast<uint32_t>(32 * lq) << 16);
#pragma unroll
  for (int j = 0; j < RB; ++j)
#pragma unroll
    for (int t8 = half * (NT / 2); t8 < (half + 1) * (NT / 2); t8 += 8) {
      uint32_t r[24];
      tmem_ld24(tl + j * ACC + 3 * t8, r);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        part[(t8 + i) * ROWS + j * kUmmaRows + 32 * lq + lane] =
            (__uint_as_float(r[3 * i]) + __uint_as_float(r[3 * i + 1])) + __uint_as_float(r[3 * i + 2]);
    }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(COLS) : "memory");
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every split's partial sums are in place
  const int per = NT * ROWS / splits;
#pragma unroll 2
  for (int e = split * per + threadIdx.x; e < (split + 1) * per; e += kThreads) {
    const float s = split_sum(cluster, part, e, splits);
    const int tok = tok0 + e / ROWS, row = row0 + e % ROWS;
    if (tok < t_total && row < n) y[static_cast<int64_t>(tok) * n + row] = s;
  }
  cluster.sync();  // no CTA leaves while another still reads its shared memory
}

// 2-D tensor map over bf16 rows (rows x k, row stride k), 64-column boxes
// of `box_rows` rows written 128-byte swizzled, zero fill past the rows.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return false;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kUmmaKStage), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool F32W, int TW, int KS = 1>
cudaError_t launch_np(cudaLaunchConfig_t& cfg, int np, const void* w, const __nv_bfloat16* xp, float* y, int n, int k,
                      int t) {
  switch (np) {
    case 1: return ::bt::launch_ex(&cfg, linear_rows_kernel<F32W, 1, TW, KS>, w, xp, y, n, k, t);
    case 2: return ::bt::launch_ex(&cfg, linear_rows_kernel<F32W, 2, TW, KS>, w, xp, y, n, k, t);
    case 4: return ::bt::launch_ex(&cfg, linear_rows_kernel<F32W, 4, TW, KS>, w, xp, y, n, k, t);
    default:  // two tiles per warp stop at 4 passes (the reduction's shared memory)
      return ::bt::launch_ex(&cfg, linear_rows_kernel<F32W, (TW == 2 ? 4 : 8), TW, KS>, w, xp, y, n, k, t);
  }
}

cudaLaunchConfig_t pdl_config(dim3 grid, cudaStream_t stream, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

int bf16_planes(const float* x, void* planes, int64_t t, int64_t k, cudaStream_t stream) {
  if (!x || !planes || t < 1 || k < 8 || k % 8) return fail(BT_ERR_INVALID, "bf16_planes: bad arguments");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(planes)) & 15)
    return fail(BT_ERR_INVALID, "bf16_planes: x and planes must be 16-byte aligned");
  const int64_t chunks = t * (k / 8);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg =
      pdl_config(dim3(static_cast<unsigned>(std::min<int64_t>((chunks + kThreads - 1) / kThreads, 4096))), stream, attr);
  const cudaError_t e = ::bt::launch_ex(&cfg, bf16_planes_kernel, x, static_cast<__nv_bfloat16*>(planes), t,
                                           static_cast<int>(k));
  if (e != cudaSuccess) return fail_cuda(e, "bf16_planes launch");
  return BT_OK;
}

int linear_rows(const void* w, int w_dtype, const void* x_planes, float* y, int64_t n, int64_t k, int64_t t,
                cudaStream_t stream) {
  if (!w || !x_planes || !y || n < 1 || k < 1 || t < 1) return fail(BT_ERR_INVALID, "linear_rows: bad arguments");
  if (w_dtype != BT_BF16 && w_dtype != BT_F32) return fail(BT_ERR_UNSUPPORTED, "linear_rows: weights bf16 or f32");
  if (n % 16 || k % 256 || n / 16 > 2147483647LL || (t + kPass - 1) / kPass > 65535)
    return fail(BT_ERR_UNSUPPORTED, "linear_rows: N must be a multiple of 16 and K of 256 (got %lld x %lld)",
                static_cast<long long>(n), static_cast<long long>(k));
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x_planes)) & 15)
    return fail(BT_ERR_INVALID, "linear_rows: w and the planes must be 16-byte aligned");
  const auto* xp = static_cast<const __nv_bfloat16*>(x_planes);
  if (w_dtype == BT_BF16 && t > kTensorMinTokens && n % kUmmaRows == 0) {
    // tensor-core path: 64 tokens per CTA (32 for T <= 32); K split over a
    // cluster as far as one token chunk's 128-row blocks still fit one wave
    // of 1 per SM.  The split depends on the rows and K only, not on T, so a
    // token's outputs are the same bits whichever tokens share the call (a
    // prefill chunk of many tokens per sequence gets the decode step's sums).
    // Two 128-row blocks per CTA (sharing each stage's planes) when one
    // block per CTA would take more than one wave (the head, prefill
    // chunks) or the K split is 8; measured on B200 at the 35B shapes: head
    // 231 -> 201 us at 64 tokens, the 2048 x 4096 out-projection (split 8)
    // 23 -> 18 us, the 8192 x 2048 one 104 -> 90 us at 512 tokens, while the
    // decode step's 4096 x 2048 (split 4) and 8192 x 2048 (split 2)
    // projections are faster with one block per CTA.  Same bits either way.
    const bool wide = t > 32;
    const int nt = wide ? 64 : 32;
    const int64_t blocks = n / kUmmaRows, chunks = (t + nt - 1) / nt;
    if (blocks > 2147483647LL || chunks > 65535)
      return fail(BT_ERR_UNSUPPORTED, "linear_rows: too many rows or tokens");
    int splits = 1;
    while (splits < kMaxSplits && blocks * splits * 2 <= sm_count() && k % (kUmmaKStage * splits * 2) == 0)
      splits *= 2;
    const int rb = (blocks * splits * chunks > sm_count() || splits >= 8) ? 2 : 1;
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = pdl_config(dim3(static_cast<unsigned>((blocks + rb - 1) / rb),
                                             static_cast<unsigned>(splits), static_cast<unsigned>(chunks)),
                                        stream, attr);
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = static_cast<unsigned>(splits);
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    const auto* wb = static_cast<const __nv_bfloat16*>(w);
    const int nn = static_cast<int>(n), kk = static_cast<int>(k), tt = static_cast<int>(t);
    CUtensorMap tmw, tmx;
    if (!make_map(&tmw, w, n, k, kUmmaRows) || !make_map(&tmx, x_planes, 3 * t, k, 3 * nt))
      return fail(BT_ERR_CUDA, "linear_rows: tensor maps could not be encoded");
    auto go = [&](auto kernel, int smem) {
      cfg.dynamicSmemBytes = smem;
      cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      return err == cudaSuccess ? ::bt::launch_ex(&cfg, kernel, tmw, tmx, wb, y, nn, kk, tt, splits) : err;
    };
    const cudaError_t e = wide ? (rb == 2 ? go(linear_rows_umma_kernel<64, 2>, umma_smem_bytes<64, 2>())
                                          : go(linear_rows_umma_kernel<64, 1>, umma_smem_bytes<64, 1>()))
                               : (rb == 2 ? go(linear_rows_umma_kernel<32, 2>, umma_smem_bytes<32, 2>())
                                          : go(linear_rows_umma_kernel<32, 1>, umma_smem_bytes<32, 1>()));
    if (e != cudaSuccess) return fail_cuda(e, "linear_rows (tcgen05) launch");
    return BT_OK;
  }
  if (w_dtype == BT_BF16 && t > kTensorMinTokens && n % kTileRows == 0) {
    // tiled path: K split over a cluster as far as one token chunk's blocks
    // still fit one wave of 2 per SM (rows and K decide it, not T)
    const int64_t blocks = n / kTileRows, chunks = (t + 63) / 64;
    if (blocks > 2147483647LL || chunks > 65535)
      return fail(BT_ERR_UNSUPPORTED, "linear_rows: too many rows or tokens");
    int splits = 1;
    while (splits < kMaxSplits && blocks * splits * 2 <= 2 * sm_count() && k % (kKStage * splits * 2) == 0)
      splits *= 2;
    const bool wide = t > 32;  // 64 tokens per block, else 32
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = pdl_config(
        dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(splits),
             static_cast<unsigned>(wide ? chunks : (t + 31) / 32)),
        stream, attr);
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = static_cast<unsigned>(splits);
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    const auto* wb = static_cast<const __nv_bfloat16*>(w);
    const int nn = static_cast<int>(n), kk = static_cast<int>(k), tt = static_cast<int>(t);
    cudaError_t e;
    if (wide) {
      cfg.dynamicSmemBytes = tiled_smem_bytes<2>();
      e = cudaFuncSetAttribute(linear_rows_tiled_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               tiled_smem_bytes<2>());
      if (e == cudaSuccess) e = ::bt::launch_ex(&cfg, linear_rows_tiled_kernel<2>, wb, xp, y, nn, kk, tt, splits);
    } else {
      cfg.dynamicSmemBytes = tiled_smem_bytes<1>();
      e = cudaFuncSetAttribute(linear_rows_tiled_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               tiled_smem_bytes<1>());
      if (e == cudaSuccess) e = ::bt::launch_ex(&cfg, linear_rows_tiled_kernel<1>, wb, xp, y, nn, kk, tt, splits);
    }
    if (e != cudaSuccess) return fail_cuda(e, "linear_rows (tiled) launch");
    return BT_OK;
  }
  // Two 16-row tiles per block when there are rows enough (each x plane load
  // then serves 32 rows): with several passes when they fill half a wave;
  // with one pass (<= 8 tokens) only when they still take several waves
  // (the head, 137 -> 123 us at 8 tokens on B200; the 8192-row qkv
  // projection, one wave either way, is faster with one tile: 9.5 vs 11.7
  // us).  Passes of 8 tokens per block: as many as keep >= 2 blocks per SM
  // busy (fewer weight re-reads), one when the matrix is small.  bf16
  // weights only: f32 ones are the small matrices.  (Per output the same
  // sums in the same order either way.)
  const int64_t tiles = n / 16, passes = (t + kPass - 1) / kPass, want = 2 * sm_count();
  const int tw = (w_dtype == BT_BF16 && tiles % 2 == 0 && tiles / 2 >= (passes > 1 ? want / 2 : 2 * want)) ? 2 : 1;
  int np = tw == 2 ? 4 : 8;
  while (np > 1 && (np > passes || tiles / tw * ((passes + np - 1) / np) < want)) np >>= 1;
  // Matrices whose row tiles, split kF32Splits ways, still fit two waves of
  // blocks (the router, the GDN beta/alpha rows; for <= 8 tokens also the
  // 2048-row bf16 out-projections, 10.3 -> 6.9 us at K = 4096 on B200, but
  // not the 4096-row ones, 6.7 -> 9.9 us at 3.5 waves): K split over a
  // cluster of kF32Splits CTAs, so each CTA's serial K loop is that much
  // shorter.  Decided by the rows and K alone, so a token's sums do not
  // depend on T (as on the tensor-core path).
  const bool ksplit = tiles * kF32Splits <= 2 * want && k % (kF32Splits * kWarps * 32) == 0;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = pdl_config(
      dim3(static_cast<unsigned>(tiles / tw), static_cast<unsigned>((passes + np - 1) / np), ksplit ? kF32Splits : 1),
      stream, attr);
  if (ksplit) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = kF32Splits;
    cfg.numAttrs = 2;
  }
  const int nn = static_cast<int>(n), kk = static_cast<int>(k), tt = static_cast<int>(t);
  const cudaError_t e = ksplit && w_dtype == BT_F32 ? launch_np<true, 1, kF32Splits>(cfg, np, w, xp, y, nn, kk, tt)
                        : ksplit               ? launch_np<false, 1, kF32Splits>(cfg, np, w, xp, y, nn, kk, tt)
                        : w_dtype == BT_F32    ? launch_np<true, 1>(cfg, np, w, xp, y, nn, kk, tt)
                        : tw == 2              ? launch_np<false, 2>(cfg, np, w, xp, y, nn, kk, tt)
                                               : launch_np<false, 1>(cfg, np, w, xp, y, nn, kk, tt);
  if (e != cudaSuccess) return fail_cuda(e, "linear_rows launch");
  return BT_OK;
}

int linear_rows_timeouts() {
  int v = 0;
  const int zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_umma_timeouts, sizeof(int)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_umma_timeouts, &zero, sizeof(int)) != cudaSuccess)
    return -1;
  return v;
}

}  // namespace bt
