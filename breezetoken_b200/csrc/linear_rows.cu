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
// More than 16 tokens with bf16 weights (the batched decode of many
// sequences) run as a tiled product instead, where the x planes would
// otherwise be re-read from L2 by every 16-row block: a block owns 64 rows
// and up to 64 tokens, and stages 32-column slices of its weight rows and of
// all its tokens' planes through a 4-deep cp.async pipeline in shared
// memory (rows padded to 80 bytes, so ldmatrix reads are conflict-free);
// 8 warps = 2 row halves x 4 token quarters, MMA operands by ldmatrix.  K is
// split over the CTAs of a thread-block cluster (up to 8), whose partial
// sums meet through distributed shared memory and are added in split order
// (deterministic, no workspace).
#include <cooperative_groups.h>
#include <cuda_bf16.h>

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

template <bool F32W, int NP, int TW>
__global__ void __launch_bounds__(kThreads) linear_rows_kernel(const void* __restrict__ w,
                                                               const __nv_bfloat16* __restrict__ xp,
                                                               float* __restrict__ y, int n, int k, int t_total) {
  using Elem = typename std::conditional<F32W, float, __nv_bfloat16>::type;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile0 = blockIdx.x * TW, c0 = blockIdx.y * kPass * NP, span = k / kWarps;
  if (lane < 16)
#pragma unroll
    for (int j = 0; j < TW; ++j)
      prefetch_l2(static_cast<const Elem*>(w) + static_cast<int64_t>(16 * (tile0 + j) + lane) * k + warp * span,
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
  for (int k0 = warp * span; k0 < (warp + 1) * span; k0 += 32) {
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
  for (int i = threadIdx.x; i < TW * 16 * kPass * NP; i += kThreads) {  // (tile j, row r, token v), K slices in order
    const int r = i & 15, v = (i >> 4) % (kPass * NP), j = (i >> 4) / (kPass * NP);
    const int p = v / kPass, vv = v % kPass;
    const int src = (r & 7) * 4 + (vv >> 1), reg = (r >> 3) * 2 + (vv & 1);
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) s += reinterpret_cast<const float*>(&red[q][j * NP + p][src])[reg];
    if (c0 + v < t_total) y[static_cast<int64_t>(c0 + v) * n + 16 * (tile0 + j) + r] = s;
  }
}

// ------------------------------------------------------------------ tiled path
constexpr int kTileRows = 64;                // weight rows per block
constexpr int kKStage = 32;                  // K columns per pipeline stage
constexpr int kStages = 4;
constexpr int kRowBytes = 2 * kKStage + 16;  // padded shared-memory row: 8 rows of a ldmatrix hit distinct banks
constexpr int kMaxSplits = 8;                // cluster size (portable limit)

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
  for (int e = split * per + threadIdx.x; e < (split + 1) * per; e += kThreads) {
    float s = 0.f;
    for (int r = 0; r < splits; ++r) s += cluster.map_shared_rank(part, r)[e];
    const int tok = tok0 + e / kTileRows;
    if (tok < t_total) y[static_cast<int64_t>(tok) * n + row0 + e % kTileRows] = s;
  }
  cluster.sync();  // no CTA leaves while another still reads its shared memory
}

template <bool F32W, int TW>
cudaError_t launch_np(cudaLaunchConfig_t& cfg, int np, const void* w, const __nv_bfloat16* xp, float* y, int n, int k,
                      int t) {
  switch (np) {
    case 1: return cudaLaunchKernelEx(&cfg, linear_rows_kernel<F32W, 1, TW>, w, xp, y, n, k, t);
    case 2: return cudaLaunchKernelEx(&cfg, linear_rows_kernel<F32W, 2, TW>, w, xp, y, n, k, t);
    case 4: return cudaLaunchKernelEx(&cfg, linear_rows_kernel<F32W, 4, TW>, w, xp, y, n, k, t);
    default:  // two tiles per warp stop at 4 passes (the reduction's shared memory)
      return cudaLaunchKernelEx(&cfg, linear_rows_kernel<F32W, (TW == 2 ? 4 : 8), TW>, w, xp, y, n, k, t);
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, bf16_planes_kernel, x, static_cast<__nv_bfloat16*>(planes), t,
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
  if (w_dtype == BT_BF16 && t > 16 && n % kTileRows == 0) {
    // tiled path: split K over a cluster until >= 2 blocks per SM
    const int64_t blocks = n / kTileRows, chunks = (t + 63) / 64;
    if (blocks > 2147483647LL || chunks > 65535)
      return fail(BT_ERR_UNSUPPORTED, "linear_rows: too many rows or tokens");
    int splits = 1;
    while (splits < kMaxSplits && blocks * chunks * splits < 2 * sm_count() && k % (kKStage * splits * 2) == 0)
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
      if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, linear_rows_tiled_kernel<2>, wb, xp, y, nn, kk, tt, splits);
    } else {
      cfg.dynamicSmemBytes = tiled_smem_bytes<1>();
      e = cudaFuncSetAttribute(linear_rows_tiled_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               tiled_smem_bytes<1>());
      if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, linear_rows_tiled_kernel<1>, wb, xp, y, nn, kk, tt, splits);
    }
    if (e != cudaSuccess) return fail_cuda(e, "linear_rows (tiled) launch");
    return BT_OK;
  }
  // Two 16-row tiles per block when there are rows enough (each x plane load
  // then serves 32 rows); passes of 8 tokens per block: as many as keep
  // >= 2 blocks per SM busy (fewer weight re-reads), one when the matrix is
  // small.  bf16 weights only: f32 ones are the small matrices.
  const int64_t tiles = n / 16, passes = (t + kPass - 1) / kPass, want = 2 * sm_count();
  const int tw = (w_dtype == BT_BF16 && tiles % 2 == 0 && tiles / 2 >= want / 2 && passes > 1) ? 2 : 1;
  int np = tw == 2 ? 4 : 8;
  while (np > 1 && (np > passes || tiles / tw * ((passes + np - 1) / np) < want)) np >>= 1;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(
      dim3(static_cast<unsigned>(tiles / tw), static_cast<unsigned>((passes + np - 1) / np)), stream, attr);
  const int nn = static_cast<int>(n), kk = static_cast<int>(k), tt = static_cast<int>(t);
  const cudaError_t e = w_dtype == BT_F32 ? launch_np<true, 1>(cfg, np, w, xp, y, nn, kk, tt)
                        : tw == 2         ? launch_np<false, 2>(cfg, np, w, xp, y, nn, kk, tt)
                                          : launch_np<false, 1>(cfg, np, w, xp, y, nn, kk, tt);
  if (e != cudaSuccess) return fail_cuda(e, "linear_rows launch");
  return BT_OK;
}

}  // namespace bt
