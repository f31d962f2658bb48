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
#include <cuda_bf16.h>

#include <algorithm>

#include "errors.h"
#include "linear_rows.cuh"

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
  const auto* xp = static_cast<const __nv_bfloat16*>(x_planes);
  const cudaError_t e = w_dtype == BT_F32 ? launch_np<true, 1>(cfg, np, w, xp, y, nn, kk, tt)
                        : tw == 2         ? launch_np<false, 2>(cfg, np, w, xp, y, nn, kk, tt)
                                          : launch_np<false, 1>(cfg, np, w, xp, y, nn, kk, tt);
  if (e != cudaSuccess) return fail_cuda(e, "linear_rows launch");
  return BT_OK;
}

}  // namespace bt
