// Gated-delta-rule (GDN) recurrent decode step.
//
// Semantics follow the reference's torch oracle `_torch_gdn_decode`
// (breezetoken/backends.py:241-271) and its tilelang kernel
// (breezetoken/kernels/cuda/gdn.py:32-139):
//   qn = q * rsqrt(|q|^2 + eps) * scale,  kn = k * rsqrt(|k|^2 + eps)
//   S  = S * exp(g)                       (per value head)
//   d  = (v - S^T kn) * sigmoid(beta)
//   S  = S + kn d^T,   o = S^T qn         (state updated in place)
// with value head h reading key head h % heads_k.
//
// Layout: state (batch, heads_v, dim_k, dim_v) f32, row d = key index.
// One CTA owns 32 value columns of one head: warp w holds rows
// [32w, 32w+32) of those columns in registers (32 floats per thread), so the
// state is read and written exactly once per step with 128-B coalesced
// accesses; the two column sums (S^T kn and S^T qn) reduce across warps in
// shared memory.  Before griddepcontrol.wait the CTA only issues L2
// prefetches of its state slice.
#include "errors.h"
#include "gdn.cuh"

namespace bt {

namespace {

constexpr int kCols = 32;

template <typename T>
__device__ __forceinline__ float load_elem(const void* p, int64_t i);
template <>
__device__ __forceinline__ float load_elem<float>(const void* p, int64_t i) {
  return static_cast<const float*>(p)[i];
}
template <>
__device__ __forceinline__ float load_elem<__nv_bfloat16>(const void* p, int64_t i) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

template <typename T>
__global__ void __launch_bounds__(256) gdn_decode_kernel(const __grid_constant__ GdnParams p) {
  __shared__ float red[8][kCols];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col_tiles = p.dim / kCols;
  const int tile = blockIdx.x % col_tiles;
  const int hv = (blockIdx.x / col_tiles) % p.heads_v;
  const int b = blockIdx.x / (col_tiles * p.heads_v);
  const int hk = hv % p.heads_k;
  const int dim = p.dim;
  const int col = tile * kCols + lane;

  float* S = p.state + ((static_cast<int64_t>(b) * p.heads_v + hv) * dim) * dim;
  const int d0 = warp * 32;
  // L2 prefetch of the warp's 32 state rows (one 128-B line each) of this
  // column tile: a cache hint only, so it is safe before the dependency wait.
  asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(S + static_cast<int64_t>(d0 + lane) * dim +
                                                            tile * kCols));
  pdl_launch_dependents();
  pdl_wait();

  // q/k of key head hk: every warp computes both norms (4-8 elements per lane).
  const int64_t qoff = static_cast<int64_t>(b) * p.q_bs + static_cast<int64_t>(hk) * dim;
  const int64_t koff = static_cast<int64_t>(b) * p.k_bs + static_cast<int64_t>(hk) * dim;
  float qss = 0.f, kss = 0.f;
  for (int i = lane; i < dim; i += 32) {
    const float qv = load_elem<T>(p.q, qoff + i), kv = load_elem<T>(p.k, koff + i);
    qss = fmaf(qv, qv, qss);
    kss = fmaf(kv, kv, kss);
  }
  qss = warp_sum(qss);
  kss = warp_sum(kss);
  const float qr = 1.0f / sqrtf(qss + p.eps), kr = 1.0f / sqrtf(kss + p.eps);
  // lane l of warp w holds qn/kn[d0 + l]; broadcast with shuffles below.
  const float qn_l = __fmul_rn(__fmul_rn(load_elem<T>(p.q, qoff + d0 + lane), qr), p.scale);
  const float kn_l = __fmul_rn(load_elem<T>(p.k, koff + d0 + lane), kr);

  const float gval = p.g[static_cast<int64_t>(b) * p.g_bs + hv];
  const float bval = p.beta[static_cast<int64_t>(b) * p.beta_bs + hv];
  const float decay = expf(gval);
  const float bsig = sigmoid_f(bval);

  float s[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) s[i] = __fmul_rn(S[static_cast<int64_t>(d0 + i) * dim + col], decay);

  float rec = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) rec = fmaf(s[i], __shfl_sync(0xffffffffu, kn_l, i), rec);
  red[warp][lane] = rec;
  __syncthreads();
  float recalled = 0.f;
  for (int w = 0; w < dim / 32; ++w) recalled += red[w][lane];
  const float vv = load_elem<T>(p.v, static_cast<int64_t>(b) * p.v_bs + static_cast<int64_t>(hv) * dim + col);
  const float delta = __fmul_rn(vv - recalled, bsig);

  float o = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    s[i] = __fadd_rn(s[i], __fmul_rn(__shfl_sync(0xffffffffu, kn_l, i), delta));
    S[static_cast<int64_t>(d0 + i) * dim + col] = s[i];
    o = fmaf(s[i], __shfl_sync(0xffffffffu, qn_l, i), o);
  }
  __syncthreads();
  red[warp][lane] = o;
  __syncthreads();
  if (warp == 0) {
    float t = 0.f;
    for (int w = 0; w < dim / 32; ++w) t += red[w][lane];
    p.out[static_cast<int64_t>(b) * p.out_bs + static_cast<int64_t>(hv) * dim + col] = t;
  }
}

}  // namespace

int gdn_decode_launch(const GdnParams& p, cudaStream_t stream, bool pdl) {
  if (p.dim % 32 != 0 || p.dim < 32 || p.dim > 256)
    return fail(BT_ERR_UNSUPPORTED, "gdn_decode serves dim in {32..256} step 32, got %d", p.dim);
  if (p.heads_k <= 0 || p.heads_v <= 0 || p.heads_v % p.heads_k != 0)
    return fail(BT_ERR_INVALID, "gdn_decode: value heads (%d) must be a positive multiple of key heads (%d)",
                p.heads_v, p.heads_k);
  if (p.batch <= 0) return fail(BT_ERR_INVALID, "gdn_decode: batch must be positive");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.batch) * p.heads_v * (p.dim / kCols));
  cfg.blockDim = dim3(p.dim);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = p.in_dtype == BT_BF16 ? cudaLaunchKernelEx(&cfg, gdn_decode_kernel<__nv_bfloat16>, p)
                                        : cudaLaunchKernelEx(&cfg, gdn_decode_kernel<float>, p);
  if (e != cudaSuccess) return fail_cuda(e, "gdn_decode launch");
  return BT_OK;
}

}  // namespace bt
