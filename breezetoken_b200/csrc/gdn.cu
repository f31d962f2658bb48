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
// One CTA of 256 threads owns 16 value columns of one head: thread t holds
// column t % 16 of the rows [R*(t/16), R*(t/16) + R) (R = dim/16) in
// registers, so the state is read and written exactly once per step
// (64-byte half-warp segments); the column sums S^T kn and S^T qn reduce
// across the 16 row groups in shared memory.  Before griddepcontrol.wait the
// CTA only issues L2 prefetches of its state slice.
#include "errors.h"
#include "gdn.cuh"

namespace bt {

namespace {

constexpr int kCols = 16;
constexpr int kRowGroups = 16;
constexpr int kThreads = kCols * kRowGroups;

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

template <typename T, int R>
__global__ void __launch_bounds__(kThreads) gdn_decode_kernel(const __grid_constant__ GdnParams p) {
  constexpr int DIM = R * kRowGroups;
  __shared__ float red[kRowGroups][kCols];
  __shared__ float sq[DIM], sk[DIM];
  const int tid = threadIdx.x, lane = tid & 31;
  const int col_l = tid % kCols, rg = tid / kCols;
  const int col_tiles = DIM / kCols;
  const int tile = blockIdx.x % col_tiles;
  const int hv = (blockIdx.x / col_tiles) % p.heads_v;
  const int b = blockIdx.x / (col_tiles * p.heads_v);
  const int hk = hv % p.heads_k;
  const int col = tile * kCols + col_l;
  const int r0 = rg * R;

  trace_entry(p.trace);
  float* S = p.state + ((static_cast<int64_t>(b) * p.heads_v + hv) * DIM) * DIM;
  // L2 prefetch of the tile's rows (64 B each): a cache hint only, safe
  // before the dependency wait.
  if (tid < DIM) asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(S + static_cast<int64_t>(tid) * DIM + tile * kCols));
  pdl_launch_dependents();
  pdl_wait();
  trace_waited(p.trace);

  // normalised q/k of key head hk: warp 0 does q, warp 1 does k
  const int warp = tid >> 5;
  if (warp < 2) {
    const void* src = warp == 0 ? p.q : p.k;
    const int64_t off = static_cast<int64_t>(b) * (warp == 0 ? p.q_bs : p.k_bs) + static_cast<int64_t>(hk) * DIM;
    float vals[DIM / 32];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < DIM / 32; ++i) {
      vals[i] = load_elem<T>(src, off + lane + 32 * i);
      ss = fmaf(vals[i], vals[i], ss);
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + p.eps);
    float* dst = warp == 0 ? sq : sk;
#pragma unroll
    for (int i = 0; i < DIM / 32; ++i)
      dst[lane + 32 * i] = warp == 0 ? __fmul_rn(__fmul_rn(vals[i], r), p.scale) : __fmul_rn(vals[i], r);
  }

  const float decay = expf(p.g[static_cast<int64_t>(b) * p.g_bs + hv]);
  const float bsig = sigmoid_f(p.beta[static_cast<int64_t>(b) * p.beta_bs + hv]);
  float s[R];
#pragma unroll
  for (int i = 0; i < R; ++i) s[i] = __fmul_rn(S[static_cast<int64_t>(r0 + i) * DIM + col], decay);
  __syncthreads();
  trace_ready(p.trace);

  float rec = 0.f;
#pragma unroll
  for (int i = 0; i < R; ++i) rec = fmaf(s[i], sk[r0 + i], rec);
  red[rg][col_l] = rec;
  __syncthreads();
  float recalled = 0.f;
#pragma unroll
  for (int w = 0; w < kRowGroups; ++w) recalled += red[w][col_l];
  const float vv = load_elem<T>(p.v, static_cast<int64_t>(b) * p.v_bs + static_cast<int64_t>(hv) * DIM + col);
  const float delta = __fmul_rn(vv - recalled, bsig);

  float o = 0.f;
#pragma unroll
  for (int i = 0; i < R; ++i) {
    s[i] = __fadd_rn(s[i], __fmul_rn(sk[r0 + i], delta));
    S[static_cast<int64_t>(r0 + i) * DIM + col] = s[i];
    o = fmaf(s[i], sq[r0 + i], o);
  }
  __syncthreads();
  red[rg][col_l] = o;
  __syncthreads();
  if (tid < kCols) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kRowGroups; ++w) t += red[w][tid];
    p.out[static_cast<int64_t>(b) * p.out_bs + static_cast<int64_t>(hv) * DIM + tile * kCols + tid] = t;
  }
  if (p.trace) {
    __syncthreads();
    trace_exit(p.trace);
  }
}

// One CTA of 256 threads per (sequence, value head) of dim 128, for batches
// with enough heads to fill the GPU: thread t owns column t % 128 of the
// head's state, rows [64 (t / 128), +64), in registers, so every warp reads
// and writes whole 512-byte rows and the step needs four barriers instead of
// the column-tiled kernel's per-tile reductions.  Same arithmetic per
// element as gdn_decode_kernel (only the row-group partition of the column
// sums differs: two halves of 64 rows instead of 16 groups of 8).
constexpr int kHeadDim = 128;
constexpr int kHeadHalves = kThreads / kHeadDim;
constexpr int kHeadRows = kHeadDim / kHeadHalves;

template <typename T>
__global__ void __launch_bounds__(kThreads) gdn_head_kernel(const __grid_constant__ GdnParams p) {
  __shared__ float sq[kHeadDim], sk[kHeadDim], red[kHeadHalves][kHeadDim];
  __shared__ float s_decay, s_bsig;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = tid % kHeadDim, half = tid / kHeadDim, r0 = half * kHeadRows;
  const int hv = blockIdx.x % p.heads_v, b = blockIdx.x / p.heads_v;
  const int hk = hv % p.heads_k;
  trace_entry(p.trace);
  float* S = p.state + (static_cast<int64_t>(b) * p.heads_v + hv) * kHeadDim * kHeadDim;
  pdl_launch_dependents();
  pdl_wait();
  trace_waited(p.trace);
  float s[kHeadRows];
#pragma unroll
  for (int i = 0; i < kHeadRows; ++i) s[i] = S[static_cast<int64_t>(r0 + i) * kHeadDim + c];
  if (warp < 2) {  // normalised q (x scale) and k of key head hk
    const void* src = warp == 0 ? p.q : p.k;
    const int64_t off = static_cast<int64_t>(b) * (warp == 0 ? p.q_bs : p.k_bs) + static_cast<int64_t>(hk) * kHeadDim;
    float vals[kHeadDim / 32];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kHeadDim / 32; ++i) {
      vals[i] = load_elem<T>(src, off + lane + 32 * i);
      ss = fmaf(vals[i], vals[i], ss);
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + p.eps);
    float* dst = warp == 0 ? sq : sk;
#pragma unroll
    for (int i = 0; i < kHeadDim / 32; ++i)
      dst[lane + 32 * i] = warp == 0 ? __fmul_rn(__fmul_rn(vals[i], r), p.scale) : __fmul_rn(vals[i], r);
  } else if (tid == 64) {
    s_decay = expf(p.g[static_cast<int64_t>(b) * p.g_bs + hv]);
    s_bsig = sigmoid_f(p.beta[static_cast<int64_t>(b) * p.beta_bs + hv]);
  }
  __syncthreads();
  trace_ready(p.trace);
  const float decay = s_decay, bsig = s_bsig;
  float rec = 0.f;
#pragma unroll
  for (int i = 0; i < kHeadRows; ++i) {
    s[i] = __fmul_rn(s[i], decay);
    rec = fmaf(s[i], sk[r0 + i], rec);
  }
  red[half][c] = rec;
  __syncthreads();
  float recalled = 0.f;
#pragma unroll
  for (int h = 0; h < kHeadHalves; ++h) recalled += red[h][c];
  const float vv = load_elem<T>(p.v, static_cast<int64_t>(b) * p.v_bs + static_cast<int64_t>(hv) * kHeadDim + c);
  const float delta = __fmul_rn(vv - recalled, bsig);
  float o = 0.f;
#pragma unroll
  for (int i = 0; i < kHeadRows; ++i) {
    s[i] = __fadd_rn(s[i], __fmul_rn(sk[r0 + i], delta));
    S[static_cast<int64_t>(r0 + i) * kHeadDim + c] = s[i];
    o = fmaf(s[i], sq[r0 + i], o);
  }
  __syncthreads();  // every thread has read red[][] above
  red[half][c] = o;
  __syncthreads();
  if (half == 0) {
    float t = 0.f;
#pragma unroll
    for (int h = 0; h < kHeadHalves; ++h) t += red[h][c];
    p.out[static_cast<int64_t>(b) * p.out_bs + static_cast<int64_t>(hv) * kHeadDim + c] = t;
  }
  if (p.trace) {
    __syncthreads();
    trace_exit(p.trace);
  }
}

// Prefill scan: the gated delta rule over `len` consecutive tokens of every
// (sequence, value head), one CTA each, with the 128 x 128 state held in the
// registers of its 256 threads for the whole scan (read once, written once)
// instead of going through HBM once per token.  Token i's q / k / v / g /
// beta sit `tok_*` elements after token i - 1's (the batch strides still
// apply), its output o_i tok_out after o_{i-1}.  Per token the arithmetic is
// gdn_head_kernel's, in the same order, so L scanned tokens give the same
// bits as L steps of the one-CTA-per-head decode.  The next token's inputs
// are loaded while the current one computes.
template <typename T>
__global__ void __launch_bounds__(kThreads) gdn_prefill_kernel(const __grid_constant__ GdnParams p,
                                                               const __grid_constant__ GdnScan sc) {
  __shared__ float sq[kHeadDim], sk[kHeadDim], red[kHeadHalves][kHeadDim];
  __shared__ float s_decay, s_bsig;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = tid % kHeadDim, half = tid / kHeadDim, r0 = half * kHeadRows;
  const int hv = blockIdx.x % p.heads_v, b = blockIdx.x / p.heads_v;
  const int hk = hv % p.heads_k;
  float* S = p.state + (static_cast<int64_t>(b) * p.heads_v + hv) * kHeadDim * kHeadDim;
  float s[kHeadRows];
#pragma unroll
  for (int i = 0; i < kHeadRows; ++i) s[i] = S[static_cast<int64_t>(r0 + i) * kHeadDim + c];
  // the next token's inputs: warps 0 / 1 hold its q / k, thread 64 its g and
  // beta logit, every thread its v column
  float vals[kHeadDim / 32];
  float gv = 0.f, bv = 0.f, vv = 0.f;
  auto load_token = [&](int i) {
    if (warp < 2) {
      const void* src = warp == 0 ? p.q : p.k;
      const int64_t off = static_cast<int64_t>(b) * (warp == 0 ? p.q_bs : p.k_bs) +
                          static_cast<int64_t>(i) * (warp == 0 ? sc.tok_q : sc.tok_k) +
                          static_cast<int64_t>(hk) * kHeadDim;
#pragma unroll
      for (int j = 0; j < kHeadDim / 32; ++j) vals[j] = load_elem<T>(src, off + lane + 32 * j);
    } else if (tid == 64) {
      gv = p.g[static_cast<int64_t>(b) * p.g_bs + static_cast<int64_t>(i) * sc.tok_g + hv];
      bv = p.beta[static_cast<int64_t>(b) * p.beta_bs + static_cast<int64_t>(i) * sc.tok_beta + hv];
    }
    vv = load_elem<T>(p.v, static_cast<int64_t>(b) * p.v_bs + static_cast<int64_t>(i) * sc.tok_v +
                               static_cast<int64_t>(hv) * kHeadDim + c);
  };
  if (sc.len > 0) load_token(0);
  for (int i = 0; i < sc.len; ++i) {
    // every thread has passed the previous token's third barrier, after its
    // last reads of sq / sk / s_decay / s_bsig, so they are free to overwrite
    if (warp < 2) {  // normalised q (x scale) and k
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < kHeadDim / 32; ++j) ss = fmaf(vals[j], vals[j], ss);
      ss = warp_sum(ss);
      const float r = 1.0f / sqrtf(ss + p.eps);
      float* dst = warp == 0 ? sq : sk;
#pragma unroll
      for (int j = 0; j < kHeadDim / 32; ++j)
        dst[lane + 32 * j] = warp == 0 ? __fmul_rn(__fmul_rn(vals[j], r), p.scale) : __fmul_rn(vals[j], r);
    } else if (tid == 64) {
      s_decay = expf(gv);
      s_bsig = sigmoid_f(bv);
    }
    const float v_now = vv;
    __syncthreads();
    if (i + 1 < sc.len) load_token(i + 1);  // in flight while this token computes
    const float decay = s_decay, bsig = s_bsig;
    float rec = 0.f;
#pragma unroll
    for (int j = 0; j < kHeadRows; ++j) {
      s[j] = __fmul_rn(s[j], decay);
      rec = fmaf(s[j], sk[r0 + j], rec);
    }
    red[half][c] = rec;
    __syncthreads();
    float recalled = 0.f;
#pragma unroll
    for (int h = 0; h < kHeadHalves; ++h) recalled += red[h][c];
    const float delta = __fmul_rn(v_now - recalled, bsig);
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < kHeadRows; ++j) {
      s[j] = __fadd_rn(s[j], __fmul_rn(sk[r0 + j], delta));
      o = fmaf(s[j], sq[r0 + j], o);
    }
    __syncthreads();  // every thread has read red[][], sq and sk above
    red[half][c] = o;
    __syncthreads();
    if (half == 0) {
      float t = 0.f;
#pragma unroll
      for (int h = 0; h < kHeadHalves; ++h) t += red[h][c];
      p.out[static_cast<int64_t>(b) * p.out_bs + static_cast<int64_t>(i) * sc.tok_out +
            static_cast<int64_t>(hv) * kHeadDim + c] = t;
    }
    // red[][] is next written after the next token's first barrier, which
    // every thread reaches only after its reads above
  }
#pragma unroll
  for (int j = 0; j < kHeadRows; ++j) S[static_cast<int64_t>(r0 + j) * kHeadDim + c] = s[j];
}

template <typename T>
cudaError_t launch_dim(const GdnParams& p, cudaLaunchConfig_t& cfg) {
  switch (p.dim) {
    case 64: return ::bt::launch_ex(&cfg, gdn_decode_kernel<T, 4>, p);
    case 128: return ::bt::launch_ex(&cfg, gdn_decode_kernel<T, 8>, p);
    default: return ::bt::launch_ex(&cfg, gdn_decode_kernel<T, 16>, p);
  }
}

}  // namespace

int gdn_prefill_launch(const GdnParams& p, const GdnScan& sc, cudaStream_t stream) {
  if (p.dim != kHeadDim) return fail(BT_ERR_UNSUPPORTED, "gdn_prefill serves head dim %d, got %d", kHeadDim, p.dim);
  if (p.heads_k <= 0 || p.heads_v <= 0 || p.heads_v % p.heads_k != 0)
    return fail(BT_ERR_INVALID, "gdn_prefill: value heads (%d) must be a positive multiple of key heads (%d)",
                p.heads_v, p.heads_k);
  if (p.batch <= 0 || sc.len < 0) return fail(BT_ERR_INVALID, "gdn_prefill: batch must be positive, steps >= 0");
  if (static_cast<int64_t>(p.batch) * p.heads_v > (1LL << 31) - 1)
    return fail(BT_ERR_UNSUPPORTED, "gdn_prefill: too many heads");
  if (sc.len == 0) return BT_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.batch) * p.heads_v);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  const cudaError_t e = p.in_dtype == BT_BF16 ? ::bt::launch_ex(&cfg, gdn_prefill_kernel<__nv_bfloat16>, p, sc)
                                              : ::bt::launch_ex(&cfg, gdn_prefill_kernel<float>, p, sc);
  return e == cudaSuccess ? BT_OK : fail_cuda(e, "gdn_prefill launch");
}

int gdn_decode_launch(const GdnParams& p, cudaStream_t stream, bool pdl) {
  if (p.dim != 64 && p.dim != 128 && p.dim != 256)
    return fail(BT_ERR_UNSUPPORTED, "gdn_decode serves dim 64, 128 or 256, got %d", p.dim);
  if (p.heads_k <= 0 || p.heads_v <= 0 || p.heads_v % p.heads_k != 0)
    return fail(BT_ERR_INVALID, "gdn_decode: value heads (%d) must be a positive multiple of key heads (%d)",
                p.heads_v, p.heads_k);
  if (p.batch <= 0) return fail(BT_ERR_INVALID, "gdn_decode: batch must be positive");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.batch) * p.heads_v * (p.dim / kCols));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e;
  if (p.dim == kHeadDim && static_cast<int64_t>(p.batch) * p.heads_v >= 4LL * sm_count()) {
    // enough heads for every SM: one CTA per head
    cfg.gridDim = dim3(static_cast<unsigned>(p.batch) * p.heads_v);
    e = p.in_dtype == BT_BF16 ? ::bt::launch_ex(&cfg, gdn_head_kernel<__nv_bfloat16>, p)
                              : ::bt::launch_ex(&cfg, gdn_head_kernel<float>, p);
  } else {
    e = p.in_dtype == BT_BF16 ? launch_dim<__nv_bfloat16>(p, cfg) : launch_dim<float>(p, cfg);
  }
  if (e != cudaSuccess) return fail_cuda(e, "gdn_decode launch");
  return BT_OK;
}

}  // namespace bt
