// Fused per-layer pieces of the Qwen3.6-MoE (qwen35moe) decode step.
//
// gdn_gated_step_kernel: the GDN mixer of model/qwen36_moe.py:459-483 from
// the conv output on, for B sequences: the decay g = a * softplus(alpha +
// dt_bias) from the alpha logits, the gated delta rule of
// _torch_gdn_decode (backends.py:241-271) with the state updated in place,
// then the output gate rms_norm(o, ssm_norm) * silu(z), written as the three
// bf16 planes the out-projection (bt_linear_rows) reads.  One CTA of 256
// threads per (sequence, value head): thread t owns column t % 128 of the
// head's 128 x 128 state, rows [64 (t / 128), 64 (t / 128) + 64), held in
// registers, so the state is read and written once per step in 512-byte
// rows; the column sums S^T k and S^T q add the two row halves in shared
// memory, and the gated norm's sum of squares is one block reduction.  It
// replaces the separate decay arithmetic, recurrence, norm, SiLU, product and
// plane-split launches of the unfused layer.  With steps > 1 the same CTA
// scans `steps` consecutive tokens of its sequence (a prefill chunk, token
// major) with the state kept in registers throughout: the per-token
// arithmetic is the decode step's, the state is read and written once.
//
// add_rms_norm_planes_kernel: h = a + b; y = rms_norm(h) * w
// (backends.py:229-238) and y's three bf16 planes (y = hi + mid + lo) in the
// same pass, so the projections that read y need no separate split.
#include "errors.h"
#include "norm_planes.cuh"
#include "qwen36_layer.cuh"

namespace bt {
namespace {

template <int DIM>
__device__ __forceinline__ float block_total(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kGdnStepThreads / 32; ++i) t += scratch[i];
  return t;
}

template <int DIM>
__global__ void __launch_bounds__(kGdnStepThreads) gdn_gated_step_kernel(const __grid_constant__ GdnStepParams p) {
  constexpr int HALF = kGdnStepThreads / DIM;  // row groups
  constexpr int R = DIM / HALF;                 // rows per thread
  static_assert(DIM * HALF == kGdnStepThreads, "one thread per (column, row group)");
  __shared__ float sq[DIM], sk[DIM], red[HALF][DIM];
  __shared__ float s_decay, s_bsig, scratch[kGdnStepThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = tid % DIM, half = tid / DIM, r0 = half * R;
  const int hv = blockIdx.x % p.heads_v, b = blockIdx.x / p.heads_v;
  const int hk = hv % p.heads_k;
  float* S = p.state + (static_cast<int64_t>(b) * p.heads_v + hv) * DIM * DIM;

  float s[R];
#pragma unroll
  for (int i = 0; i < R; ++i) s[i] = S[static_cast<int64_t>(r0 + i) * DIM + c];

  // The inputs of token j of sequence b sit in row j * batch + b of mixed,
  // ba and z; they are loaded one token ahead: warps 0 / 1 hold q / k, thread
  // 64 the beta and alpha logits, every thread its v column, the threads of
  // row group 0 their z column.
  float vals[DIM / 32];
  float beta_l = 0.f, alpha_l = 0.f, vv = 0.f, zz = 0.f;
  auto load_token = [&](int j) {
    const int64_t r = static_cast<int64_t>(j) * p.batch + b;
    const float* row = p.mixed + r * p.mixed_bs;
    if (warp < 2) {
      const float* src = row + (warp == 0 ? 0 : static_cast<int64_t>(p.heads_k) * DIM) + static_cast<int64_t>(hk) * DIM;
#pragma unroll
      for (int i = 0; i < DIM / 32; ++i) vals[i] = src[lane + 32 * i];
    } else if (tid == 64) {
      const float* ba = p.ba + r * p.ba_bs;
      beta_l = ba[hv];
      alpha_l = ba[p.heads_v + hv];
    }
    vv = row[static_cast<int64_t>(2 * p.heads_k) * DIM + static_cast<int64_t>(hv) * DIM + c];
    if (half == 0) zz = p.z[r * p.z_bs + static_cast<int64_t>(hv) * DIM + c];
  };
  load_token(0);
  for (int j = 0; j < p.steps; ++j) {
    // every thread has passed this token's predecessor's block_total, after
    // its last reads of sq / sk / s_decay / s_bsig, so they are free to overwrite
    if (warp < 2) {  // L2-normalised q (x scale) and k of key head hk
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < DIM / 32; ++i) ss = fmaf(vals[i], vals[i], ss);
      ss = warp_sum(ss);
      const float r = 1.0f / sqrtf(ss + p.l2_eps);
      float* dst = warp == 0 ? sq : sk;
#pragma unroll
      for (int i = 0; i < DIM / 32; ++i)
        dst[lane + 32 * i] = warp == 0 ? __fmul_rn(__fmul_rn(vals[i], r), p.scale) : __fmul_rn(vals[i], r);
    } else if (tid == 64) {
      // decay: a * softplus(alpha + dt_bias) (model/qwen36_moe.py:474-476)
      const float g = __fmul_rn(p.a_log[hv], softplus_f(__fadd_rn(alpha_l, p.dt_bias[hv])));
      s_decay = expf(g);
      s_bsig = sigmoid_f(beta_l);
    }
    const float v_now = vv, z_now = zz;
    __syncthreads();
    if (j + 1 < p.steps) load_token(j + 1);  // in flight while this token computes
    const float decay = s_decay, bsig = s_bsig;
    float rec = 0.f;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      s[i] = __fmul_rn(s[i], decay);
      rec = fmaf(s[i], sk[r0 + i], rec);
    }
    red[half][c] = rec;
    __syncthreads();
    float recalled = 0.f;
#pragma unroll
    for (int h = 0; h < HALF; ++h) recalled += red[h][c];
    const float delta = __fmul_rn(v_now - recalled, bsig);
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      s[i] = __fadd_rn(s[i], __fmul_rn(sk[r0 + i], delta));
      o = fmaf(s[i], sq[r0 + i], o);
    }
    __syncthreads();  // every thread has read red[][] above
    red[half][c] = o;
    __syncthreads();
    float out = 0.f;
#pragma unroll
    for (int h = 0; h < HALF; ++h) out += red[h][c];
    // gated norm: rms_norm(o) * w * silu(z) over the head's DIM outputs
    // (threads of row group 0 hold one output each; the others add zero);
    // block_total's first barrier also orders the reads of red[][] above
    // before the next token's writes
    const float total = block_total<DIM>(half == 0 ? out * out : 0.f, scratch);
    if (half == 0) {
      const float r = 1.0f / sqrtf(total / static_cast<float>(DIM) + p.norm_eps);
      const float y = __fmul_rn(__fmul_rn(__fmul_rn(out, r), p.norm_w[c]), silu_f(z_now));
      float hi, mid, lo;
      split3(y, hi, mid, lo);
      const int64_t width = static_cast<int64_t>(p.heads_v) * DIM;
      __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(p.planes) +
                           (static_cast<int64_t>(j) * p.batch + b) * 3 * width + static_cast<int64_t>(hv) * DIM + c;
      dst[0] = __float2bfloat16_rn(hi);
      dst[width] = __float2bfloat16_rn(mid);
      dst[2 * width] = __float2bfloat16_rn(lo);
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i) S[static_cast<int64_t>(r0 + i) * DIM + c] = s[i];
}

// One block of 256 threads per row, n % 8 == 0 (add_rms_norm_planes_row).
__global__ void __launch_bounds__(256) add_rms_norm_planes_kernel(const float* __restrict__ a,
                                                                   const float* __restrict__ b,
                                                                   const float* __restrict__ w, float* __restrict__ h,
                                                                   float* __restrict__ y, __nv_bfloat16* planes,
                                                                   int n, float eps) {
  __shared__ float scratch[8];
  const int64_t row = blockIdx.x;
  const float* br = b ? b + row * n : nullptr;
  auto b_of = [&](int i0, float (&bb)[8]) {
    const float4 b0 = *reinterpret_cast<const float4*>(br + i0), b1 = *reinterpret_cast<const float4*>(br + i0 + 4);
    bb[0] = b0.x, bb[1] = b0.y, bb[2] = b0.z, bb[3] = b0.w, bb[4] = b1.x, bb[5] = b1.y, bb[6] = b1.z, bb[7] = b1.w;
  };
  add_rms_norm_planes_row(a + row * n, br != nullptr, b_of, w, h ? h + row * n : nullptr, y + row * n,
                          planes + row * 3 * n, n, eps, scratch);
}

}  // namespace

int gdn_gated_step_launch(const GdnStepParams& p, cudaStream_t stream) {
  if (!p.mixed || !p.ba || !p.a_log || !p.dt_bias || !p.state || !p.z || !p.norm_w || !p.planes)
    return fail(BT_ERR_INVALID, "gdn gated step: null pointer");
  if (p.steps < 1) return fail(BT_ERR_INVALID, "gdn gated step: steps must be >= 1");
  if (p.batch < 1 || p.heads_k < 1 || p.heads_v < 1 || p.heads_v % p.heads_k)
    return fail(BT_ERR_INVALID, "gdn gated step: value heads must be a positive multiple of key heads");
  if (p.dim != 128) return fail(BT_ERR_UNSUPPORTED, "gdn gated step serves head dim 128, got %d", p.dim);
  if (static_cast<int64_t>(p.batch) * p.heads_v > (1LL << 31) - 1)
    return fail(BT_ERR_UNSUPPORTED, "gdn gated step: too many heads");
  const int64_t mixed_need = static_cast<int64_t>(2 * p.heads_k + p.heads_v) * p.dim;
  if (p.mixed_bs < mixed_need || p.ba_bs < 2 * p.heads_v || p.z_bs < static_cast<int64_t>(p.heads_v) * p.dim)
    return fail(BT_ERR_INVALID, "gdn gated step: row strides shorter than the rows");
  note_launch();
  gdn_gated_step_kernel<128><<<static_cast<unsigned>(p.batch * p.heads_v), kGdnStepThreads, 0, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BT_OK : fail_cuda(e, "gdn gated step launch");
}

int add_rms_norm_planes(const float* a, const float* b, const float* w, float* h, float* y, void* planes,
                        int64_t rows, int64_t n, float eps, cudaStream_t stream) {
  if (!a || !w || !y || !planes || (b && !h) || rows < 0 || n < 8 || n % 8)
    return fail(BT_ERR_INVALID, "add_rms_norm_planes: bad arguments (n %% 8 == 0)");
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(w) |
       reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(planes)) & 15 ||
      rows > 2147483647LL || n > 2147483647LL)
    return fail(BT_ERR_INVALID, "add_rms_norm_planes: every buffer must be 16-byte aligned");
  if (rows == 0) return BT_OK;
  note_launch();
  add_rms_norm_planes_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(
      a, b, w, h, y, static_cast<__nv_bfloat16*>(planes), static_cast<int>(n), eps);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BT_OK : fail_cuda(e, "add_rms_norm_planes launch");
}

}  // namespace bt
