// Residual add + RMSNorm + bf16 plane split of one row (backends.py:229-238:
// h = a + b, y = rms_norm(h) * w), shared by add_rms_norm_planes_kernel and
// the MoE layer's fused combine (moe.cu): both produce the same bits for the
// same a, b.
#pragma once

#include "common.cuh"

namespace bt {

__device__ __forceinline__ uint32_t bf16_pair_rn(float lo, float hi) {
  const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return a | (b << 16);
}

// v = hi + mid + lo with each remainder exact in f32 (bf16 keeps 8 bits).
__device__ __forceinline__ void split3(float v, float& hi, float& mid, float& lo) {
  hi = __bfloat162float(__float2bfloat16_rn(v));
  const float r1 = v - hi;
  mid = __bfloat162float(__float2bfloat16_rn(r1));
  lo = r1 - mid;
}

// One row of n (n % 8 == 0) by a block of 256 threads: thread t owns the 8
// consecutive elements at 8 t + 2048 i.  b_of(i0, bb) gives b[i0 .. i0+8)
// (has_b false: b = 0, h not written).  Rows of up to 2048 elements are read
// once (kept in registers through the block reduction); longer rows take a
// second pass, which calls b_of again.  `scratch`: 8 floats of shared memory.
template <class BOf>
__device__ __forceinline__ void add_rms_norm_planes_row(const float* __restrict__ ar, bool has_b, BOf b_of,
                                                        const float* __restrict__ w, float* __restrict__ hr,
                                                        float* __restrict__ yr, __nv_bfloat16* pr, int n, float eps,
                                                        float* scratch) {
  const bool one_pass = n <= 8 * static_cast<int>(blockDim.x);
  float v[8];
  float ss = 0.f;
  for (int i0 = 8 * threadIdx.x; i0 < n; i0 += 8 * blockDim.x) {
    const float4 a0 = *reinterpret_cast<const float4*>(ar + i0), a1 = *reinterpret_cast<const float4*>(ar + i0 + 4);
    float x[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    if (has_b) {
      float bb[8];
      b_of(i0, bb);
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = x[j] + bb[j];
      if (hr) {
        *reinterpret_cast<float4*>(hr + i0) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4*>(hr + i0 + 4) = make_float4(x[4], x[5], x[6], x[7]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ss = fmaf(x[j], x[j], ss);
      v[j] = x[j];
    }
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) total += scratch[i];
  const float r = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
  for (int i0 = 8 * threadIdx.x; i0 < n; i0 += 8 * blockDim.x) {
    if (!one_pass) {
      float bb[8];
      if (has_b) b_of(i0, bb);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = has_b ? ar[i0 + j] + bb[j] : ar[i0 + j];
    }
    const float4 w0 = *reinterpret_cast<const float4*>(w + i0), w1 = *reinterpret_cast<const float4*>(w + i0 + 4);
    const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(__fmul_rn(v[j], r), ww[j]);
    *reinterpret_cast<float4*>(yr + i0) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(yr + i0 + 4) = make_float4(o[4], o[5], o[6], o[7]);
    uint32_t pk[3][4];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      float h0, m0, l0, h1, m1, l1;
      split3(o[j], h0, m0, l0);
      split3(o[j + 1], h1, m1, l1);
      pk[0][j / 2] = bf16_pair_rn(h0, h1);
      pk[1][j / 2] = bf16_pair_rn(m0, m1);
      pk[2][j / 2] = bf16_pair_rn(l0, l1);
    }
#pragma unroll
    for (int q = 0; q < 3; ++q)
      *reinterpret_cast<uint4*>(pr + static_cast<int64_t>(q) * n + i0) =
          make_uint4(pk[q][0], pk[q][1], pk[q][2], pk[q][3]);
  }
}

}  // namespace bt
