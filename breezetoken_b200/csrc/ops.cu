// Stand-alone Backend operations (breezetoken/backends.py:28-98) and the
// weight-format kernels: GGUF Q8_0 -> q8 rows repacking, q8 and IQ3_S
// dequantisation, dense (K, N) GEMV, RMSNorm, residual + RMSNorm, SiLU-mul,
// partial RoPE and argmax.  These serve the op-level C ABI; the fused
// decode step uses the GEMV/GDN/attention kernels directly.
#include "errors.h"
#include "ops.cuh"

namespace bt {

__device__ const uint32_t g_iq3s_grid[512] = {
#include "iq3s_grid.inc"
};

namespace {

// ------------------------------------------------------------- repacking
// One thread per 32-weight block: 34 source bytes (fp16 d, 32 x int8) ->
// scale slot + 32 quant bytes of the destination row.
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t rows,
                                   int64_t k, int64_t dst_row0, int64_t dst_row_step, int64_t row_bytes,
                                   int64_t sb) {
  const int64_t nb = k / 32;
  const int64_t total = rows * nb;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nb, j = i % nb;
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src + i * 34);
    uint8_t* drow = dst + (dst_row0 + r * dst_row_step) * row_bytes;
    reinterpret_cast<uint16_t*>(drow)[j] = s[0];
    uint32_t w[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) w[t] = static_cast<uint32_t>(s[1 + 2 * t]) | (static_cast<uint32_t>(s[2 + 2 * t]) << 16);
    uint4* q = reinterpret_cast<uint4*>(drow + sb + 32 * j);
    q[0] = make_uint4(w[0], w[1], w[2], w[3]);
    q[1] = make_uint4(w[4], w[5], w[6], w[7]);
    if (j == 0)
      for (int64_t b = 2 * nb; b < sb; ++b) drow[b] = 0;
  }
}

__global__ void dequant_q8_rows_kernel(const uint8_t* __restrict__ w, float* __restrict__ out, int64_t rows,
                                       int64_t k, int64_t row_bytes, int64_t sb) {
  const int64_t total = rows * k;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / k, c = i % k;
    const uint8_t* row = w + r * row_bytes;
    const float d = __half2float(reinterpret_cast<const __half*>(row)[c >> 5]);
    out[i] = static_cast<float>(static_cast<int8_t>(row[sb + c])) * d;
  }
}

// IQ3_S: lane (p, s, l) of a warp decodes the 8 weights
// e = 64p + 32s + 8l + [0, 8) of one 256-weight block
// (quant/dequant.py:164-185).
__global__ void dequant_iq3_s_kernel(const uint8_t* __restrict__ raw, float* __restrict__ out, int64_t n_blocks) {
  __shared__ uint32_t grid_s[512];
  for (int i = threadIdx.x; i < 512; i += blockDim.x) grid_s[i] = g_iq3s_grid[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int p = lane >> 3, s = (lane >> 2) & 1, l = lane & 3;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t blk = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); blk < n_blocks;
       blk += warps) {
    const uint8_t* b = raw + blk * 110;
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(b[0] | (b[1] << 8))));
    const int qs0 = b[2 + p * 16 + s * 8 + 2 * l], qs1 = b[2 + p * 16 + s * 8 + 2 * l + 1];
    const int qh = b[66 + p * 2 + s];
    const int sign = b[74 + p * 8 + s * 4 + l];
    const int sc = b[106 + p];
    const float db = d * static_cast<float>(1 + 2 * (s ? (sc >> 4) : (sc & 0xF)));
    const uint32_t g1 = grid_s[qs0 | (((qh >> (2 * l)) & 1) << 8)];
    const uint32_t g2 = grid_s[qs1 | (((qh >> (2 * l + 1)) & 1) << 8)];
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j] = db * static_cast<float>((g1 >> (8 * j)) & 0xFF) * ((sign >> j) & 1 ? -1.f : 1.f);
      v[4 + j] = db * static_cast<float>((g2 >> (8 * j)) & 0xFF) * ((sign >> (4 + j)) & 1 ? -1.f : 1.f);
    }
    float4* o = reinterpret_cast<float4*>(out + blk * 256 + p * 64 + s * 32 + l * 8);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// ------------------------------------------------------------- dense GEMV
// y[n] = sum_k x[k] W[k][n] for the reference's (K, N) layout; thread per 8
// consecutive columns, 16-byte loads along N.
template <typename T>
__global__ void linear_kn_kernel(const T* __restrict__ w, const float* __restrict__ x, float* __restrict__ y,
                                 int64_t k, int64_t n) {
  const int64_t c0 = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) * 8;
  if (c0 >= n) return;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const bool full = c0 + 8 <= n;
  for (int64_t kk = 0; kk < k; ++kk) {
    const float xv = x[kk];
    const T* row = w + kk * n + c0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (full || c0 + j < n) acc[j] = fmaf(xv, static_cast<float>(row[j]), acc[j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (c0 + j < n) y[c0 + j] = acc[j];
}

// ------------------------------------------------------------- row ops
__device__ float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += scratch[i];
  return t;
}

// One block per row: y = x * rsqrt(mean(x^2) + eps) * w (backends.py:187-189);
// with `b`, first h = a + b (backends.py:229-238).
__global__ void rms_norm_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                const float* __restrict__ w, float* __restrict__ h, float* __restrict__ y,
                                int64_t n, float eps) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const float* ar = a + row * n;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float v = ar[i];
    if (b) {
      v = v + b[row * n + i];
      h[row * n + i] = v;
    }
    ss = fmaf(v, v, ss);
  }
  const float total = block_sum(ss, scratch);
  const float r = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = b ? ar[i] + b[row * n + i] : ar[i];
    y[row * n + i] = __fmul_rn(__fmul_rn(v, r), w[i]);
  }
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ y,
                                int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = silu_f(g[i]) * u[i];
}

// One block per row (backends.py:218-226).
__global__ void rope_kernel(const float* __restrict__ x, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, const int32_t* __restrict__ pos,
                            float* __restrict__ y, int64_t dim, int64_t rope_dim, int64_t cap, int32_t* status) {
  int64_t p = pos[0];
  if (p < 0 || p >= cap) {
    if (threadIdx.x == 0 && blockIdx.x == 0)
      report_status(status, BT_ERR_INVALID, SITE_ROPE_POS, static_cast<int32_t>(p), static_cast<int32_t>(cap));
    p = p < 0 ? 0 : cap - 1;
  }
  const int64_t row = blockIdx.x;
  const float* xr = x + row * dim;
  const int64_t half = rope_dim / 2;
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = xr[i];
    if (i < rope_dim) {
      const float partner = i < half ? -xr[i + half] : xr[i - half];
      v = __fadd_rn(__fmul_rn(v, cos_t[p * rope_dim + i]), __fmul_rn(partner, sin_t[p * rope_dim + i]));
    }
    y[row * dim + i] = v;
  }
}

// Short causal conv of the GDN projection (model/qwen36_moe.py:465-468):
// window = [state (K-1 taps) | entry], out = silu(sum_j window[j] * w[j])
// (products rounded, summed in tap order), state <- window[1:].  One thread
// per (sequence, channel), scanning `steps` tokens (token-major rows:
// token s of sequence b at row s * batch + b) with the window in registers.
__global__ void conv_silu_kernel(const float* __restrict__ entry, float* __restrict__ state,
                                 const float* __restrict__ w, float* __restrict__ out, int64_t steps,
                                 int64_t batch, int64_t channels, int taps) {
  const int64_t total = batch * channels;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = i % channels;
    float* st = state + i * (taps - 1);
    float win[8];
    for (int j = 0; j < taps - 1; ++j) win[j] = st[j];
    for (int64_t s = 0; s < steps; ++s) {
      win[taps - 1] = entry[s * total + i];
      float acc = __fmul_rn(win[0], w[c * taps]);
      for (int j = 1; j < taps; ++j) acc = __fadd_rn(acc, __fmul_rn(win[j], w[c * taps + j]));
      out[s * total + i] = silu_f(acc);
      for (int j = 0; j < taps - 1; ++j) win[j] = win[j + 1];
    }
    for (int j = 0; j < taps - 1; ++j) st[j] = win[j];
  }
}

// Argmax over rows: each block reduces a slice to a packed key, one atomicMax
// per block; the last block of a row writes the index and re-arms the slots.
__global__ void argmax_kernel(const float* __restrict__ x, int64_t n, int32_t* __restrict__ out,
                              unsigned long long* best, uint32_t* counters) {
  __shared__ unsigned long long sk[32];
  const int64_t row = blockIdx.y;
  const float* xr = x + row * n;
  unsigned long long key = 0ull;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t bits = __float_as_uint(xr[i]);
    bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
    const unsigned long long k2 = (static_cast<unsigned long long>(bits) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
    key = k2 > key ? k2 : key;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, key, o);
    key = t > key ? t : key;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sk[warp] = key;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) key = sk[w] > key ? sk[w] : key;
    atomicMax(best + row, key);
    __threadfence();
    if (atomicAdd(counters + row, 1u) == gridDim.x - 1) {
      __threadfence();
      const unsigned long long b = atomicExch(best + row, 0ull);
      out[row] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(b & 0xFFFFFFFFull));
      atomicExch(counters + row, 0u);
    }
  }
}

int grid_for(int64_t work, int threads) {
  const int64_t blocks = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BT_OK : fail_cuda(e, what);
}

}  // namespace

int repack_q8_0(const void* src, void* dst, int64_t rows, int64_t k, int64_t dst_row0, int64_t dst_row_step,
                cudaStream_t stream) {
  if (!src || !dst || rows < 0 || k < 32 || k % 32) return fail(BT_ERR_INVALID, "repack_q8_0: bad arguments (k=%lld)", (long long)k);
  if ((reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 1))
    return fail(BT_ERR_INVALID, "repack_q8_0: dst must be 16-byte and src 2-byte aligned");
  if (rows == 0) return BT_OK;
  const int64_t row_bytes = bt_q8_row_bytes(k);
  ::bt::note_launch();
  repack_q8_0_kernel<<<grid_for(rows * (k / 32), 256), 256, 0, stream>>>(
      static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), rows, k, dst_row0, dst_row_step, row_bytes,
      row_bytes - k);
  return check_launch("repack_q8_0");
}

int dequant_q8_rows(const void* w, float* out, int64_t rows, int64_t k, cudaStream_t stream) {
  if (!w || !out || rows < 0 || k < 32 || k % 32) return fail(BT_ERR_INVALID, "dequant_q8_rows: bad arguments");
  if (rows == 0) return BT_OK;
  const int64_t row_bytes = bt_q8_row_bytes(k);
  ::bt::note_launch();
  dequant_q8_rows_kernel<<<grid_for(rows * k, 256), 256, 0, stream>>>(static_cast<const uint8_t*>(w), out, rows, k,
                                                                     row_bytes, row_bytes - k);
  return check_launch("dequant_q8_rows");
}

int dequant_iq3_s(const void* raw, float* out, int64_t rows, int64_t cols, cudaStream_t stream) {
  if (!raw || !out || rows < 0 || cols % 256) return fail(BT_ERR_INVALID, "dequant_iq3_s: cols must be a multiple of 256");
  if (reinterpret_cast<uintptr_t>(out) & 15) return fail(BT_ERR_INVALID, "dequant_iq3_s: out must be 16-byte aligned");
  const int64_t n_blocks = rows * (cols / 256);
  if (n_blocks == 0) return BT_OK;
  ::bt::note_launch();
  dequant_iq3_s_kernel<<<grid_for(n_blocks * 32, 256), 256, 0, stream>>>(static_cast<const uint8_t*>(raw), out,
                                                                        n_blocks);
  return check_launch("dequant_iq3_s");
}

int linear_kn(const void* w, int w_dtype, const float* x, float* y, int64_t k, int64_t n, cudaStream_t stream) {
  if (!w || !x || !y || k < 1 || n < 1) return fail(BT_ERR_INVALID, "linear_kn: bad arguments");
  const int threads = 128;
  const int blocks = static_cast<int>((n + 8 * threads - 1) / (8 * threads));
  if (w_dtype != BT_BF16 && w_dtype != BT_F32) return fail(BT_ERR_UNSUPPORTED, "linear_kn: weight dtype %d", w_dtype);
  ::bt::note_launch();
  if (w_dtype == BT_BF16)
    linear_kn_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(w), x, y, k, n);
  else
    linear_kn_kernel<float><<<blocks, threads, 0, stream>>>(static_cast<const float*>(w), x, y, k, n);
  return check_launch("linear_kn");
}

int rms_norm(const float* a, const float* b, const float* w, float* h, float* y, int64_t rows, int64_t n, float eps,
             cudaStream_t stream) {
  if (!a || !w || !y || rows < 0 || n < 1 || (b && !h)) return fail(BT_ERR_INVALID, "rms_norm: bad arguments");
  if (rows == 0) return BT_OK;
  if (rows > 2147483647LL) return fail(BT_ERR_UNSUPPORTED, "rms_norm: too many rows");
  ::bt::note_launch();
  rms_norm_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(a, b, w, h, y, n, eps);
  return check_launch("rms_norm");
}

int silu_mul(const float* g, const float* u, float* y, int64_t n, cudaStream_t stream) {
  if (!g || !u || !y || n < 0) return fail(BT_ERR_INVALID, "silu_mul: bad arguments");
  if (n == 0) return BT_OK;
  ::bt::note_launch();
  silu_mul_kernel<<<grid_for(n, 256), 256, 0, stream>>>(g, u, y, n);
  return check_launch("silu_mul");
}

int rope(const float* x, const float* cos_t, const float* sin_t, const int32_t* pos, float* y, int64_t rows,
         int64_t dim, int64_t rope_dim, int64_t cap, cudaStream_t stream) {
  if (!x || !cos_t || !sin_t || !pos || !y || rows < 0 || rope_dim < 0 || rope_dim > dim || rope_dim % 2 || cap < 1)
    return fail(BT_ERR_INVALID, "rope: bad arguments");
  if (rows == 0) return BT_OK;
  ::bt::note_launch();
  rope_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(x, cos_t, sin_t, pos, y, dim, rope_dim, cap, nullptr);
  return check_launch("rope");
}

int conv_silu(const float* entry, float* state, const float* w, float* out, int64_t steps, int64_t batch,
              int64_t channels, int64_t taps, cudaStream_t stream) {
  if (!entry || !state || !w || !out || steps < 1 || batch < 1 || channels < 1 || taps < 2 || taps > 8)
    return fail(BT_ERR_INVALID, "conv_silu: bad arguments (steps >= 1, taps in [2, 8])");
  ::bt::note_launch();
  conv_silu_kernel<<<grid_for(batch * channels, 256), 256, 0, stream>>>(entry, state, w, out, steps, batch, channels,
                                                                          static_cast<int>(taps));
  return check_launch("conv_silu");
}

int argmax(const float* x, int64_t rows, int64_t n, int32_t* out, void* workspace, cudaStream_t stream) {
  if (!x || !out || !workspace || rows < 1 || n < 1 || rows > 65535 || n > 0x7fffffffLL)
    return fail(BT_ERR_INVALID, "argmax: bad arguments");
  auto* best = static_cast<unsigned long long*>(workspace);
  auto* counters = reinterpret_cast<uint32_t*>(best + rows);
  // about four blocks per SM over all rows (a batch's rows share the grid)
  const int64_t per_row = std::max<int64_t>(1, (static_cast<int64_t>(sm_count()) * 4 + rows - 1) / rows);
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, per_row);
  ::bt::note_launch();
  argmax_kernel<<<dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(rows)), 256, 0, stream>>>(x, n, out, best,
                                                                                                     counters);
  return check_launch("argmax");
}

}  // namespace bt
