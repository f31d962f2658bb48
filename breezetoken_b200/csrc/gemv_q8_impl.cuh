// Device code of the Q8_0 GEMV (gemv_q8.cuh), specialised at compile time on
// its prologue and epilogue.
//
// A decode step launches ~120 short kernels; each starts with a cold
// instruction cache, and a taken branch to code that has not been fetched
// yet costs an L2 round trip.  So every (prologue, epilogue) pair the step
// uses is its own kernel with straight-line code for exactly that pair, and
// the launch table (launch_kind) is instantiated per pair in the
// gemv_q8_k_*.cu files, which compile in parallel.
#pragma once

#include <cuda_fp16.h>

#include "errors.h"
#include "gemv_q8.cuh"

namespace bt {
namespace gemv_detail {

// L2 prefetch issue granularity (one cp.async.bulk.prefetch per piece).
constexpr int64_t kPrefetchPiece = 16 * 1024;
// float4 per thread per vector in the prologue: K <= 4 * 256 * kMaxF4.
constexpr int kMaxF4 = 4;
// Dynamic shared memory the kernels may use (activations of 8 vectors at K = 4096).
constexpr int kMaxDynSmem = 120 * 1024;

__device__ __forceinline__ float4 f4_mul(float4 a, float4 b) {
  return make_float4(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z), __fmul_rn(a.w, b.w));
}
__device__ __forceinline__ float4 f4_scale(float4 a, float r) {
  return make_float4(__fmul_rn(a.x, r), __fmul_rn(a.y, r), __fmul_rn(a.z, r), __fmul_rn(a.w, r));
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 255u) | ((static_cast<uint32_t>(b) & 255u) << 8) |
         ((static_cast<uint32_t>(c) & 255u) << 16) | ((static_cast<uint32_t>(d) & 255u) << 24);
}

// Power-of-two fixed-point scale of a block with max |x| = m: inv = 2^e with
// m * 2^e < 2^22 <= 2 m * 2^e, and sx = 2^-e.  Scaling by inv is exact, and
// inv * sx == 1 exactly.  Blocks with m < 2^-105 (all-zero ones included)
// encode as zero.
__device__ __forceinline__ void block_scale(float m, float& inv, float& sx) {
  const uint32_t be = (__float_as_uint(m) >> 23) & 255u;  // biased exponent; m >= 0
  const bool ok = be >= 22u;
  inv = ok ? __uint_as_float((275u - be) << 23) : 0.f;
  sx = ok ? __uint_as_float((be - 21u) << 23) : 0.f;
}

// X = rint(x * inv), |X| <= 2^22, as three signed base-256 digits.
__device__ __forceinline__ void encode_digits(float x, float inv, int& d2, int& d1, int& d0) {
  const int X = __float2int_rn(x * inv);
  d0 = ((X + 128) & 255) - 128;
  const int x1 = (X - d0) >> 8;
  d1 = ((x1 + 128) & 255) - 128;
  d2 = (x1 - d1) >> 8;
}

// ------------------------------------------------------------------ prologue
// Builds each activation vector and encodes it for the dp4a inner loop.
// Thread t owns float4 number f = t + 256*i of the vector; every global load
// of the prologue (x, residual, norm weights or the embedding row) is issued
// before any is used, at clamped indices (entries past the vector are zeroed
// afterwards), so the loads carry no control dependence.  A 32-element block
// is 8 consecutive float4 = 8 consecutive lanes, so its max is 3
// xor-shuffles and the digits go straight from registers to shared memory.
template <int PRO, int NV, int NIT>
__device__ __forceinline__ void gemv_prologue(const GemvQ8Params& p, uint8_t* xd, float* sx, float* scratch) {
  const int tid = threadIdx.x;
  const int K = p.k, nf4 = K >> 2, nb = K >> 5, J = (K + 511) / 512;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll(NV <= 2 ? NV : 1)
  for (int v = 0; v < NV; ++v) {
    float4 h[NIT], a2[NIT], w4[NIT];
    if constexpr (PRO == PRO_EMBED_NORM) {
      int64_t tok = p.tokens[v];
      if (tok < 0 || tok >= p.embed_rows) {
        if (tid == 0) report_status(p.status, BT_ERR_INVALID, SITE_EMBED_TOKEN, static_cast<int32_t>(tok), v);
        tok = 0;
      }
      const uint8_t* erow = p.embed + tok * static_cast<int64_t>(p.row_bytes);
      uint32_t q[NIT];
      float d[NIT];
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        const int fc = min(tid + kConsumerThreads * i, nf4 - 1);
        d[i] = __half2float(reinterpret_cast<const __half*>(erow)[fc >> 3]);
        q[i] = *reinterpret_cast<const uint32_t*>(erow + p.sb + 4 * fc);
        w4[i] = reinterpret_cast<const float4*>(p.norm_w)[fc];
      }
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        h[i] = make_float4(static_cast<float>(static_cast<int8_t>(q[i] & 255)) * d[i],
                           static_cast<float>(static_cast<int8_t>((q[i] >> 8) & 255)) * d[i],
                           static_cast<float>(static_cast<int8_t>((q[i] >> 16) & 255)) * d[i],
                           static_cast<float>(static_cast<int8_t>(q[i] >> 24)) * d[i]);
        a2[i] = zero4;
      }
    } else {
      const float4* x4 = reinterpret_cast<const float4*>(p.x + v * p.x_bs);
      const float4* x24 = reinterpret_cast<const float4*>(p.x2 + v * p.x2_bs);
      const float4* n4 = reinterpret_cast<const float4*>(p.norm_w);
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        const int fc = min(tid + kConsumerThreads * i, nf4 - 1);
        if constexpr (PRO == PRO_SILU_PAIR) {
          // interleaved (gate, up) pairs: float4s 2fc and 2fc+1 give x[4fc .. 4fc+3]
          h[i] = x4[2 * fc];
          a2[i] = x4[2 * fc + 1];
        } else {
          h[i] = x4[fc];
          a2[i] = (PRO == PRO_RESID_NORM || PRO == PRO_GATED_NORM) ? x24[fc] : zero4;
        }
        if constexpr (PRO == PRO_RESID_NORM)
          w4[i] = n4[fc];
        else if constexpr (PRO == PRO_GATED_NORM)
          w4[i] = n4[fc % (p.group >> 2)];
        else
          w4[i] = zero4;
      }
    }
#pragma unroll
    for (int i = 0; i < NIT; ++i)
      if (tid + kConsumerThreads * i >= nf4) h[i] = a2[i] = w4[i] = zero4;
    if (p.trace && v == 0) trace_loaded(p.trace, h[NIT - 1].x + a2[NIT - 1].x + w4[NIT - 1].x);

    if constexpr (PRO == PRO_SILU_PAIR) {
#pragma unroll
      for (int i = 0; i < NIT; ++i)
        h[i] = make_float4(silu_f(h[i].x) * h[i].y, silu_f(h[i].z) * h[i].w, silu_f(a2[i].x) * a2[i].y,
                           silu_f(a2[i].z) * a2[i].w);
    }
    if constexpr (PRO == PRO_RESID_NORM || PRO == PRO_EMBED_NORM) {
      // residual add (the sum is the new residual stream, stored by CTA 0),
      // then RMSNorm over the whole vector
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        const int f = tid + kConsumerThreads * i;
        if constexpr (PRO == PRO_RESID_NORM)
          h[i] = make_float4(h[i].x + a2[i].x, h[i].y + a2[i].y, h[i].z + a2[i].z, h[i].w + a2[i].w);
        if (blockIdx.x == 0 && f < nf4) reinterpret_cast<float4*>(p.h_out + static_cast<int64_t>(v) * K)[f] = h[i];
        ss = fmaf(h[i].x, h[i].x, ss);
        ss = fmaf(h[i].y, h[i].y, ss);
        ss = fmaf(h[i].z, h[i].z, ss);
        ss = fmaf(h[i].w, h[i].w, ss);
      }
      const float total = group_sum<1>(ss, scratch, kConsumerWarps, kConsumerThreads);
      const float r = 1.0f / sqrtf(total / static_cast<float>(K) + p.eps);
#pragma unroll
      for (int i = 0; i < NIT; ++i) h[i] = f4_mul(f4_scale(h[i], r), w4[i]);
    } else if constexpr (PRO == PRO_GATED_NORM) {
      // per-group RMSNorm (a group of G elements = G/4 consecutive lanes of
      // one warp, G = 64 or 128) times the norm weight and silu(z)
      const int lanes = p.group >> 2;
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        float ss = fmaf(h[i].x, h[i].x, fmaf(h[i].y, h[i].y, fmaf(h[i].z, h[i].z, h[i].w * h[i].w)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float t = __shfl_xor_sync(0xffffffffu, ss, o);
          ss = o < lanes ? ss + t : ss;
        }
        const float r = 1.0f / sqrtf(ss / static_cast<float>(p.group) + p.eps);
        h[i] = f4_mul(f4_mul(f4_scale(h[i], r), w4[i]), a2[i]);
      }
    }

    // ---- encode: block max over 8 lanes, digits from registers
    uint8_t* xdv = xd + static_cast<int64_t>(v) * J * 1536;
#pragma unroll
    for (int i = 0; i < NIT; ++i) {
      const int f = tid + kConsumerThreads * i;
      float m = fmaxf(fmaxf(fabsf(h[i].x), fabsf(h[i].y)), fmaxf(fabsf(h[i].z), fabsf(h[i].w)));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      float inv, scale;
      block_scale(m, inv, scale);
      int a[4], b[4], c[4];
      encode_digits(h[i].x, inv, a[0], b[0], c[0]);
      encode_digits(h[i].y, inv, a[1], b[1], c[1]);
      encode_digits(h[i].z, inv, a[2], b[2], c[2]);
      encode_digits(h[i].w, inv, a[3], b[3], c[3]);
      if (f < nf4) {
        const int ch = f >> 2;  // 16-element chunk
        uint32_t* w = reinterpret_cast<uint32_t*>(xdv + ((ch >> 5) * 96 + (ch & 31)) * 16) + (f & 3);
        w[0] = pack4(a[0], a[1], a[2], a[3]);
        w[32 * 4] = pack4(b[0], b[1], b[2], b[3]);
        w[64 * 4] = pack4(c[0], c[1], c[2], c[3]);
        if ((f & 7) == 0) sx[v * nb + (f >> 3)] = scale;
      }
    }
  }
}

// ------------------------------------------------------------------ epilogue
// Operands of the GDN in-projection epilogue for one row: the conv window
// (taps <= 3) and conv weights (conv_k <= 4) of a qkv channel, or a_log and
// dt_bias of an alpha row.  Batches of <= 2 vectors load them before the
// row's dot products, so their latency hides behind the math.
struct EpiOperands {
  float cs[3], cw[4], a_log, dt_bias;
};

__device__ __forceinline__ void gdn_operands(const GemvQ8Params& p, int v, int64_t r, EpiOperands& o) {
  if (r < p.n_conv) {
    const int taps = p.conv_k - 1;
    const float* cs = p.conv_state + (static_cast<int64_t>(v) * p.n_conv + r) * taps;
    const float* cw = p.conv_w + r * p.conv_k;
#pragma unroll
    for (int t = 0; t < 3; ++t) o.cs[t] = t < taps ? cs[t] : 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) o.cw[t] = t < p.conv_k ? cw[t] : 0.f;
  } else if (r >= p.n_conv + p.n_z && r < p.n_conv + p.n_z + p.n_gh) {
    const int h = static_cast<int>(r - p.n_conv - p.n_z);
    o.a_log = p.a_log[h];
    o.dt_bias = p.dt_bias[h];
  }
}

// Causal conv window + SiLU of conv channel ch with its new input a
// (model/layers.py:90-93); shifts the channel's conv state.
__device__ __forceinline__ float conv_silu(const GemvQ8Params& p, int v, int64_t ch, float a, const EpiOperands& o) {
  const int taps = p.conv_k - 1;
  float sum = 0.f;
#pragma unroll
  for (int t = 0; t < 3; ++t)
    if (t < taps) sum = __fadd_rn(sum, __fmul_rn(o.cs[t], o.cw[t]));
  float last = 0.f;
#pragma unroll
  for (int t = 0; t < 4; ++t)
    if (t == taps) last = o.cw[t];
  sum = __fadd_rn(sum, __fmul_rn(a, last));
  float* cs = p.conv_state + (static_cast<int64_t>(v) * p.n_conv + ch) * taps;
#pragma unroll
  for (int t = 0; t < 3; ++t)
    if (t + 1 < taps) cs[t] = o.cs[t + 1];
  cs[taps - 1] = a;
  return silu_f(sum);
}

// GDN in-projection epilogue of row r (value a): conv + SiLU of a qkv
// channel, silu(z), the decay g = a_log * softplus(alpha + dt_bias)
// (model/layers.py:99-103), beta logits as they are.
__device__ __forceinline__ void gdn_epilogue(const GemvQ8Params& p, int v, int64_t r, float a,
                                             const EpiOperands& o) {
  float* y = p.y + static_cast<int64_t>(v) * p.y_stride;
  if (r < p.n_conv) {
    y[r] = conv_silu(p, v, r, a, o);
  } else if (r < p.n_conv + p.n_z) {
    y[r] = silu_f(a);
  } else if (r < p.n_conv + p.n_z + p.n_gh) {
    y[r] = o.a_log * softplus_f(a + o.dt_bias);
  } else {
    y[r] = a;
  }
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  return v;
}

// ------------------------------------------------------------------ weights
// Weight stream: 16 bytes of int8 quants and the fp16 scale of their block,
// read once without L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned short ldg_u16(const uint8_t* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
// Bulk prefetch of global bytes into L2 (no shared memory, no completion).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// The weights of one row group as one lane holds them: chunk j of row r is
// bytes [16c, 16c + 16) of the row's quants, c = lane + 32 j.
template <int GR, int J>
struct Tile {
  uint4 q[GR][J];
  unsigned short s[GR][J];
};

template <int GR, int J>
__device__ __forceinline__ void load_tile(Tile<GR, J>& t, const GemvQ8Params& p, int64_t r0, int nr, int lane,
                                          int nchunks) {
#pragma unroll
  for (int r = 0; r < GR; ++r) {
    const uint8_t* row = p.w + (r0 + r) * static_cast<int64_t>(p.row_bytes);
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      if (r < nr && c < nchunks) {
        t.q[r][j] = ldg_stream(row + p.sb + 16 * c);
        t.s[r][j] = ldg_u16(row + 2 * (c >> 1));
      } else {
        t.q[r][j] = make_uint4(0u, 0u, 0u, 0u);
        t.s[r][j] = 0;
      }
    }
  }
}

// Finish row `row` of vector v with value c (every epilogue but the SiLU pair).
template <int EPI, int NV, bool EPF>
__device__ __forceinline__ void finish_row(const GemvQ8Params& p, int v, int64_t row, float c,
                                           const EpiOperands* eo, unsigned long long (&best)[NV]) {
  if constexpr (EPI == EPI_STORE) {
    p.y[static_cast<int64_t>(v) * p.y_stride + row] = c;
  } else if constexpr (EPI == EPI_ARGMAX) {
    if (p.y) p.y[static_cast<int64_t>(v) * p.y_stride + row] = c;
    const unsigned long long key = argmax_key(c, row);
    best[v] = key > best[v] ? key : best[v];
  } else if constexpr (EPI == EPI_GDN_IN) {
    if constexpr (EPF) {
      gdn_epilogue(p, v, row, c, eo[v]);
    } else {
      EpiOperands o;
      gdn_operands(p, v, row, o);
      gdn_epilogue(p, v, row, c, o);
    }
  }
}

// Per-lane partial dot products of a row group with the NV encoded vectors
// (summed over the lane's chunks; the warp reduction follows).
template <int NV, int GR, int J>
__device__ __forceinline__ void tile_dot(const Tile<GR, J>& t, int lane, int nchunks, int nb, const uint4* xd4,
                                         const float* sx, float (&acc)[GR][NV]) {
#pragma unroll
  for (int r = 0; r < GR; ++r)
#pragma unroll
    for (int v = 0; v < NV; ++v) acc[r][v] = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = lane + 32 * j;
    if (c < nchunks) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const uint4 d2 = xd4[(v * J + j) * 96 + lane];
        const uint4 d1 = xd4[(v * J + j) * 96 + 32 + lane];
        const uint4 d0 = xd4[(v * J + j) * 96 + 64 + lane];
        const float xsc = sx[v * nb + (c >> 1)];
#pragma unroll
        for (int r = 0; r < GR; ++r) {
          const float d = __half2float(__ushort_as_half(t.s[r][j]));
          acc[r][v] = fmaf(d * xsc, dot16_digits(t.q[r][j], d2, d1, d0), acc[r][v]);
        }
      }
    }
  }
}

// 4-row reduce-scatter of vector v: lane l ends with the total of row l >> 3
// (lanes 0, 8, 16, 24 hold rows 0..3; 6 shuffles for the 4 rows).
template <int NV>
__device__ __forceinline__ float reduce_rows4(const float (&acc)[4][NV], int v, int lane) {
  const bool hi16 = (lane & 16) != 0, hi8 = (lane & 8) != 0;
  const float s0 = hi16 ? acc[0][v] : acc[2][v];
  const float s1 = hi16 ? acc[1][v] : acc[3][v];
  const float r0v = __shfl_xor_sync(0xffffffffu, s0, 16);
  const float r1v = __shfl_xor_sync(0xffffffffu, s1, 16);
  const float b0 = (hi16 ? acc[2][v] : acc[0][v]) + r0v;
  const float b1 = (hi16 ? acc[3][v] : acc[1][v]) + r1v;
  const float send = hi8 ? b0 : b1;
  float c = (hi8 ? b1 : b0) + __shfl_xor_sync(0xffffffffu, send, 8);
  c += __shfl_xor_sync(0xffffffffu, c, 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

template <int EPI, int NV, int GR, int J>
__device__ __forceinline__ void process_tile(const Tile<GR, J>& t, const GemvQ8Params& p, int64_t r0, int nr,
                                             int lane, int nchunks, const uint4* xd4, const float* sx,
                                             unsigned long long (&best)[NV]) {
  const int nb = p.k >> 5;
  // GDN epilogue operands of the row this lane finishes, in flight during the math
  constexpr bool EPF = EPI == EPI_GDN_IN && NV <= 2;
  EpiOperands eo[EPF ? NV : 1];
  if constexpr (EPF) {
    const int my_r = GR == 4 ? (lane >> 3) : 0;
    const bool mine = GR == 4 ? (lane & 7) == 0 : lane == 0;
    if (mine && my_r < nr)
#pragma unroll
      for (int v = 0; v < NV; ++v) gdn_operands(p, v, r0 + my_r, eo[v]);
  }
  float acc[GR][NV];
  tile_dot<NV, GR, J>(t, lane, nchunks, nb, xd4, sx, acc);

  if constexpr (GR == 4) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const float c = reduce_rows4<NV>(acc, v, lane);
      const int lr = lane >> 3;  // row held by lanes 0, 8, 16, 24
      if constexpr (EPI == EPI_SILU_PAIR) {
        // rows (2j, 2j+1) = (gate_j, up_j): lanes 0 and 16 hold the gates
        const float up = __shfl_down_sync(0xffffffffu, c, 8);
        if ((lane & 15) == 0 && lr + 1 < nr) {
          const int64_t pair = (r0 + lr) >> 1;
          p.y[static_cast<int64_t>(v) * p.y_stride + pair] = silu_f(c) * up;
        }
      } else {
        if ((lane & 7) == 0 && lr < nr) finish_row<EPI, NV, EPF>(p, v, r0 + lr, c, eo, best);
      }
    }
  } else {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
#pragma unroll
      for (int r = 0; r < GR; ++r) {
        const float c = warp_sum(acc[r][v]);
        if (lane == 0 && r < nr) finish_row<EPI, NV, EPF>(p, v, r0 + r, c, eo, best);
      }
    }
  }
}

// ------------------------------------------------------------------ kernel
// One CTA (or two, for long matrices) per SM streams a contiguous range of
// rows.  Warp w takes row groups w, w+8, ...; each warp double-buffers its
// groups in registers (the load of group g+8 is in flight while group g is
// computed).  Before the dependency wait -- weights never depend on earlier
// kernels -- the CTA prefetches the head of its weight slice into L2 and
// each warp loads its first two groups into registers, so a short slice
// needs no memory round trip after the wait.  Past the prefetched head, each
// warp keeps a bulk L2 prefetch running two groups ahead of its loads.
template <int PRO, int EPI, int NV, int GR, int J>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_q8_kernel(const __grid_constant__ GemvQ8Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  float* scratch = reinterpret_cast<float*>(smem);
  unsigned long long* amax = reinterpret_cast<unsigned long long*>(scratch + 64);
  const XLayout xl = gemv_x_layout(p.k, NV);
  uint8_t* xd = smem + GemvSmem::kHeader + xl.xd;
  float* sx = reinterpret_cast<float*>(smem + GemvSmem::kHeader + xl.sx);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_units = (p.n_rows + 3) >> 2;
  const int64_t u0 = n_units * blockIdx.x / gridDim.x;
  const int64_t u1 = n_units * (blockIdx.x + 1) / gridDim.x;
  const int64_t row0 = u0 * 4;
  const int64_t row1 = u1 * 4 < p.n_rows ? u1 * 4 : p.n_rows;
  const int cta_rows = static_cast<int>(row1 - row0);
  const int n_groups = (cta_rows + GR - 1) / GR;
  const int nchunks = p.k >> 4;
  trace_entry(p.trace);

  // ---- before the dependency wait: weights only
  {
    const int64_t slice = static_cast<int64_t>(cta_rows) * p.row_bytes;
    const int64_t pf = slice < p.prefetch_bytes ? slice : p.prefetch_bytes;
    const int pieces = static_cast<int>((pf + kPrefetchPiece - 1) / kPrefetchPiece);
    if (threadIdx.x < pieces) {
      const int64_t off = static_cast<int64_t>(threadIdx.x) * kPrefetchPiece;
      const int64_t n = pf - off < kPrefetchPiece ? pf - off : kPrefetchPiece;
      prefetch_l2_bulk(p.w + row0 * p.row_bytes + off, static_cast<uint32_t>(n & ~15LL));
    }
  }
  Tile<GR, J> A, B;
  int g = warp;
  if (g < n_groups)
    load_tile<GR, J>(A, p, row0 + static_cast<int64_t>(g) * GR, min(GR, cta_rows - g * GR), lane, nchunks);
  // (the second group waits for the prologue where both together would
  // leave the prologue too few registers: long rows with a normalising one)
  constexpr bool kEarlyB = J <= 4 || PRO == PRO_LOAD;
  if (kEarlyB && g + kConsumerWarps < n_groups)
    load_tile<GR, J>(B, p, row0 + static_cast<int64_t>(g + kConsumerWarps) * GR,
                     min(GR, cta_rows - (g + kConsumerWarps) * GR), lane, nchunks);
  pdl_launch_dependents();

  // ---- activations (after the wait)
  pdl_wait();
  trace_waited(p.trace);
  gemv_prologue<PRO, NV, (J > 1 ? J / 2 : 1)>(p, xd, sx, scratch);
  if (!kEarlyB && g + kConsumerWarps < n_groups)
    load_tile<GR, J>(B, p, row0 + static_cast<int64_t>(g + kConsumerWarps) * GR,
                     min(GR, cta_rows - (g + kConsumerWarps) * GR), lane, nchunks);
  __syncthreads();
  trace_ready(p.trace);

  unsigned long long best[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) best[v] = 0ull;
  const uint4* xd4 = reinterpret_cast<const uint4*>(xd);
  // group gl's rows start gl*GR*row_bytes into the slice; the pre-wait
  // prefetch covered the first prefetch_bytes of it
  const int64_t group_bytes = static_cast<int64_t>(GR) * p.row_bytes;
  auto refill = [&](Tile<GR, J>& t, int gl) {
    if (gl >= n_groups) return;
    load_tile<GR, J>(t, p, row0 + static_cast<int64_t>(gl) * GR, min(GR, cta_rows - gl * GR), lane, nchunks);
    const int gp = gl + 2 * kConsumerWarps;
    if (lane == 0 && gp < n_groups && gp * group_bytes >= p.prefetch_bytes)
      prefetch_l2_bulk(p.w + (row0 + static_cast<int64_t>(gp) * GR) * p.row_bytes,
                       static_cast<uint32_t>(min(GR, cta_rows - gp * GR) * p.row_bytes));
  };
  while (g < n_groups) {
    process_tile<EPI, NV, GR, J>(A, p, row0 + static_cast<int64_t>(g) * GR, min(GR, cta_rows - g * GR), lane,
                                 nchunks, xd4, sx, best);
    refill(A, g + 2 * kConsumerWarps);
    g += kConsumerWarps;
    if (g >= n_groups) break;
    process_tile<EPI, NV, GR, J>(B, p, row0 + static_cast<int64_t>(g) * GR, min(GR, cta_rows - g * GR), lane,
                                 nchunks, xd4, sx, best);
    refill(B, g + 2 * kConsumerWarps);
    g += kConsumerWarps;
  }

  if constexpr (EPI != EPI_ARGMAX) {
    if (p.trace) {
      __syncthreads();
      trace_exit(p.trace);
    }
    return;
  } else {
    // ---------------- argmax: CTA reduce, one atomic per vector, last CTA finalises
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const unsigned long long b = warp_max_u64(best[v]);
      if (lane == 0) amax[warp * kMaxVec + v] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int v = 0; v < p.n_vec && v < NV; ++v) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kConsumerWarps; ++w) b = amax[w * kMaxVec + v] > b ? amax[w * kMaxVec + v] : b;
        if (b) atomicMax(p.best + v, b);
      }
      __threadfence();
      const uint32_t ticket = atomicAdd(p.counter, 1u);
      if (ticket == gridDim.x - 1) {
        __threadfence();
        for (int v = 0; v < p.n_vec && v < NV; ++v) {
          const unsigned long long b = atomicExch(p.best + v, 0ull);
          const int32_t tok = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(b & 0xFFFFFFFFull));
          if (p.token_out) p.token_out[v] = tok;
          if (p.pos) {
            const int32_t next = p.pos[v] + 1;
            if (p.history && next < p.history_stride)
              p.history[static_cast<int64_t>(v) * p.history_stride + next] = tok;
            p.pos[v] = next;
          }
        }
        atomicExch(p.counter, 0u);
        __threadfence();
      }
    }
    trace_exit(p.trace);
  }
}

// ------------------------------------------------------------------ host side
template <int PRO, int EPI, int NV, int GR, int J>
int launch_impl(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  auto kern = gemv_q8_kernel<PRO, EPI, NV, GR, J>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
    if (e != cudaSuccess) return fail_cuda(e, "gemv_q8 set smem");
    configured_device = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(L.grid);
  cfg.blockDim = dim3(L.threads);
  cfg.dynamicSmemBytes = L.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = ::bt::launch_ex(&cfg, kern, p);
  if (e != cudaSuccess) return fail_cuda(e, "gemv_q8 launch");
  return BT_OK;
}

template <int PRO, int EPI, int NV, int GR>
int launch_j(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  const int J = (p.k + 511) / 512;
  if (J <= 1) return launch_impl<PRO, EPI, NV, GR, 1>(p, L, stream, pdl);
  if (J <= 2) return launch_impl<PRO, EPI, NV, GR, 2>(p, L, stream, pdl);
  if constexpr (GR == 1) {
    if (J <= 4) return launch_impl<PRO, EPI, NV, GR, 4>(p, L, stream, pdl);
    return launch_impl<PRO, EPI, NV, GR, 8>(p, L, stream, pdl);
  }
  return fail(BT_ERR_UNSUPPORTED, "q8 GEMV: 4-row groups serve K <= 1024");
}

// Launch table of one (prologue, epilogue) pair over batch width, row group
// and K.  The SiLU-pair epilogue needs 4-row groups (<= 2 vectors); the
// SiLU-pair prologue serves the wider batches that store gate/up unpaired.
template <int PRO, int EPI>
int launch_kind(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  const bool g4 = p.group_rows == 4;
  if constexpr (EPI == EPI_SILU_PAIR) {
    if (!g4) return fail(BT_ERR_UNSUPPORTED, "q8 GEMV: the SiLU-pair epilogue needs 4-row groups");
    if (p.n_vec == 1) return launch_j<PRO, EPI, 1, 4>(p, L, stream, pdl);
    if (p.n_vec == 2) return launch_j<PRO, EPI, 2, 4>(p, L, stream, pdl);
  } else if constexpr (PRO == PRO_SILU_PAIR) {
    if (p.n_vec == 4) return launch_j<PRO, EPI, 4, 1>(p, L, stream, pdl);
    if (p.n_vec == 8) return launch_j<PRO, EPI, 8, 1>(p, L, stream, pdl);
  } else {
    switch (p.n_vec) {
      case 1: return g4 ? launch_j<PRO, EPI, 1, 4>(p, L, stream, pdl) : launch_j<PRO, EPI, 1, 1>(p, L, stream, pdl);
      case 2: return g4 ? launch_j<PRO, EPI, 2, 4>(p, L, stream, pdl) : launch_j<PRO, EPI, 2, 1>(p, L, stream, pdl);
      case 4: return launch_j<PRO, EPI, 4, 1>(p, L, stream, pdl);
      case 8: return launch_j<PRO, EPI, 8, 1>(p, L, stream, pdl);
      default: break;
    }
  }
  return fail(BT_ERR_UNSUPPORTED, "q8 GEMV: prologue %d / epilogue %d do not serve %d vectors", PRO, EPI, p.n_vec);
}

#define BT_GEMV_KINDS(X)                  \
  X(PRO_LOAD, EPI_STORE)                  \
  X(PRO_RESID_NORM, EPI_STORE)            \
  X(PRO_RESID_NORM, EPI_GDN_IN)           \
  X(PRO_RESID_NORM, EPI_SILU_PAIR)        \
  X(PRO_RESID_NORM, EPI_ARGMAX)           \
  X(PRO_EMBED_NORM, EPI_STORE)            \
  X(PRO_EMBED_NORM, EPI_GDN_IN)           \
  X(PRO_GATED_NORM, EPI_STORE)            \
  X(PRO_SILU_PAIR, EPI_STORE)

#define BT_GEMV_EXTERN(P, E) \
  extern template int launch_kind<P, E>(const GemvQ8Params&, const GemvQ8Launch&, cudaStream_t, bool);
#define BT_GEMV_INSTANTIATE(P, E) \
  template int launch_kind<P, E>(const GemvQ8Params&, const GemvQ8Launch&, cudaStream_t, bool);

}  // namespace gemv_detail
}  // namespace bt
