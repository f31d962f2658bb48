// Q8_0 GEMV kernel and its host-side planner.  See gemv_q8.cuh for the design.
#include <algorithm>
#include <cstdlib>

#include "errors.h"
#include "gemv_q8.cuh"

namespace bt {

namespace {

// Bytes of its weight slice each CTA prefetches into L2 before the
// dependency wait (BT_GEMV_PREFETCH_KB overrides it for tuning sweeps).
constexpr int64_t kPrefetchPiece = 16 * 1024;

struct GemvTuning {
  int64_t prefetch_bytes = 64 * 1024;
  int early_tile = 1;  // load the first register tile before the wait (BT_GEMV_EARLY_TILE)
};

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

const GemvTuning& tuning() {
  static const GemvTuning t = [] {
    GemvTuning g;
    g.prefetch_bytes = static_cast<int64_t>(std::min(1024, std::max(0, env_int("BT_GEMV_PREFETCH_KB", 64)))) * 1024;
    g.early_tile = env_int("BT_GEMV_EARLY_TILE", 1) != 0;
    return g;
  }();
  return t;
}

// ------------------------------------------------------------------ prologue
// Builds each activation vector and encodes it for the dp4a inner loop (see
// gemv_q8.cuh).  Thread t owns float4 number f = t + 256*i of the vector, so
// every global load of the prologue (x, residual, norm weights or the
// embedding row) is issued before any is used: one memory latency on the
// critical path instead of one per element loop.  A 32-element block is 8
// consecutive float4 = 8 consecutive lanes, so its max is 3 xor-shuffles and
// the digits go straight from registers to shared memory.
constexpr int kMaxF4 = 4;  // float4 per thread per vector: K <= 4096

__device__ __forceinline__ float4 f4_mul(float4 a, float4 b) {
  return make_float4(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z), __fmul_rn(a.w, b.w));
}
__device__ __forceinline__ float4 f4_scale(float4 a, float r) {
  return make_float4(__fmul_rn(a.x, r), __fmul_rn(a.y, r), __fmul_rn(a.z, r), __fmul_rn(a.w, r));
}

__device__ __forceinline__ void encode_digits(float x, float inv, int& d2, int& d1, int& d0) {
  int X = __float2int_rn(x * inv);
  X = X > kXMax ? kXMax : (X < -kXMax ? -kXMax : X);
  d0 = ((X + 128) & 255) - 128;
  const int x1 = (X - d0) >> 8;
  d1 = ((x1 + 128) & 255) - 128;
  d2 = (x1 - d1) >> 8;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 255u) | ((static_cast<uint32_t>(b) & 255u) << 8) |
         ((static_cast<uint32_t>(c) & 255u) << 16) | ((static_cast<uint32_t>(d) & 255u) << 24);
}

template <int NV, int NIT>
__device__ void gemv_prologue(const GemvQ8Params& p, uint8_t* xd, float* sx, float* scratch) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int K = p.k, nf4 = K >> 2, nb = K >> 5, J = (K + 511) / 512;
  const int n_it = NIT;
  const int64_t xbs = p.x_bs ? p.x_bs : K, x2bs = p.x2_bs ? p.x2_bs : K;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int v = 0; v < NV; ++v) {
    float4 h[NIT], a2[NIT], w4[NIT];
    // ---- all loads first, unconditionally: indices past the vector are
    //      clamped onto its last float4 and zeroed afterwards, so the loads
    //      carry no control dependence and are all in flight at once.
    if (p.prologue == PRO_EMBED_NORM) {
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
      for (int i = 0; i < NIT; ++i)
        h[i] = make_float4(static_cast<float>(static_cast<int8_t>(q[i] & 255)) * d[i],
                           static_cast<float>(static_cast<int8_t>((q[i] >> 8) & 255)) * d[i],
                           static_cast<float>(static_cast<int8_t>((q[i] >> 16) & 255)) * d[i],
                           static_cast<float>(static_cast<int8_t>(q[i] >> 24)) * d[i]);
    } else {
      const float4* x4 = reinterpret_cast<const float4*>(p.x + v * xbs);
      const float4* x24 = reinterpret_cast<const float4*>(p.x2 + v * x2bs);
      const float4* n4 = reinterpret_cast<const float4*>(p.norm_w);
      const int gq = p.group >> 2;
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        const int fc = min(tid + kConsumerThreads * i, nf4 - 1);
        if (p.prologue == PRO_SILU_PAIR) {
          // interleaved (gate, up) pairs: float4s 2fc and 2fc+1 give x[4fc .. 4fc+3]
          h[i] = x4[2 * fc];
          a2[i] = x4[2 * fc + 1];
        } else {
          h[i] = x4[fc];
          a2[i] = p.prologue != PRO_LOAD ? x24[fc] : zero4;
        }
        w4[i] = p.prologue == PRO_RESID_NORM ? n4[fc] : (p.prologue == PRO_GATED_NORM ? n4[fc % gq] : zero4);
      }
    }
#pragma unroll
    for (int i = 0; i < NIT; ++i)
      if (tid + kConsumerThreads * i >= nf4) h[i] = a2[i] = w4[i] = zero4;
    if (p.prologue == PRO_SILU_PAIR) {
#pragma unroll
      for (int i = 0; i < NIT; ++i)
        h[i] = make_float4(silu_f(h[i].x) * h[i].y, silu_f(h[i].z) * h[i].w, silu_f(a2[i].x) * a2[i].y,
                           silu_f(a2[i].z) * a2[i].w);
    }
    // ---- residual add and normalisation
    if (p.prologue == PRO_RESID_NORM || p.prologue == PRO_EMBED_NORM) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        const int f = tid + kConsumerThreads * i;
        if (i < n_it && f < nf4) {
          if (p.prologue == PRO_RESID_NORM)
            h[i] = make_float4(h[i].x + a2[i].x, h[i].y + a2[i].y, h[i].z + a2[i].z, h[i].w + a2[i].w);
          if (blockIdx.x == 0) reinterpret_cast<float4*>(p.h_out + static_cast<int64_t>(v) * K)[f] = h[i];
          ss = fmaf(h[i].x, h[i].x, ss);
          ss = fmaf(h[i].y, h[i].y, ss);
          ss = fmaf(h[i].z, h[i].z, ss);
          ss = fmaf(h[i].w, h[i].w, ss);
        }
      }
      const float total = group_sum<1>(ss, scratch, kConsumerWarps, kConsumerThreads);
      const float r = 1.0f / sqrtf(total / static_cast<float>(K) + p.eps);
#pragma unroll
      for (int i = 0; i < NIT; ++i) h[i] = f4_mul(f4_scale(h[i], r), w4[i]);
    } else if (p.prologue == PRO_GATED_NORM) {
      // group of G elements = G/4 consecutive lanes of one warp
      const int lanes = p.group >> 2;
#pragma unroll
      for (int i = 0; i < NIT; ++i) {
        if (i >= n_it) break;
        float ss = fmaf(h[i].x, h[i].x, fmaf(h[i].y, h[i].y, fmaf(h[i].z, h[i].z, h[i].w * h[i].w)));
        for (int o = lanes >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = 1.0f / sqrtf(ss / static_cast<float>(p.group) + p.eps);
        h[i] = f4_mul(f4_mul(f4_scale(h[i], r), w4[i]), a2[i]);
      }
    }
    // ---- encode: block max over 8 lanes, digits from registers
    uint8_t* xdv = xd + static_cast<int64_t>(v) * J * 1536;
#pragma unroll
    for (int i = 0; i < NIT; ++i) {
      if (i >= n_it) break;
      const int f = tid + kConsumerThreads * i;
      float m = fmaxf(fmaxf(fabsf(h[i].x), fabsf(h[i].y)), fmaxf(fabsf(h[i].z), fabsf(h[i].w)));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
      if (f < nf4) {
        const float inv = m > 0.f ? static_cast<float>(kXMax) / m : 0.f;
        int a[4], b[4], c[4];
        encode_digits(h[i].x, inv, a[0], b[0], c[0]);
        encode_digits(h[i].y, inv, a[1], b[1], c[1]);
        encode_digits(h[i].z, inv, a[2], b[2], c[2]);
        encode_digits(h[i].w, inv, a[3], b[3], c[3]);
        const int ch = f >> 2;  // 16-element chunk
        uint32_t* w = reinterpret_cast<uint32_t*>(xdv + ((ch >> 5) * 96 + (ch & 31)) * 16) + (f & 3);
        w[0] = pack4(a[0], a[1], a[2], a[3]);
        w[32 * 4] = pack4(b[0], b[1], b[2], b[3]);
        w[64 * 4] = pack4(c[0], c[1], c[2], c[3]);
        if ((f & 7) == 0) sx[v * nb + (f >> 3)] = m / static_cast<float>(kXMax);
      }
    }
  }
  (void)lane;
}

// ------------------------------------------------------------------ epilogue
// Operands of the GDN in-projection epilogue for one row, loaded before the
// row's dot products so their latency hides behind the math: the conv window
// (taps <= 3) and conv weights (conv_k <= 4) of a qkv channel, or a_log and
// dt_bias of an alpha row.
struct EpiOperands {
  float cs[3], cw[4], a_log, dt_bias;
};

__device__ __forceinline__ void epi_prefetch(const GemvQ8Params& p, int v, int64_t r, EpiOperands& o) {
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

__device__ __forceinline__ void epilogue_row(const GemvQ8Params& p, int v, int64_t r, float a,
                                             const EpiOperands& o) {
  float* y = p.y + static_cast<int64_t>(v) * p.y_stride;
  if (p.epilogue == EPI_STORE) {
    y[r] = a;
    return;
  }
  // EPI_GDN_IN: conv window + SiLU (model/layers.py:90-93), silu(z),
  // g = a_log * softplus(alpha + dt_bias) (:99-103), beta logits as they are
  if (r < p.n_conv) {
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
    float* cs = p.conv_state + (static_cast<int64_t>(v) * p.n_conv + r) * taps;
#pragma unroll
    for (int t = 0; t < 3; ++t)
      if (t + 1 < taps) cs[t] = o.cs[t + 1];
    cs[taps - 1] = a;
    y[r] = silu_f(sum);
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

// ------------------------------------------------------------------ kernel
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

// EPF: the GDN in-projection epilogue with its operands loaded before the
// math (batches of <= 2 vectors); otherwise they are loaded here.
template <bool EPF, int NE>
__device__ __forceinline__ void epilogue_late(const GemvQ8Params& p, int v, int64_t row, float c,
                                              const EpiOperands (&eo)[NE]) {
  if constexpr (EPF) {
    epilogue_row(p, v, row, c, eo[v]);
  } else {
    EpiOperands o;
    if (p.epilogue == EPI_GDN_IN) epi_prefetch(p, v, row, o);
    epilogue_row(p, v, row, c, o);
  }
}

template <int NV, int GR, int J, bool EPF>
__device__ __forceinline__ void process_tile(const Tile<GR, J>& t, const GemvQ8Params& p, int64_t r0, int nr,
                                             int lane, int nchunks, const uint4* xd4, const float* sx,
                                             unsigned long long (&best)[NV]) {
  const int nb = p.k >> 5;
  // epilogue operands of the row this lane will finish, in flight during the math
  constexpr int NE = EPF ? NV : 1;
  EpiOperands eo[NE];
  if constexpr (EPF) {
    const int my_r = GR == 4 ? (lane >> 3) : 0;
    const bool mine = GR == 4 ? (lane & 7) == 0 : lane == 0;
    if (mine && my_r < nr)
#pragma unroll
      for (int v = 0; v < NE; ++v) epi_prefetch(p, v, r0 + my_r, eo[v]);
  }
  float acc[GR][NV];
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

  if constexpr (GR == 4) {
    // reduce-scatter: lane l ends with the sum of row 2*bit4(l) + bit3(l)
    const bool hi16 = (lane & 16) != 0, hi8 = (lane & 8) != 0;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
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
      const int lr = lane >> 3;  // row held by lanes 0, 8, 16, 24
      if (p.epilogue == EPI_SILU_PAIR) {
        const float up = __shfl_down_sync(0xffffffffu, c, 8);
        if ((lane & 15) == 0 && lr + 1 < nr) {
          const int64_t pair = (r0 + lr) >> 1;
          p.y[static_cast<int64_t>(v) * p.y_stride + pair] = silu_f(c) * up;
        }
      } else if ((lane & 7) == 0 && lr < nr) {
        const int64_t row = r0 + lr;
        if (p.epilogue == EPI_ARGMAX) {
          if (p.y) p.y[static_cast<int64_t>(v) * p.y_stride + row] = c;
          const unsigned long long key = argmax_key(c, row);
          best[v] = key > best[v] ? key : best[v];
        } else {
          epilogue_late<EPF>(p, v, row, c, eo);
        }
      }
    }
  } else {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
#pragma unroll
      for (int r = 0; r < GR; ++r) {
        const float c = warp_sum(acc[r][v]);
        if (lane == 0 && r < nr) {
          const int64_t row = r0 + r;
          if (p.epilogue == EPI_ARGMAX) {
            if (p.y) p.y[static_cast<int64_t>(v) * p.y_stride + row] = c;
            const unsigned long long key = argmax_key(c, row);
            best[v] = key > best[v] ? key : best[v];
          } else {
            epilogue_late<EPF>(p, v, row, c, eo);
          }
        }
      }
    }
  }
}

// One CTA per SM streams a contiguous range of rows.  Warp w takes row groups
// w, w+8, ...; each warp double-buffers its groups in registers (loads of
// group g+8 are in flight while group g is computed).  Before the dependency
// wait the CTA prefetches the head of its weight slice into L2 and loads its
// first groups into registers: weights never depend on earlier kernels.
template <int NV, int GR, int J, bool EPF>
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
  if (p.early_tile && g < n_groups)
    load_tile<GR, J>(A, p, row0 + static_cast<int64_t>(g) * GR, min(GR, cta_rows - g * GR), lane, nchunks);
  pdl_launch_dependents();

  // ---- activations (after the wait)
  pdl_wait();
  trace_waited(p.trace);
  gemv_prologue<NV, (J > 1 ? J / 2 : 1)>(p, xd, sx, scratch);
  if (!p.early_tile && g < n_groups)
    load_tile<GR, J>(A, p, row0 + static_cast<int64_t>(g) * GR, min(GR, cta_rows - g * GR), lane, nchunks);
  __syncthreads();
  trace_ready(p.trace);

  unsigned long long best[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) best[v] = 0ull;
  const uint4* xd4 = reinterpret_cast<const uint4*>(xd);
  while (g < n_groups) {
    int gn = g + kConsumerWarps;
    if (gn < n_groups) load_tile<GR, J>(B, p, row0 + static_cast<int64_t>(gn) * GR, min(GR, cta_rows - gn * GR), lane, nchunks);
    process_tile<NV, GR, J, EPF>(A, p, row0 + static_cast<int64_t>(g) * GR, min(GR, cta_rows - g * GR), lane, nchunks, xd4, sx, best);
    g = gn;
    if (g >= n_groups) break;
    gn = g + kConsumerWarps;
    if (gn < n_groups) load_tile<GR, J>(A, p, row0 + static_cast<int64_t>(gn) * GR, min(GR, cta_rows - gn * GR), lane, nchunks);
    process_tile<NV, GR, J, EPF>(B, p, row0 + static_cast<int64_t>(g) * GR, min(GR, cta_rows - g * GR), lane, nchunks, xd4, sx, best);
    g = gn;
  }

  if (p.epilogue != EPI_ARGMAX) {
    if (p.trace) {
      __syncthreads();
      trace_exit(p.trace);
    }
    return;
  }

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

template <int NV, int GR, int J, bool EPF>
int launch_impl(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  auto kern = gemv_q8_kernel<NV, GR, J, EPF>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return fail_cuda(e, "gemv_q8 launch");
  return BT_OK;
}

template <int NV, int GR, bool EPF = false>
int launch_j(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  const int J = (p.k + 511) / 512;
  if (J <= 1) return launch_impl<NV, GR, 1, EPF>(p, L, stream, pdl);
  if (J <= 2) return launch_impl<NV, GR, 2, EPF>(p, L, stream, pdl);
  if constexpr (GR == 1) {
    if (J <= 4) return launch_impl<NV, GR, 4, EPF>(p, L, stream, pdl);
    return launch_impl<NV, GR, 8, EPF>(p, L, stream, pdl);
  }
  return fail(BT_ERR_UNSUPPORTED, "q8 GEMV: 4-row groups serve K <= 1024");
}

}  // namespace

int gemv_q8_plan(GemvQ8Params& p, int sm_count, GemvQ8Launch& L) {
  if (p.k < 32 || p.k % 32 != 0) return fail(BT_ERR_UNSUPPORTED, "q8 GEMV needs K %% 32 == 0, got K=%d", p.k);
  if (p.n_rows < 1) return fail(BT_ERR_INVALID, "q8 GEMV needs at least one row");
  if (p.n_vec < 1 || p.n_vec > kMaxVec) return fail(BT_ERR_UNSUPPORTED, "q8 GEMV serves 1..8 vectors, got %d", p.n_vec);
  if (!p.w || (reinterpret_cast<uintptr_t>(p.w) & 15))
    return fail(BT_ERR_INVALID, "q8 GEMV weights must be 16-byte aligned");
  if (p.epilogue == EPI_ARGMAX && (!p.best || !p.counter))
    return fail(BT_ERR_INVALID, "argmax epilogue needs its workspace");
  if (p.k > kMaxF4 * kConsumerThreads * 4)
    return fail(BT_ERR_UNSUPPORTED, "q8 GEMV serves K <= %d, got %d", kMaxF4 * kConsumerThreads * 4, p.k);
  {
    // the prologue reads activations and norm weights as float4
    const uintptr_t a = reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.x2) |
                        reinterpret_cast<uintptr_t>(p.norm_w) | reinterpret_cast<uintptr_t>(p.h_out);
    if ((a & 15) || (p.x_bs & 3) || (p.x2_bs & 3))
      return fail(BT_ERR_INVALID, "q8 GEMV activations must be 16-byte aligned with strides a multiple of 4");
    if (p.prologue == PRO_GATED_NORM && p.group != 64 && p.group != 128)
      return fail(BT_ERR_UNSUPPORTED, "gated-norm prologue serves groups of 64 or 128, got %d", p.group);
    if (p.prologue == PRO_SILU_PAIR && p.x_bs == 0) p.x_bs = 2LL * p.k;
  }
  p.sb = static_cast<int32_t>(bt_q8_row_bytes(p.k) - p.k);
  p.row_bytes = static_cast<int32_t>(bt_q8_row_bytes(p.k));
  const int64_t n_units = (p.n_rows + 3) / 4;
  const int grid = static_cast<int>(std::min<int64_t>(sm_count, n_units));
  const int64_t rows_per_cta = ((n_units + grid - 1) / grid) * 4;
  // 4-row groups reuse each activation chunk across rows (K <= 1024: a
  // double-buffered 4-row tile stays within the register budget)
  const bool g4_ok = p.k <= 1024 && p.n_vec <= 2;
  int gr = 1;
  if (p.epilogue == EPI_SILU_PAIR || (g4_ok && rows_per_cta >= 32)) gr = 4;
  if (p.epilogue == EPI_SILU_PAIR && !g4_ok)
    return fail(BT_ERR_UNSUPPORTED, "SiLU-pair epilogue serves at most 2 vectors and K <= 1024");
  p.group_rows = gr;
  p.prefetch_bytes = tuning().prefetch_bytes;
  p.early_tile = tuning().early_tile;
  L.grid = grid;
  L.threads = kGemvThreads;
  L.smem = GemvSmem::kHeader + gemv_x_layout(p.k, p.n_vec).total;
  return BT_OK;
}

int gemv_q8_launch(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  const bool g4 = p.group_rows == 4, epf = p.epilogue == EPI_GDN_IN;
  switch (p.n_vec) {
    case 1:
      if (epf) return g4 ? launch_j<1, 4, true>(p, L, stream, pdl) : launch_j<1, 1, true>(p, L, stream, pdl);
      return g4 ? launch_j<1, 4>(p, L, stream, pdl) : launch_j<1, 1>(p, L, stream, pdl);
    case 2:
      if (epf) return g4 ? launch_j<2, 4, true>(p, L, stream, pdl) : launch_j<2, 1, true>(p, L, stream, pdl);
      return g4 ? launch_j<2, 4>(p, L, stream, pdl) : launch_j<2, 1>(p, L, stream, pdl);
    case 4: return launch_j<4, 1>(p, L, stream, pdl);
    default: return launch_j<8, 1>(p, L, stream, pdl);
  }
}

}  // namespace bt
