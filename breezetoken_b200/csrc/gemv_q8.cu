// Q8_0 GEMV kernel and its host-side planner.  See gemv_q8.cuh for the design.
#include <algorithm>

#include "errors.h"
#include "gemv_q8.cuh"

namespace bt {

namespace {

constexpr int kSmemBudget = 104 * 1024;  // two CTAs (this kernel + the PDL successor) per SM

// ------------------------------------------------------------------ prologue
// Phase 1: the f32 activation vector(s) in natural layout (xf[v*K + k]).
template <int NV>
__device__ void gemv_build_x(const GemvQ8Params& p, float* xs, float* scratch) {
  const int tid = threadIdx.x;
  const int K = p.k;
  const int64_t xbs = p.x_bs ? p.x_bs : K, x2bs = p.x2_bs ? p.x2_bs : K;
  if (p.prologue == PRO_LOAD) {
    for (int v = 0; v < NV && v < p.n_vec; ++v)
      for (int k = tid; k < K; k += kConsumerThreads) xs[v * K + k] = p.x[v * xbs + k];
    return;
  }
  if (p.prologue == PRO_RESID_NORM || p.prologue == PRO_EMBED_NORM) {
    for (int v = 0; v < NV && v < p.n_vec; ++v) {
      float* xv = xs + v * K;
      const uint8_t* erow = nullptr;
      if (p.prologue == PRO_EMBED_NORM) {
        int64_t tok = p.tokens[v];
        if (tok < 0 || tok >= p.embed_rows) {
          if (tid == 0) report_status(p.status, BT_ERR_INVALID, SITE_EMBED_TOKEN, static_cast<int32_t>(tok), v);
          tok = 0;
        }
        erow = p.embed + tok * static_cast<int64_t>(p.row_bytes);
      }
      float ss = 0.f;
      for (int k = tid; k < K; k += kConsumerThreads) {
        float h;
        if (p.prologue == PRO_RESID_NORM) {
          h = p.x[v * xbs + k] + p.x2[v * x2bs + k];
        } else {
          const float d = __half2float(reinterpret_cast<const __half*>(erow)[k >> 5]);
          const float q = static_cast<float>(static_cast<int8_t>(erow[p.sb + k]));
          h = q * d;
        }
        xv[k] = h;
        ss = fmaf(h, h, ss);
        if (blockIdx.x == 0) p.h_out[static_cast<int64_t>(v) * K + k] = h;
      }
      const float total = group_sum<1>(ss, scratch, kConsumerWarps, kConsumerThreads);
      const float r = 1.0f / sqrtf(total / static_cast<float>(K) + p.eps);
      for (int k = tid; k < K; k += kConsumerThreads) xv[k] = __fmul_rn(__fmul_rn(xv[k], r), p.norm_w[k]);
    }
    return;
  }
  // PRO_GATED_NORM: one warp per normalisation group
  const int warp = tid >> 5, lane = tid & 31;
  const int G = p.group, n_groups = K / G;
  for (int v = 0; v < NV && v < p.n_vec; ++v) {
    const float* o = p.x + v * xbs;
    const float* z = p.x2 + v * x2bs;
    for (int g = warp; g < n_groups; g += kConsumerWarps) {
      float ss = 0.f;
      for (int i = lane; i < G; i += 32) {
        const float t = o[g * G + i];
        ss = fmaf(t, t, ss);
      }
      ss = warp_sum(ss);
      const float r = 1.0f / sqrtf(ss / static_cast<float>(G) + p.eps);
      for (int i = lane; i < G; i += 32) {
        const int k = g * G + i;
        const float normed = __fmul_rn(__fmul_rn(o[k], r), p.norm_w[i]);
        xs[v * K + k] = __fmul_rn(normed, z[k]);
      }
    }
  }
}

// Phase 2: per 32-element block, scale sx and three int8 digits of the
// fixed-point value (see gemv_q8.cuh); one warp per block.
template <int NV>
__device__ void gemv_encode_x(const GemvQ8Params& p, const float* xf, uint8_t* xd, float* sx) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = p.k, nb = K / 32, J = (K + 511) / 512;
  for (int item = warp; item < NV * nb; item += kConsumerWarps) {
    const int v = item / nb, b = item % nb;
    if (v >= p.n_vec) break;
    const float x = xf[v * K + 32 * b + lane];
    const float amax = warp_max(fabsf(x));
    const float inv = amax > 0.f ? static_cast<float>(kXMax) / amax : 0.f;
    int X = __float2int_rn(x * inv);
    X = X > kXMax ? kXMax : (X < -kXMax ? -kXMax : X);
    const int d0 = ((X + 128) & 255) - 128;
    const int x1 = (X - d0) >> 8;
    const int d1 = ((x1 + 128) & 255) - 128;
    const int d2 = (x1 - d1) >> 8;
    const int c = 2 * b + (lane >> 4), e = lane & 15;
    uint8_t* base = xd + static_cast<int64_t>(v) * J * 1536 + ((c >> 5) * 3 * 32 + (c & 31)) * 16 + e;
    base[0] = static_cast<uint8_t>(d2);
    base[32 * 16] = static_cast<uint8_t>(d1);
    base[64 * 16] = static_cast<uint8_t>(d0);
    if (lane == 0) sx[v * nb + b] = amax / static_cast<float>(kXMax);
  }
}

// ------------------------------------------------------------------ epilogue
__device__ __forceinline__ void epilogue_row(const GemvQ8Params& p, int v, int64_t r, float a) {
  float* y = p.y + static_cast<int64_t>(v) * p.y_stride;
  if (p.epilogue == EPI_STORE) {
    y[r] = a;
    return;
  }
  // EPI_GDN_IN
  if (r < p.n_conv) {
    const int taps = p.conv_k - 1;
    float* cs = p.conv_state + (static_cast<int64_t>(v) * p.n_conv + r) * taps;
    const float* cw = p.conv_w + r * p.conv_k;
    float sum = 0.f;
    for (int t = 0; t < taps; ++t) sum = __fadd_rn(sum, __fmul_rn(cs[t], cw[t]));
    sum = __fadd_rn(sum, __fmul_rn(a, cw[taps]));
    for (int t = 0; t + 1 < taps; ++t) cs[t] = cs[t + 1];
    cs[taps - 1] = a;
    y[r] = silu_f(sum);
  } else if (r < p.n_conv + p.n_z) {
    y[r] = silu_f(a);
  } else if (r < p.n_conv + p.n_z + p.n_gh) {
    const int h = static_cast<int>(r - p.n_conv - p.n_z);
    y[r] = p.a_log[h] * softplus_f(a + p.dt_bias[h]);
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
template <int NV, int GR>
__global__ void __launch_bounds__(kGemvThreads, 2)
    gemv_q8_kernel(const __grid_constant__ GemvQ8Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  float* scratch = reinterpret_cast<float*>(empty + kMaxStages);
  unsigned long long* amax = reinterpret_cast<unsigned long long*>(scratch + 64);
  const XLayout xl = gemv_x_layout(p.k, NV);
  float* xf = reinterpret_cast<float*>(smem + GemvSmem::kHeader + xl.xf);
  uint8_t* xd = smem + GemvSmem::kHeader + xl.xd;
  float* sx = reinterpret_cast<float*>(smem + GemvSmem::kHeader + xl.sx);
  uint8_t* ring = smem + GemvSmem::kHeader + xl.total;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_units = (p.n_rows + 3) >> 2;
  const int64_t u0 = n_units * blockIdx.x / gridDim.x;
  const int64_t u1 = n_units * (blockIdx.x + 1) / gridDim.x;
  const int64_t row0 = u0 * 4;
  const int64_t row1 = u1 * 4 < p.n_rows ? u1 * 4 : p.n_rows;
  const int cta_rows = static_cast<int>(row1 - row0);
  const int n_iters = (cta_rows + p.stage_rows - 1) / p.stage_rows;
  // Per-warp rings: iteration `it` belongs to consumer warp it % 8, which owns
  // slots [w * SPW, (w + 1) * SPW) and consumes them strictly in order.  A
  // waiter is therefore never more than one phase ahead of its barrier, so the
  // mbarrier parity test cannot alias (a shared ring with more consumers than
  // stages would let a warp pass on the parity of a phase two fills old).
  const int SPW = p.stages;
  const uint32_t stage_bytes = static_cast<uint32_t>(p.stage_rows) * p.row_bytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kConsumerWarps * SPW; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kConsumerWarps) {
    // ---------------- producer: weights only, so no pdl_wait needed
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      int issued = 0;
      for (int it = 0; it < n_iters; ++it) {
        const int i = it / kConsumerWarps;  // this warp's i-th stage
        const int s = (it % kConsumerWarps) * SPW + i % SPW;
        if (i >= SPW && !mbar_wait(&empty[s], ((i / SPW) - 1) & 1)) {
          report_status(p.status, BT_ERR_TIMEOUT, SITE_GEMV_PRODUCER_EMPTY, it, n_iters, SPW);
          break;
        }
        const int64_t r = row0 + static_cast<int64_t>(it) * p.stage_rows;
        const int nr = static_cast<int>(min(static_cast<int64_t>(p.stage_rows), row1 - r));
        const uint32_t bytes = static_cast<uint32_t>(nr) * p.row_bytes;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(ring + static_cast<size_t>(s) * stage_bytes, p.w + r * p.row_bytes, bytes,
                 &full[s], policy);
        issued = it + 1;
      }
      // Do not leave the CTA with copies in flight (bounded): wait for the
      // last fill of every slot.
      for (int it = max(0, issued - kConsumerWarps * SPW); it < issued; ++it) {
        const int i = it / kConsumerWarps;
        const int s = (it % kConsumerWarps) * SPW + i % SPW;
        if (!mbar_wait(&full[s], (i / SPW) & 1)) {
          report_status(p.status, BT_ERR_TIMEOUT, SITE_GEMV_PRODUCER_DRAIN, it, n_iters, SPW);
          break;
        }
      }
    }
    return;
  }

  // ---------------- consumers
  pdl_wait();
  gemv_build_x<NV>(p, xf, scratch);
  named_sync(1, kConsumerThreads);
  gemv_encode_x<NV>(p, xf, xd, sx);
  named_sync(1, kConsumerThreads);

  unsigned long long best[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) best[v] = 0ull;

  const int nchunks = p.k >> 4;
  const int J = (nchunks + 31) >> 5;
  const int nb = p.k >> 5;
  const uint4* xd4 = reinterpret_cast<const uint4*>(xd);

  for (int it = warp, i = 0; it < n_iters; it += kConsumerWarps, ++i) {
    const int s = warp * SPW + i % SPW;
    if (!mbar_wait(&full[s], (i / SPW) & 1)) {
      report_status(p.status, BT_ERR_TIMEOUT, SITE_GEMV_CONSUMER_FULL, it, n_iters, (warp << 16) | SPW);
      break;
    }
    const uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    const int64_t r0 = row0 + static_cast<int64_t>(it) * p.stage_rows;
    const int nr = static_cast<int>(min(static_cast<int64_t>(p.stage_rows), row1 - r0));

    for (int g = 0; g < nr; g += GR) {
      float acc[GR][NV];
#pragma unroll
      for (int r = 0; r < GR; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = 0.f;

      for (int j = 0; j < J; ++j) {
        const int c = lane + (j << 5);
        if (c < nchunks) {
          uint4 dg[NV][3];
          float xsc[NV];
#pragma unroll
          for (int v = 0; v < NV; ++v) {
#pragma unroll
            for (int t = 0; t < 3; ++t) dg[v][t] = xd4[(v * J + j) * 96 + t * 32 + lane];
            xsc[v] = sx[v * nb + (c >> 1)];
          }
#pragma unroll
          for (int r = 0; r < GR; ++r) {
            if (g + r < nr) {
              const uint8_t* row = st + static_cast<size_t>(g + r) * p.row_bytes;
              const float d = __half2float(reinterpret_cast<const __half*>(row)[c >> 1]);
              const uint4 q = *reinterpret_cast<const uint4*>(row + p.sb + (c << 4));
#pragma unroll
              for (int v = 0; v < NV; ++v)
                acc[r][v] = fmaf(d * xsc[v], dot16_digits(q, dg[v][0], dg[v][1], dg[v][2]), acc[r][v]);
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
          const int lr = g + (lane >> 3);  // local row held by lanes 0, 8, 16, 24
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
              epilogue_row(p, v, row, c);
            }
          }
        }
      } else {
#pragma unroll
        for (int v = 0; v < NV; ++v) {
          const float c = warp_sum(acc[0][v]);
          if (lane == 0 && g < nr) {
            const int64_t row = r0 + g;
            if (p.epilogue == EPI_ARGMAX) {
              if (p.y) p.y[static_cast<int64_t>(v) * p.y_stride + row] = c;
              const unsigned long long key = argmax_key(c, row);
              best[v] = key > best[v] ? key : best[v];
            } else {
              epilogue_row(p, v, row, c);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  if (p.epilogue != EPI_ARGMAX) return;

  // ---------------- argmax: CTA reduce, one atomic per vector, last CTA finalises
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const unsigned long long b = warp_max_u64(best[v]);
    if (lane == 0) amax[warp * kMaxVec + v] = b;
  }
  named_sync(1, kConsumerThreads);
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
}

template <int NV, int GR>
int launch_impl(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  auto kern = gemv_q8_kernel<NV, GR>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBudget + GemvSmem::kHeader + 1024);
    if (e != cudaSuccess) return fail_cuda(e, "gemv_q8 set smem");
    // full shared-memory carveout, so the PDL successor's CTA fits beside this one
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return fail_cuda(e, "gemv_q8 set carveout");
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

}  // namespace

int gemv_q8_plan(GemvQ8Params& p, int sm_count, GemvQ8Launch& L) {
  if (p.k < 32 || p.k % 32 != 0) return fail(BT_ERR_UNSUPPORTED, "q8 GEMV needs K %% 32 == 0, got K=%d", p.k);
  if (p.n_rows < 1) return fail(BT_ERR_INVALID, "q8 GEMV needs at least one row");
  if (p.n_vec < 1 || p.n_vec > kMaxVec) return fail(BT_ERR_UNSUPPORTED, "q8 GEMV serves 1..8 vectors, got %d", p.n_vec);
  if (!p.w || (reinterpret_cast<uintptr_t>(p.w) & 15))
    return fail(BT_ERR_INVALID, "q8 GEMV weights must be 16-byte aligned (bulk copies)");
  if (p.epilogue == EPI_ARGMAX && (!p.best || !p.counter))
    return fail(BT_ERR_INVALID, "argmax epilogue needs its workspace");
  p.sb = static_cast<int32_t>(bt_q8_row_bytes(p.k) - p.k);
  p.row_bytes = static_cast<int32_t>(bt_q8_row_bytes(p.k));
  const int64_t n_units = (p.n_rows + 3) / 4;
  const int grid = static_cast<int>(std::min<int64_t>(sm_count, n_units));
  const int64_t rows_per_cta = ((n_units + grid - 1) / grid) * 4;
  const int64_t x_bytes = gemv_x_layout(p.k, p.n_vec).total;
  const int64_t ring_budget = kSmemBudget - x_bytes;
  // 4-row groups reuse each activation chunk across rows; they need one
  // 4-row stage per consumer warp in the ring.
  const bool fits4 = kConsumerWarps * 4LL * p.row_bytes <= ring_budget;
  int gr = 1;
  if (p.epilogue == EPI_SILU_PAIR || (p.n_vec <= 2 && rows_per_cta >= 32 && fits4)) gr = 4;
  if (p.epilogue == EPI_SILU_PAIR && (p.n_vec > 2 || !fits4))
    return fail(BT_ERR_UNSUPPORTED, "SiLU-pair epilogue serves at most 2 vectors and K <= %lld",
                static_cast<long long>(ring_budget / (4 * kConsumerWarps)));
  p.group_rows = gr;
  // stage = gr * f rows, ~8 KB at most, and no more rows than keep all 8
  // consumer warps busy
  const int64_t f_rows = std::max<int64_t>(1, rows_per_cta / (kConsumerWarps * gr));
  const int64_t f_bytes = std::max<int64_t>(1, 8192 / (static_cast<int64_t>(gr) * p.row_bytes));
  const int64_t f = std::min(f_rows, f_bytes);
  p.stage_rows = static_cast<int32_t>(gr * f);
  const int64_t stage_bytes = static_cast<int64_t>(p.stage_rows) * p.row_bytes;
  if (kConsumerWarps * stage_bytes > ring_budget)
    return fail(BT_ERR_UNSUPPORTED, "q8 GEMV row of K=%d does not fit the stage budget", p.k);
  // stages per consumer warp (each warp owns its own ring)
  const int64_t iters = (rows_per_cta + p.stage_rows - 1) / p.stage_rows;
  const int64_t per_warp = (iters + kConsumerWarps - 1) / kConsumerWarps;
  p.stages = static_cast<int32_t>(std::min<int64_t>(
      {kMaxStages / kConsumerWarps, ring_budget / (kConsumerWarps * stage_bytes), std::max<int64_t>(1, per_warp)}));
  L.grid = grid;
  L.threads = kGemvThreads;
  L.smem = GemvSmem::kHeader + x_bytes + static_cast<size_t>(kConsumerWarps) * p.stages * stage_bytes;
  return BT_OK;
}

int gemv_q8_launch(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  const bool g4 = p.group_rows == 4;
  switch (p.n_vec) {
    case 1: return g4 ? launch_impl<1, 4>(p, L, stream, pdl) : launch_impl<1, 1>(p, L, stream, pdl);
    case 2: return g4 ? launch_impl<2, 4>(p, L, stream, pdl) : launch_impl<2, 1>(p, L, stream, pdl);
    case 3:
    case 4: return launch_impl<4, 1>(p, L, stream, pdl);
    default: return launch_impl<8, 1>(p, L, stream, pdl);
  }
}

}  // namespace bt
