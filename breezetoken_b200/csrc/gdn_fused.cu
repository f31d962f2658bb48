// One kernel for the Gated DeltaNet half of a Qwen3.5 linear-attention layer
// at decode: in-projection GEMV (with the residual/embedding RMSNorm in
// front), causal conv + SiLU, q/k L2 norms, the gated-delta recurrence and
// the gated RMSNorm (model/layers.py:84-118 with the recurrence of
// backends.py:241-271).  The out-projection that follows reads its output as
// is.
//
// Each value head is a cluster of 8 CTAs (head dim 128).  CTA j of head h
// owns the 16-column slice [16j, 16j+16) of everything per head: it computes
// in-projection rows 16j..16j+15 of the head's q, k, v and z (64 q8 rows),
// the conv of those q/k/v channels, and the recurrence for value columns
// 16j..16j+15 (a 128 x 16 slice of the state).  The recurrence needs the
// whole normalised q and k of the head, so the slices are exchanged through
// distributed shared memory: each CTA stores its slices into every CTA of
// the cluster, then one cluster barrier; the gated norm's sum of squares over
// the head's 128 outputs is a second such exchange.  CTAs 0 and 1 also
// compute the head's alpha and beta rows.  Before the dependency wait a CTA
// prefetches its 70 KB of weights and its state slice into L2 and loads its
// first row groups into registers; after it the state slice streams into
// shared memory (cp.async) while the activation prologue and the GEMV run.
//
// Compared with three kernels (in-projection, recurrence, gated-norm
// out-projection) this removes one kernel boundary per layer and the
// round trips of q/k/v/z/g/beta and of the state through global memory.
#include <cooperative_groups.h>

#include "gdn_fused.cuh"
#include "gemv_q8_impl.cuh"

namespace cg = cooperative_groups;

namespace bt {

namespace {

using namespace gemv_detail;

constexpr int kC = 8;          // CTAs per head (cluster size)
constexpr int kDim = 128;      // head dim served
constexpr int kSeg = 16;       // rows of each of q, k, v, z per CTA (= value columns per CTA)
constexpr int kR = kDim / 16;  // state rows per thread in the recurrence
constexpr int kMaxSmem = 200 * 1024;

// Dynamic shared memory: [gemv header][fused vectors][state slices][activations]
struct FusedLayout {
  int64_t sv, sz, gdec, gbeta, qf, kf, ot, ssq, red, st, x, total;
};

__host__ __device__ inline FusedLayout fused_layout(int k, int nv) {
  FusedLayout l;
  int64_t o = GemvSmem::kHeader;  // bytes
  auto take = [&](int64_t floats) {
    const int64_t at = o;
    o += ((floats * 4 + 15) / 16) * 16;
    return at;
  };
  l.sv = take(nv * kSeg);
  l.sz = take(nv * kSeg);
  l.gdec = take(nv);
  l.gbeta = take(nv);
  l.qf = take(nv * kDim);
  l.kf = take(nv * kDim);
  l.ot = take(nv * kSeg);
  l.ssq = take(nv * kC);
  l.red = take(16 * 16);
  l.st = take(static_cast<int64_t>(nv) * kDim * kSeg);
  o = (o + 127) / 128 * 128;
  l.x = o;
  l.total = o + gemv_x_layout(k, nv).total;
  return l;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Split cluster barrier: every thread of every CTA arrives, then waits.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// Store v into the same shared-memory slot of every CTA of the cluster.
__device__ __forceinline__ void push_all(cg::cluster_group& cluster, float* slot, float v) {
#pragma unroll
  for (int r = 0; r < kC; ++r) *cluster.map_shared_rank(slot, r) = v;
}

template <int PRO, int NV, int GR, int J>
__global__ void __launch_bounds__(kGemvThreads, (J <= 4 ? 2 : 1)) gdn_fused_kernel(const __grid_constant__ GdnFusedParams P) {
  constexpr int GPS = kSeg / GR;  // row groups per segment
  constexpr int NG = 4 * GPS;     // row groups of the CTA (q, k, v, z segments)
  const GemvQ8Params& p = P.g;
  extern __shared__ __align__(128) uint8_t smem[];
  const FusedLayout L = fused_layout(p.k, NV);
  float* scratch = reinterpret_cast<float*>(smem);
  float* sv = reinterpret_cast<float*>(smem + L.sv);      // conv(v) slice [v][16]
  float* sz = reinterpret_cast<float*>(smem + L.sz);      // silu(z) slice
  float* gdec = reinterpret_cast<float*>(smem + L.gdec);  // decay logit g (pushed by CTA 0)
  float* gbeta = reinterpret_cast<float*>(smem + L.gbeta);  // beta logit (pushed by CTA 1)
  float* qf = reinterpret_cast<float*>(smem + L.qf);      // q of the head [v][128] (every CTA's slice)
  float* kf = reinterpret_cast<float*>(smem + L.kf);
  float* ot = reinterpret_cast<float*>(smem + L.ot);      // recurrence output slice [v][16]
  float* ssq = reinterpret_cast<float*>(smem + L.ssq);    // per-CTA sums of squares of the output [v][8]
  float (*red)[16] = reinterpret_cast<float (*)[16]>(smem + L.red);
  float* st = reinterpret_cast<float*>(smem + L.st);      // state slices [v][128][16]
  const XLayout xl = gemv_x_layout(p.k, NV);
  uint8_t* xd = smem + L.x + xl.xd;
  float* sx = reinterpret_cast<float*>(smem + L.x + xl.sx);

  cg::cluster_group cluster = cg::this_cluster();
  const int j = static_cast<int>(cluster.block_rank());
  const int h = blockIdx.x / kC;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int inner = P.heads * kDim;
  const int nchunks = p.k >> 4, nb = p.k >> 5;
  trace_entry(p.trace);
  // every CTA of the cluster has started once this barrier completes (it is
  // waited on before the first store into another CTA's shared memory)
  cluster_arrive_relaxed();

  // first row of segment s (0 q, 1 k, 2 v, 3 z) of this CTA
  auto seg_row = [&](int s) -> int64_t { return static_cast<int64_t>(s) * inner + h * kDim + j * kSeg; };
  auto group_row = [&](int gi) -> int64_t { return seg_row(gi / GPS) + (gi % GPS) * GR; };
  // CTA 0 computes the head's alpha row, CTA 1 its beta row (warp 0)
  const bool has_e = j < 2 && warp == 0;
  const int64_t e_row = 4LL * inner + (j == 0 ? 0 : P.heads) + h;
  const float* S = P.state + static_cast<int64_t>(h) * kDim * kDim + j * kSeg;  // + b*heads*dim*dim

  // ---- before the dependency wait: weights and parameters only
  if (tid < 4) prefetch_l2_bulk(p.w + seg_row(tid) * p.row_bytes, static_cast<uint32_t>(kSeg * p.row_bytes));
  if (has_e && lane == 0) prefetch_l2_bulk(p.w + e_row * p.row_bytes, static_cast<uint32_t>(p.row_bytes));
  for (int i = tid; i < NV * kDim; i += kGemvThreads) {
    const int v = i / kDim, r = i % kDim;
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(S + static_cast<int64_t>(v) * P.heads * kDim * kDim +
                                                              static_cast<int64_t>(r) * kDim));
  }
  Tile<GR, J> A, B;
  Tile<1, J> E;
  int g = warp;
  if (g < NG) load_tile<GR, J>(A, p, group_row(g), GR, lane, nchunks);
  if (g + kConsumerWarps < NG) load_tile<GR, J>(B, p, group_row(g + kConsumerWarps), GR, lane, nchunks);
  if (has_e) load_tile<1, J>(E, p, e_row, 1, lane, nchunks);
  // conv weights of the rows this lane finishes in its first two groups
  const int my_r = GR == 4 ? (lane >> 3) : 0;
  const bool mine = GR == 4 ? (lane & 7) == 0 : lane == 0;
  float cwA[4] = {0.f, 0.f, 0.f, 0.f}, cwB[4] = {0.f, 0.f, 0.f, 0.f};
  auto conv_w = [&](int gi, float (&cw)[4]) {
    if (mine && gi < NG && gi / GPS < 3) {
      const float* w = p.conv_w + (group_row(gi) + my_r) * p.conv_k;
#pragma unroll
      for (int t = 0; t < 4; ++t) cw[t] = t < p.conv_k ? w[t] : 0.f;
    }
  };
  conv_w(g, cwA);
  conv_w(g + kConsumerWarps, cwB);
  const float a_log = has_e && j == 0 ? p.a_log[h] : 0.f, dt_bias = has_e && j == 0 ? p.dt_bias[h] : 0.f;
  const float gnw = tid < NV * kSeg ? P.norm_w[j * kSeg + tid % kSeg] : 0.f;
  pdl_launch_dependents();

  pdl_wait();
  trace_waited(p.trace);
  // state slices -> shared memory, in flight during the prologue and the GEMV
  for (int i = tid; i < NV * kDim * 4; i += kGemvThreads) {
    const int v = i / (kDim * 4), r = (i / 4) % kDim, c4 = i % 4;
    cp_async16(st + (static_cast<int64_t>(v) * kDim + r) * kSeg + c4 * 4,
               S + static_cast<int64_t>(v) * P.heads * kDim * kDim + static_cast<int64_t>(r) * kDim + c4 * 4);
  }
  cp_async_commit();
  gemv_prologue<PRO, NV, (J > 1 ? J / 2 : 1)>(p, xd, sx, scratch);
  __syncthreads();
  trace_ready(p.trace);
  cluster_wait();

  // ---- in-projection rows of the slice: q/k after conv + SiLU go to every
  //      CTA of the cluster, v and silu(z) stay here
  const uint4* xd4 = reinterpret_cast<const uint4*>(xd);
  auto run_group = [&](const Tile<GR, J>& t, int gi, const float (&cw)[4]) {
    const int s = gi / GPS, ri = (gi % GPS) * GR + my_r;
    const bool conv_row = s < 3;
    // conv state of the row this lane finishes (batches of <= 2 vectors:
    // loaded before the math; wider ones: at the epilogue, for registers)
    constexpr bool kEarly = NV <= 2;
    const int taps = p.conv_k - 1;
    auto load_ops = [&](int v, EpiOperands& o) {
      const float* cs = p.conv_state + (static_cast<int64_t>(v) * p.n_conv + group_row(gi) + my_r) * taps;
#pragma unroll
      for (int tp = 0; tp < 3; ++tp) o.cs[tp] = tp < taps ? cs[tp] : 0.f;
#pragma unroll
      for (int tp = 0; tp < 4; ++tp) o.cw[tp] = cw[tp];
    };
    EpiOperands eo[kEarly ? NV : 1];
    if constexpr (kEarly) {
      if (mine && conv_row)
#pragma unroll
        for (int v = 0; v < NV; ++v) load_ops(v, eo[v]);
    }
    float acc[GR][NV];
    tile_dot<NV, GR, J>(t, lane, nchunks, nb, xd4, sx, acc);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      float c;
      if constexpr (GR == 4)
        c = reduce_rows4<NV>(acc, v, lane);
      else
        c = warp_sum(acc[0][v]);
      if (mine) {
        if (conv_row) {
          EpiOperands o;
          if constexpr (kEarly)
            o = eo[v];
          else
            load_ops(v, o);
          const float y = conv_silu(p, v, group_row(gi) + my_r, c, o);
          if (s == 2)
            sv[v * kSeg + ri] = y;
          else
            push_all(cluster, (s == 0 ? qf : kf) + v * kDim + j * kSeg + ri, y);
        } else {
          sz[v * kSeg + ri] = silu_f(c);
        }
      }
    }
  };
  while (g < NG) {
    float cw[4] = {0.f, 0.f, 0.f, 0.f};
    if (g < 2 * kConsumerWarps) {
#pragma unroll
      for (int t = 0; t < 4; ++t) cw[t] = cwA[t];
    } else {
      conv_w(g, cw);
    }
    run_group(A, g, cw);
    if (g + 2 * kConsumerWarps < NG) load_tile<GR, J>(A, p, group_row(g + 2 * kConsumerWarps), GR, lane, nchunks);
    g += kConsumerWarps;
    if (g >= NG) break;
    if (g < 2 * kConsumerWarps) {
#pragma unroll
      for (int t = 0; t < 4; ++t) cw[t] = cwB[t];
    } else {
      conv_w(g, cw);
    }
    run_group(B, g, cw);
    if (g + 2 * kConsumerWarps < NG) load_tile<GR, J>(B, p, group_row(g + 2 * kConsumerWarps), GR, lane, nchunks);
    g += kConsumerWarps;
  }
  if (has_e) {
    float acc[1][NV];
    tile_dot<NV, 1, J>(E, lane, nchunks, nb, xd4, sx, acc);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const float c = warp_sum(acc[0][v]);
      if (lane == 0) {
        if (j == 0)
          push_all(cluster, gdec + v, a_log * softplus_f(c + dt_bias));  // decay logit (model/layers.py:99-103)
        else
          push_all(cluster, gbeta + v, c);
      }
    }
  }
  cluster.sync();  // q, k, g and beta of the head are now in every CTA

  // ---- L2 norms (backends.py:251-253): one warp per (vector, q|k)
  for (int t = warp; t < 2 * NV; t += kConsumerWarps) {
    const int v = t >> 1;
    float* x = ((t & 1) ? kf : qf) + v * kDim;
    float vals[kDim / 32];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kDim / 32; ++i) {
      vals[i] = x[lane + 32 * i];
      ss = fmaf(vals[i], vals[i], ss);
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + P.l2_eps);
#pragma unroll
    for (int i = 0; i < kDim / 32; ++i)
      x[lane + 32 * i] = (t & 1) ? __fmul_rn(vals[i], r) : __fmul_rn(__fmul_rn(vals[i], r), P.scale);
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- recurrence on the slice (backends.py:255-268): thread t holds column
  //      t % 16 of rows [8 (t/16), 8 (t/16) + 8)
  const int col_l = tid % kSeg, rg = tid / kSeg, r0 = rg * kR;
  for (int v = 0; v < NV; ++v) {
    const float decay = expf(gdec[v]);
    const float bsig = sigmoid_f(gbeta[v]);
    const float* stv = st + static_cast<int64_t>(v) * kDim * kSeg;
    const float* kv = kf + v * kDim;
    const float* qv = qf + v * kDim;
    float s[kR];
#pragma unroll
    for (int i = 0; i < kR; ++i) s[i] = __fmul_rn(stv[(r0 + i) * kSeg + col_l], decay);
    float rec = 0.f;
#pragma unroll
    for (int i = 0; i < kR; ++i) rec = fmaf(s[i], kv[r0 + i], rec);
    red[rg][col_l] = rec;
    __syncthreads();
    float recalled = 0.f;
#pragma unroll
    for (int w = 0; w < 16; ++w) recalled += red[w][col_l];
    const float delta = __fmul_rn(sv[v * kSeg + col_l] - recalled, bsig);
    float o = 0.f;
    float* Sg = P.state + static_cast<int64_t>(v) * P.heads * kDim * kDim + static_cast<int64_t>(h) * kDim * kDim +
                j * kSeg;
#pragma unroll
    for (int i = 0; i < kR; ++i) {
      s[i] = __fadd_rn(s[i], __fmul_rn(kv[r0 + i], delta));
      Sg[static_cast<int64_t>(r0 + i) * kDim + col_l] = s[i];
      o = fmaf(s[i], qv[r0 + i], o);
    }
    __syncthreads();
    red[rg][col_l] = o;
    __syncthreads();
    if (tid < kSeg) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < 16; ++w) t += red[w][tid];
      ot[v * kSeg + tid] = t;
    }
    __syncthreads();
  }

  // ---- gated RMSNorm over the head's 128 outputs (model/layers.py:113-116):
  //      each CTA's sum of squares goes to every CTA, which add them in rank order
  if (warp == 0) {
    for (int v = 0; v < NV; ++v) {
      const float x = lane < kSeg ? ot[v * kSeg + lane] : 0.f;
      float ss = x * x;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) push_all(cluster, ssq + v * kC + j, ss);
    }
  }
  cluster.sync();  // (no shared memory of another CTA is touched after this)
  if (tid < NV * kSeg) {
    const int v = tid / kSeg, c = tid % kSeg;
    float total = 0.f;
#pragma unroll
    for (int r = 0; r < kC; ++r) total += ssq[v * kC + r];
    const float rn = 1.0f / sqrtf(total / static_cast<float>(kDim) + P.norm_eps);
    const float y = __fmul_rn(__fmul_rn(__fmul_rn(ot[v * kSeg + c], rn), gnw), sz[v * kSeg + c]);
    P.out[static_cast<int64_t>(v) * P.out_bs + static_cast<int64_t>(h) * kDim + j * kSeg + c] = y;
  }
  trace_exit(p.trace);
}

template <int PRO, int NV, int GR, int J>
int launch_fused(const GdnFusedParams& P, cudaStream_t stream, bool pdl) {
  auto kern = gdn_fused_kernel<PRO, NV, GR, J>;
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return fail_cuda(e, "gdn_fused set smem");
    configured_device = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(P.heads) * kC);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = fused_layout(P.g.k, NV).total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = kC;
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = ::bt::launch_ex(&cfg, kern, P);
  if (e != cudaSuccess) return fail_cuda(e, "gdn_fused launch");
  return BT_OK;
}

template <int PRO, int NV>
int launch_nv(const GdnFusedParams& P, cudaStream_t stream, bool pdl) {
  const int J = (P.g.k + 511) / 512;
  if constexpr (NV <= 2) {
    // 4-row groups reuse each activation chunk across rows (K <= 1024)
    if (P.g.k <= 1024) {
      if (J <= 1) return launch_fused<PRO, NV, 4, 1>(P, stream, pdl);
      return launch_fused<PRO, NV, 4, 2>(P, stream, pdl);
    }
  }
  if (J <= 1) return launch_fused<PRO, NV, 1, 1>(P, stream, pdl);
  if (J <= 2) return launch_fused<PRO, NV, 1, 2>(P, stream, pdl);
  if (J <= 4) return launch_fused<PRO, NV, 1, 4>(P, stream, pdl);
  return launch_fused<PRO, NV, 1, 8>(P, stream, pdl);
}

template <int PRO>
int launch_pro(const GdnFusedParams& P, cudaStream_t stream, bool pdl) {
  switch (P.g.n_vec) {
    case 1: return launch_nv<PRO, 1>(P, stream, pdl);
    case 2: return launch_nv<PRO, 2>(P, stream, pdl);
    case 4: return launch_nv<PRO, 4>(P, stream, pdl);
    default: return launch_nv<PRO, 8>(P, stream, pdl);
  }
}

}  // namespace

bool gdn_fused_supported(int64_t hidden, int heads_k, int heads_v, int dim, int batch) {
  return dim == kDim && heads_k == heads_v && heads_v > 0 && hidden >= 32 && hidden % 32 == 0 && hidden <= 4096 &&
         (batch == 1 || batch == 2 || batch == 4 || batch == 8) &&
         fused_layout(static_cast<int>(hidden), batch).total <= kMaxSmem;
}

int gdn_fused_launch(GdnFusedParams& P, cudaStream_t stream, bool pdl) {
  GemvQ8Params& p = P.g;
  if (!gdn_fused_supported(p.k, P.heads, P.heads, P.dim, p.n_vec))
    return fail(BT_ERR_UNSUPPORTED, "fused GDN layer: unsupported shape (hidden %d, heads %d, dim %d, batch %d)", p.k,
                P.heads, P.dim, p.n_vec);
  if (p.prologue != PRO_RESID_NORM && p.prologue != PRO_EMBED_NORM)
    return fail(BT_ERR_UNSUPPORTED, "fused GDN layer: the in-projection normalises its input");
  if (p.conv_k < 2 || p.conv_k > 4) return fail(BT_ERR_UNSUPPORTED, "fused GDN layer: conv kernel of 2..4 taps");
  if (!p.w || (reinterpret_cast<uintptr_t>(p.w) & 15) ||
      ((reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.x2) |
        reinterpret_cast<uintptr_t>(p.norm_w) | reinterpret_cast<uintptr_t>(p.h_out) |
        reinterpret_cast<uintptr_t>(P.state)) & 15))
    return fail(BT_ERR_INVALID, "fused GDN layer: weights, activations and state must be 16-byte aligned");
  p.sb = static_cast<int32_t>(bt_q8_row_bytes(p.k) - p.k);
  p.row_bytes = static_cast<int32_t>(bt_q8_row_bytes(p.k));
  if (p.x_bs == 0) p.x_bs = p.k;
  if (p.x2_bs == 0) p.x2_bs = p.k;
  if ((p.x_bs & 3) || (p.x2_bs & 3)) return fail(BT_ERR_INVALID, "fused GDN layer: strides must be multiples of 4");
  p.n_conv = 3 * P.heads * kDim;
  p.n_z = P.heads * kDim;
  p.n_gh = P.heads;
  return p.prologue == PRO_EMBED_NORM ? launch_pro<PRO_EMBED_NORM>(P, stream, pdl)
                                      : launch_pro<PRO_RESID_NORM>(P, stream, pdl);
}

}  // namespace bt
