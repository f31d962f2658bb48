// Split-KV GQA flash-decode with an in-kernel combine.
//
// Replaces the reference's tilelang split + combine kernels
// (breezetoken/kernels/cuda/attention.py:55-366) and matches its torch
// oracle `_torch_attention` (breezetoken/backends.py:196-215):
//   out[h] = softmax(q[h] . K[:, h / (heads/kv_heads)] * scale) V
//
// Grid (splits, kv_heads, batch); 4 warps per CTA.  A CTA owns one KV head
// (group) of one sequence and a contiguous slice of positions, and serves all
// GS = heads/kv_heads query heads of the group, so every K/V byte is read
// once.  Lane l holds dims [l*DPL, l*DPL + DPL) of the GS queries.  A warp
// takes PB = 32/GS positions at a time: each lane forms GS*PB partial dot
// products, a 31-shuffle reduce-scatter leaves score (head l/PB, position
// l%PB) in lane l, the online softmax runs in base 2 with per-head running
// max/sum, and P.V accumulates with the probabilities broadcast by shuffle.
// Warps merge in shared memory; with several splits the last CTA of a group
// (atomic ticket in the workspace) merges the splits' (max, sum, o) records
// and re-arms the counter, so no second kernel is needed.
//
// Model mode fuses the surrounding ops of the Qwen3.5 attention layer
// (model/layers.py:55-82 / graph.py:35-64): per-head q/k RMSNorm, partial
// rotate-half RoPE at the device position, the KV-cache write at that
// position and the sigmoid output gate.
#include <cooperative_groups.h>

#include "attention.cuh"
#include "errors.h"

namespace cg = cooperative_groups;

namespace bt {

namespace {

constexpr int kAttnWarps = 4;
// A split takes part only with at least this many positions: short contexts
// run in one CTA per group and skip the cross-CTA merge.
constexpr int kMinSplitLen = 64;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr float kLog2e = 1.4426950408889634f;
// K/V rows per CTA prefetched into L2 as soon as the slice is known.
constexpr int kPrefetchRows = 64;
// Model mode with a cluster merge: the first kStageRows K and V rows of a
// CTA's slice are copied into shared memory (cp.async) during the prologue.
constexpr int kStageRows = 16;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Loads issued exactly where they stand (volatile asm keeps their order):
// the model prologue puts every load that does not depend on the position
// ahead of the position load, so the two L2 round trips overlap.
__device__ __forceinline__ float4 ld_f4_now(const float* p) {
  float4 v;
  asm volatile("ld.global.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_f32_now(const float* p) {
  float v;
  asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ int ld_s32_now(const int32_t* p) {
  int v;
  asm volatile("ld.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Sum 32 per-lane values across the warp; lane l returns the total of value l.
__device__ __forceinline__ float reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int stage = 16; stage >= 1; stage >>= 1) {
    const bool upper = (lane & stage) != 0;
#pragma unroll
    for (int i = 0; i < stage; ++i) {
      const float send = upper ? v[i] : v[i + stage];
      const float keep = upper ? v[i + stage] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, stage);
    }
  }
  return v[0];
}

template <typename KV, int DPL>
struct KvRow;

template <int DPL>
struct KvRow<float, DPL> {
  __device__ static __forceinline__ void load(const void* base, int64_t off, float (&o)[DPL]) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
#pragma unroll
    for (int i = 0; i < DPL / 4; ++i) {
      const float4 t = p[i];
      o[4 * i] = t.x;
      o[4 * i + 1] = t.y;
      o[4 * i + 2] = t.z;
      o[4 * i + 3] = t.w;
    }
  }
};

template <>
struct KvRow<__nv_bfloat16, 8> {
  __device__ static __forceinline__ void load(const void* base, int64_t off, float (&o)[8]) {
    const uint4 t = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + off);
    o[0] = bf16_lo(t.x); o[1] = bf16_hi(t.x);
    o[2] = bf16_lo(t.y); o[3] = bf16_hi(t.y);
    o[4] = bf16_lo(t.z); o[5] = bf16_hi(t.z);
    o[6] = bf16_lo(t.w); o[7] = bf16_hi(t.w);
  }
};

template <>
struct KvRow<__nv_bfloat16, 4> {
  __device__ static __forceinline__ void load(const void* base, int64_t off, float (&o)[4]) {
    const uint2 t = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(base) + off);
    o[0] = bf16_lo(t.x); o[1] = bf16_hi(t.x);
    o[2] = bf16_lo(t.y); o[3] = bf16_hi(t.y);
  }
};

// CL = the splits of one (sequence, group) form a thread-block cluster and
// merge through distributed shared memory instead of the global workspace.
template <typename KV, int DPL, int GS, bool CL, bool MODEL>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnParams p) {
  constexpr int DIM = DPL * 32;
  constexpr int PB = 32 / GS;
  __shared__ __align__(16) float qs[GS][DIM];
  // cluster mode: the partials other CTAs store here for the elements this
  // CTA finishes ([split][element], `per` elements per split), and every
  // split's max / sum per head
  __shared__ __align__(16) float rx[CL ? GS * DIM + 8 : 1];
  __shared__ float rm[CL ? 8 : 1][GS], rl[CL ? 8 : 1][GS];
  extern __shared__ __align__(16) float kv_stage[];  // CL && MODEL: [K rows][V rows] of kStageRows x DIM
  __shared__ __align__(16) float kvn[2][DIM];
  __shared__ float wm[kAttnWarps][GS], wl[kAttnWarps][GS];
  __shared__ __align__(16) float wacc[kAttnWarps][GS][DIM];
  __shared__ uint32_t s_ticket;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  trace_entry(p.trace);
  // (cluster mode: every CTA of the cluster has started once this barrier
  // completes; it is waited on before the first store into another CTA)
  if constexpr (CL) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  // model mode: the q/k/v values of this warp's items and the norm weights
  // (items: GS query heads, then k and v of the group; warp w takes items
  // w, w + 4, ...); the weights before the dependency wait
  constexpr int NI = (GS + 2 + kAttnWarps - 1) / kAttnWarps;
  float x[MODEL ? NI : 1][DPL], nwv[MODEL ? NI : 1][DPL];
  if constexpr (MODEL) {
#pragma unroll
    for (int it = 0; it < NI; ++it) {
      const int item = min(warp + it * kAttnWarps, GS + 1);
      const float* nw = (item < GS ? p.q_norm : p.k_norm) + lane * DPL;
#pragma unroll
      for (int i = 0; i < DPL; i += 4) {
        const float4 t = reinterpret_cast<const float4*>(nw)[i / 4];
        nwv[it][i] = t.x, nwv[it][i + 1] = t.y, nwv[it][i + 2] = t.z, nwv[it][i + 3] = t.w;
      }
    }
  }
  pdl_launch_dependents();
  pdl_wait();
  trace_waited(p.trace);

  float gate_first = 0.f;
  const int e_first0 = split * ((GS * DIM + p.splits - 1) / p.splits) + threadIdx.x;
  int L;
  if constexpr (MODEL) {
#pragma unroll
    for (int it = 0; it < NI; ++it) {
      const int item = min(warp + it * kAttnWarps, GS + 1);
      const float* src = item < GS ? p.q + static_cast<int64_t>(b) * p.q_bs + static_cast<int64_t>(g * GS + item) * p.q_hs
                                   : (item == GS ? p.k_new : p.v_new) + static_cast<int64_t>(b) * p.q_bs + g * DIM;
#pragma unroll
      for (int i = 0; i < DPL; i += 4) {
        const float4 t = ld_f4_now(src + lane * DPL + i);
        x[it][i] = t.x, x[it][i + 1] = t.y, x[it][i + 2] = t.z, x[it][i + 3] = t.w;
      }
    }
    // (cluster mode: every CTA merges per = GS*DIM/splits outputs, 1 per thread here)
    if (CL && e_first0 < min(GS * DIM, (split + 1) * ((GS * DIM + p.splits - 1) / p.splits)))
      gate_first = ld_f32_now(p.gate + static_cast<int64_t>(b) * p.q_bs +
                              static_cast<int64_t>(g * GS + e_first0 / DIM) * p.q_hs + e_first0 % DIM);
    L = ld_s32_now(p.pos + b) + 1;
  } else {
    L = p.lens[b];
  }
  if (L < 0 || L > p.cap) {
    if (threadIdx.x == 0 && split == 0) report_status(p.status, BT_ERR_INVALID, SITE_ATTN_LENGTH, L, p.cap, b);
    L = L < 0 ? 0 : p.cap;
  }
  // Only as many splits as keep >= kMinSplitLen positions each take part; the
  // others leave at once and are not counted by the merge ticket.
  // (in cluster mode every CTA of the cluster takes part, possibly with no
  // positions, because all of them meet at the cluster barriers)
  const int splits = CL ? p.splits : max(1, min(p.splits, (L + kMinSplitLen - 1) / kMinSplitLen));
  if (!CL && split >= splits) return;
  const int chunk = (L + splits - 1) / splits;
  const int t0 = min(L, split * chunk), t1 = min(L, t0 + chunk);
  // CL && MODEL: the first kStageRows K and V rows of the slice -> shared memory
  const int staged = (CL && MODEL) ? min(t1 - t0, kStageRows) : 0;
  if constexpr (CL && MODEL) {
    constexpr int C16 = DIM / 4;  // 16-byte pieces per row
    for (int i = threadIdx.x; i < 2 * staged * C16; i += kAttnThreads) {
      const int kv = i / (staged * C16), r = (i / C16) % staged, c = i % C16;
      const float* src = static_cast<const float*>(kv ? p.v : p.k) + static_cast<int64_t>(b) * p.kv_bs +
                         static_cast<int64_t>(t0 + r) * p.kv_ts + g * DIM + 4 * c;
      cp_async16(kv_stage + (kv * kStageRows + r) * DIM + 4 * c, src);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  {
    // K/V rows of the next positions of the slice on their way into L2 while
    // the queries are prepared (one bulk prefetch per row)
    const int n = min(t1 - t0 - staged, kPrefetchRows);
    const int r = threadIdx.x < n ? threadIdx.x : threadIdx.x - n;
    if (threadIdx.x < 2 * n) {
      const KV* base = static_cast<const KV*>(threadIdx.x < n ? p.k : p.v);
      prefetch_l2_bulk(base + static_cast<int64_t>(b) * p.kv_bs + static_cast<int64_t>(t0 + staged + r) * p.kv_ts +
                           g * DIM,
                       DIM * sizeof(KV));
    }
  }
  // the output element this thread finishes first in a cluster merge
  // (cluster mode uses all p.splits CTAs)
  const int per = (GS * DIM + splits - 1) / splits;
  const int e_first = split * per + threadIdx.x;

  if constexpr (!MODEL) {
    for (int i = threadIdx.x; i < GS * DIM; i += kAttnThreads)
      qs[i / DIM][i % DIM] =
          p.q[static_cast<int64_t>(b) * p.q_bs + static_cast<int64_t>(g * GS + i / DIM) * p.q_hs + i % DIM];
    __syncthreads();
  } else {
    const int pos = max(L - 1, 0);  // (L == 0 only after a reported invalid position)
    // the RoPE row at the position (the values and weights are in flight or here)
    const float* crow = p.rope_cos + static_cast<int64_t>(pos) * p.rope_dim;
    const float* srow = p.rope_sin + static_cast<int64_t>(pos) * p.rope_dim;
    float cv[DPL], sv[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      const int dc = min(lane * DPL + i, p.rope_dim - 1);
      cv[i] = ld_f32_now(crow + dc);
      sv[i] = ld_f32_now(srow + dc);
    }
#pragma unroll
    for (int it = 0; it < NI; ++it) {
      const int item = warp + it * kAttnWarps;
      if (item >= GS + 2) break;
      float* dst = item < GS ? qs[item] : kvn[item - GS];
      if (item <= GS) {
        // RMSNorm then rotate-half RoPE on the first rope_dim dims (q and k)
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) ss = fmaf(x[it][i], x[it][i], ss);
        ss = warp_sum(ss);
        const float r = 1.0f / sqrtf(ss / static_cast<float>(DIM) + p.eps);
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          x[it][i] = __fmul_rn(__fmul_rn(x[it][i], r), nwv[it][i]);
          dst[lane * DPL + i] = x[it][i];
        }
        __syncwarp();
        const int half = p.rope_dim >> 1;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          const int d = lane * DPL + i;
          if (d < p.rope_dim) {
            const float partner = d < half ? -dst[d + half] : dst[d - half];
            x[it][i] = __fadd_rn(__fmul_rn(x[it][i], cv[i]), __fmul_rn(partner, sv[i]));
          }
        }
        __syncwarp();
      }
#pragma unroll
      for (int i = 0; i < DPL; ++i) dst[lane * DPL + i] = x[it][i];
    }
    __syncthreads();
    if (pos >= t0 && pos < t1) {
      float* kc = const_cast<float*>(static_cast<const float*>(p.k)) + static_cast<int64_t>(b) * p.kv_bs +
                  static_cast<int64_t>(pos) * p.kv_ts + g * DIM;
      float* vc = const_cast<float*>(static_cast<const float*>(p.v)) + static_cast<int64_t>(b) * p.kv_bs +
                  static_cast<int64_t>(pos) * p.kv_ts + g * DIM;
      for (int i = threadIdx.x; i < DIM; i += kAttnThreads) {
        kc[i] = kvn[0][i];
        vc[i] = kvn[1][i];
      }
      __threadfence_block();
    }
    if constexpr (CL) {
      // the staged rows are in; the new position's row replaces its stale copy
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncthreads();
      if (pos >= t0 && pos < t0 + staged)
        for (int i = threadIdx.x; i < DIM; i += kAttnThreads) {
          kv_stage[(pos - t0) * DIM + i] = kvn[0][i];
          kv_stage[(kStageRows + pos - t0) * DIM + i] = kvn[1][i];
        }
    }
    __syncthreads();
  }

  trace_ready(p.trace);
  float qr[GS][DPL], acc[GS][DPL];
#pragma unroll
  for (int h = 0; h < GS; ++h)
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      qr[h][i] = qs[h][lane * DPL + i];
      acc[h][i] = 0.f;
    }
  float m_run = -INFINITY, l_run = 0.f;
  const float sl = p.scale * kLog2e;
  const int64_t kvbase = static_cast<int64_t>(b) * p.kv_bs + g * DIM + lane * DPL;

  for (int tb = t0 + warp * PB; tb < t1; tb += kAttnWarps * PB) {
    // All PB key rows are loaded before any is used (positions past t1 read
    // the last valid row and are masked below), so a batch costs one memory
    // latency rather than PB.
    // (rows staged in shared memory are read from there)
    float kf[PB][DPL];
#pragma unroll
    for (int pp = 0; pp < PB; ++pp) {
      const int t = min(tb + pp, t1 - 1);
      if (CL && MODEL && t - t0 < staged)
        KvRow<KV, DPL>::load(kv_stage, (t - t0) * DIM + lane * DPL, kf[pp]);
      else
        KvRow<KV, DPL>::load(p.k, kvbase + static_cast<int64_t>(t) * p.kv_ts, kf[pp]);
    }
    float part[32];
#pragma unroll
    for (int pp = 0; pp < PB; ++pp) {
#pragma unroll
      for (int h = 0; h < GS; ++h) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) s = fmaf(qr[h][i], kf[pp][i], s);
        part[h * PB + pp] = s;
      }
    }
    // value rows of the batch, issued before the softmax bookkeeping
    float vf[PB][DPL];
#pragma unroll
    for (int pp = 0; pp < PB; ++pp) {
      const int t = min(tb + pp, t1 - 1);
      if (CL && MODEL && t - t0 < staged)
        KvRow<KV, DPL>::load(kv_stage, (kStageRows + t - t0) * DIM + lane * DPL, vf[pp]);
      else
        KvRow<KV, DPL>::load(p.v, kvbase + static_cast<int64_t>(t) * p.kv_ts, vf[pp]);
    }
    float score = reduce_scatter32(part, lane) * sl;
    const bool valid = tb + (lane % PB) < t1;
    if (!valid) score = -INFINITY;
    float mx = score;
#pragma unroll
    for (int o = PB / 2; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float m_new = fmaxf(m_run, mx);
    const float alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
    const float pe = valid ? exp2f(score - m_new) : 0.f;
    float ps = pe;
#pragma unroll
    for (int o = PB / 2; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    l_run = l_run * alpha + ps;
    m_run = m_new;
#pragma unroll
    for (int h = 0; h < GS; ++h) {
      const float a = __shfl_sync(0xffffffffu, alpha, h * PB);
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[h][i] *= a;
    }
#pragma unroll
    for (int pp = 0; pp < PB; ++pp) {
#pragma unroll
      for (int h = 0; h < GS; ++h) {
        const float w = __shfl_sync(0xffffffffu, pe, h * PB + pp);  // 0 for masked positions
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[h][i] = fmaf(w, vf[pp][i], acc[h][i]);
      }
    }
  }

  // ---------------- merge the warps
  if (lane % PB == 0) {
    wm[warp][lane / PB] = m_run;
    wl[warp][lane / PB] = l_run;
  }
#pragma unroll
  for (int h = 0; h < GS; ++h)
#pragma unroll
    for (int i = 0; i < DPL; ++i) wacc[warp][h][lane * DPL + i] = acc[h][i];
  __syncthreads();

  if constexpr (CL) {
    // ---------------- cluster merge: each CTA stores its partial of element e
    // into the CTA that finishes e (rank e / per), and its per-head max / sum
    // into every CTA; after one cluster barrier each CTA combines locally,
    // splits in rank order.
    cg::cluster_group cluster = cg::this_cluster();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA has started
    for (int e = threadIdx.x; e < GS * DIM; e += kAttnThreads) {
      const int h = e / DIM, d = e % DIM;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][h]);
      float Ls = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        if (wm[w][h] != -INFINITY) {
          const float f = exp2f(wm[w][h] - M);
          Ls = fmaf(wl[w][h], f, Ls);
          O = fmaf(wacc[w][h][d], f, O);
        }
      }
      const int owner = e / per;
      *cluster.map_shared_rank(&rx[split * per + (e - owner * per)], owner) = O;
      if (d == 0)
        for (int r = 0; r < splits; ++r) {
          *cluster.map_shared_rank(&rm[split][h], r) = M;
          *cluster.map_shared_rank(&rl[split][h], r) = Ls;
        }
    }
    cluster.sync();  // (no shared memory of another CTA is touched after this)
    for (int e = split * per + threadIdx.x; e < min(GS * DIM, (split + 1) * per); e += kAttnThreads) {
      const int h = e / DIM, d = e % DIM;
      float M = -INFINITY;
      for (int s2 = 0; s2 < splits; ++s2) M = fmaxf(M, rm[s2][h]);
      float Ls = 0.f, O = 0.f;
      for (int s2 = 0; s2 < splits; ++s2) {
        const float ms = rm[s2][h];
        if (ms != -INFINITY) {
          const float f = exp2f(ms - M);
          Ls = fmaf(rl[s2][h], f, Ls);
          O = fmaf(rx[s2 * per + (e - split * per)], f, O);
        }
      }
      float o = Ls > 0.f ? O / Ls : 0.f;
      if constexpr (MODEL) {
        const float gt = e == e_first ? gate_first
                                      : p.gate[static_cast<int64_t>(b) * p.q_bs +
                                               static_cast<int64_t>(g * GS + h) * p.q_hs + d];
        o *= sigmoid_f(gt);
      }
      p.out[static_cast<int64_t>(b) * p.out_bs + static_cast<int64_t>(g * GS + h) * DIM + d] = o;
    }
    trace_exit(p.trace);
    return;
  }

  // records of this (sequence, group): split s, head h at rec0 + s*GS + h
  const int64_t rec0 = ((static_cast<int64_t>(b) * p.kv_heads + g) * p.splits) * GS;
  for (int e = threadIdx.x; e < GS * DIM; e += kAttnThreads) {
    const int h = e / DIM, d = e % DIM;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][h]);
    float Ls = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      if (wm[w][h] != -INFINITY) {
        const float f = exp2f(wm[w][h] - M);
        Ls = fmaf(wl[w][h], f, Ls);
        O = fmaf(wacc[w][h][d], f, O);
      }
    }
    if (splits == 1) {
      float o = Ls > 0.f ? O / Ls : 0.f;
      if constexpr (MODEL)
        o *= sigmoid_f(p.gate[static_cast<int64_t>(b) * p.q_bs + static_cast<int64_t>(g * GS + h) * p.q_hs + d]);
      p.out[static_cast<int64_t>(b) * p.out_bs + static_cast<int64_t>(g * GS + h) * DIM + d] = o;
    } else {
      float* rec = p.part + (rec0 + static_cast<int64_t>(split) * GS + h) * (DIM + 2);
      rec[d] = O;
      if (d == 0) {
        rec[DIM] = M;
        rec[DIM + 1] = Ls;
      }
    }
  }
  if (splits == 1) {
    if (p.trace) {
      __syncthreads();
      trace_exit(p.trace);
    }
    return;
  }

  // ---------------- merge the splits: the last CTA of a (sequence, group)
  // merges them, in two levels past kMergeGroup splits (the last CTA of each
  // group of kMergeGroup splits merges its group into a group record)
  const int ngrp = static_cast<int>(attn_groups(splits));
  const int64_t bg = static_cast<int64_t>(b) * p.kv_heads + g;
  const int64_t grec0 = static_cast<int64_t>(p.batch) * p.kv_heads * p.splits * GS + bg * ngrp * GS;
  uint32_t* const top_counter = p.counters + bg;
  float* fw = &wacc[0][0][0];  // (the warp-partial buffer is free again: GS x records weights)
  __shared__ float s_sum[GS];
  // merges `count` records starting at record index r0 (stride GS records);
  // final: output (normalised, gated), else one record at record index dst
  auto merge = [&](int64_t r0, int count, bool final, int64_t dst) {
    for (int h = warp; h < GS; h += kAttnWarps) {
      float M = -INFINITY;
      for (int s = lane; s < count; s += 32)
        M = fmaxf(M, __ldcg(p.part + (r0 + static_cast<int64_t>(s) * GS + h) * (DIM + 2) + DIM));
      M = warp_max(M);
      float Ls = 0.f;
      for (int s = lane; s < count; s += 32) {
        const float* rec = p.part + (r0 + static_cast<int64_t>(s) * GS + h) * (DIM + 2);
        const float ms = __ldcg(rec + DIM);
        const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
        fw[h * count + s] = f;
        Ls = fmaf(__ldcg(rec + DIM + 1), f, Ls);
      }
      Ls = warp_sum(Ls);
      if (lane == 0) {
        s_sum[h] = Ls;
        if (!final) {
          float* out_rec = p.part + (dst + h) * (DIM + 2);
          out_rec[DIM] = M;
          out_rec[DIM + 1] = Ls;
        }
      }
    }
    __syncthreads();
    const int64_t rstride = static_cast<int64_t>(GS) * (DIM + 2);
    for (int e = threadIdx.x; e < GS * DIM; e += kAttnThreads) {
      const int h = e / DIM, d = e % DIM;
      const float* base = p.part + (r0 + h) * (DIM + 2) + d;
      const float* f = fw + h * count;
      float O0 = 0.f, O1 = 0.f, O2 = 0.f, O3 = 0.f;
      int s = 0;
      for (; s + 4 <= count; s += 4) {
        const float a0 = __ldcg(base + s * rstride), a1 = __ldcg(base + (s + 1) * rstride);
        const float a2 = __ldcg(base + (s + 2) * rstride), a3 = __ldcg(base + (s + 3) * rstride);
        O0 = fmaf(a0, f[s], O0);
        O1 = fmaf(a1, f[s + 1], O1);
        O2 = fmaf(a2, f[s + 2], O2);
        O3 = fmaf(a3, f[s + 3], O3);
      }
      for (; s < count; ++s) O0 = fmaf(__ldcg(base + s * rstride), f[s], O0);
      const float O = (O0 + O1) + (O2 + O3);
      if (final) {
        const float Ls = s_sum[h];
        float o = Ls > 0.f ? O / Ls : 0.f;
        if constexpr (MODEL)
          o *= sigmoid_f(p.gate[static_cast<int64_t>(b) * p.q_bs + static_cast<int64_t>(g * GS + h) * p.q_hs + d]);
        p.out[static_cast<int64_t>(b) * p.out_bs + static_cast<int64_t>(g * GS + h) * DIM + d] = o;
      } else {
        p.part[(dst + h) * (DIM + 2) + d] = O;
      }
    }
  };
  // arrival: returns true in the last of `n` CTAs counted by *counter (then re-armed)
  auto last_of = [&](uint32_t* counter, int n) -> bool {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      s_ticket = atomicAdd(counter, 1u);
      if (s_ticket == static_cast<uint32_t>(n - 1)) atomicExch(counter, 0u);
    }
    __syncthreads();
    const bool last = s_ticket == static_cast<uint32_t>(n - 1);
    if (last) __threadfence();
    return last;
  };
  if (ngrp == 0) {
    if (!last_of(top_counter, splits)) {
      trace_exit(p.trace);
      return;
    }
    merge(rec0, splits, true, 0);
  } else {
    const int grp = split / kMergeGroup;
    const int in_grp = min(kMergeGroup, splits - grp * kMergeGroup);
    if (!last_of(p.counters + static_cast<int64_t>(p.batch) * p.kv_heads + bg * ngrp + grp, in_grp)) {
      trace_exit(p.trace);
      return;
    }
    merge(rec0 + static_cast<int64_t>(grp) * kMergeGroup * GS, in_grp, false, grec0 + grp * GS);
    if (!last_of(top_counter, ngrp)) {
      trace_exit(p.trace);
      return;
    }
    merge(grec0, ngrp, true, 0);
  }
  if (p.trace) {
    __syncthreads();
    trace_exit(p.trace);
  }
}

template <typename KV, int DPL, int GS>
int launch_t(const AttnParams& p, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.kv_heads, p.batch);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  const bool cl = p.cluster && GS == 4;
  if (cl) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = p.splits;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e;
  if (p.model) {
    // the model keeps an f32 cache (checked by attention_launch)
    if (cl) {
      auto kern = attn_decode_kernel<float, DPL, GS, (GS == 4), true>;
      const int stage_bytes = 2 * kStageRows * DPL * 32 * static_cast<int>(sizeof(float));
      static int configured_device = -1;
      int dev = 0;
      cudaGetDevice(&dev);
      if (configured_device != dev) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, stage_bytes);
        if (e != cudaSuccess) return fail_cuda(e, "attention set smem");
        configured_device = dev;
      }
      cfg.dynamicSmemBytes = stage_bytes;
      e = ::bt::launch_ex(&cfg, kern, p);
    } else {
      e = ::bt::launch_ex(&cfg, attn_decode_kernel<float, DPL, GS, false, true>, p);
    }
  } else {
    e = cl ? ::bt::launch_ex(&cfg, attn_decode_kernel<KV, DPL, GS, (GS == 4), false>, p)
           : ::bt::launch_ex(&cfg, attn_decode_kernel<KV, DPL, GS, false, false>, p);
  }
  if (e != cudaSuccess) return fail_cuda(e, "attention launch");
  return BT_OK;
}

template <typename KV>
int launch_dtype(const AttnParams& p, cudaStream_t stream, bool pdl) {
  const int gs = p.heads / p.kv_heads;
  if (p.dim == 256 && gs == 4) return launch_t<KV, 8, 4>(p, stream, pdl);
  if (p.dim == 256 && gs == 8) return launch_t<KV, 8, 8>(p, stream, pdl);
  if (p.dim == 128 && gs == 4) return launch_t<KV, 4, 4>(p, stream, pdl);
  if (p.dim == 128 && gs == 8) return launch_t<KV, 4, 8>(p, stream, pdl);
  return fail(BT_ERR_UNSUPPORTED, "attention serves head_dim {128, 256} with 4 or 8 query heads per KV head (got dim %d, %d)",
              p.dim, gs);
}

}  // namespace

int attention_launch(const AttnParams& p, cudaStream_t stream, bool pdl) {
  if (p.batch <= 0 || p.kv_heads <= 0 || p.heads <= 0 || p.heads % p.kv_heads != 0)
    return fail(BT_ERR_INVALID, "attention: heads (%d) must be a positive multiple of kv_heads (%d)", p.heads,
                p.kv_heads);
  if (p.splits < 1 || p.splits > 4 * p.dim)
    return fail(BT_ERR_INVALID, "attention: splits must be in [1, %d]", 4 * p.dim);
  if (p.model && p.kv_dtype != BT_F32) return fail(BT_ERR_UNSUPPORTED, "model-mode attention keeps an f32 cache");
  if ((reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v)) & 15)
    return fail(BT_ERR_INVALID, "attention: K/V must be 16-byte aligned (vector loads)");
  if ((p.kv_ts * (p.kv_dtype == BT_BF16 ? 2 : 4)) % 16 || (p.kv_bs * (p.kv_dtype == BT_BF16 ? 2 : 4)) % 16)
    return fail(BT_ERR_INVALID, "attention: K/V strides must be multiples of 16 bytes");
  if (p.model && (p.rope_dim < 2 || p.rope_dim > p.dim || p.rope_dim % 2))
    return fail(BT_ERR_INVALID, "attention: invalid rope_dim %d", p.rope_dim);
  if (p.model && (((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k_new) |
                    reinterpret_cast<uintptr_t>(p.v_new) | reinterpret_cast<uintptr_t>(p.q_norm) |
                    reinterpret_cast<uintptr_t>(p.k_norm)) & 15) ||
                  (p.q_bs & 3) || (p.q_hs & 3)))
    return fail(BT_ERR_INVALID, "model-mode attention reads q/k/v and norm weights as float4: 16-byte aligned, "
                                "strides a multiple of 4");
  if (p.cluster && (p.splits > 8 || p.heads != 4 * p.kv_heads))
    return fail(BT_ERR_UNSUPPORTED, "cluster-merged attention serves <= 8 splits and 4 query heads per KV head");
  return p.kv_dtype == BT_BF16 ? launch_dtype<__nv_bfloat16>(p, stream, pdl) : launch_dtype<float>(p, stream, pdl);
}

}  // namespace bt
