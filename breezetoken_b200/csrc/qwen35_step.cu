// The Qwen3.5 decode step as a fixed schedule of fused kernels.
//
// One step of the reference (`Qwen35.forward_token`, model/qwen35.py:252-286,
// with the in-graph argmax and position increment of GraphMixin._graph_body,
// model/graph.py:66-91) becomes, per layer:
//
//   GDN layer (model/layers.py:84-112)           full-attention layer (:55-82)
//   1 GEMV  resid+RMSNorm | qkv,z,a,b -> conv,   1 GEMV  resid+RMSNorm | q,gate,k,v
//           SiLU, silu(z), softplus decay        2 attention: q/k norm, RoPE, KV write,
//   2 GDN   recurrent step                                    split-KV, sigmoid gate
//   3 GEMV  per-head RMSNorm*silu(z) | out       3 GEMV  o projection
//   4 GEMV  resid+RMSNorm | gate/up -> silu(g)*u (MLP, :114-119)
//   5 GEMV  down
//
// and a final head GEMV with resid+RMSNorm in front and argmax behind.  Every
// kernel is launched with programmatic stream serialization, so each GEMV's
// weight stream starts while its predecessor finishes; every write of a
// kernel happens after its griddepcontrol.wait, so reusing buffers across
// kernels is race-free.  The residual stream ping-pongs between h0 and h1.
#include <cstdlib>
#include <vector>

#include "attention.cuh"
#include "errors.h"
#include "gdn.cuh"
#include "gdn_fused.cuh"
#include "gemv_q8.cuh"

namespace bt {

namespace {

constexpr int kAttnSplits = 8;

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

struct Workspace {
  unsigned long long* best;
  uint32_t* counter;
  float* attn_part;
  uint32_t* attn_counters;
};

Workspace carve(const BtQwen35Dims& d, void* base) {
  Workspace w{};
  uint8_t* p = static_cast<uint8_t*>(base);
  w.best = reinterpret_cast<unsigned long long*>(p);
  p += align256(8LL * d.batch);
  w.counter = reinterpret_cast<uint32_t*>(p);
  p += 256;
  w.attn_part = reinterpret_cast<float*>(p);
  p += align256(4 * attn_part_floats(d.batch, d.n_kv, d.n_heads, d.head_dim, kAttnSplits));
  w.attn_counters = reinterpret_cast<uint32_t*>(p);
  return w;
}

__global__ void advance_pos_kernel(int32_t* pos, int n) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x < n) pos[threadIdx.x] += 1;
}

int validate(const BtQwen35Dims& d) {
  if (d.batch < 1 || d.batch > kMaxVec || (d.batch > 2 && d.batch != 4 && d.batch != 8))
    return fail(BT_ERR_UNSUPPORTED, "decode step serves batch 1, 2, 4 or 8 per GPU (got %d)", d.batch);
  if (d.n_layers < 1 || d.hidden < 32 || d.hidden % 32) return fail(BT_ERR_INVALID, "bad hidden/layers");
  if (d.ssm_heads * d.ssm_state != d.ssm_inner) return fail(BT_ERR_INVALID, "ssm heads * state != inner");
  if (d.n_heads % d.n_kv) return fail(BT_ERR_INVALID, "n_heads must be a multiple of n_kv");
  if (d.conv_k < 2 || d.conv_k > 4) return fail(BT_ERR_UNSUPPORTED, "conv kernel must be in [2, 4]");
  return BT_OK;
}

GemvQ8Params base_gemv(const BtQwen35Dims& d, const BtQwen35Runtime& rt) {
  GemvQ8Params p{};
  p.n_vec = d.batch;
  p.eps = d.eps;
  p.status = rt.status;
  return p;
}

// Programmatic dependent launch between the step's kernels: each kernel's
// weight prefetch and first row loads run while its predecessor finishes.
constexpr bool kUsePdl = true;

// The fused GDN layer kernel where it serves the shapes (on by default;
// BT_GDN_FUSED=0 runs in-projection, recurrence and gated-norm out-projection
// as three kernels, for measurements).
bool gdn_fused_enabled(const BtQwen35Dims& d) {
  static const bool on = [] {
    const char* v = getenv("BT_GDN_FUSED");
    return !(v && v[0] == '0');
  }();
  return on && gdn_fused_supported(d.hidden, d.ssm_heads, d.ssm_heads, d.ssm_state, d.batch);
}

int run_gemv(GemvQ8Params& p, cudaStream_t s) {
  GemvQ8Launch L{};
  int rc = gemv_q8_plan(p, sm_count(), L);
  if (rc) return rc;
  return gemv_q8_launch(p, L, s, kUsePdl);
}

}  // namespace

int qwen35_kernels_per_step(const BtQwen35Model& m) {
  const BtQwen35Dims& d = m.dims;
  int n = 1;  // the head
  for (int i = 0; i < d.n_layers; ++i) n += (!m.layers[i].is_attn && gdn_fused_enabled(d)) ? 4 : 5;
  return n;
}

int64_t qwen35_proj_elems(const BtQwen35Dims& d) {
  const int64_t gdn = 4LL * d.ssm_inner + 2LL * d.ssm_heads;
  const int64_t attn = 2LL * d.n_heads * d.head_dim + 2LL * d.n_kv * d.head_dim;
  const int64_t n = gdn > attn ? gdn : attn;
  return (n + 3) / 4 * 4;  // rows of the buffer stay 16-byte aligned
}

int64_t qwen35_workspace_bytes(const BtQwen35Dims& d) {
  return align256(8LL * d.batch) + 256 +
         align256(4 * attn_part_floats(d.batch, d.n_kv, d.n_heads, d.head_dim, kAttnSplits)) +
         align256(4 * attn_counters(d.batch, d.n_kv, kAttnSplits));
}

int qwen35_step(const BtQwen35Model& m, const BtQwen35Runtime& rt, int with_logits, cudaStream_t s) {
  const BtQwen35Dims& d = m.dims;
  int rc = validate(d);
  if (rc) return rc;
  if (!m.embed || !m.layers || !rt.pos || !rt.token || !rt.h0 || !rt.h1 || !rt.delta || !rt.proj || !rt.mix ||
      !rt.act || !rt.workspace)
    return fail(BT_ERR_INVALID, "decode step: null model/runtime pointer");
  const Workspace ws = carve(d, rt.workspace);
  const int64_t proj_stride = qwen35_proj_elems(d);
  const int64_t mix_stride = d.ssm_inner > d.n_heads * d.head_dim ? d.ssm_inner : d.n_heads * d.head_dim;
  float* hc = rt.h0;
  float* ho = rt.h1;
  int kidx = 0;  // launch index within the step, for the optional tracer
  auto trace = [&]() -> TraceRec* { return rt.trace ? static_cast<TraceRec*>(rt.trace) + kidx++ : nullptr; };

  for (int i = 0; i < d.n_layers; ++i) {
    const BtQwen35Layer& ly = m.layers[i];
    // ---- 1: in-projection with residual + RMSNorm in front
    GemvQ8Params p1 = base_gemv(d, rt);
    p1.w = static_cast<const uint8_t*>(ly.w_in);
    p1.k = d.hidden;
    p1.norm_w = ly.norm_in;
    p1.y = rt.proj;
    p1.y_stride = proj_stride;
    if (i == 0) {
      p1.prologue = PRO_EMBED_NORM;
      p1.embed = static_cast<const uint8_t*>(m.embed);
      p1.embed_rows = d.vocab;
      p1.tokens = rt.token;
      p1.h_out = hc;
    } else {
      p1.prologue = PRO_RESID_NORM;
      p1.x = hc;
      p1.x2 = rt.delta;
      p1.h_out = ho;
      std::swap(hc, ho);
    }
    const bool fused = !ly.is_attn && gdn_fused_enabled(d);
    if (!ly.is_attn) {
      p1.n_rows = 4LL * d.ssm_inner + 2LL * d.ssm_heads;
      p1.epilogue = EPI_GDN_IN;
      p1.conv_state = ly.conv_state;
      p1.conv_w = ly.conv_w;
      p1.a_log = ly.a_log;
      p1.dt_bias = ly.dt_bias;
      p1.n_conv = 3 * d.ssm_inner;
      p1.n_z = d.ssm_inner;
      p1.n_gh = d.ssm_heads;
      p1.conv_k = d.conv_k;
    } else {
      p1.n_rows = 2LL * d.n_heads * d.head_dim + 2LL * d.n_kv * d.head_dim;
      p1.epilogue = EPI_STORE;
    }
    p1.trace = trace();
    if (fused) {
      // ---- 1+2: in-projection, conv, recurrence and gated norm in one kernel
      GdnFusedParams f{};
      f.g = p1;
      f.heads = d.ssm_heads;
      f.dim = d.ssm_state;
      f.state = ly.rec_state;
      f.scale = 1.0f / sqrtf(static_cast<float>(d.ssm_state));
      f.l2_eps = d.l2_eps;
      f.norm_w = ly.ssm_norm;
      f.norm_eps = d.eps;
      f.out = rt.mix;
      f.out_bs = mix_stride;
      if ((rc = gdn_fused_launch(f, s, kUsePdl))) return rc;
    } else if ((rc = run_gemv(p1, s))) {
      return rc;
    }

    // ---- 2: the mixer
    if (fused) {
      // done above
    } else if (!ly.is_attn) {
      GdnParams g{};
      g.q = rt.proj;
      g.k = rt.proj + d.ssm_inner;
      g.v = rt.proj + 2LL * d.ssm_inner;
      g.in_dtype = BT_F32;
      g.q_bs = g.k_bs = g.v_bs = proj_stride;
      g.g = rt.proj + 4LL * d.ssm_inner;
      g.beta = rt.proj + 4LL * d.ssm_inner + d.ssm_heads;
      g.g_bs = g.beta_bs = proj_stride;
      g.state = ly.rec_state;
      g.out = rt.mix;
      g.out_bs = mix_stride;
      g.batch = d.batch;
      g.heads_k = d.ssm_heads;
      g.heads_v = d.ssm_heads;
      g.dim = d.ssm_state;
      g.scale = 1.0f / sqrtf(static_cast<float>(d.ssm_state));
      g.eps = d.l2_eps;
      g.status = rt.status;
      g.trace = trace();
      if ((rc = gdn_decode_launch(g, s, kUsePdl))) return rc;
    } else {
      AttnParams a{};
      const int64_t qsz = 2LL * d.n_heads * d.head_dim;
      a.q = rt.proj;
      a.q_bs = proj_stride;
      a.q_hs = 2 * d.head_dim;
      a.gate = rt.proj + d.head_dim;
      a.k_new = rt.proj + qsz;
      a.v_new = rt.proj + qsz + static_cast<int64_t>(d.n_kv) * d.head_dim;
      a.k = ly.k_cache;
      a.v = ly.v_cache;
      a.kv_dtype = BT_F32;
      a.kv_ts = d.n_kv * d.head_dim;
      a.kv_bs = static_cast<int64_t>(d.max_ctx) * a.kv_ts;
      a.out = rt.mix;
      a.out_bs = mix_stride;
      a.batch = d.batch;
      a.heads = d.n_heads;
      a.kv_heads = d.n_kv;
      a.dim = d.head_dim;
      a.cap = d.max_ctx;
      a.splits = kAttnSplits;
      a.cluster = (d.n_heads == 4 * d.n_kv) ? 1 : 0;
      a.scale = 1.0f / sqrtf(static_cast<float>(d.head_dim));
      a.model = 1;
      a.pos = rt.pos;
      a.q_norm = ly.q_norm;
      a.k_norm = ly.k_norm;
      a.rope_cos = m.rope_cos;
      a.rope_sin = m.rope_sin;
      a.rope_dim = d.rope_dim;
      a.eps = d.eps;
      a.part = ws.attn_part;
      a.counters = ws.attn_counters;
      a.status = rt.status;
      a.trace = trace();
      if ((rc = attention_launch(a, s, kUsePdl))) return rc;
    }

    // ---- 3: out-projection
    GemvQ8Params p3 = base_gemv(d, rt);
    p3.w = static_cast<const uint8_t*>(ly.w_out);
    p3.n_rows = d.hidden;
    p3.x = rt.mix;
    p3.x_bs = mix_stride;
    p3.y = rt.delta;
    p3.y_stride = d.hidden;
    p3.epilogue = EPI_STORE;
    if (fused) {
      p3.k = d.ssm_inner;
      p3.prologue = PRO_LOAD;
    } else if (!ly.is_attn) {
      p3.k = d.ssm_inner;
      p3.prologue = PRO_GATED_NORM;
      p3.x2 = rt.proj + 3LL * d.ssm_inner;
      p3.x2_bs = proj_stride;
      p3.norm_w = ly.ssm_norm;
      p3.group = d.ssm_state;
    } else {
      p3.k = d.n_heads * d.head_dim;
      p3.prologue = PRO_LOAD;
    }
    p3.trace = trace();
    if ((rc = run_gemv(p3, s))) return rc;

    // ---- 4: gate/up with residual + RMSNorm in front, SiLU-gate behind
    GemvQ8Params p4 = base_gemv(d, rt);
    p4.w = static_cast<const uint8_t*>(ly.w_gu);
    p4.n_rows = 2LL * d.ffn;
    p4.k = d.hidden;
    p4.prologue = PRO_RESID_NORM;
    p4.x = hc;
    p4.x2 = rt.delta;
    p4.h_out = ho;
    std::swap(hc, ho);
    p4.norm_w = ly.norm_post;
    // batches of <= 2 pair gate/up rows in the epilogue (4-row groups);
    // wider batches store them interleaved and the down projection pairs them
    const bool pair_late = d.batch > 2;
    p4.epilogue = pair_late ? EPI_STORE : EPI_SILU_PAIR;
    p4.y = rt.act;
    p4.y_stride = pair_late ? 2LL * d.ffn : d.ffn;
    p4.trace = trace();
    if ((rc = run_gemv(p4, s))) return rc;

    // ---- 5: down
    GemvQ8Params p5 = base_gemv(d, rt);
    p5.w = static_cast<const uint8_t*>(ly.w_down);
    p5.n_rows = d.hidden;
    p5.k = d.ffn;
    p5.prologue = pair_late ? PRO_SILU_PAIR : PRO_LOAD;
    p5.x = rt.act;
    p5.x_bs = pair_late ? 2LL * d.ffn : d.ffn;
    p5.epilogue = EPI_STORE;
    p5.y = rt.delta;
    p5.y_stride = d.hidden;
    p5.trace = trace();
    if ((rc = run_gemv(p5, s))) return rc;
  }

  if (!with_logits) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = kUsePdl ? 1 : 0;
    cudaError_t e = ::bt::launch_ex(&cfg, advance_pos_kernel, rt.pos, static_cast<int>(d.batch));
    return e == cudaSuccess ? BT_OK : fail_cuda(e, "advance_pos");
  }

  // ---- head: final residual + output_norm, tied-embedding GEMV, argmax
  GemvQ8Params ph = base_gemv(d, rt);
  ph.w = static_cast<const uint8_t*>(m.embed);
  ph.n_rows = d.vocab;
  ph.k = d.hidden;
  ph.prologue = PRO_RESID_NORM;
  ph.x = hc;
  ph.x2 = rt.delta;
  ph.h_out = ho;
  ph.norm_w = m.layers[d.n_layers - 1].norm_next;
  ph.epilogue = EPI_ARGMAX;
  ph.y = rt.logits;
  ph.y_stride = d.vocab;
  ph.best = ws.best;
  ph.counter = ws.counter;
  ph.token_out = rt.token;
  ph.pos = rt.pos;
  ph.history = rt.history;
  ph.history_stride = d.max_ctx;
  ph.trace = trace();
  return run_gemv(ph, s);
}

}  // namespace bt
