// extern "C" entry points declared in include/bt_b200.h.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "attention.cuh"
#include "qwen36_layer.cuh"
#include "errors.h"
#include "gdn.cuh"
#include "gemv_q8.cuh"
#include "linear_rows.cuh"
#include "moe.cuh"
#include "ops.cuh"

namespace bt {

int64_t qwen35_proj_elems(const BtQwen35Dims& d);
int qwen35_kernels_per_step(const BtQwen35Model& m);
int64_t qwen35_workspace_bytes(const BtQwen35Dims& d);
int qwen35_step(const BtQwen35Model& m, const BtQwen35Runtime& rt, int with_logits, cudaStream_t s);

namespace {
thread_local char g_last_error[512] = "";
std::mutex g_sm_mutex;
std::vector<int> g_sm_counts;
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int fail_cuda(cudaError_t err, const char* what) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", what, cudaGetErrorString(err),
           cudaGetErrorName(err));
  return BT_ERR_CUDA;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  if (dev >= static_cast<int>(g_sm_counts.size())) g_sm_counts.resize(dev + 1, 0);
  if (!g_sm_counts[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_counts[dev] = n;
  }
  return g_sm_counts[dev];
}

}  // namespace bt

using bt::fail;

namespace {
inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
}  // namespace

extern "C" {

const char* bt_last_error(void) { return bt::g_last_error; }

int bt_version(void) { return 100; }

int bt_sm_count(void) { return bt::sm_count(); }

int64_t bt_q8_row_bytes(int64_t k) {
  const int64_t scale_bytes = (k / 32) * 2;
  return (scale_bytes + 15) / 16 * 16 + k;
}

int bt_repack_q8_0(const void* src, void* dst, int64_t rows, int64_t k, int64_t dst_row0, int64_t dst_row_step,
                   void* stream) {
  return bt::repack_q8_0(src, dst, rows, k, dst_row0, dst_row_step, as_stream(stream));
}

int bt_dequant_q8_rows(const void* w, float* out, int64_t rows, int64_t k, void* stream) {
  return bt::dequant_q8_rows(w, out, rows, k, as_stream(stream));
}

int bt_dequant_iq3_s(const void* raw, float* out, int64_t rows, int64_t cols, void* stream) {
  return bt::dequant_iq3_s(raw, out, rows, cols, as_stream(stream));
}

int64_t bt_iq3s_row_bytes(int64_t k) { return k > 0 && k % 256 == 0 ? bt::iq3s_row_bytes(k) : 0; }

int bt_repack_iq3_s(const void* src, void* dst, int64_t rows, int64_t k, void* stream) {
  return bt::repack_iq3_s(src, dst, rows, k, as_stream(stream));
}

int bt_moe_route(const float* logits, int64_t t, int64_t n_experts, int top_k, int32_t* ids, float* weights,
                 void* stream) {
  return bt::moe_route(logits, t, n_experts, top_k, ids, weights, as_stream(stream));
}

int64_t bt_moe_workspace_bytes(int64_t t, int64_t hidden, int64_t ffn, int64_t n_experts, int top_k) {
  return bt::moe_workspace_bytes(t, hidden, ffn, 0, n_experts, top_k);
}

int bt_moe_experts_iq3s(const void* gate, const void* up, const void* down, const float* x, int64_t t,
                        int64_t hidden, int64_t ffn, int64_t n_experts, const int32_t* ids, const float* weights,
                        int top_k, float* out, void* workspace, void* stream) {
  return bt::moe_layer_iq3s(gate, up, down, nullptr, x, t, hidden, ffn, n_experts, ids, weights, top_k, out,
                            workspace, as_stream(stream));
}

int64_t bt_moe_layer_workspace_bytes(int64_t t, int64_t hidden, int64_t ffn, int64_t shared_ffn, int64_t n_experts,
                                     int top_k) {
  return bt::moe_workspace_bytes(t, hidden, ffn, shared_ffn, n_experts, top_k);
}

int bt_moe_layer_iq3s(const void* gate, const void* up, const void* down, const BtMoeShared* shared, const float* x,
                      int64_t t, int64_t hidden, int64_t ffn, int64_t n_experts, const int32_t* ids,
                      const float* weights, int top_k, float* out, void* workspace, void* stream) {
  if (!shared)
    return bt::moe_layer_iq3s(gate, up, down, nullptr, x, t, hidden, ffn, n_experts, ids, weights, top_k, out,
                              workspace, as_stream(stream));
  const bt::MoeShared sh{shared->gate, shared->up, shared->down, shared->gate_inp, shared->ffn};
  return bt::moe_layer_iq3s(gate, up, down, &sh, x, t, hidden, ffn, n_experts, ids, weights, top_k, out, workspace,
                            as_stream(stream));
}

namespace {
int moe_add_norm(const void* gate, const void* up, const void* down, const BtMoeShared* shared, const float* x,
                 int64_t t, int64_t hidden, int64_t ffn, int64_t n_experts, const int32_t* ids, const float* weights,
                 int top_k, const float* h, const float* w, float eps, float* h_out, float* y, void* planes,
                 float* out, void* workspace, void* stream, int prep_part) {
  const bt::MoeNorm nm{h, w, h_out, y, planes, eps};
  if (!shared)
    return bt::moe_layer_iq3s(gate, up, down, nullptr, x, t, hidden, ffn, n_experts, ids, weights, top_k, out,
                              workspace, as_stream(stream), &nm, prep_part);
  const bt::MoeShared sh{shared->gate, shared->up, shared->down, shared->gate_inp, shared->ffn};
  return bt::moe_layer_iq3s(gate, up, down, &sh, x, t, hidden, ffn, n_experts, ids, weights, top_k, out, workspace,
                            as_stream(stream), &nm, prep_part);
}
}  // namespace

int bt_moe_layer_iq3s_add_norm(const void* gate, const void* up, const void* down, const BtMoeShared* shared,
                               const float* x, int64_t t, int64_t hidden, int64_t ffn, int64_t n_experts,
                               const int32_t* ids, const float* weights, int top_k, const float* h, const float* w,
                               float eps, float* h_out, float* y, void* planes, float* out, void* workspace,
                               void* stream) {
  return moe_add_norm(gate, up, down, shared, x, t, hidden, ffn, n_experts, ids, weights, top_k, h, w, eps, h_out, y,
                      planes, out, workspace, stream, bt::kPrepAll);
}

int bt_moe_layer_iq3s_add_norm_prepared(const void* gate, const void* up, const void* down,
                                        const BtMoeShared* shared, const float* x, int64_t t, int64_t hidden,
                                        int64_t ffn, int64_t n_experts, const int32_t* ids, const float* weights,
                                        int top_k, const float* h, const float* w, float eps, float* h_out, float* y,
                                        void* planes, float* out, void* workspace, void* stream) {
  return moe_add_norm(gate, up, down, shared, x, t, hidden, ffn, n_experts, ids, weights, top_k, h, w, eps, h_out, y,
                      planes, out, workspace, stream, bt::kPrepNone);
}

int bt_moe_route_sort_iq3s(const float* logits, const float* x, int64_t t, int64_t hidden, int64_t ffn,
                           int64_t n_experts, int top_k, int64_t shared_ffn, int32_t* ids, float* weights,
                           void* workspace, void* stream) {
  return bt::moe_route_sort_iq3s(logits, x, t, hidden, ffn, n_experts, top_k, shared_ffn, ids, weights, workspace,
                                 as_stream(stream));
}

int bt_linear_q8(const void* w, const float* x, float* y, int64_t n, int64_t k, int n_vec, void* stream) {
  if (!w || !x || !y) return fail(BT_ERR_INVALID, "linear_q8: null pointer");
  if (k > (1 << 20)) return fail(BT_ERR_UNSUPPORTED, "linear_q8: K too large");
  if (n_vec != 1 && n_vec != 2 && n_vec != 4 && n_vec != 8)
    return fail(BT_ERR_UNSUPPORTED, "linear_q8: n_vec must be 1, 2, 4 or 8 (got %d)", n_vec);
  bt::GemvQ8Params p{};
  p.w = static_cast<const uint8_t*>(w);
  p.n_rows = n;
  p.k = static_cast<int32_t>(k);
  p.n_vec = n_vec;
  p.prologue = bt::PRO_LOAD;
  p.x = x;
  p.epilogue = bt::EPI_STORE;
  p.y = y;
  p.y_stride = n;
  bt::GemvQ8Launch L{};
  int rc = bt::gemv_q8_plan(p, bt::sm_count(), L);
  if (rc) return rc;
  return bt::gemv_q8_launch(p, L, as_stream(stream), false);
}

int bt_linear_kn(const void* w, int w_dtype, const float* x, float* y, int64_t k, int64_t n, void* stream) {
  return bt::linear_kn(w, w_dtype, x, y, k, n, as_stream(stream));
}

int bt_conv_silu(const float* entry, float* state, const float* w, float* out, int64_t batch, int64_t channels,
                 int64_t taps, void* stream) {
  return bt::conv_silu(entry, state, w, out, 1, batch, channels, taps, as_stream(stream));
}

int bt_conv_silu_scan(const float* entry, float* state, const float* w, float* out, int64_t steps, int64_t batch,
                      int64_t channels, int64_t taps, void* stream) {
  return bt::conv_silu(entry, state, w, out, steps, batch, channels, taps, as_stream(stream));
}

int bt_bf16_planes(const float* x, void* planes, int64_t t, int64_t k, void* stream) {
  return bt::bf16_planes(x, planes, t, k, as_stream(stream));
}

int bt_linear_rows(const void* w, int w_dtype, const void* x_planes, float* y, int64_t n, int64_t k, int64_t t,
                   void* stream) {
  return bt::linear_rows(w, w_dtype, x_planes, y, n, k, t, as_stream(stream));
}

int bt_linear_rows_timeouts(void) { return bt::linear_rows_timeouts(); }

long long bt_launch_count(void) { return bt::g_launch_count.load(std::memory_order_relaxed); }

int bt_rms_norm(const float* x, const float* w, float* y, int64_t rows, int64_t n, float eps, void* stream) {
  return bt::rms_norm(x, nullptr, w, nullptr, y, rows, n, eps, as_stream(stream));
}

int bt_fused_add_rms_norm(const float* a, const float* b, const float* w, float* h, float* xn, int64_t rows,
                          int64_t n, float eps, void* stream) {
  if (!b || !h) return fail(BT_ERR_INVALID, "fused_add_rms_norm: null pointer");
  return bt::rms_norm(a, b, w, h, xn, rows, n, eps, as_stream(stream));
}

int bt_silu_mul(const float* g, const float* u, float* y, int64_t n, void* stream) {
  return bt::silu_mul(g, u, y, n, as_stream(stream));
}

int bt_rope(const float* x, const float* cos_t, const float* sin_t, const int32_t* pos, float* y, int64_t rows,
            int64_t dim, int64_t rope_dim, int64_t cap, void* stream) {
  return bt::rope(x, cos_t, sin_t, pos, y, rows, dim, rope_dim, cap, as_stream(stream));
}

int64_t bt_attention_workspace_bytes(int64_t batch, int64_t kv_heads, int64_t heads, int64_t dim, int splits) {
  if (batch < 1 || kv_heads < 1 || heads < 1 || dim < 1 || splits < 1) return 0;
  const int64_t part = (4 * bt::attn_part_floats(batch, kv_heads, heads, dim, splits) + 255) / 256 * 256;
  return part + (4 * bt::attn_counters(batch, kv_heads, splits) + 255) / 256 * 256;
}

int bt_attention_decode(const float* q, const void* k, const void* v, int kv_dtype, const int32_t* lens, float* out,
                        int64_t batch, int64_t heads, int64_t kv_heads, int64_t dim, int64_t cap, float scale,
                        int splits, void* workspace, void* stream) {
  if (!q || !k || !v || !lens || !out) return fail(BT_ERR_INVALID, "attention: null pointer");
  if (splits > 1 && !workspace) return fail(BT_ERR_INVALID, "attention: splits > 1 needs a workspace");
  if (batch > 65535 || cap < 1 || cap > (1LL << 30) || kv_heads > 65535)
    return fail(BT_ERR_UNSUPPORTED, "attention: shape out of range");
  bt::AttnParams p{};
  p.q = q;
  p.q_bs = heads * dim;
  p.q_hs = static_cast<int32_t>(dim);
  p.k = k;
  p.v = v;
  p.kv_dtype = kv_dtype;
  p.kv_ts = static_cast<int32_t>(kv_heads * dim);
  p.kv_bs = cap * kv_heads * dim;
  p.lens = lens;
  p.out = out;
  p.out_bs = heads * dim;
  p.batch = static_cast<int32_t>(batch);
  p.heads = static_cast<int32_t>(heads);
  p.kv_heads = static_cast<int32_t>(kv_heads);
  p.dim = static_cast<int32_t>(dim);
  p.cap = static_cast<int32_t>(cap);
  p.splits = splits;
  p.scale = scale;
  if (splits > 1) {
    p.part = static_cast<float*>(workspace);
    const int64_t part_bytes = (4 * bt::attn_part_floats(batch, kv_heads, heads, dim, splits) + 255) / 256 * 256;
    p.counters = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + part_bytes);
  }
  return bt::attention_launch(p, as_stream(stream), false);
}

int bt_attention_layer(const float* proj, int64_t proj_bs, const float* q_norm, const float* k_norm,
                       const float* rope_cos, const float* rope_sin, int64_t rope_dim, const int32_t* pos,
                       float* k_cache, float* v_cache, float* out, int64_t batch, int64_t heads, int64_t kv_heads,
                       int64_t dim, int64_t cap, float scale, float eps, int splits, void* workspace,
                       int32_t* status, void* stream) {
  if (!proj || !q_norm || !k_norm || !rope_cos || !rope_sin || !pos || !k_cache || !v_cache || !out)
    return fail(BT_ERR_INVALID, "attention layer: null pointer");
  if (splits > 1 && !workspace) return fail(BT_ERR_INVALID, "attention layer: splits > 1 needs a workspace");
  if (batch < 1 || batch > 65535 || heads < 1 || heads > 65535 || kv_heads < 1 || kv_heads > 65535 || dim < 1 ||
      dim > 1024 || cap < 1 || cap > (1LL << 30) || rope_dim < 2 || rope_dim > dim)
    return fail(BT_ERR_INVALID, "attention layer: shape out of range");
  const int64_t need = (2 * heads + 2 * kv_heads) * dim;
  if (proj_bs < need) return fail(BT_ERR_INVALID, "attention layer: projection rows of %lld < %lld elements",
                                  static_cast<long long>(proj_bs), static_cast<long long>(need));
  bt::AttnParams p{};
  p.q = proj;
  p.q_bs = proj_bs;
  p.q_hs = static_cast<int32_t>(2 * dim);
  p.gate = proj + dim;
  p.k_new = proj + 2 * heads * dim;
  p.v_new = proj + (2 * heads + kv_heads) * dim;
  p.k = k_cache;
  p.v = v_cache;
  p.kv_dtype = BT_F32;
  p.kv_ts = static_cast<int32_t>(kv_heads * dim);
  p.kv_bs = cap * kv_heads * dim;
  p.out = out;
  p.out_bs = heads * dim;
  p.batch = static_cast<int32_t>(batch);
  p.heads = static_cast<int32_t>(heads);
  p.kv_heads = static_cast<int32_t>(kv_heads);
  p.dim = static_cast<int32_t>(dim);
  p.cap = static_cast<int32_t>(cap);
  p.splits = splits;
  p.cluster = (heads == 4 * kv_heads && splits <= 8) ? 1 : 0;
  p.scale = scale;
  p.model = 1;
  p.pos = pos;
  p.q_norm = q_norm;
  p.k_norm = k_norm;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.rope_dim = static_cast<int32_t>(rope_dim);
  p.eps = eps;
  p.status = status;
  if (splits > 1) {
    p.part = static_cast<float*>(workspace);
    const int64_t part_bytes = (4 * bt::attn_part_floats(batch, kv_heads, heads, dim, splits) + 255) / 256 * 256;
    p.counters = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + part_bytes);
  }
  return bt::attention_launch(p, as_stream(stream), false);
}

int bt_gdn_gated_step(const float* mixed, int64_t mixed_bs, const float* ba, int64_t ba_bs, const float* a_log,
                      const float* dt_bias, float* state, const float* z, int64_t z_bs, const float* norm_w,
                      void* planes, int64_t batch, int64_t heads_k, int64_t heads_v, int64_t dim, float scale,
                      float l2_eps, float norm_eps, void* stream) {
  return bt_gdn_gated_scan(mixed, mixed_bs, ba, ba_bs, a_log, dt_bias, state, z, z_bs, norm_w, planes, 1, batch,
                           heads_k, heads_v, dim, scale, l2_eps, norm_eps, stream);
}

int bt_gdn_gated_scan(const float* mixed, int64_t mixed_bs, const float* ba, int64_t ba_bs, const float* a_log,
                      const float* dt_bias, float* state, const float* z, int64_t z_bs, const float* norm_w,
                      void* planes, int64_t steps, int64_t batch, int64_t heads_k, int64_t heads_v, int64_t dim,
                      float scale, float l2_eps, float norm_eps, void* stream) {
  if (batch < 1 || batch > (1LL << 24) || heads_k < 1 || heads_k > 65535 || heads_v < 1 || heads_v > 65535 ||
      steps < 1 || steps * batch > 0x7fffffffLL)
    return fail(BT_ERR_INVALID, "gdn gated step: shape out of range");
  bt::GdnStepParams p{};
  p.steps = static_cast<int32_t>(steps);
  p.mixed = mixed;
  p.mixed_bs = mixed_bs;
  p.ba = ba;
  p.ba_bs = ba_bs;
  p.a_log = a_log;
  p.dt_bias = dt_bias;
  p.state = state;
  p.z = z;
  p.z_bs = z_bs;
  p.norm_w = norm_w;
  p.planes = planes;
  p.batch = static_cast<int32_t>(batch);
  p.heads_k = static_cast<int32_t>(heads_k);
  p.heads_v = static_cast<int32_t>(heads_v);
  p.dim = static_cast<int32_t>(dim);
  p.scale = scale;
  p.l2_eps = l2_eps;
  p.norm_eps = norm_eps;
  return bt::gdn_gated_step_launch(p, as_stream(stream));
}

int bt_add_rms_norm_planes(const float* a, const float* b, const float* w, float* h, float* y, void* planes,
                           int64_t rows, int64_t n, float eps, void* stream) {
  return bt::add_rms_norm_planes(a, b, w, h, y, planes, rows, n, eps, as_stream(stream));
}

int bt_gdn_decode(const void* q, const void* k, const void* v, int in_dtype, const float* g, const float* beta,
                  float* state, float* out, int64_t batch, int64_t heads_k, int64_t heads_v, int64_t dim, float scale,
                  float eps, void* stream) {
  return bt_gdn_decode_strided(q, k, v, in_dtype, heads_k * dim, heads_k * dim, heads_v * dim, g, heads_v, beta,
                               heads_v, state, out, heads_v * dim, batch, heads_k, heads_v, dim, scale, eps, stream);
}

int bt_gdn_prefill(const void* q, const void* k, const void* v, int in_dtype, int64_t q_bs, int64_t k_bs,
                   int64_t v_bs, int64_t q_ts, int64_t k_ts, int64_t v_ts, const float* g, int64_t g_bs, int64_t g_ts,
                   const float* beta, int64_t beta_bs, int64_t beta_ts, float* state, float* out, int64_t out_bs,
                   int64_t out_ts, int64_t steps, int64_t batch, int64_t heads_k, int64_t heads_v, int64_t dim,
                   float scale, float eps, void* stream) {
  if (!q || !k || !v || !g || !beta || !state || !out) return fail(BT_ERR_INVALID, "gdn_prefill: null pointer");
  if (steps < 0 || steps > 0x7fffffffLL || batch < 1 || heads_k < 1 || heads_v < 1 || dim < 1)
    return fail(BT_ERR_INVALID, "gdn_prefill: bad shape");
  if (q_bs < 0 || k_bs < 0 || v_bs < 0 || g_bs < 0 || beta_bs < 0 || out_bs < 0 || q_ts < 0 || k_ts < 0 ||
      v_ts < 0 || g_ts < 0 || beta_ts < 0 || out_ts < 0)
    return fail(BT_ERR_INVALID, "gdn_prefill: negative stride");
  if (in_dtype != BT_F32 && in_dtype != BT_BF16) return fail(BT_ERR_UNSUPPORTED, "gdn_prefill: dtype %d", in_dtype);
  bt::GdnParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.in_dtype = in_dtype;
  p.q_bs = q_bs;
  p.k_bs = k_bs;
  p.v_bs = v_bs;
  p.g = g;
  p.beta = beta;
  p.g_bs = g_bs;
  p.beta_bs = beta_bs;
  p.state = state;
  p.out = out;
  p.out_bs = out_bs;
  p.batch = static_cast<int32_t>(std::min<int64_t>(batch, 0x7fffffffLL));
  p.heads_k = static_cast<int32_t>(std::min<int64_t>(heads_k, 0x7fffffffLL));
  p.heads_v = static_cast<int32_t>(std::min<int64_t>(heads_v, 0x7fffffffLL));
  p.dim = static_cast<int32_t>(std::min<int64_t>(dim, 0x7fffffffLL));
  p.scale = scale;
  p.eps = eps;
  bt::GdnScan sc{};
  sc.len = static_cast<int32_t>(steps);
  sc.tok_q = q_ts;
  sc.tok_k = k_ts;
  sc.tok_v = v_ts;
  sc.tok_g = g_ts;
  sc.tok_beta = beta_ts;
  sc.tok_out = out_ts;
  return bt::gdn_prefill_launch(p, sc, as_stream(stream));
}

int bt_gdn_decode_strided(const void* q, const void* k, const void* v, int in_dtype, int64_t q_bs, int64_t k_bs,
                          int64_t v_bs, const float* g, int64_t g_bs, const float* beta, int64_t beta_bs, float* state,
                          float* out, int64_t out_bs, int64_t batch, int64_t heads_k, int64_t heads_v, int64_t dim,
                          float scale, float eps, void* stream) {
  if (!q || !k || !v || !g || !beta || !state || !out) return fail(BT_ERR_INVALID, "gdn_decode: null pointer");
  if (q_bs < heads_k * dim || k_bs < heads_k * dim || v_bs < heads_v * dim || g_bs < heads_v ||
      beta_bs < heads_v || out_bs < heads_v * dim)
    return fail(BT_ERR_INVALID, "gdn_decode: a batch stride is shorter than its row");
  if (in_dtype != BT_F32 && in_dtype != BT_BF16) return fail(BT_ERR_UNSUPPORTED, "gdn_decode: dtype %d", in_dtype);
  if (batch * heads_v * (dim / 32) > 0x7fffffffLL) return fail(BT_ERR_UNSUPPORTED, "gdn_decode: grid too large");
  bt::GdnParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.in_dtype = in_dtype;
  p.q_bs = q_bs;
  p.k_bs = k_bs;
  p.v_bs = v_bs;
  p.g = g;
  p.beta = beta;
  p.g_bs = g_bs;
  p.beta_bs = beta_bs;
  p.state = state;
  p.out = out;
  p.out_bs = out_bs;
  p.batch = static_cast<int32_t>(batch);
  p.heads_k = static_cast<int32_t>(heads_k);
  p.heads_v = static_cast<int32_t>(heads_v);
  p.dim = static_cast<int32_t>(dim);
  p.scale = scale;
  p.eps = eps;
  return bt::gdn_decode_launch(p, as_stream(stream), false);
}

int64_t bt_argmax_workspace_bytes(int64_t rows) { return rows < 1 ? 0 : 12 * rows; }

int bt_argmax(const float* x, int64_t rows, int64_t n, int32_t* out, void* workspace, void* stream) {
  return bt::argmax(x, rows, n, out, workspace, as_stream(stream));
}

int bt_qwen35_kernels_per_step(const BtQwen35Model* model) {
  return model && model->layers ? bt::qwen35_kernels_per_step(*model) : 0;
}

int64_t bt_qwen35_proj_elems(const BtQwen35Dims* dims) { return dims ? bt::qwen35_proj_elems(*dims) : 0; }

int64_t bt_qwen35_workspace_bytes(const BtQwen35Dims* dims) { return dims ? bt::qwen35_workspace_bytes(*dims) : 0; }

int bt_qwen35_step(const BtQwen35Model* model, const BtQwen35Runtime* rt, int with_logits, void* stream) {
  if (!model || !rt) return fail(BT_ERR_INVALID, "qwen35_step: null model or runtime");
  return bt::qwen35_step(*model, *rt, with_logits, as_stream(stream));
}

int bt_qwen35_graph_create(const BtQwen35Model* model, const BtQwen35Runtime* rt, int n_steps, void* stream,
                           void** graph_out) {
  if (!model || !rt || !graph_out || n_steps < 1) return fail(BT_ERR_INVALID, "graph_create: bad arguments");
  if (!stream) return fail(BT_ERR_INVALID, "graph_create: capture needs a non-default stream");
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return bt::fail_cuda(e, "begin capture");
  int rc = BT_OK;
  for (int i = 0; i < n_steps && rc == BT_OK; ++i) rc = bt::qwen35_step(*model, *rt, 1, s);
  cudaGraph_t graph = nullptr;
  e = cudaStreamEndCapture(s, &graph);
  if (rc != BT_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return bt::fail_cuda(e, "end capture");
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return bt::fail_cuda(e, "graph instantiate");
  // upload now, so the first launch does not pay for it
  e = cudaGraphUpload(exec, s);
  if (e != cudaSuccess) {
    cudaGraphExecDestroy(exec);
    return bt::fail_cuda(e, "graph upload");
  }
  *graph_out = exec;
  return BT_OK;
}

int bt_graph_launch(void* graph, void* stream) {
  if (!graph) return fail(BT_ERR_INVALID, "graph_launch: null graph");
  cudaError_t e = cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph), as_stream(stream));
  return e == cudaSuccess ? BT_OK : bt::fail_cuda(e, "graph launch");
}

int bt_graph_destroy(void* graph) {
  if (!graph) return BT_OK;
  cudaError_t e = cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph));
  return e == cudaSuccess ? BT_OK : bt::fail_cuda(e, "graph destroy");
}

}  // extern "C"
