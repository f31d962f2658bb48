/*
 * bt_b200.h -- C ABI of the B200 (sm_100a) decode-step library.
 *
 * Every entry point takes raw device pointers, element counts and a CUDA
 * stream passed as `void*` (a cudaStream_t; NULL = legacy default stream).
 * None of them allocates device memory or synchronises the stream: outputs
 * and workspaces are owned by the caller, so every call can be captured in
 * a CUDA graph.  Each returns a BT_* status code; bt_last_error() gives the
 * message of the last failure on the calling thread.
 *
 * The entry points replace the operations of breezetoken's `Backend`
 * interface (breezetoken/backends.py:28-98) and the per-token decode step of
 * `Qwen35.forward_token` (breezetoken/model/qwen35.py:252-286) /
 * `GraphMixin._graph_body` (breezetoken/model/graph.py:66-91).
 *
 * Weight layout used by the Q8_0 entry points ("q8 rows"): one row of K
 * weights is stored as [K/32 fp16 block scales, zero-padded to a multiple of
 * 16 bytes][K int8 quants]; rows are contiguous.  bt_q8_row_bytes(K) gives
 * the row stride.  bt_repack_q8_0 converts GGUF Q8_0 blocks into it.
 */
#ifndef BT_B200_H
#define BT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BT_API __attribute__((visibility("default")))
#else
#define BT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define BT_OK 0
#define BT_ERR_INVALID 1     /* bad pointer, shape or argument        */
#define BT_ERR_UNSUPPORTED 2 /* shape/dtype this build does not serve */
#define BT_ERR_CUDA 3        /* a CUDA runtime call failed            */
#define BT_ERR_TIMEOUT 4     /* a bounded device-side wait gave up    */

/* int32 words of a device status record (see BtQwen35Runtime.status) */
#define BT_STATUS_WORDS 8

/* element types for the dtype arguments */
#define BT_F32 0
#define BT_BF16 1

/* Message of the last failed call on this thread ("" if none). */
BT_API const char* bt_last_error(void);
/* Library ABI version (major*100 + minor). */
BT_API int bt_version(void);
/* Number of SMs of the current device (cached per device). */
BT_API int bt_sm_count(void);
/* Bytes of one q8 row of K weights (see the header comment). */
BT_API int64_t bt_q8_row_bytes(int64_t k);

/* ------------------------------------------------------- weight repacking */
/* GGUF Q8_0 rows -> q8 rows.  `src` holds `rows` rows of K/32 34-byte blocks
 * (fp16 d, 32 x int8), as stored in the GGUF file (gguf.py:184-212).  Source
 * row i is written to destination row dst_row0 + i * dst_row_step, so two
 * matrices can be interleaved row by row (gate/up) or concatenated.        */
BT_API int bt_repack_q8_0(const void* src, void* dst, int64_t rows, int64_t k,
                   int64_t dst_row0, int64_t dst_row_step, void* stream);

/* Dequantise q8 rows to f32 (rows x k), exactly d * q
 * (quant/dequant.py:72-75).                                               */
BT_API int bt_dequant_q8_rows(const void* w, float* out, int64_t rows, int64_t k,
                       void* stream);

/* GGUF IQ3_S blocks (110 bytes per 256 weights) to f32, bit-exact with
 * quant/dequant.py:164-185 (`_deq_iq3_s`).                                */
BT_API int bt_dequant_iq3_s(const void* raw, float* out, int64_t rows, int64_t cols,
                     void* stream);

/* ------------------------------------------------------- Backend ops */
/* Backend.linear with Q8_0 weights (backends.py:109-112):
 * y[m][n] = sum_k x[m][k] * dequant(W)[n][k] for m < n_vec (<= 8).        */
BT_API int bt_linear_q8(const void* w, const float* x, float* y, int64_t n, int64_t k,
                 int n_vec, void* stream);

/* Backend.linear with a dense (K, N) weight as the reference stores it
 * (model/qwen35.py:148-153): y[n] = sum_k x[k] * W[k][n].
 * w_dtype is BT_BF16 or BT_F32.                                           */
BT_API int bt_linear_kn(const void* w, int w_dtype, const float* x, float* y,
                 int64_t k, int64_t n, void* stream);

/* x (T, K) f32 -> planes (T, 3, K) bf16 with x = hi + mid + lo (each
 * remainder exact in f32, so the planes carry x's 24 bits): the input form
 * of bt_linear_rows, split once per activation and shared by every
 * projection of it.  K % 8 == 0; both 16-byte aligned.                    */
BT_API int bt_bf16_planes(const float* x, void* planes, int64_t t, int64_t k,
                   void* stream);

/* Qwen36Moe._linear / _linear_b (model/qwen36_moe.py:352-358) for T
 * tokens: y[t][n] = sum_k W[n][k] * x[t][k] with W (N, K) rows in the GGUF
 * (out, in) orientation, bf16 or f32 (w_dtype), x given as the planes of
 * bt_bf16_planes, on the tensor cores (both operands to 24 bits).  y (T, N)
 * f32; N % 16 == 0, K % 256 == 0; w and the planes 16-byte aligned.       */
BT_API int bt_linear_rows(const void* w, int w_dtype, const void* x_planes, float* y,
                   int64_t n, int64_t k, int64_t t, void* stream);

/* Diagnostic without a reference counterpart: how many bounded mbarrier
 * waits of bt_linear_rows' tensor-core path (tcgen05, > 8 tokens, N % 128
 * == 0) gave up since the last call (0 unless the pipeline broke).
 * Synchronises the device and resets the count; -1 if it cannot be read.  */
BT_API int bt_linear_rows_timeouts(void);

/* Diagnostic without a reference counterpart: kernels this library has
 * launched in this process, each launch recorded into a CUDA graph under
 * stream capture counted once (replays launch it again and are not
 * counted).  The difference across one captured step is that step's kernel
 * count.                                                                  */
BT_API long long bt_launch_count(void);

/* Backend.rms_norm (backends.py:119-123) over rows of length n.           */
BT_API int bt_rms_norm(const float* x, const float* w, float* y, int64_t rows,
                int64_t n, float eps, void* stream);

/* Backend.fused_add_rms_norm (backends.py:229-238): h = a + b,
 * xn = rms_norm(h, w, eps).                                               */
BT_API int bt_fused_add_rms_norm(const float* a, const float* b, const float* w,
                          float* h, float* xn, int64_t rows, int64_t n,
                          float eps, void* stream);

/* Backend.silu_mul (backends.py:160-163): y = silu(g) * u.                */
BT_API int bt_silu_mul(const float* g, const float* u, float* y, int64_t n,
                void* stream);

/* Backend.rope (backends.py:218-226): partial rotate-half RoPE on the first
 * rope_dim of each row at position *pos (device int32); cos/sin are
 * (cap, rope_dim) f32 tables.                                             */
BT_API int bt_rope(const float* x, const float* cos_t, const float* sin_t,
            const int32_t* pos, float* y, int64_t rows, int64_t dim,
            int64_t rope_dim, int64_t cap, void* stream);

/* Backend.attention / attention_fixed (backends.py:196-215, 682-706):
 * GQA decode, one query per sequence.
 *   q:   (batch, heads, dim) f32
 *   k,v: (batch, cap, kv_heads, dim) in kv_dtype (BT_F32 or BT_BF16)
 *   lens: (batch,) int32 device lengths (keys [0, lens[b]) are attended)
 *   out: (batch, heads, dim) f32
 * workspace: bt_attention_workspace_bytes() bytes, zeroed once before the
 * first call (the kernel leaves it zeroed again).                         */
BT_API int64_t bt_attention_workspace_bytes(int64_t batch, int64_t kv_heads,
                                     int64_t heads, int64_t dim, int splits);
BT_API int bt_attention_decode(const float* q, const void* k, const void* v,
                        int kv_dtype, const int32_t* lens, float* out,
                        int64_t batch, int64_t heads, int64_t kv_heads,
                        int64_t dim, int64_t cap, float scale, int splits,
                        void* workspace, void* stream);

/* The attention layer after its in-projection, for `batch` sequences each at
 * its own position: Qwen36Moe._attn (model/qwen36_moe.py:432-457) and the
 * Qwen3.5 layer (model/layers.py:55-82) from the projection output on.
 *   proj: row b (stride proj_bs elements) = [q_h | gate_h for each head h
 *         (2*dim each)] [k (kv_heads*dim)] [v (kv_heads*dim)], f32
 * Per head RMSNorm of q and k (q_norm, k_norm: (dim,), eps), partial
 * rotate-half RoPE of the first rope_dim dims at pos[b] (rope_cos/sin:
 * (cap, rope_dim) f32, the cos|cos and sin|sin halves), k and v written to
 * the f32 caches (batch, cap, kv_heads, dim) at pos[b], attention over
 * positions [0, pos[b]] (value head h uses KV head h / (heads/kv_heads)),
 * out = attention * sigmoid(gate): (batch, heads, dim) f32.  workspace:
 * bt_attention_workspace_bytes(batch, kv_heads, heads, dim, splits), zeroed
 * once.  status: NULL or BT_STATUS_WORDS device int32 zeroed by the caller;
 * a position outside [0, cap) is recorded there ([0] = BT_ERR_INVALID).   */
BT_API int bt_attention_layer(const float* proj, int64_t proj_bs, const float* q_norm,
                              const float* k_norm, const float* rope_cos, const float* rope_sin,
                              int64_t rope_dim, const int32_t* pos, float* k_cache, float* v_cache,
                              float* out, int64_t batch, int64_t heads, int64_t kv_heads,
                              int64_t dim, int64_t cap, float scale, float eps, int splits,
                              void* workspace, int32_t* status, void* stream);

/* bt_attention_decode without a caller workspace, for callers that cannot
 * allocate device memory at call time (a pre-sized arena or memory pool that
 * owns every allocation, or a binding that only holds the buffers it was
 * handed).  No counterpart in the reference: it is an addition of this
 * library.  The split partials and merge counters live in one static device
 * array of BT_NOALLOC_ATTN_SCRATCH_BYTES bytes that every GPU loading the
 * library holds until the process exits; shapes needing more
 * (4*batch*kv_heads*splits*(heads/kv_heads)*(dim+2) bytes rounded up to 256,
 * plus 4*batch*kv_heads) are rejected with BT_ERR_INVALID.  The first call on
 * a device looks up the array's device address (cudaGetSymbolAddress with
 * that device current), so make that first call before any stream capture.
 * All calls on a device share that device's array and it keeps the last
 * call's contents: calls whose kernels overlap on the same GPU (for example
 * on two streams) race on it, so the caller must serialise them.  The call
 * allocates nothing; it clears the merge counters with an asynchronous
 * memset on `stream` before the kernel.                                    */
#define BT_NOALLOC_ATTN_SCRATCH_BYTES (8 * 1024 * 1024)
BT_API int bt_attention_decode_noalloc(const float* q, const void* k, const void* v,
                                       int kv_dtype, const int32_t* lens, float* out,
                                       int64_t batch, int64_t heads, int64_t kv_heads,
                                       int64_t dim, int64_t cap, float scale, int splits,
                                       void* stream);

/* Backend.gdn_decode (backends.py:241-271): one gated-delta-rule step.
 *   q,k: (batch, heads_k, dim), v: (batch, heads_v, dim) in in_dtype
 *   g (log decay), beta (logits): (batch, heads_v) f32
 *   state: (batch, heads_v, dim, dim) f32, updated in place
 *   out: (batch, heads_v, dim) f32
 * Value head h reads key head h % heads_k.                                */
BT_API int bt_gdn_decode(const void* q, const void* k, const void* v, int in_dtype,
                  const float* g, const float* beta, float* state, float* out,
                  int64_t batch, int64_t heads_k, int64_t heads_v, int64_t dim,
                  float scale, float eps, void* stream);

/* bt_gdn_decode on strided views, as the model layer hands them over
 * (model/qwen36_moe.py:459-483 slices q, k and v out of the conv output and
 * beta / alpha out of their projections): row b of q, k, v, g, beta and out
 * starts b * q_bs, k_bs, v_bs, g_bs, beta_bs and out_bs elements after the
 * first; inside a row the heads are contiguous as above.                  */
BT_API int bt_gdn_decode_strided(const void* q, const void* k, const void* v, int in_dtype,
                          int64_t q_bs, int64_t k_bs, int64_t v_bs, const float* g,
                          int64_t g_bs, const float* beta, int64_t beta_bs, float* state,
                          float* out, int64_t out_bs, int64_t batch, int64_t heads_k,
                          int64_t heads_v, int64_t dim, float scale, float eps,
                          void* stream);

/* The prefill loop of model/prefill.py:106-110 and
 * model/qwen36_moe.py:520-530 (a gdn_decode step once per prompt token) as
 * one launch: `steps` consecutive gated-delta-rule steps of each of `batch`
 * sequences, with the state kept on chip between tokens (read and written
 * once).  Element (token s, sequence b, head h, i) of q sits at
 * s * q_ts + b * q_bs + h * dim + i, likewise k, v (k_ts, k_bs, v_ts,
 * v_bs) and out (out_ts, out_bs); g and beta at s * g_ts + b * g_bs + h
 * (beta_ts, beta_bs).  Each token's step is bt_gdn_decode's arithmetic.
 * dim == 128 (the reference models' head size); steps == 0 is a no-op.  */
BT_API int bt_gdn_prefill(const void* q, const void* k, const void* v, int in_dtype,
                          int64_t q_bs, int64_t k_bs, int64_t v_bs, int64_t q_ts,
                          int64_t k_ts, int64_t v_ts, const float* g, int64_t g_bs,
                          int64_t g_ts, const float* beta, int64_t beta_bs, int64_t beta_ts,
                          float* state, float* out, int64_t out_bs, int64_t out_ts,
                          int64_t steps, int64_t batch, int64_t heads_k, int64_t heads_v,
                          int64_t dim, float scale, float eps, void* stream);

/* The GDN mixer of Qwen36Moe._gdn (model/qwen36_moe.py:459-483) from the
 * conv output on, for `batch` sequences, with dim == 128:
 *   mixed: row b (stride mixed_bs) = q (heads_k*dim) | k (heads_k*dim) |
 *          v (heads_v*dim), the SiLU conv output
 *   ba:    row b (stride ba_bs) = beta logits (heads_v) | alpha logits (heads_v)
 *   g = a_log * softplus(alpha + dt_bias); the gated delta rule of
 *   bt_gdn_decode on L2-normalised q (times scale) and k, state (batch,
 *   heads_v, dim, dim) f32 updated in place; then per value head
 *   y = rms_norm(o, norm_w, norm_eps) * silu(z) with z row b (stride z_bs),
 *   written as three bf16 planes (batch, 3, heads_v*dim), the input form of
 *   bt_linear_rows for the out-projection.                                 */
BT_API int bt_gdn_gated_step(const float* mixed, int64_t mixed_bs, const float* ba, int64_t ba_bs,
                             const float* a_log, const float* dt_bias, float* state, const float* z,
                             int64_t z_bs, const float* norm_w, void* planes, int64_t batch,
                             int64_t heads_k, int64_t heads_v, int64_t dim, float scale, float l2_eps,
                             float norm_eps, void* stream);

/* bt_gdn_gated_step over a prompt chunk of `steps` tokens per sequence
 * (the GDN mixer of Qwen36Moe._gdn_batch, model/qwen36_moe.py:485-534,
 * whose recurrence runs token by token): mixed, ba, z and planes hold
 * steps * batch rows, token s of sequence b in row s * batch + b; each
 * (sequence, head) scans its tokens in order with the state on chip, and
 * each token's arithmetic is bt_gdn_gated_step's.                         */
BT_API int bt_gdn_gated_scan(const float* mixed, int64_t mixed_bs, const float* ba, int64_t ba_bs,
                             const float* a_log, const float* dt_bias, float* state, const float* z,
                             int64_t z_bs, const float* norm_w, void* planes, int64_t steps,
                             int64_t batch, int64_t heads_k, int64_t heads_v, int64_t dim,
                             float scale, float l2_eps, float norm_eps, void* stream);

/* bt_fused_add_rms_norm that also writes y's three bf16 planes (rows, 3, n)
 * (the form of bt_bf16_planes) in the same pass: h = a + b (b may be NULL:
 * then y = rms_norm(a) and h is not written), y = rms_norm(h, w, eps).
 * n % 8 == 0; every buffer 16-byte aligned.                              */
BT_API int bt_add_rms_norm_planes(const float* a, const float* b, const float* w, float* h,
                                  float* y, void* planes, int64_t rows, int64_t n, float eps,
                                  void* stream);

/* The GDN short conv (model/qwen36_moe.py:465-468) for `batch` sequences:
 * window = [state (taps-1 per channel) | entry], out = silu(sum_j window[j] *
 * w[c][j]) in tap order, state <- window[1:] (in place).  entry, out:
 * (batch, channels); state: (batch, channels, taps-1); w: (channels, taps);
 * taps in [2, 8].                                                         */
BT_API int bt_conv_silu(const float* entry, float* state, const float* w, float* out,
                 int64_t batch, int64_t channels, int64_t taps, void* stream);

/* bt_conv_silu over `steps` consecutive tokens of every sequence, the
 * prompt-chunk form of the batched prefill's conv1d over [state | entries]
 * (model/qwen36_moe.py:493-501, model/prefill.py:90-93): entry and out are
 * (steps, batch, channels), token s of sequence b in row s * batch + b;
 * the state ends as the window after the last token.  Per token the same
 * arithmetic as bt_conv_silu.                                             */
BT_API int bt_conv_silu_scan(const float* entry, float* state, const float* w, float* out,
                             int64_t steps, int64_t batch, int64_t channels, int64_t taps,
                             void* stream);

/* argmax with torch.argmax's first-index tie rule over rows of length n.
 * workspace: bt_argmax_workspace_bytes(rows) bytes, zeroed before first use. */
BT_API int64_t bt_argmax_workspace_bytes(int64_t rows);
BT_API int bt_argmax(const float* x, int64_t rows, int64_t n, int32_t* out,
              void* workspace, void* stream);

/* ------------------------------------------------------- MoE experts */
/* Bytes per IQ3_S row of K weights in the device layout (K % 256 == 0):
 * K / 256 * 136.  Every weight d * (1 + 2 * scale nibble) * v, v an odd
 * codebook value in [-15, 15], is stored as the 4-bit code (v + 15) / 2 (a
 * lossless re-encoding of the GGUF block's codebook index, high bit and
 * sign); rows in tiles of 16; a tile's 16 GGUF blocks of one 256-weight
 * column block form one 2176-byte chunk (codes ordered for the fp16
 * tensor-core MMA's operand fragments, then each row's scales and d),
 * chunks of a tile contiguous, tiles in row order.                        */
BT_API int64_t bt_iq3s_row_bytes(int64_t k);

/* GGUF IQ3_S rows (110-byte blocks, quant/dequant.py:164-185) -> the device
 * layout (rows % 16 == 0); replaces the reference's per-step byte staging of
 * the selected experts (model/moe.py:64-120): they stay resident in HBM.  */
BT_API int bt_repack_iq3_s(const void* src, void* dst, int64_t rows, int64_t k,
                    void* stream);

/* route() for T tokens (model/moe.py:33-39): softmax over each token's
 * n_experts router logits, top-k (ties to the lower id), weights
 * renormalised by max(sum, 6.1035e-5).  ids/weights: (T, top_k).         */
BT_API int bt_moe_route(const float* logits, int64_t t, int64_t n_experts, int top_k,
                 int32_t* ids, float* weights, void* stream);

/* Workspace of bt_moe_experts_iq3s: zeroed once before first use; the
 * calls leave it reusable (its arrival counters are re-armed).            */
BT_API int64_t bt_moe_workspace_bytes(int64_t t, int64_t hidden, int64_t ffn,
                               int64_t n_experts, int top_k);

/* ExpertPool.forward (model/moe.py:205-233) for T tokens at once:
 * out[t] = sum_k weights[t,k] * down_e(silu(gate_e x_t) * up_e x_t), e =
 * ids[t,k], with the IQ3_S experts decoded inside the GEMVs.  gate/up:
 * (n_experts * ffn) rows of K = hidden, down: (n_experts * hidden) rows of
 * K = ffn, all in the bt_repack_iq3_s layout.  x, out: (T, hidden) f32.
 * (hidden, ffn) in {(1024, 512), (2048, 512), (2048, 1024)}.
 * Each selected expert is read once for all the tokens that selected it.
 * Pairs with an id outside [0, n_experts) contribute nothing.             */
BT_API int bt_moe_experts_iq3s(const void* gate, const void* up, const void* down,
                        const float* x, int64_t t, int64_t hidden, int64_t ffn,
                        int64_t n_experts, const int32_t* ids, const float* weights,
                        int top_k, float* out, void* workspace, void* stream);

/* Qwen36Moe._moe (model/qwen36_moe.py:634-642) for T tokens: the routed
 * experts as bt_moe_experts_iq3s plus, when `shared` is not NULL, the
 * shared expert: out[t] = routed[t] + sigmoid(x_t . gate_inp) *
 * down(silu(gate x_t) * up x_t).  Shared weights are bf16 rows in the GGUF
 * (out, in) orientation (gate, up: (ffn, hidden); down: (hidden, ffn)),
 * 16-byte aligned; gate_inp is f32 (hidden,); ffn % 256 == 0.
 * workspace: bt_moe_layer_workspace_bytes() bytes, zeroed once.           */
typedef struct BtMoeShared {
  const void* gate;
  const void* up;
  const void* down;
  const float* gate_inp;
  int64_t ffn;
} BtMoeShared;
BT_API int64_t bt_moe_layer_workspace_bytes(int64_t t, int64_t hidden, int64_t ffn,
                                     int64_t shared_ffn, int64_t n_experts, int top_k);
BT_API int bt_moe_layer_iq3s(const void* gate, const void* up, const void* down,
                      const BtMoeShared* shared, const float* x, int64_t t,
                      int64_t hidden, int64_t ffn, int64_t n_experts,
                      const int32_t* ids, const float* weights, int top_k,
                      float* out, void* workspace, void* stream);

/* bt_moe_layer_iq3s followed by the decoder's residual add + RMSNorm + bf16
 * planes (bt_add_rms_norm_planes(h, out, w, eps, h_out, y, planes):
 * model/qwen36_moe.py:658-662 with the next layer's input norm), the same
 * bits as the two calls.  For T > 1 the combine and the norm run as one
 * kernel and `out` (T x hidden f32) is not written; for T == 1 it is the
 * layer's output.  All buffers 16-byte aligned.                          */
BT_API int bt_moe_layer_iq3s_add_norm(const void* gate, const void* up, const void* down,
                                      const BtMoeShared* shared, const float* x, int64_t t,
                                      int64_t hidden, int64_t ffn, int64_t n_experts,
                                      const int32_t* ids, const float* weights, int top_k,
                                      const float* h, const float* w, float eps, float* h_out,
                                      float* y, void* planes, float* out, void* workspace,
                                      void* stream);

/* bt_moe_route + bt_moe_layer_iq3s_add_norm as two calls on one workspace
 * that chain without a gap: bt_moe_route_sort_iq3s routes the router
 * logits (T x n_experts f32) into ids / weights exactly like bt_moe_route
 * and, in the same launch, sorts the pairs and encodes the T tokens of x
 * into the workspace (the last routing block sorts; shared_ffn: the layer's
 * shared expert's ffn, 0 for none, as the layer call will get it);
 * bt_moe_layer_iq3s_add_norm_prepared, ordered after it, does the rest with
 * the same x, ids, weights, shapes, shared expert and workspace (for T > 1
 * the shared expert's blocks ride in the expert kernels, no prep launch).
 * Together they give the bits of bt_moe_route followed by
 * bt_moe_layer_iq3s_add_norm.  No reference counterpart: a regrouping of
 * model/moe.py:33-39 and model/qwen36_moe.py:634-642.                      */
BT_API int bt_moe_route_sort_iq3s(const float* logits, const float* x, int64_t t,
                                  int64_t hidden, int64_t ffn, int64_t n_experts, int top_k,
                                  int64_t shared_ffn, int32_t* ids, float* weights,
                                  void* workspace, void* stream);
BT_API int bt_moe_layer_iq3s_add_norm_prepared(const void* gate, const void* up,
                                               const void* down, const BtMoeShared* shared,
                                               const float* x, int64_t t, int64_t hidden,
                                               int64_t ffn, int64_t n_experts,
                                               const int32_t* ids, const float* weights,
                                               int top_k, const float* h, const float* w,
                                               float eps, float* h_out, float* y, void* planes,
                                               float* out, void* workspace, void* stream);

/* ------------------------------------------------- Qwen3.5 decode step */
typedef struct BtQwen35Dims {
  int32_t hidden, n_layers, n_heads, n_kv, head_dim, rope_dim, ffn, vocab;
  int32_t ssm_inner, ssm_state, ssm_heads, conv_k, max_ctx, batch;
  float eps, l2_eps;
} BtQwen35Dims;

typedef struct BtQwen35Layer {
  int32_t is_attn, pad_;
  const float* norm_in;   /* (hidden,) f32 */
  const float* norm_post; /* (hidden,) */
  const float* norm_next; /* next layer's norm_in, or output_norm */
  const void* w_in;   /* GDN: q8 rows [qkv | z | alpha | beta]; attn: [q|gate per head, k, v] */
  const void* w_out;  /* GDN: ssm_out (hidden x inner); attn: attn_output */
  const void* w_gu;   /* q8 rows gate/up interleaved: row 2j = gate_j, 2j+1 = up_j */
  const void* w_down; /* (hidden x ffn) */
  const float* conv_w;   /* GDN (3*inner, conv_k) */
  const float* a_log;    /* GDN (ssm_heads,) = -exp(A_log) */
  const float* dt_bias;  /* GDN (ssm_heads,) */
  const float* ssm_norm; /* GDN (ssm_state,) */
  const float* q_norm;   /* attn (head_dim,) */
  const float* k_norm;   /* attn (head_dim,) */
  float* conv_state;     /* GDN (batch, 3*inner, conv_k-1) */
  float* rec_state;      /* GDN (batch, ssm_heads, ssm_state, ssm_state) */
  float* k_cache;        /* attn (batch, max_ctx, n_kv*head_dim) f32 */
  float* v_cache;
} BtQwen35Layer;

typedef struct BtQwen35Model {
  BtQwen35Dims dims;
  const void* embed;     /* q8 rows (vocab x hidden): token_embd == tied head */
  const float* rope_cos; /* (max_ctx, rope_dim) */
  const float* rope_sin;
  const BtQwen35Layer* layers; /* host array of n_layers */
} BtQwen35Model;

typedef struct BtQwen35Runtime {
  int32_t* pos;       /* (batch,) device positions of the token being consumed */
  int32_t* token;     /* (batch,) device token ids consumed by the next step */
  int32_t* history;   /* (batch, max_ctx) tokens produced, indexed by pos+1; may be NULL */
  float* logits;      /* (batch, vocab) or NULL (argmax only) */
  float* h0;          /* (batch, hidden) residual ping */
  float* h1;          /* (batch, hidden) residual pong */
  float* delta;       /* (batch, hidden) mixer / mlp output */
  float* proj;        /* (batch, bt_qwen35_proj_elems) in-projection outputs */
  float* mix;         /* (batch, max(ssm_inner, n_heads*head_dim)) mixer output */
  float* act;         /* (batch, 2*ffn): silu(gate)*up, or (gate, up) pairs when batch > 2 */
  void* workspace;    /* bt_qwen35_workspace_bytes(), zeroed once */
  void* trace;        /* optional timeline: bt_qwen35_kernels_per_step() records of
                         BtTraceRecord, or NULL (no tracing) */
  int32_t* status;    /* BT_STATUS_WORDS device int32, zeroed by the caller: on a
                         device-side failure [0] = BT_ERR_TIMEOUT or
                         BT_ERR_INVALID, [1] = site, [2] = block, [3..5] =
                         site-specific detail; the first failure wins */
} BtQwen35Runtime;

/* One launch of the step as seen by the device-side tracer: %globaltimer
 * nanoseconds folded over the launch's CTAs.  Set the *_min fields to
 * UINT64_MAX and the others to 0 before a traced step. */
typedef struct BtTraceRecord {
  uint64_t entry_min, entry_max;   /* first / last CTA start                 */
  uint64_t waited_min, waited_max; /* first / last CTA past the dependency wait */
  uint64_t ready_max;              /* last CTA past its prologue             */
  uint64_t exit_min, exit_max;     /* first / last CTA end                   */
  uint64_t loaded_max;             /* GEMV: last CTA with its activation loads
                                      back (0 for other kernels)             */
} BtTraceRecord;

/* Kernels one decode step of `model` launches (with logits): the trace
 * record count.  0 for a null model. */
BT_API int bt_qwen35_kernels_per_step(const BtQwen35Model* model);
BT_API int64_t bt_qwen35_proj_elems(const BtQwen35Dims* dims);
BT_API int64_t bt_qwen35_workspace_bytes(const BtQwen35Dims* dims);

/* Enqueue one decode step for every sequence in the batch: consume token[b]
 * at pos[b], write logits (if rt->logits), token[b] = argmax, history, and
 * pos[b] += 1.  Mirrors Qwen35.forward_token + the in-graph argmax and
 * position increment of GraphMixin._graph_body.  `with_logits` = 0 skips
 * the head and leaves token/pos untouched except pos += 1 (prefill).     */
BT_API int bt_qwen35_step(const BtQwen35Model* model, const BtQwen35Runtime* rt,
                   int with_logits, void* stream);

/* Capture `n_steps` consecutive decode steps into one CUDA graph (native
 * stream capture; the stream must not be the legacy default stream).  The
 * model and runtime structs are copied into the graph; the device buffers
 * they point to must outlive it.                                          */
BT_API int bt_qwen35_graph_create(const BtQwen35Model* model, const BtQwen35Runtime* rt,
                           int n_steps, void* stream, void** graph_out);
BT_API int bt_graph_launch(void* graph, void* stream);
BT_API int bt_graph_destroy(void* graph);

#ifdef __cplusplus
}
#endif
#endif /* BT_B200_H */
