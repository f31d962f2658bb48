// Q8_0 GEMV: host-side planner and the launch switch over (prologue,
// epilogue) kinds.  The kernels are in gemv_q8_impl.cuh and are instantiated
// per kind in the gemv_q8_k_*.cu files.  See gemv_q8.cuh for the design.
#include <algorithm>

#include "errors.h"
#include "gemv_q8_impl.cuh"

namespace bt {

namespace gemv_detail {
BT_GEMV_KINDS(BT_GEMV_EXTERN)
}  // namespace gemv_detail

namespace {

// Weight bytes per CTA prefetched into L2 before the dependency wait.
constexpr int64_t kPrefetchBytes = 64 * 1024;
// Long matrices (at least kBigUnits row units of 4 rows per SM) run
// kBigGrid CTAs per SM: twice the weight bytes in flight and half the rows
// per CTA after the dependency wait.
constexpr int kBigGrid = 2;
constexpr int kBigUnits = 8;

}  // namespace

int gemv_q8_plan(GemvQ8Params& p, int sm_count, GemvQ8Launch& L) {
  if (p.k < 32 || p.k % 32 != 0) return fail(BT_ERR_UNSUPPORTED, "q8 GEMV needs K %% 32 == 0, got K=%d", p.k);
  if (p.n_rows < 1) return fail(BT_ERR_INVALID, "q8 GEMV needs at least one row");
  if (p.n_vec != 1 && p.n_vec != 2 && p.n_vec != 4 && p.n_vec != 8)
    return fail(BT_ERR_UNSUPPORTED, "q8 GEMV serves 1, 2, 4 or 8 vectors, got %d", p.n_vec);
  if (!p.w || (reinterpret_cast<uintptr_t>(p.w) & 15))
    return fail(BT_ERR_INVALID, "q8 GEMV weights must be 16-byte aligned");
  if (p.epilogue == EPI_ARGMAX && (!p.best || !p.counter))
    return fail(BT_ERR_INVALID, "argmax epilogue needs its workspace");
  constexpr int kMaxK = gemv_detail::kMaxF4 * kConsumerThreads * 4;
  if (p.k > kMaxK) return fail(BT_ERR_UNSUPPORTED, "q8 GEMV serves K <= %d, got %d", kMaxK, p.k);
  {
    // the prologue reads activations and norm weights as float4
    const uintptr_t a = reinterpret_cast<uintptr_t>(p.x) | reinterpret_cast<uintptr_t>(p.x2) |
                        reinterpret_cast<uintptr_t>(p.norm_w) | reinterpret_cast<uintptr_t>(p.h_out);
    if ((a & 15) || (p.x_bs & 3) || (p.x2_bs & 3))
      return fail(BT_ERR_INVALID, "q8 GEMV activations must be 16-byte aligned with strides a multiple of 4");
    if (p.prologue == PRO_GATED_NORM && p.group != 64 && p.group != 128)
      return fail(BT_ERR_UNSUPPORTED, "gated-norm prologue serves groups of 64 or 128, got %d", p.group);
    if (p.x_bs == 0) p.x_bs = p.prologue == PRO_SILU_PAIR ? 2LL * p.k : p.k;
    if (p.x2_bs == 0) p.x2_bs = p.k;
  }
  p.sb = static_cast<int32_t>(bt_q8_row_bytes(p.k) - p.k);
  p.row_bytes = static_cast<int32_t>(bt_q8_row_bytes(p.k));
  const int64_t n_units = (p.n_rows + 3) / 4;
  const int64_t ctas = n_units >= static_cast<int64_t>(kBigUnits) * sm_count
                           ? static_cast<int64_t>(kBigGrid) * sm_count
                           : sm_count;
  const int grid = static_cast<int>(std::min<int64_t>(ctas, n_units));
  const int64_t rows_per_cta = ((n_units + grid - 1) / grid) * 4;
  // 4-row groups reuse each activation chunk across rows (K <= 1024: a
  // double-buffered 4-row tile stays within the register budget)
  const bool g4_ok = p.k <= 1024 && p.n_vec <= 2;
  int gr = 1;
  if (p.epilogue == EPI_SILU_PAIR || (g4_ok && rows_per_cta >= 32)) gr = 4;
  if (p.epilogue == EPI_SILU_PAIR && !g4_ok)
    return fail(BT_ERR_UNSUPPORTED, "SiLU-pair epilogue serves at most 2 vectors and K <= 1024");
  p.group_rows = gr;
  p.prefetch_bytes = kPrefetchBytes;
  L.grid = grid;
  L.threads = kGemvThreads;
  L.smem = GemvSmem::kHeader + gemv_x_layout(p.k, p.n_vec).total;
  if (L.smem > static_cast<size_t>(gemv_detail::kMaxDynSmem))
    return fail(BT_ERR_UNSUPPORTED, "q8 GEMV: %zu bytes of activations exceed the shared-memory budget", L.smem);
  return BT_OK;
}

int gemv_q8_launch(const GemvQ8Params& p, const GemvQ8Launch& L, cudaStream_t stream, bool pdl) {
  using namespace gemv_detail;
#define BT_GEMV_CASE(P, E) \
  if (p.prologue == P && p.epilogue == E) return launch_kind<P, E>(p, L, stream, pdl);
  BT_GEMV_KINDS(BT_GEMV_CASE)
#undef BT_GEMV_CASE
  return fail(BT_ERR_UNSUPPORTED, "q8 GEMV: no kernel for prologue %d with epilogue %d", p.prologue, p.epilogue);
}

}  // namespace bt
