// Q8_0 GEMV kernels of the kinds below (one file per group so the
// instantiations compile in parallel).
#include "gemv_q8_impl.cuh"

namespace bt {
namespace gemv_detail {
BT_GEMV_INSTANTIATE(PRO_RESID_NORM, EPI_ARGMAX)
BT_GEMV_INSTANTIATE(PRO_GATED_NORM, EPI_STORE)
}  // namespace gemv_detail
}  // namespace bt
