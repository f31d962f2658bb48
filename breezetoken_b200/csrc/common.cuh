// Device-side helpers shared by every kernel of the library: programmatic
// dependent launch (PDL), mbarrier + bulk-copy (TMA engine, non-tensor form)
// wrappers, bounded waits, block reductions and exact-by-construction number
// conversions.  sm_100a only.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/bt_b200.h"

namespace bt {

// ----------------------------------------------------------------- PDL
// A kernel launched with programmatic stream serialization may start while
// its predecessor still runs.  Before pdl_wait() it may only read data that
// no kernel of the step writes (weights); pdl_wait() returns once every
// predecessor grid has completed and its writes are visible.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------- timers
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Every spin-wait in the library gives up after this many nanoseconds and
// reports BT_ERR_TIMEOUT through the caller's status word.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ------------------------------------------------------------ step tracer
// Optional per-launch timeline: every CTA folds %globaltimer stamps of four
// points into one record per launch (first/last CTA entry, last CTA past the
// dependency wait, last CTA past its prologue, first/last CTA exit).  Off
// (null) in normal runs; the layout matches BtTraceRecord in bt_b200.h.
struct TraceRec {
  unsigned long long entry_min, entry_max, waited_min, waited_max, ready_max, exit_min, exit_max, loaded_max;
};
__device__ __forceinline__ void trace_entry(TraceRec* t) {
  if (t && threadIdx.x == 0) {
    const unsigned long long now = global_ns();
    atomicMin(&t->entry_min, now);
    atomicMax(&t->entry_max, now);
  }
}
__device__ __forceinline__ void trace_waited(TraceRec* t) {
  if (t && threadIdx.x == 0) {
    const unsigned long long now = global_ns();
    atomicMin(&t->waited_min, now);
    atomicMax(&t->waited_max, now);
  }
}
// `dep` is a value computed from the loads being timed; the branch on it
// orders the timer read after their arrival.
__device__ __forceinline__ void trace_loaded(TraceRec* t, float dep) {
  if (t && threadIdx.x == 0 && __float_as_uint(dep) != 0x7fbadbadu) atomicMax(&t->loaded_max, global_ns());
}
__device__ __forceinline__ void trace_ready(TraceRec* t) {
  if (t && threadIdx.x == 0) atomicMax(&t->ready_max, global_ns());
}
__device__ __forceinline__ void trace_exit(TraceRec* t) {
  if (t && threadIdx.x == 0) {
    const unsigned long long now = global_ns();
    atomicMin(&t->exit_min, now);
    atomicMax(&t->exit_max, now);
  }
}

// Where a device-side check fired (status word 1).
enum StatusSite : int32_t {
  SITE_GEMV_PRODUCER_EMPTY = 1,  // producer waiting for a consumed stage
  SITE_GEMV_PRODUCER_DRAIN = 2,  // producer waiting for its last copies to land
  SITE_GEMV_CONSUMER_FULL = 3,   // consumer waiting for a stage's bytes
  SITE_EMBED_TOKEN = 4,          // token id outside the vocabulary
  SITE_ATTN_LENGTH = 5,          // attended length outside [0, cap]
  SITE_ROPE_POS = 6,             // RoPE position outside the table
};

// The caller's status record is BT_STATUS_WORDS int32: [code, site, block,
// a, b, c, ...].  The first failure wins and fills the record.
__device__ __forceinline__ void report_status(int32_t* status, int32_t code, int32_t site = 0, int32_t a = 0,
                                              int32_t b = 0, int32_t c = 0) {
  if (!status) return;
  if (atomicCAS(reinterpret_cast<int*>(status), 0, code) == 0) {
    status[1] = site;
    status[2] = static_cast<int32_t>(blockIdx.x);
    status[3] = a;
    status[4] = b;
    status[5] = c;
    __threadfence();
  }
}

// ----------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of `bar`; false on timeout (the caller
// reports where).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
}

// L2 policy for data read exactly once per step (weights): evict first, so
// activations, states and caches keep their L2 residency.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bulk (non-tensor) global->shared copy on the TMA engine, completing on
// `bar` with a transaction count of `bytes`.  dst/src 16-B aligned, bytes a
// multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// --------------------------------------------------------- conversions
// int8 -> f32 without the I2F pipe: bias the byte to unsigned, place it in
// the mantissa of 2^23 and subtract 2^23 + 128.  Exact for every int8.
// `u` is a 32-bit word of four int8 already XORed with 0x80808080.
template <int kByte>
__device__ __forceinline__ float biased_byte_to_f32(uint32_t u) {
  return __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u + kByte)) - 8388736.0f;
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// ------------------------------------------------------- elementwise math
// Reference formulas: torch.nn.functional.silu, torch.sigmoid,
// torch.nn.functional.softplus (beta=1, threshold=20).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// ------------------------------------------------------------ reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Named barrier over the first `nthreads` threads (whole warps).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Sum over a group of `nwarps` warps using `scratch` (>= nwarps floats);
// every participating thread gets the total.  Caller provides the barrier.
template <int kNamedBarrier>
__device__ __forceinline__ float group_sum(float v, float* scratch, int nwarps, int nthreads) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  named_sync(kNamedBarrier, nthreads);
  if (lane == 0) scratch[warp] = v;
  named_sync(kNamedBarrier, nthreads);
  float t = 0.f;
  for (int i = 0; i < nwarps; ++i) t += scratch[i];
  return t;
}

}  // namespace bt
