// Allocation-free variant of the split-KV decode attention entry point.
//
// Some callers of this library cannot allocate device memory when they call
// it: code running inside a memory pool or arena that owns every allocation
// (an inference server's pre-sized pool), hosts that forbid cudaMalloc after
// start-up, or language bindings whose only handle on the GPU is the buffers
// they were given.  For them, bt_attention_decode_noalloc keeps the split
// partials and merge counters in this file's static device array instead of
// a caller workspace.  The array is sized once, at load time, for every GPU
// that loads the library, and stays resident until the process exits.
#include <mutex>
#include <vector>

#include "attention.cuh"
#include "errors.h"

namespace bt {
namespace {

constexpr int64_t kNoallocScratchBytes = BT_NOALLOC_ATTN_SCRATCH_BYTES;

// Scratch of the allocation-free entry point.  In host code this symbol is a
// host-side stand-in, not a device address: the kernels get the address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_attn_scratch[kNoallocScratchBytes];

std::mutex g_mutex;
std::vector<void*> g_scratch_by_device;

// Device address of g_attn_scratch on the current device, resolved once per
// device (with that device current).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "noalloc attention: cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (dev >= static_cast<int>(g_scratch_by_device.size())) g_scratch_by_device.resize(dev + 1, nullptr);
  if (!g_scratch_by_device[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_attn_scratch);
    if (e != cudaSuccess || !ptr) return fail_cuda(e, "noalloc attention: cudaGetSymbolAddress");
    g_scratch_by_device[dev] = ptr;
  }
  *out = g_scratch_by_device[dev];
  return BT_OK;
}

}  // namespace
}  // namespace bt

extern "C" int bt_attention_decode_noalloc(const float* q, const void* k, const void* v, int kv_dtype,
                                           const int32_t* lens, float* out, int64_t batch, int64_t heads,
                                           int64_t kv_heads, int64_t dim, int64_t cap, float scale, int splits,
                                           void* stream) {
  using bt::fail;
  if (!q || !k || !v || !lens || !out) return fail(BT_ERR_INVALID, "noalloc attention: null pointer");
  // bounded before any size arithmetic, so the scratch size below cannot
  // overflow and every field fits the kernel's 32-bit parameters
  if (batch < 1 || batch > 65535 || heads < 1 || heads > 65535 || kv_heads < 1 || kv_heads > 65535 || dim < 1 ||
      dim > 1024 || cap < 1 || cap > (1LL << 30) || splits < 1 || splits > 65535)
    return fail(BT_ERR_INVALID, "noalloc attention: shape out of range");
  if (heads % kv_heads != 0)
    return fail(BT_ERR_INVALID, "noalloc attention: heads (%lld) must be a multiple of kv_heads (%lld)",
                static_cast<long long>(heads), static_cast<long long>(kv_heads));
  const int64_t part_bytes = (4 * bt::attn_part_floats(batch, kv_heads, heads, dim, splits) + 255) / 256 * 256;
  const int64_t counter_bytes = 4 * bt::attn_counters(batch, kv_heads, splits);
  if (part_bytes + counter_bytes > bt::kNoallocScratchBytes)
    return fail(BT_ERR_INVALID,
                "noalloc attention: batch %lld x kv_heads %lld x splits %d needs %lld scratch bytes, above the "
                "fixed maximum of %lld (BT_NOALLOC_ATTN_SCRATCH_BYTES); use fewer splits or bt_attention_decode",
                static_cast<long long>(batch), static_cast<long long>(kv_heads), splits,
                static_cast<long long>(part_bytes + counter_bytes),
                static_cast<long long>(bt::kNoallocScratchBytes));
  void* scratch = nullptr;
  int rc = bt::scratch_address(&scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  // The merge counters must start at zero; the array keeps whatever the last
  // call (possibly an interrupted one) left there.
  cudaError_t e = cudaMemsetAsync(base + part_bytes, 0, counter_bytes, s);
  if (e != cudaSuccess) return bt::fail_cuda(e, "noalloc attention: clear counters");
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
  p.part = reinterpret_cast<float*>(base);
  p.counters = reinterpret_cast<uint32_t*>(base + part_bytes);
  return bt::attention_launch(p, s, false);
}
