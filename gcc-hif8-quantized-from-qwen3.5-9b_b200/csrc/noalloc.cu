// Paged attention whose split-KV scratch lives inside the library.
//
// hif8_paged_attention wants a caller-provided workspace for the partial
// results of its split-KV pass.  Some callers have no way to provide one: a
// plain C host that only receives the tensors and a stream from its
// framework (the framework's caching allocator is out of its reach), or a
// serving engine that has reserved every free byte of HBM for its KV-page
// pool up front.  This entry point serves them from a fixed scratch array in
// the library's own device image, so it allocates nothing.
//
// Limits and rules, all stated in include/hif8_b200.h:
//   * the arguments are checked first, exactly as hif8_paged_attention
//     checks them (a bad call gets HIF8_ERR_INVALID_ARGUMENT whatever its
//     size); then at most HIF8_NOALLOC_ATTENTION_SCRATCH_BYTES of partials
//     per call (hif8_paged_attention_workspace_size() of the call's sizes,
//     SIZE_MAX where that product overflows); larger calls are rejected with
//     HIF8_ERR_WORKSPACE before anything is enqueued;
//   * nothing in the scratch needs to start at zero: every partial the merge
//     kernel reads was written by the split kernel of the same call;
//   * the scratch is one array per device, shared by every call on that
//     device: two calls in flight at once (different streams, or host
//     threads without ordering) race on it.  Calls on one stream are ordered
//     and safe;
//   * the first call on each device resolves the array's device address with
//     cudaGetSymbolAddress (which may load the library's device code on that
//     device); make that first call before any stream capture.
#include <atomic>
#include <mutex>

#include "hif8_common.cuh"

namespace {

constexpr size_t kScratchBytes = HIF8_NOALLOC_ATTENTION_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attention_scratch[kScratchBytes];

std::mutex g_scratch_mutex;
std::atomic<void *> g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's scratch array, resolved once per device
// with that device current; nullptr (and the last-error text set) on failure.
// After the first call on a device this is one atomic load: host threads
// driving different devices do not contend on the lock.
void *scratch_for_current_device() {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    hif8::set_last_error(err);
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    hif8::set_last_error(cudaErrorInvalidDevice);
    return nullptr;
  }
  void *ptr = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (ptr) return ptr;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ptr = g_scratch_ptr[dev].load(std::memory_order_relaxed);
  if (!ptr) {
    err = cudaGetSymbolAddress(&ptr, g_attention_scratch);
    if (err != cudaSuccess) {
      hif8::set_last_error(err);
      return nullptr;
    }
    g_scratch_ptr[dev].store(ptr, std::memory_order_release);
  }
  return ptr;
}

}  // namespace

extern "C" int hif8_paged_attention_noalloc(const uint16_t *query, const uint8_t *key_cache,
                                            const uint8_t *value_cache, const int32_t *block_tables,
                                            const int32_t *seq_lens, const int32_t *query_start, int64_t batch,
                                            int64_t num_tokens, int64_t num_heads, int64_t kv_heads,
                                            int64_t head_size, int64_t num_blocks, int64_t block_size,
                                            int64_t max_blocks, int64_t max_seq_len, float softmax_scale,
                                            int causal, uint16_t *out, void *stream) {
  // the same argument checks as hif8_paged_attention, before the scratch
  // test: an invalid call is an invalid call at any size
  const int args_status = hif8::paged_attention_args_status(
      query, key_cache, value_cache, block_tables, seq_lens, query_start, out, batch, num_tokens, num_heads,
      kv_heads, head_size, num_blocks, block_size, max_blocks, max_seq_len);
  if (args_status != HIF8_OK) return args_status;
  // overflow-checked: SIZE_MAX for sizes whose partials do not fit size_t
  const size_t need = hif8_paged_attention_workspace_size(num_tokens, num_heads, head_size, max_seq_len);
  if (need > kScratchBytes) return HIF8_ERR_WORKSPACE;
  void *scratch = nullptr;
  if (need > 0) {
    scratch = scratch_for_current_device();
    if (!scratch) return HIF8_ERR_CUDA;
  }
  return hif8_paged_attention(query, key_cache, value_cache, block_tables, seq_lens, query_start, batch,
                              num_tokens, num_heads, kv_heads, head_size, num_blocks, block_size, max_blocks,
                              max_seq_len, softmax_scale, causal, out, scratch, need, stream);
}
