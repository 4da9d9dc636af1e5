// Library-wide C-ABI plumbing: status strings, last-error text, codec tables.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "hif8_common.cuh"

namespace hif8 {

static thread_local char g_last_error[256] = "no error";

void set_last_error(cudaError_t err) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(err),
                cudaGetErrorString(err));
}

int check_launch() {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_last_error(err);
    return HIF8_ERR_CUDA;
  }
  return HIF8_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("HIF8_DISABLE_PDL");
    return !(v && v[0] == '1');
  }();
  return on;
}

int num_sms() {
  static std::atomic<int> cache[128];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

int ensure_smem_limit(const void *kernel, size_t bytes) {
  struct Entry {
    const void *kernel;
    int device;
    size_t bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (Entry &e : done) {
    if (e.kernel == kernel && e.device == dev) {
      if (e.bytes >= bytes) return HIF8_OK;
      const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
      if (err != cudaSuccess) {
        cudaGetLastError();  // reported through the status; must not surface at the next launch check
        set_last_error(err);
        return HIF8_ERR_CUDA;
      }
      e.bytes = bytes;
      return HIF8_OK;
    }
  }
  const cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (err != cudaSuccess) {
    cudaGetLastError();  // reported through the status; must not surface at the next launch check
    set_last_error(err);
    return HIF8_ERR_CUDA;
  }
  done.push_back({kernel, dev, bytes});
  return HIF8_OK;
}

}  // namespace hif8

extern "C" {

const char *hif8_status_string(int status) {
  switch (status) {
    case HIF8_OK: return "ok";
    case HIF8_ERR_INVALID_ARGUMENT: return "invalid argument";
    case HIF8_ERR_CUDA: return "CUDA error";
    case HIF8_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}

const char *hif8_last_error(void) { return hif8::g_last_error; }

const char *hif8_version(void) { return "0.1.0"; }

void hif8_decode_table_bf16(uint16_t out[256]) {
  for (uint32_t b = 0; b < 256u; ++b) out[b] = (uint16_t)hif8::decode_bf16(b);
}

void hif8_encode_table(uint8_t out[4096]) {
  for (uint32_t i = 0; i < 4096u; ++i) out[i] = (uint8_t)hif8::encode_grid(i);
}

}  // extern "C"
