// Prefill GEMM entry (tcgen05).  Until the tcgen05 kernel is enabled every
// shape reports "unsupported" and soft_hif8_gemm runs the split-K kernel on
// 16-token slices.
#include "linear.cuh"

namespace hif8 {

bool hif8_gemm_tc_supported(int64_t, int64_t, int64_t) { return false; }
size_t hif8_gemm_tc_workspace(int64_t, int64_t, int64_t) { return 0; }
int hif8_gemm_tc(const GemvArgs &, int, void *, size_t, cudaStream_t) { return HIF8_ERR_INVALID_ARGUMENT; }

}  // namespace hif8
