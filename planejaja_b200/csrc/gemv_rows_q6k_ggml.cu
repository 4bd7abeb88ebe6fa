// Fused decode GEMV instantiations for one weight format (gemv_rows.cuh).
#include "gemv_rows.cuh"

namespace nsq {
template cudaError_t launch_fused_code<kQ6KG>(bool, int, int, const FusedParams&, int, size_t, cudaStream_t, int*);
}  // namespace nsq
