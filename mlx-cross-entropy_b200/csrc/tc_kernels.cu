// tcgen05 kernels (placeholder until the tensor-core path lands).
#include "kernels.cuh"

namespace cce {
bool tc_supported(const void*, const void*, int64_t, int) { return false; }
cudaError_t tc_forward(const FwdArgs&, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t tc_dlogits(const BwdChunkArgs&, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t tc_grad_e(const BwdChunkArgs&, float*, bool, void*, bool, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t tc_grad_c(const BwdChunkArgs&, void*, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace cce
