// Tensor-core (tcgen05 + TMA) attention kernels for 16-bit inputs.
#include "common.cuh"
#include "params.cuh"

namespace hfan {
bool tc_supported(int dtype, const AttnParams& p) { (void)dtype; (void)p; return false; }
cudaError_t tc_attention_fwd(int, const AttnParams&, int, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t tc_attention_bwd(int, const AttnParams&, int, int, cudaStream_t) { return cudaErrorNotSupported; }
}  // namespace hfan
