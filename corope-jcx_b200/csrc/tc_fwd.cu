// Tensor-core (tcgen05) CoRoPE forward for sm_100a.
#include "common.cuh"

namespace corope {

bool tc_fwd_supported(const FwdArgs& a, int dtype) { return false; }

cudaError_t tc_fwd_launch(const FwdArgs& a, int dtype, cudaStream_t st) {
  return cudaErrorNotSupported;
}

}  // namespace corope
