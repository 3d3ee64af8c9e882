// fp16 backward on tcgen05 (dQ and dK/dV kernels). Placeholder until the tensor-core kernels land.
#include "common.cuh"
#include "kernels.h"

namespace tattn {

cudaError_t launch_bwd_dq_f16(int, bool, int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                              const CUtensorMap&, const BwdArgs&, cudaStream_t) {
  return cudaErrorNotSupported;
}

cudaError_t launch_bwd_dkdv_f16(int, bool, int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                                const CUtensorMap&, const BwdArgs&, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace tattn
