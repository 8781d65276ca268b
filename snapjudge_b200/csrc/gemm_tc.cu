// gemm_tc.cu — tcgen05 GEMM (placeholder until the tensor-core kernel lands).
#include "kernels.h"

namespace sjb {
bool gemm_tc_supported(int, int, int, bool) { return false; }
cudaError_t gemm_tc(const bf16*, const bf16*, const float*, bf16*, float*, int, int, int, int,
                    int, TcRope, int*, cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace sjb
