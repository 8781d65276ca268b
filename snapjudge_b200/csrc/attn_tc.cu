// attn_tc.cu — tcgen05 flash attention (placeholder until the tensor-core kernel lands).
#include "kernels.h"

namespace sjb {
bool attn_tc_supported(int) { return false; }
cudaError_t attn_tc(const bf16*, const int32_t*, const int32_t*, bf16*, int, int, int,
                    const int2*, int, int, int, int*, cudaStream_t) {
  return cudaErrorNotSupported;
}
}  // namespace sjb
