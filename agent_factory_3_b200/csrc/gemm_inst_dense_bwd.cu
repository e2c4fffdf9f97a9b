// Dense backward GEMMs: data gradients dY x W (MN-major weight operand, optional fused LoRA
// branch) and weight gradients X^T x dY (both operands MN-major).
#include "gemm_dispatch.h"
#include "gemm_launch.cuh"

namespace af3 {
bool gemm_dispatch_dense_bwd(const GemmKey& k, const GemmOperands& o, const GemmArgs& args,
                             int max_ctas, cudaStream_t stream) {
  AF3_GEMM_TRY(256, false, true, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(192, false, true, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(128, false, true, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(64, false, true, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(256, false, true, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(192, false, true, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(128, false, true, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(64, false, true, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(256, false, true, false, kSchedPlain, kEpiBf16, true)
  AF3_GEMM_TRY(192, false, true, false, kSchedPlain, kEpiBf16, true)
  AF3_GEMM_TRY(256, true, true, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(192, true, true, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(128, true, true, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(64, true, true, false, kSchedPlain, kEpiF32, false)
  return false;
}
}  // namespace af3
