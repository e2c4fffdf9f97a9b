// Dense forward GEMMs: activations x weight^T (projections with fused LoRA, router, LoRA
// down-projections, LM head with fused log-sum-exp and its backward logits).
#include "gemm_dispatch.h"
#include "gemm_launch.cuh"

namespace af3 {
bool gemm_dispatch_dense_fwd(const GemmKey& k, const GemmOperands& o, const GemmArgs& args,
                             int max_ctas, cudaStream_t stream) {
  AF3_GEMM_TRY(256, false, false, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(192, false, false, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(128, false, false, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(64, false, false, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(32, false, false, false, kSchedPlain, kEpiBf16, false)
  AF3_GEMM_TRY(256, false, false, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(192, false, false, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(128, false, false, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(64, false, false, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(32, false, false, false, kSchedPlain, kEpiF32, false)
  AF3_GEMM_TRY(256, false, false, false, kSchedPlain, kEpiBf16, true)
  AF3_GEMM_TRY(192, false, false, false, kSchedPlain, kEpiBf16, true)
  AF3_GEMM_TRY(128, false, false, false, kSchedPlain, kEpiBf16, true)
  AF3_GEMM_TRY(256, false, false, false, kSchedPlain, kEpiLse, false)
  AF3_GEMM_TRY(256, false, false, false, kSchedPlain, kEpiLogprobBwd, false)
  return false;
}
}  // namespace af3
