// Routed-MoE backward GEMMs: expert data gradients dY_sorted x W_e (MN-major weights, fused
// SwiGLU backward, optional LoRA branch) and ragged-K per-expert LoRA weight gradients.
#include "gemm_dispatch.h"
#include "gemm_launch.cuh"

namespace af3 {
bool gemm_dispatch_grouped_bwd(const GemmKey& k, const GemmOperands& o, const GemmArgs& args,
                               int max_ctas, cudaStream_t stream) {
  AF3_GEMM_TRY(256, false, true, true, kSchedGroupedM, kEpiSwigluBwd, false)
  AF3_GEMM_TRY(192, false, true, true, kSchedGroupedM, kEpiSwigluBwd, false)
  AF3_GEMM_TRY(128, false, true, true, kSchedGroupedM, kEpiSwigluBwd, false)
  AF3_GEMM_TRY(256, false, true, true, kSchedGroupedM, kEpiSwigluBwd, true)
  AF3_GEMM_TRY(192, false, true, true, kSchedGroupedM, kEpiSwigluBwd, true)
  AF3_GEMM_TRY(256, false, true, true, kSchedGroupedM, kEpiBf16, false)
  AF3_GEMM_TRY(192, false, true, true, kSchedGroupedM, kEpiBf16, false)
  AF3_GEMM_TRY(128, false, true, true, kSchedGroupedM, kEpiBf16, false)
  AF3_GEMM_TRY(64, false, true, true, kSchedGroupedM, kEpiBf16, false)
  AF3_GEMM_TRY(256, false, true, true, kSchedGroupedM, kEpiBf16, true)
  AF3_GEMM_TRY(192, false, true, true, kSchedGroupedM, kEpiBf16, true)
  AF3_GEMM_TRY(256, true, true, false, kSchedGroupedK, kEpiF32, false)
  AF3_GEMM_TRY(192, true, true, false, kSchedGroupedK, kEpiF32, false)
  AF3_GEMM_TRY(128, true, true, false, kSchedGroupedK, kEpiF32, false)
  AF3_GEMM_TRY(64, true, true, false, kSchedGroupedK, kEpiF32, false)
  return false;
}
}  // namespace af3
