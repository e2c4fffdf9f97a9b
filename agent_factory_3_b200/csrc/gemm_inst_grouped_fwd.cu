// Routed-MoE forward GEMMs over 128-row padded expert segments: gate_up with fused clamped
// SwiGLU, down with fused gate weights, both optionally with the per-expert LoRA branch.
#include "gemm_dispatch.h"
#include "gemm_launch.cuh"

namespace af3 {
bool gemm_dispatch_grouped_fwd(const GemmKey& k, const GemmOperands& o, const GemmArgs& args,
                               int max_ctas, cudaStream_t stream) {
  AF3_GEMM_TRY(256, false, false, true, kSchedGroupedM, kEpiSwiglu, false)
  AF3_GEMM_TRY(192, false, false, true, kSchedGroupedM, kEpiSwiglu, false)
  AF3_GEMM_TRY(128, false, false, true, kSchedGroupedM, kEpiSwiglu, false)
  AF3_GEMM_TRY(256, false, false, true, kSchedGroupedM, kEpiSwiglu, true)
  AF3_GEMM_TRY(192, false, false, true, kSchedGroupedM, kEpiSwiglu, true)
  AF3_GEMM_TRY(256, false, false, true, kSchedGroupedM, kEpiRowScale, false)
  AF3_GEMM_TRY(192, false, false, true, kSchedGroupedM, kEpiRowScale, false)
  AF3_GEMM_TRY(128, false, false, true, kSchedGroupedM, kEpiRowScale, false)
  AF3_GEMM_TRY(256, false, false, true, kSchedGroupedM, kEpiRowScale, true)
  AF3_GEMM_TRY(192, false, false, true, kSchedGroupedM, kEpiRowScale, true)
  AF3_GEMM_TRY(256, false, false, true, kSchedGroupedM, kEpiBf16, false)
  AF3_GEMM_TRY(192, false, false, true, kSchedGroupedM, kEpiBf16, false)
  AF3_GEMM_TRY(128, false, false, true, kSchedGroupedM, kEpiBf16, false)
  AF3_GEMM_TRY(32, false, false, true, kSchedGroupedM, kEpiBf16, false)
  return false;
}
}  // namespace af3
