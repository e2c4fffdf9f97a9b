// Instantiations of the tcgen05 GEMM for routed-MoE problems: ragged-M expert GEMMs
// (forward gate_up with fused clamped SwiGLU, down with fused gate weights, data gradients
// with fused SwiGLU backward) and ragged-K per-expert weight gradients.
#include "gemm_dispatch.h"
#include "gemm_launch.cuh"

namespace af3 {

#define AF3_TRYG(BN_, AMN, BMN, B3D, SCH, EP)                                          \
  if (bn == BN_ && a_mn == AMN && b_mn == BMN && b_3d == B3D && sched == SCH && epi == EP) { \
    launch_gemm<BN_, AMN, BMN, B3D, SCH, EP>(o, args, max_ctas, stream);               \
    return true;                                                                        \
  }

bool gemm_dispatch_grouped(int bn, bool a_mn, bool b_mn, bool b_3d, int sched, int epi,
                           const GemmOperands& o, const GemmArgs& args, int max_ctas,
                           cudaStream_t stream) {
  // forward: x_sorted x W_e^T
  AF3_TRYG(256, false, false, true, kSchedGroupedM, kEpiSwiglu)
  AF3_TRYG(192, false, false, true, kSchedGroupedM, kEpiSwiglu)
  AF3_TRYG(128, false, false, true, kSchedGroupedM, kEpiSwiglu)
  AF3_TRYG(256, false, false, true, kSchedGroupedM, kEpiRowScale)
  AF3_TRYG(192, false, false, true, kSchedGroupedM, kEpiRowScale)
  AF3_TRYG(128, false, false, true, kSchedGroupedM, kEpiRowScale)
  AF3_TRYG(256, false, false, true, kSchedGroupedM, kEpiBf16)
  AF3_TRYG(192, false, false, true, kSchedGroupedM, kEpiBf16)
  AF3_TRYG(128, false, false, true, kSchedGroupedM, kEpiBf16)
  AF3_TRYG(32, false, false, true, kSchedGroupedM, kEpiBf16)
  // backward data gradient: dY_sorted x W_e (MN-major B)
  AF3_TRYG(256, false, true, true, kSchedGroupedM, kEpiSwigluBwd)
  AF3_TRYG(192, false, true, true, kSchedGroupedM, kEpiSwigluBwd)
  AF3_TRYG(128, false, true, true, kSchedGroupedM, kEpiSwigluBwd)
  AF3_TRYG(256, false, true, true, kSchedGroupedM, kEpiBf16)
  AF3_TRYG(192, false, true, true, kSchedGroupedM, kEpiBf16)
  AF3_TRYG(128, false, true, true, kSchedGroupedM, kEpiBf16)
  AF3_TRYG(64, false, true, true, kSchedGroupedM, kEpiBf16)
  // ragged-K weight gradients (both operands MN-major activations)
  AF3_TRYG(256, true, true, false, kSchedGroupedK, kEpiF32)
  AF3_TRYG(192, true, true, false, kSchedGroupedK, kEpiF32)
  AF3_TRYG(128, true, true, false, kSchedGroupedK, kEpiF32)
  AF3_TRYG(64, true, true, false, kSchedGroupedK, kEpiF32)
  return false;
}

}  // namespace af3
