// Dispatch of the tcgen05 GEMM over its compile-time variants (tile width, operand majors,
// scheduling mode, epilogue, dual operand).  Variants are instantiated in gemm_inst_*.cu so
// they compile in parallel; each file contributes one dispatch function.
#pragma once
#include "gemm_sm100.cuh"
#include "host_utils.h"

namespace af3 {
struct GemmOperands;
struct GemmKey {
  int bn;
  bool a_mn, b_mn, b_3d;
  int sched, epi;
  bool dual;
};
using GemmDispatchFn = bool (*)(const GemmKey&, const GemmOperands&, const GemmArgs&, int,
                                cudaStream_t);
bool gemm_dispatch_dense_fwd(const GemmKey&, const GemmOperands&, const GemmArgs&, int,
                             cudaStream_t);
bool gemm_dispatch_dense_bwd(const GemmKey&, const GemmOperands&, const GemmArgs&, int,
                             cudaStream_t);
bool gemm_dispatch_grouped_fwd(const GemmKey&, const GemmOperands&, const GemmArgs&, int,
                               cudaStream_t);
bool gemm_dispatch_grouped_bwd(const GemmKey&, const GemmOperands&, const GemmArgs&, int,
                               cudaStream_t);
}  // namespace af3

#define AF3_GEMM_TRY(BN_, AMN, BMN, B3D, SCH, EP, DU)                                      \
  if (k.bn == BN_ && k.a_mn == AMN && k.b_mn == BMN && k.b_3d == B3D && k.sched == SCH &&   \
      k.epi == EP && k.dual == DU) {                                                        \
    launch_gemm<BN_, AMN, BMN, B3D, SCH, EP, DU>(o, args, max_ctas, stream);                \
    return true;                                                                            \
  }
