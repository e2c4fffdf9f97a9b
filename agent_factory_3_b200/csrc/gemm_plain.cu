// Instantiations of the tcgen05 GEMM for dense (non-grouped) problems: projections, router,
// LM head with fused log-prob epilogues, data and weight gradients.
#include "gemm_dispatch.h"
#include "gemm_launch.cuh"

namespace af3 {

#define AF3_TRY(BN_, AMN, BMN, EP)                                                    \
  if (bn == BN_ && a_mn == AMN && b_mn == BMN && epi == EP) {                        \
    launch_gemm<BN_, AMN, BMN, false, kSchedPlain, EP>(o, args, max_ctas, stream);   \
    return true;                                                                      \
  }

bool gemm_dispatch_plain(int bn, bool a_mn, bool b_mn, int epi, const GemmOperands& o,
                         const GemmArgs& args, int max_ctas, cudaStream_t stream) {
  // activations x weights^T
  AF3_TRY(256, false, false, kEpiBf16)
  AF3_TRY(128, false, false, kEpiBf16)
  AF3_TRY(64, false, false, kEpiBf16)
  AF3_TRY(32, false, false, kEpiBf16)
  AF3_TRY(256, false, false, kEpiF32)
  AF3_TRY(128, false, false, kEpiF32)
  AF3_TRY(64, false, false, kEpiF32)
  AF3_TRY(32, false, false, kEpiF32)
  AF3_TRY(256, false, false, kEpiLse)
  AF3_TRY(256, false, false, kEpiLogprobBwd)
  // data gradients: dY x W (W row-major [K, N] -> MN-major B)
  AF3_TRY(256, false, true, kEpiBf16)
  AF3_TRY(128, false, true, kEpiBf16)
  AF3_TRY(64, false, true, kEpiBf16)
  AF3_TRY(256, false, true, kEpiF32)
  AF3_TRY(128, false, true, kEpiF32)
  AF3_TRY(64, false, true, kEpiF32)
  // weight gradients: X^T x dY (both MN-major)
  AF3_TRY(256, true, true, kEpiF32)
  AF3_TRY(128, true, true, kEpiF32)
  AF3_TRY(64, true, true, kEpiF32)
  return false;
}

}  // namespace af3
