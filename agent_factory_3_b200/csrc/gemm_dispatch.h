// Dispatch of the tcgen05 GEMM over its compile-time variants (tile width, operand majors,
// scheduling mode, epilogue).  The variants are instantiated in gemm_plain.cu and
// gemm_grouped.cu so they compile in parallel.
#pragma once
#include "gemm_sm100.cuh"
#include "host_utils.h"

namespace af3 {
struct GemmOperands;
bool gemm_dispatch_plain(int bn, bool a_mn, bool b_mn, int epi, const GemmOperands& o,
                         const GemmArgs& args, int max_ctas, cudaStream_t stream);
bool gemm_dispatch_grouped(int bn, bool a_mn, bool b_mn, bool b_3d, int sched, int epi,
                           const GemmOperands& o, const GemmArgs& args, int max_ctas,
                           cudaStream_t stream);
}  // namespace af3
