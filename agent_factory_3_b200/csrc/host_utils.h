// Host-side helpers shared by the extension's launchers: TMA tensor-map encoding through the
// driver entry point (no link-time dependency on libcuda), argument checks and the
// device-error word.
#pragma once
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <mutex>
#include <stdexcept>
#include <string>

namespace af3 {

#define AF3_CHECK(cond, msg)                                                        \
  do {                                                                              \
    if (!(cond)) throw std::runtime_error(std::string("af3: ") + (msg));            \
  } while (0)

#define AF3_CUDA_CHECK(expr)                                                        \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    if (_e != cudaSuccess)                                                          \
      throw std::runtime_error(std::string("af3 CUDA error: ") + cudaGetErrorString(_e) + \
                               " at " + __FILE__ + ":" + std::to_string(__LINE__)); \
  } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("af3: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Row-major tensor of `rank` (2 or 3) dims given innermost-first.  strides_bytes has rank-1
// entries (dims 1..rank-1).  The box is innermost-first as well.
inline CUtensorMap make_tmap(const void* ptr, CUtensorMapDataType dtype, int rank,
                             const uint64_t* dims, const uint64_t* strides_bytes,
                             const uint32_t* box, CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t gd[5];
  cuuint64_t gs[4];
  cuuint32_t bx[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    gs[i] = strides_bytes[i];
    AF3_CHECK(strides_bytes[i] % 16 == 0, "TMA stride must be a multiple of 16 bytes");
  }
  AF3_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base must be 16-byte aligned");
  CUresult r = get_encode_tiled()(&m, dtype, rank, const_cast<void*>(ptr), gd, gs, bx, es,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  AF3_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return m;
}

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    AF3_CUDA_CHECK(cudaGetDevice(&dev));
    AF3_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

inline void check_cuda_bf16(const torch::Tensor& t, const char* name) {
  AF3_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
  AF3_CHECK(t.scalar_type() == torch::kBFloat16, std::string(name) + " must be bfloat16");
}

}  // namespace af3
