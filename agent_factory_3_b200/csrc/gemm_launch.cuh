// Host-side launch of the tcgen05 GEMM: builds the TMA descriptors for the operand layouts
// and launches the persistent kernel with one CTA per SM.
#pragma once
#include "gemm_sm100.cuh"
#include "host_utils.h"

namespace af3 {

struct GemmOperands {
  const void* a;
  bool a_mn;
  int64_t lda;  // elements between consecutive rows of the stored matrix
  int64_t a_rows, a_cols;  // stored shape (rows x cols, row-major)
  const void* b;
  bool b_mn;
  bool b_3d;
  int64_t ldb;
  int64_t b_rows, b_cols;  // per group (3-D: group g starts at b + g*b_gstride)
  int64_t b_groups;
  int64_t b_gstride;       // elements
  // second operand pair (dual mode); same majors as (a, b)
  const void* a2 = nullptr;
  int64_t lda2 = 0, a2_rows = 0, a2_cols = 0;
  const void* b2 = nullptr;
  int64_t ldb2 = 0, b2_rows = 0, b2_cols = 0, b2_gstride = 0;
};

// F8: operands are e4m3 bytes (K-major only); a 128-byte row of a box is 128 K elements.
// With f8_as_u16 the e4m3 bytes are described as 16-bit elements (half the count, same
// bytes and swizzle); the kernel then halves its K coordinates (GemmArgs::kx_shift).
template <int BN, bool F8 = false>
inline void build_tmaps(const GemmOperands& o, CUtensorMap& ta, CUtensorMap& tb, bool second,
                        bool f8_as_u16 = false) {
  const bool u16 = F8 && f8_as_u16;
  const auto bf16 = !F8 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                        : (u16 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8);
  constexpr int esz = F8 ? 1 : 2;   // bytes per logical K element
  const uint32_t kbox = F8 ? (u16 ? 64 : 128) : kBK;
  const int64_t cdiv = u16 ? 2 : 1;  // logical columns per TMA element
  const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const void* pa = second ? o.a2 : o.a;
  const int64_t lda = second ? o.lda2 : o.lda, a_rows = second ? o.a2_rows : o.a_rows,
                a_cols = second ? o.a2_cols : o.a_cols;
  const void* pb = second ? o.b2 : o.b;
  const int64_t ldb = second ? o.ldb2 : o.ldb, b_rows = second ? o.b2_rows : o.b_rows,
                b_cols = second ? o.b2_cols : o.b_cols,
                b_gstride = second ? o.b2_gstride : o.b_gstride;
  {
    uint64_t dims[2] = {(uint64_t)(a_cols / cdiv), (uint64_t)a_rows};
    uint64_t strides[1] = {(uint64_t)lda * esz};
    uint32_t box[2];
    if (!o.a_mn) { box[0] = kbox; box[1] = kBM; }  // [M, K]: K inner
    else { box[0] = 64; box[1] = kBK; }            // [K, M]: M inner, 64-wide chunks
    ta = make_tmap(pa, bf16, 2, dims, strides, box, sw);
  }
  {
    uint32_t box[3];
    if (!o.b_mn) { box[0] = kbox; box[1] = BN; box[2] = 1; }
    else { box[0] = 64; box[1] = kBK; box[2] = 1; }
    if (o.b_3d) {
      uint64_t dims[3] = {(uint64_t)(b_cols / cdiv), (uint64_t)b_rows, (uint64_t)o.b_groups};
      uint64_t strides[2] = {(uint64_t)ldb * esz, (uint64_t)b_gstride * esz};
      tb = make_tmap(pb, bf16, 3, dims, strides, box, sw);
    } else {
      uint64_t dims[2] = {(uint64_t)(b_cols / cdiv), (uint64_t)b_rows};
      uint64_t strides[1] = {(uint64_t)ldb * esz};
      tb = make_tmap(pb, bf16, 2, dims, strides, box, sw);
    }
  }
}

template <int BN, bool A_MN, bool B_MN, bool B_3D, int SCHED, int EPI, bool DUAL = false,
          bool F8 = false>
inline void launch_gemm(const GemmOperands& o, const GemmArgs& args, int max_ctas,
                        cudaStream_t stream) {
  CUtensorMap ta, tb, ta2, tb2;
  build_tmaps<BN, F8>(o, ta, tb, false, args.kx_shift == 1);
  if (DUAL) build_tmaps<BN, F8>(o, ta2, tb2, true);
  else { ta2 = ta; tb2 = tb; }
  auto kern = gemm_sm100_kernel<BN, A_MN, B_MN, B_3D, SCHED, EPI, DUAL, F8>;
  constexpr int smem = GemmCfg<BN>::SMEM_BYTES;
  static bool attr_set[64] = {};  // per device
  int dev = 0;
  AF3_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev >= 64 || !attr_set[dev]) {
    AF3_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (dev < 64) attr_set[dev] = true;
  }
  int ctas;
  if (SCHED == kSchedPlain) {
    const int64_t tiles = ((args.M + kBM - 1) / kBM) * (int64_t)((args.N + BN - 1) / BN);
    ctas = (int)std::min<int64_t>(tiles, max_ctas);
  } else {
    ctas = max_ctas;  // tile count lives on the device
  }
  if (ctas <= 0) return;
  kern<<<ctas, kGemmThreads, smem, stream>>>(ta, tb, ta2, tb2, args);
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
