// FP8 (e4m3) path of the routed-MoE expert GEMMs: the B200 form of the reference's fp8
// dequantisation mode (models/gpt_oss/kernels.py K1 / K3 / K4 and quantizer_config.py in the
// reference, which dequantise MXFP4 experts to fp8 and quantise activations per token).
//
//   * mxfp4_to_e4m3: MXFP4 experts [E, N, K/32, 16] + e8m0 scales -> e4m3 bytes [E, N, K] with
//     one fp32 scale per expert.  The expert scale is 2^(s_max - 133), s_max the expert's
//     largest block-scale byte, so every e2m1 value x 2^(s - 127) becomes e2m1 x 2^(s - s_max
//     + 6): exact in e4m3 (max 448 = 1.75 x 2^8, smallest subnormal 2^-9) for every block
//     within 14 octaves of the expert's largest; blocks further down lose low bits / flush to
//     zero (their weights are below 2^-14 of the expert's largest).
//   * transpose_u8: [G, R, C] -> [G, C, R] bytes, the K-major copy of the weights that the
//     backward's dX = dY W needs (the reference's column-major fp8 copy, K3).
//   * quant_rows_e4m3: bf16 [M, K] -> e4m3 [M, K] with one fp32 scale per row (amax / 448),
//     the per-token activation quantisation (K4).
//   * gemm_f8: the tcgen05 GEMM template with F8 = true (kind::f8f6f4, K-major operands); the
//     epilogue multiplies by a_scale[row] * b_scale[group] before bias and the fused epilogue.
#include <cstdlib>
#include <string>

#include "common.h"
#include "gemm_launch.cuh"
#include "host_utils.h"

namespace af3 {
namespace f8 {

__device__ __forceinline__ uint16_t e4m3x2_of(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// value of an e2m1 code (sign, 2-bit exponent with bias 1, 1-bit mantissa)
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t e = (c >> 1) & 3u, m = c & 1u;
  float v = (e == 0) ? 0.5f * (float)m
                     : __uint_as_float(((e + 126u) << 23) | (m << 22));   // (1 + m/2) 2^(e-1)
  return (c & 8u) ? -v : v;
}

// max block-scale byte per expert
__global__ void expert_scale_max_kernel(const uint8_t* __restrict__ scales, int64_t per_expert,
                                        int* __restrict__ out) {
  const int e = blockIdx.y;
  const uint8_t* s = scales + (int64_t)e * per_expert;
  int m = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per_expert;
       i += (int64_t)gridDim.x * blockDim.x)
    m = max(m, (int)s[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out + e, m);
}

// one thread per 32-element block: 16 packed bytes -> 32 e4m3 bytes
__global__ void mxfp4_to_e4m3_kernel(const uint4* __restrict__ blocks, const uint8_t* __restrict__ scales,
                                     const int* __restrict__ smax, int64_t blocks_per_expert,
                                     int64_t n_blocks, uint4* __restrict__ out,
                                     float* __restrict__ expert_scale) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_blocks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)(i / blocks_per_expert);
    const int sm = smax[e];
    if (i % blocks_per_expert == 0) expert_scale[e] = exp2f((float)(sm - 133));
    // factor 2^(s - s_max + 6), built from its exponent bits (clamped at 2^-126)
    const int k = max((int)scales[i] - sm + 6, -126);
    const float f = __uint_as_float((uint32_t)(k + 127) << 23);
    const uint4 w = blocks[i];
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      // 8 codes of one word: byte b holds elements 2b (low nibble) and 2b+1 (high nibble)
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = e2m1_value((words[q] >> (4 * j)) & 15u) * f;
      o[2 * q] = (uint32_t)e4m3x2_of(v[0], v[1]) | ((uint32_t)e4m3x2_of(v[2], v[3]) << 16);
      o[2 * q + 1] = (uint32_t)e4m3x2_of(v[4], v[5]) | ((uint32_t)e4m3x2_of(v[6], v[7]) << 16);
    }
    out[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
    out[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// [G, R, C] -> [G, C, R] bytes through a 64 x 64 shared tile
__global__ void transpose_u8_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out,
                                    int R, int C) {
  __shared__ uint8_t tile[64][65];
  const int g = blockIdx.z;
  const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  const uint8_t* src = in + (int64_t)g * R * C;
  uint8_t* dst = out + (int64_t)g * R * C;
  for (int i = threadIdx.y; i < 64; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < R && c < C) ? src[(int64_t)r * C + c] : 0;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 64; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (c < C && r < R) dst[(int64_t)c * R + r] = tile[threadIdx.x][i];
  }
}

// one warp per row: amax, then x * 448 / amax rounded to e4m3 (saturating)
__global__ void quant_rows_e4m3_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                       uint8_t* __restrict__ out, int64_t ldo,
                                       float* __restrict__ scale, int64_t M, int K) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= M) return;
  const __nv_bfloat16* xr = x + row * ldx;
  float amax = 0.f;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 w = *reinterpret_cast<const uint4*>(xr + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = amax > 0.f ? amax / 448.f : 1.f;
  const float inv = amax > 0.f ? 448.f / amax : 1.f;
  if (lane == 0) scale[row] = sc;
  uint8_t* orow = out + row * ldo;
  for (int c = lane * 8; c < K; c += 256) {
    const uint4 w = *reinterpret_cast<const uint4*>(xr + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
    uint32_t q[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float2 a = __bfloat1622float2(h[2 * e]), b = __bfloat1622float2(h[2 * e + 1]);
      q[e] = (uint32_t)e4m3x2_of(a.x * inv, a.y * inv) |
             ((uint32_t)e4m3x2_of(b.x * inv, b.y * inv) << 16);
    }
    *reinterpret_cast<uint2*>(orow + c) = make_uint2(q[0], q[1]);
  }
}

}  // namespace f8

void mxfp4_to_e4m3(torch::Tensor blocks, torch::Tensor scales, torch::Tensor out,
                   torch::Tensor expert_scale) {
  AF3_CHECK(blocks.is_cuda() && blocks.scalar_type() == torch::kUInt8 && blocks.is_contiguous() &&
                blocks.dim() == 4 && blocks.size(3) == 16, "blocks must be uint8 [E, N, K/32, 16]");
  AF3_CHECK(scales.is_cuda() && scales.scalar_type() == torch::kUInt8 && scales.is_contiguous() &&
                scales.numel() * 16 == blocks.numel(), "scales must be uint8 [E, N, K/32]");
  AF3_CHECK(out.is_cuda() && out.scalar_type() == torch::kUInt8 && out.is_contiguous() &&
                out.numel() == blocks.numel() * 2, "out must be uint8 [E, N, K]");
  AF3_CHECK(expert_scale.is_cuda() && expert_scale.scalar_type() == torch::kFloat32 &&
                expert_scale.numel() == blocks.size(0), "expert_scale must be fp32 [E]");
  AF3_CHECK(reinterpret_cast<uintptr_t>(blocks.data_ptr()) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "16-byte aligned buffers");
  const c10::cuda::CUDAGuard guard(blocks.device());
  const int64_t E = blocks.size(0);
  const int64_t per = blocks.numel() / 16 / E;   // 32-element blocks per expert
  if (E == 0 || per == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto smax = torch::zeros({E}, blocks.options().dtype(torch::kInt32));
  f8::expert_scale_max_kernel<<<dim3((unsigned)std::min<int64_t>(64, (per + 255) / 256), (unsigned)E),
                                256, 0, stream>>>(scales.data_ptr<uint8_t>(), per,
                                                  smax.data_ptr<int>());
  AF3_CUDA_CHECK(cudaGetLastError());
  const int64_t n = E * per;
  f8::mxfp4_to_e4m3_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, num_sms() * 16), 256, 0,
                             stream>>>(reinterpret_cast<const uint4*>(blocks.data_ptr()),
                                       scales.data_ptr<uint8_t>(), smax.data_ptr<int>(), per, n,
                                       reinterpret_cast<uint4*>(out.data_ptr()),
                                       expert_scale.data_ptr<float>());
  AF3_CUDA_CHECK(cudaGetLastError());
}

void transpose_u8(torch::Tensor in, torch::Tensor out) {
  AF3_CHECK(in.is_cuda() && in.scalar_type() == torch::kUInt8 && in.is_contiguous() && in.dim() == 3,
            "in must be contiguous uint8 [G, R, C]");
  AF3_CHECK(out.is_cuda() && out.scalar_type() == torch::kUInt8 && out.is_contiguous() &&
                out.dim() == 3 && out.size(0) == in.size(0) && out.size(1) == in.size(2) &&
                out.size(2) == in.size(1), "out must be contiguous uint8 [G, C, R]");
  const c10::cuda::CUDAGuard guard(in.device());
  const int64_t G = in.size(0), R = in.size(1), C = in.size(2);
  if (G == 0 || R == 0 || C == 0) return;
  AF3_CHECK(R < (1 << 30) && C < (1 << 30) && G < 65536, "transpose_u8: shape too large");
  dim3 grid((unsigned)((C + 63) / 64), (unsigned)((R + 63) / 64), (unsigned)G);
  f8::transpose_u8_kernel<<<grid, dim3(64, 8), 0, at::cuda::getCurrentCUDAStream()>>>(
      in.data_ptr<uint8_t>(), out.data_ptr<uint8_t>(), (int)R, (int)C);
  AF3_CUDA_CHECK(cudaGetLastError());
}

void quant_rows_e4m3(torch::Tensor x, torch::Tensor out, torch::Tensor scale) {
  check_cuda_bf16(x, "x");
  AF3_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be 2-D with unit inner stride");
  AF3_CHECK(out.is_cuda() && out.scalar_type() == torch::kUInt8 && out.dim() == 2 &&
                out.stride(1) == 1 && out.size(0) == x.size(0) && out.size(1) == x.size(1),
            "out must be uint8 [M, K]");
  AF3_CHECK(scale.is_cuda() && scale.scalar_type() == torch::kFloat32 &&
                scale.numel() == x.size(0), "scale must be fp32 [M]");
  const int64_t M = x.size(0), K = x.size(1);
  AF3_CHECK(K % 8 == 0 && x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0 &&
                reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(out.data_ptr()) % 8 == 0,
            "quant_rows_e4m3: K and row strides must be multiples of 8, buffers aligned");
  const c10::cuda::CUDAGuard guard(x.device());
  if (M == 0) return;
  const int64_t threads = M * 32;
  f8::quant_rows_e4m3_kernel<<<(unsigned)((threads + 255) / 256), 256, 0,
                               at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), out.data_ptr<uint8_t>(),
      out.stride(0), scale.data_ptr<float>(), M, (int)K);
  AF3_CUDA_CHECK(cudaGetLastError());
}

#define AF3_GEMM_F8_TRY(BN_, B3D, SCH, EP)                                                  \
  if (bn == BN_ && b3d == B3D && sched == SCH && epi == EP) {                               \
    launch_gemm<BN_, false, false, B3D, SCH, EP, false, true>(o, args, ctas, stream);       \
    ok = true;                                                                              \
  }

void gemm_f8(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t epi, int64_t sched,
             int64_t M, int64_t N, int64_t K, c10::optional<torch::Tensor> group_offsets,
             int64_t num_groups, torch::Tensor a_scale, torch::Tensor b_scale,
             c10::optional<torch::Tensor> bias, int64_t bias_group_stride,
             c10::optional<torch::Tensor> row_scale, c10::optional<torch::Tensor> aux,
             c10::optional<torch::Tensor> out2, c10::optional<torch::Tensor> acc_add,
             double alpha, double act_alpha, double act_limit, int64_t bn, int64_t band,
             int64_t max_ctas) {
  AF3_CHECK(a.is_cuda() && a.scalar_type() == torch::kUInt8 && a.dim() == 2 && a.stride(1) == 1,
            "a must be uint8 (e4m3) [M, K] with unit inner stride");
  AF3_CHECK(b.is_cuda() && b.scalar_type() == torch::kUInt8 && (b.dim() == 2 || b.dim() == 3) &&
                b.stride(-1) == 1, "b must be uint8 (e4m3) [N, K] or [G, N, K]");
  AF3_CHECK(a.stride(0) % 16 == 0 && b.stride(-2) % 16 == 0 && (b.dim() == 2 || b.stride(0) % 16 == 0),
            "e4m3 row strides must be multiples of 16 bytes");
  AF3_CHECK(a_scale.is_cuda() && a_scale.scalar_type() == torch::kFloat32 && a_scale.numel() >= M,
            "a_scale must be fp32 [M]");
  AF3_CHECK(b_scale.is_cuda() && b_scale.scalar_type() == torch::kFloat32 &&
                b_scale.numel() >= (b.dim() == 3 ? b.size(0) : 1), "b_scale must be fp32 [G]");
  AF3_CHECK(M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31),
            "bad GEMM shape");
  const c10::cuda::CUDAGuard guard(a.device());
  if (M == 0) return;
  GemmOperands o;
  o.a = a.data_ptr();
  o.a_mn = false;
  o.lda = a.stride(0);
  o.a_rows = a.size(0);
  o.a_cols = a.size(1);
  o.b = b.data_ptr();
  o.b_mn = false;
  o.b_3d = b.dim() == 3;
  o.ldb = b.stride(-2);
  o.b_rows = b.size(-2);
  o.b_cols = b.size(-1);
  o.b_groups = o.b_3d ? b.size(0) : 1;
  o.b_gstride = o.b_3d ? b.stride(0) : 0;
  GemmArgs args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.num_groups = (int)num_groups;
  args.group_offsets = group_offsets.has_value() ? group_offsets->data_ptr<int>() : nullptr;
  args.band = (int)std::max<int64_t>(band, 1);
  args.out = out.data_ptr();
  args.ldo = out.stride(out.dim() - 2);
  args.bias = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  args.bias_group_stride = bias_group_stride;
  args.row_scale = row_scale.has_value() ? row_scale->data_ptr<float>() : nullptr;
  args.aux = aux.has_value() ? reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr()) : nullptr;
  args.ld_aux = aux.has_value() ? aux->stride(0) : 0;
  args.out2 = out2.has_value() ? out2->data_ptr() : nullptr;
  args.ldo2 = out2.has_value() ? out2->stride(0) : 0;
  args.acc_add = acc_add.has_value() ? reinterpret_cast<const __nv_bfloat16*>(acc_add->data_ptr())
                                     : nullptr;
  args.ld_acc_add = acc_add.has_value() ? acc_add->stride(0) : 0;
  args.a_scale = a_scale.data_ptr<float>();
  args.b_scale = b_scale.data_ptr<float>();
  args.alpha = (float)alpha;
  args.act_alpha = (float)act_alpha;
  args.act_limit = (float)act_limit;
  args.err = device_error_ptr();
  // describe the e4m3 bytes to TMA as 16-bit elements (AF3_F8_TMA=u16, default) or as bytes
  static const int kx_shift = [] {
    const char* e = std::getenv("AF3_F8_TMA");
    return (e && std::string(e) == "u8") ? 0 : 1;
  }();
  args.kx_shift = (K % 2 == 0) ? kx_shift : 0;
  if (sched != kSchedPlain) {
    AF3_CHECK(sched == kSchedGroupedM && group_offsets.has_value() && b.dim() == 3,
              "grouped FP8 GEMM: ragged M with a 3-D weight stack");
    AF3_CHECK(num_groups >= 1 && num_groups <= kMaxGroups, "num_groups out of range");
  }
  const int ctas = max_ctas > 0 ? (int)max_ctas : num_sms();
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  const bool b3d = o.b_3d;
  bool ok = false;
  AF3_GEMM_F8_TRY(256, false, kSchedPlain, kEpiBf16)
  else AF3_GEMM_F8_TRY(128, false, kSchedPlain, kEpiBf16)
  else AF3_GEMM_F8_TRY(256, true, kSchedGroupedM, kEpiBf16)
  else AF3_GEMM_F8_TRY(192, true, kSchedGroupedM, kEpiBf16)
  else AF3_GEMM_F8_TRY(128, true, kSchedGroupedM, kEpiBf16)
  else AF3_GEMM_F8_TRY(256, true, kSchedGroupedM, kEpiSwiglu)
  else AF3_GEMM_F8_TRY(192, true, kSchedGroupedM, kEpiSwiglu)
  else AF3_GEMM_F8_TRY(128, true, kSchedGroupedM, kEpiSwiglu)
  else AF3_GEMM_F8_TRY(256, true, kSchedGroupedM, kEpiRowScale)
  else AF3_GEMM_F8_TRY(192, true, kSchedGroupedM, kEpiRowScale)
  else AF3_GEMM_F8_TRY(128, true, kSchedGroupedM, kEpiRowScale)
  else AF3_GEMM_F8_TRY(256, true, kSchedGroupedM, kEpiSwigluBwd)
  else AF3_GEMM_F8_TRY(192, true, kSchedGroupedM, kEpiSwigluBwd)
  else AF3_GEMM_F8_TRY(128, true, kSchedGroupedM, kEpiSwigluBwd)
  AF3_CHECK(ok, "no FP8 GEMM variant for bn=" + std::to_string(bn) + " b_3d=" +
                    std::to_string(b3d) + " sched=" + std::to_string(sched) +
                    " epi=" + std::to_string(epi));
}

}  // namespace af3
