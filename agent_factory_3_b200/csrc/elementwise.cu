// Memory-bound kernels of the gpt-oss block for sm_100a: RMSNorm forward/backward, rotary
// embedding (NeoX halves, YaRN-scaled tables), the cross-tile merge of the fused
// log-prob/entropy, and a standalone clamped SwiGLU (forward/backward) used outside the GEMM
// epilogues.
//
// RMSNorm follows HF GptOssRMSNorm (fp32 statistics, weight applied in fp32, cast to bf16).
// RoPE follows HF gpt_oss _apply_rotary_emb (first/second half rotation).
#include "common.h"
#include "host_utils.h"
#include "sm100.cuh"

namespace af3 {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float2 t = __bfloat1622float2(h[q]);
    f[2 * q] = t.x;
    f[2 * q + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 o;
  o.x = pack_bf16x2(f[0], f[1]);
  o.y = pack_bf16x2(f[2], f[3]);
  o.z = pack_bf16x2(f[4], f[5]);
  o.w = pack_bf16x2(f[6], f[7]);
  return o;
}

// ------------------------------------ RMSNorm ------------------------------------------
// One warp per row.  y = bf16(w * (x * rstd)), rstd = 1/sqrt(mean(x^2) + eps).
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                   const float* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                   int64_t ldy, float* __restrict__ rstd_out, int64_t T, int H,
                                   float eps) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= T) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
  const int vec = H / 8;
  float ss = 0.f;
  for (int j = lane; j < vec; j += 32) {
    float f[8];
    unpack8(xr[j], f);
#pragma unroll
    for (int q = 0; q < 8; ++q) ss += f[q] * f[q];
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / H + eps);
  if (rstd_out && lane == 0) rstd_out[row] = rstd;
  uint4* yr = reinterpret_cast<uint4*>(y + row * ldy);
  for (int j = lane; j < vec; j += 32) {
    float f[8];
    unpack8(xr[j], f);
    const float4 w0 = reinterpret_cast<const float4*>(w)[2 * j];
    const float4 w1 = reinterpret_cast<const float4*>(w)[2 * j + 1];
    const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int q = 0; q < 8; ++q) f[q] = ww[q] * (f[q] * rstd);
    yr[j] = pack8(f);
  }
}

// dx = rstd * (w*dy - xhat * mean(w*dy*xhat)) (+ dres).  Optional dw += sum_rows dy*xhat.
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                   const float* __restrict__ w, const __nv_bfloat16* __restrict__ dy,
                                   int64_t lddy, const float* __restrict__ rstd_in,
                                   const __nv_bfloat16* __restrict__ dres, int64_t lddr,
                                   __nv_bfloat16* __restrict__ dx, int64_t lddx,
                                   float* __restrict__ dw, int64_t T, int H) {
  const int lane = threadIdx.x % 32;
  const int64_t warps_total = (int64_t)gridDim.x * blockDim.x / 32;
  const int vec = H / 8;
  for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32; row < T;
       row += warps_total) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * ldx);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + row * lddy);
    const float rstd = rstd_in[row];
    float dot = 0.f;
    for (int j = lane; j < vec; j += 32) {
      float f[8], g[8];
      unpack8(xr[j], f);
      unpack8(gr[j], g);
      const float4 w0 = reinterpret_cast<const float4*>(w)[2 * j];
      const float4 w1 = reinterpret_cast<const float4*>(w)[2 * j + 1];
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) dot += ww[q] * g[q] * f[q] * rstd;
    }
    dot = warp_sum(dot) / H;
    uint4* dxr = reinterpret_cast<uint4*>(dx + row * lddx);
    for (int j = lane; j < vec; j += 32) {
      float f[8], g[8], r[8];
      unpack8(xr[j], f);
      unpack8(gr[j], g);
      const float4 w0 = reinterpret_cast<const float4*>(w)[2 * j];
      const float4 w1 = reinterpret_cast<const float4*>(w)[2 * j + 1];
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      if (dres) unpack8(reinterpret_cast<const uint4*>(dres + row * lddr)[j], r);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float xh = f[q] * rstd;
        float v = rstd * (ww[q] * g[q] - xh * dot);
        if (dres) v += r[q];
        f[q] = v;
        if (dw) atomicAdd(&dw[j * 8 + q], g[q] * xh);
      }
      dxr[j] = pack8(f);
    }
  }
}

void rmsnorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y,
                 c10::optional<torch::Tensor> rstd, double eps) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(y, "y");
  AF3_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous(), "rmsnorm weight must be fp32");
  const int64_t T = x.size(0);
  const int H = (int)x.size(1);
  AF3_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  const c10::cuda::CUDAGuard guard(x.device());
  if (T == 0) return;
  const int threads = 256;
  const int64_t grid = (T * 32 + threads - 1) / threads;
  rmsnorm_fwd_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), w.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0),
      rstd.has_value() ? rstd->data_ptr<float>() : nullptr, T, H, (float)eps);
  AF3_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm_bwd(torch::Tensor x, torch::Tensor w, torch::Tensor dy, torch::Tensor rstd,
                 c10::optional<torch::Tensor> dres, torch::Tensor dx,
                 c10::optional<torch::Tensor> dw) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(dy, "dy");
  check_cuda_bf16(dx, "dx");
  const int64_t T = x.size(0);
  const int H = (int)x.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  if (T == 0) return;
  const int threads = 256;
  const int64_t grid = std::min<int64_t>((T * 32 + threads - 1) / threads, (int64_t)num_sms() * 8);
  rmsnorm_bwd_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), w.data_ptr<float>(),
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), dy.stride(0), rstd.data_ptr<float>(),
      dres.has_value() ? reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr()) : nullptr,
      dres.has_value() ? dres->stride(0) : 0, reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()),
      dx.stride(0), dw.has_value() ? dw->data_ptr<float>() : nullptr, T, H);
  AF3_CUDA_CHECK(cudaGetLastError());
}

// -------------------------------------- RoPE -------------------------------------------
// In place on the first `n_rot_heads` heads (q then k) of each row of qkv [T, n_heads*D].
// cos/sin tables [P, D/2] fp32 (attention scaling already folded in).  sign=-1 applies the
// inverse rotation (backward).
template <int D>
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld, int n_rot_heads,
                            const int* __restrict__ pos, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, int64_t T, float sign) {
  constexpr int HALF = D / 2;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // (row, head, pair-of-8)
  constexpr int GROUPS = HALF / 8;
  const int64_t total = T * n_rot_heads * GROUPS;
  if (idx >= total) return;
  const int gi = idx % GROUPS;
  const int64_t rh = idx / GROUPS;
  const int h = rh % n_rot_heads;
  const int64_t row = rh / n_rot_heads;
  const int p = pos[row];
  __nv_bfloat16* base = qkv + row * ld + h * D;
  uint4* lo = reinterpret_cast<uint4*>(base + gi * 8);
  uint4* hi = reinterpret_cast<uint4*>(base + HALF + gi * 8);
  float a[8], b[8];
  unpack8(*lo, a);
  unpack8(*hi, b);
  const float* c = cos_t + (int64_t)p * HALF + gi * 8;
  const float* s = sin_t + (int64_t)p * HALF + gi * 8;
  float ra[8], rb[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float cq = c[q], sq = sign * s[q];
    ra[q] = a[q] * cq - b[q] * sq;
    rb[q] = b[q] * cq + a[q] * sq;
  }
  *lo = pack8(ra);
  *hi = pack8(rb);
}

void rope_apply(torch::Tensor qkv, int64_t n_rot_heads, int64_t head_dim, torch::Tensor pos,
                torch::Tensor cos_t, torch::Tensor sin_t, bool inverse) {
  check_cuda_bf16(qkv, "qkv");
  AF3_CHECK(head_dim == 16 || head_dim == 32 || head_dim == 64 || head_dim == 128,
            "rope: head_dim must be 16, 32, 64 or 128");
  const int64_t T = qkv.size(0);
  const c10::cuda::CUDAGuard guard(qkv.device());
  if (T == 0) return;
  const int64_t total = T * n_rot_heads * (head_dim / 16);
  const int threads = 256;
  const int64_t grid = (total + threads - 1) / threads;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto* p = reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr());
  const float sign = inverse ? -1.f : 1.f;
#define AF3_ROPE(D)                                                                          \
  rope_kernel<D><<<grid, threads, 0, stream>>>(p, qkv.stride(0), (int)n_rot_heads,           \
                                              pos.data_ptr<int>(), cos_t.data_ptr<float>(),   \
                                              sin_t.data_ptr<float>(), T, sign)
  if (head_dim == 16) AF3_ROPE(16);
  else if (head_dim == 32) AF3_ROPE(32);
  else if (head_dim == 64) AF3_ROPE(64);
  else AF3_ROPE(128);
#undef AF3_ROPE
  AF3_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------- log-prob merge ----------------------------------------
// parts [T, nt, 3] = (max, sumexp, sum z*exp) per vocab tile -> logZ, entropy, logprob.
__global__ void lse_merge_kernel(const float* __restrict__ parts, int nt,
                                 const float* __restrict__ label_logit, int64_t T,
                                 float* __restrict__ logprob, float* __restrict__ entropy,
                                 float* __restrict__ logz) {
  const int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= T) return;
  const float* p = parts + row * nt * 3;
  float m = -INFINITY;
  for (int i = lane; i < nt; i += 32) m = fmaxf(m, p[i * 3]);
  m = warp_max(m);
  float s = 0.f, t = 0.f;
  for (int i = lane; i < nt; i += 32) {
    const float mi = p[i * 3];
    if (mi == -INFINITY) continue;
    const float sc = __expf(mi - m);
    s += p[i * 3 + 1] * sc;
    t += p[i * 3 + 2] * sc;
  }
  s = warp_sum(s);
  t = warp_sum(t);
  if (lane == 0) {
    const float lz = m + __logf(s);
    logz[row] = lz;
    entropy[row] = lz - t / s;
    logprob[row] = label_logit[row] - lz;
  }
}

void lse_merge(torch::Tensor parts, torch::Tensor label_logit, torch::Tensor logprob,
               torch::Tensor entropy, torch::Tensor logz) {
  const int64_t T = parts.size(0);
  const int nt = (int)parts.size(1);
  const c10::cuda::CUDAGuard guard(parts.device());
  if (T == 0) return;
  const int threads = 256;
  lse_merge_kernel<<<(T * 32 + threads - 1) / threads, threads, 0,
                     at::cuda::getCurrentCUDAStream()>>>(
      parts.data_ptr<float>(), nt, label_logit.data_ptr<float>(), T, logprob.data_ptr<float>(),
      entropy.data_ptr<float>(), logz.data_ptr<float>());
  AF3_CUDA_CHECK(cudaGetLastError());
}

// ----------------------------- standalone clamped SwiGLU --------------------------------
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }

// gate_up [M, 2I] interleaved -> out [M, I].  Each thread handles 8 (gate, up) pairs: two
// 16-byte loads and one 16-byte store (scalar tail for counts not divisible by 8).
__device__ __forceinline__ float swiglu_one(float g, float u, float alpha, float limit) {
  const float gc = fminf(g, limit);
  const float uc = fminf(fmaxf(u, -limit), limit);
  return gc * sigmoidf_(alpha * gc) * (uc + 1.f);
}

__device__ __forceinline__ void swiglu_grad_one(float g, float u, float d, float alpha,
                                                float limit, float& dg, float& du) {
  const float gc = fminf(g, limit);
  const float uc = fminf(fmaxf(u, -limit), limit);
  const float s = sigmoidf_(alpha * gc);
  du = (u >= -limit && u <= limit) ? d * gc * s : 0.f;
  dg = (g <= limit) ? d * (uc + 1.f) * (s + gc * alpha * s * (1.f - s)) : 0.f;
}

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out,
                                  int64_t n_pairs, int64_t n8, float alpha, float limit) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += stride) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(gu) + 2 * i);
    const uint4 b = __ldcs(reinterpret_cast<const uint4*>(gu) + 2 * i + 1);
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
    float h[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = __bfloat1622float2(pa[e]);
      const float2 y = __bfloat1622float2(pb[e]);
      h[e] = swiglu_one(x.x, x.y, alpha, limit);
      h[4 + e] = swiglu_one(y.x, y.y, alpha, limit);
    }
    uint4 o;
    o.x = pack_bf16x2(h[0], h[1]);
    o.y = pack_bf16x2(h[2], h[3]);
    o.z = pack_bf16x2(h[4], h[5]);
    o.w = pack_bf16x2(h[6], h[7]);
    __stcs(reinterpret_cast<uint4*>(out) + i, o);
  }
  for (int64_t i = n8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_pairs; i += stride) {
    const float2 gv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(gu)[i]);
    out[i] = __float2bfloat16(swiglu_one(gv.x, gv.y, alpha, limit));
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  const __nv_bfloat16* __restrict__ dout,
                                  __nv_bfloat16* __restrict__ dgu, int64_t n_pairs, int64_t n8,
                                  float alpha, float limit) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += stride) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(gu) + 2 * i);
    const uint4 b = __ldcs(reinterpret_cast<const uint4*>(gu) + 2 * i + 1);
    const uint4 dv = __ldcs(reinterpret_cast<const uint4*>(dout) + i);
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
    const __nv_bfloat162* pd = reinterpret_cast<const __nv_bfloat162*>(&dv);
    uint32_t r[8];
    // pairs 0..3 come from `a`, 4..7 from `b`; their output gradients are dout[8i .. 8i+7]
    float dd[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 d = __bfloat1622float2(pd[e]);
      dd[2 * e] = d.x;
      dd[2 * e + 1] = d.y;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = __bfloat1622float2(pa[e]);
      const float2 y = __bfloat1622float2(pb[e]);
      float dg, du;
      swiglu_grad_one(x.x, x.y, dd[e], alpha, limit, dg, du);
      r[e] = pack_bf16x2(dg, du);
      swiglu_grad_one(y.x, y.y, dd[4 + e], alpha, limit, dg, du);
      r[4 + e] = pack_bf16x2(dg, du);
    }
    __stcs(reinterpret_cast<uint4*>(dgu) + 2 * i, make_uint4(r[0], r[1], r[2], r[3]));
    __stcs(reinterpret_cast<uint4*>(dgu) + 2 * i + 1, make_uint4(r[4], r[5], r[6], r[7]));
  }
  for (int64_t i = n8 * 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_pairs; i += stride) {
    const float2 gv = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(gu)[i]);
    float dg, du;
    swiglu_grad_one(gv.x, gv.y, __bfloat162float(dout[i]), alpha, limit, dg, du);
    reinterpret_cast<__nv_bfloat162*>(dgu)[i] = __floats2bfloat162_rn(dg, du);
  }
}

void swiglu_fwd(torch::Tensor gu, torch::Tensor out, double alpha, double limit) {
  check_cuda_bf16(gu, "gate_up");
  AF3_CHECK(gu.is_contiguous() && out.is_contiguous(), "swiglu needs contiguous tensors");
  const int64_t n = out.numel();
  const c10::cuda::CUDAGuard guard(gu.device());
  if (n == 0) return;
  // 8 pairs per thread through 16-byte accesses when every operand is 16-byte aligned
  const bool vec = aligned16(gu.data_ptr()) && aligned16(out.data_ptr());
  const int64_t n8 = vec ? n / 8 : 0;
  swiglu_fwd_kernel<<<std::min<int64_t>((std::max<int64_t>(n8, n - n8 * 8) + 255) / 256,
                                        num_sms() * 8), 256, 0,
                      at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n, n8, (float)alpha, (float)limit);
  AF3_CUDA_CHECK(cudaGetLastError());
}

void swiglu_bwd(torch::Tensor gu, torch::Tensor dout, torch::Tensor dgu, double alpha,
                double limit) {
  AF3_CHECK(gu.is_contiguous() && dout.is_contiguous() && dgu.is_contiguous(),
            "swiglu needs contiguous tensors");
  const int64_t n = dout.numel();
  const c10::cuda::CUDAGuard guard(gu.device());
  if (n == 0) return;
  const bool vec = aligned16(gu.data_ptr()) && aligned16(dout.data_ptr()) && aligned16(dgu.data_ptr());
  const int64_t n8 = vec ? n / 8 : 0;
  swiglu_bwd_kernel<<<std::min<int64_t>((std::max<int64_t>(n8, n - n8 * 8) + 255) / 256,
                                        num_sms() * 8), 256, 0,
                      at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), n, n8, (float)alpha, (float)limit);
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
