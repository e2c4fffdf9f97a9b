// Torch entry points of the paged decode attention (kernels in decode_attention_kernels.cuh)
// and the KV page store / gather kernels of the rollout engine.
#include "common.h"
#include "decode_attention_kernels.cuh"
#include "host_utils.h"
#include "sm100.cuh"

namespace af3 {
namespace dec {

// k/v of the new tokens -> their page slots.  kv [N, 2, Hkv, 64] rows given by qkv's k, v
// parts; slot[n] = page * page_size + offset.
__global__ void kv_store_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld, int k_off,
                                int v_off, const int* __restrict__ slots, __nv_bfloat16* __restrict__ kp,
                                __nv_bfloat16* __restrict__ vp, int n, int kv_width) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const int64_t slot = slots[i];
  if (slot < 0) return;
  const uint4* src_k = reinterpret_cast<const uint4*>(qkv + (int64_t)i * ld + k_off);
  const uint4* src_v = reinterpret_cast<const uint4*>(qkv + (int64_t)i * ld + v_off);
  uint4* dk = reinterpret_cast<uint4*>(kp + slot * kv_width);
  uint4* dv = reinterpret_cast<uint4*>(vp + slot * kv_width);
  for (int j = threadIdx.x; j < kv_width / 8; j += blockDim.x) {
    dk[j] = src_k[j];
    dv[j] = src_v[j];
  }
}

// Gather cached k/v of positions into a packed qkv buffer (prefill with a cached prefix).
__global__ void kv_gather_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld, int k_off, int v_off,
                                 const int* __restrict__ slots, const __nv_bfloat16* __restrict__ kp,
                                 const __nv_bfloat16* __restrict__ vp, int n, int kv_width) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const int64_t slot = slots[i];
  if (slot < 0) return;
  uint4* dk = reinterpret_cast<uint4*>(qkv + (int64_t)i * ld + k_off);
  uint4* dv = reinterpret_cast<uint4*>(qkv + (int64_t)i * ld + v_off);
  const uint4* sk = reinterpret_cast<const uint4*>(kp + slot * kv_width);
  const uint4* sv = reinterpret_cast<const uint4*>(vp + slot * kv_width);
  for (int j = threadIdx.x; j < kv_width / 8; j += blockDim.x) {
    dk[j] = sk[j];
    dv[j] = sv[j];
  }
}

}  // namespace dec

void decode_attention(torch::Tensor q, torch::Tensor k_pages, torch::Tensor v_pages,
                      torch::Tensor page_table, torch::Tensor seq_lens, torch::Tensor sinks,
                      torch::Tensor out, c10::optional<torch::Tensor> lse, int64_t hq, int64_t hkv,
                      int64_t window, double scale, int64_t max_seq_len) {
  using namespace dec;
  check_cuda_bf16(q, "q");
  check_cuda_bf16(k_pages, "k_pages");
  AF3_CHECK(k_pages.size(-1) == kD && k_pages.size(-2) == hkv, "k_pages must be [P, page, Hkv, 64]");
  const int G = (int)(hq / hkv);
  AF3_CHECK(hq % hkv == 0 && G <= kMaxG, "unsupported GQA group");
  const int B = (int)seq_lens.size(0);
  const c10::cuda::CUDAGuard guard(q.device());
  if (B == 0) return;
  const int page_size = (int)k_pages.size(1);
  const int chunk_tokens = kChunkPages * page_size;
  const int chunks = (int)std::max<int64_t>(1, (max_seq_len + chunk_tokens - 1) / chunk_tokens);
  auto part_o = torch::empty({B, hq, chunks, kD}, q.options().dtype(torch::kFloat32));
  auto part_ml = torch::empty({B, hq, chunks, 2}, q.options().dtype(torch::kFloat32));
  Params p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.ld_q = q.stride(0);
  p.kp = reinterpret_cast<const __nv_bfloat16*>(k_pages.data_ptr());
  p.vp = reinterpret_cast<const __nv_bfloat16*>(v_pages.data_ptr());
  p.page_table = page_table.data_ptr<int>();
  p.max_pages = (int)page_table.size(1);
  p.seq_lens = seq_lens.data_ptr<int>();
  p.part_o = part_o.data_ptr<float>();
  p.part_ml = part_ml.data_ptr<float>();
  p.page_size = page_size;
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.window = (int)window;
  p.chunks = chunks;
  p.scale_log2 = (float)scale * 1.4426950408889634f;
  auto stream = at::cuda::getCurrentCUDAStream();
  dim3 grid(chunks, (unsigned)hkv, B);
  switch (G) {
    case 1: decode_attn_kernel<1><<<grid, kWarps * 32, 0, stream>>>(p); break;
    case 2: decode_attn_kernel<2><<<grid, kWarps * 32, 0, stream>>>(p); break;
    case 4: decode_attn_kernel<4><<<grid, kWarps * 32, 0, stream>>>(p); break;
    case 8: decode_attn_mma_kernel<<<grid, kWarps * 32, 0, stream>>>(p); break;   // tensor cores
    case 16: decode_attn_kernel<16><<<grid, kWarps * 32, 0, stream>>>(p); break;
    default: AF3_CHECK(false, "GQA group must be 1, 2, 4, 8 or 16");
  }
  AF3_CUDA_CHECK(cudaGetLastError());
  decode_combine_kernel<<<dim3((unsigned)hq, B), kD, 0, stream>>>(
      part_o.data_ptr<float>(), part_ml.data_ptr<float>(), sinks.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), (int)hq, chunks,
      lse.has_value() ? lse->data_ptr<float>() : nullptr);
  AF3_CUDA_CHECK(cudaGetLastError());
}

void kv_store(torch::Tensor qkv, int64_t k_off, int64_t v_off, torch::Tensor slots,
              torch::Tensor k_pages, torch::Tensor v_pages) {
  check_cuda_bf16(qkv, "qkv");
  const int n = (int)slots.numel();
  const int kv_width = (int)(k_pages.size(-1) * k_pages.size(-2));
  const c10::cuda::CUDAGuard guard(qkv.device());
  if (n == 0) return;
  dec::kv_store_kernel<<<n, 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), (int)k_off, (int)v_off,
      slots.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(k_pages.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v_pages.data_ptr()), n, kv_width);
  AF3_CUDA_CHECK(cudaGetLastError());
}

void kv_gather(torch::Tensor qkv, int64_t k_off, int64_t v_off, torch::Tensor slots,
               torch::Tensor k_pages, torch::Tensor v_pages) {
  check_cuda_bf16(qkv, "qkv");
  const int n = (int)slots.numel();
  const int kv_width = (int)(k_pages.size(-1) * k_pages.size(-2));
  const c10::cuda::CUDAGuard guard(qkv.device());
  if (n == 0) return;
  dec::kv_gather_kernel<<<n, 64, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), (int)k_off, (int)v_off,
      slots.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(k_pages.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(v_pages.data_ptr()), n, kv_width);
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
