// Routed-MoE support kernels for sm_100a:
//   * MXFP4 (e2m1 values + e8m0 block scales) -> bf16 dequantisation
//   * router: top-k (or replay of recorded expert ids) with softmax over the chosen logits
//   * deterministic stable grouping of (token, slot) pairs by expert into 128-row padded
//     segments, so every GEMM tile belongs to exactly one expert
//   * row gather into the expert-sorted buffer and the top-k combine back to token order
//
// Semantics follow the reference's torch paths: MXFP4 decode as in
// models/gpt_oss/quantization.py:102-122 (_mxfp4_to_bf16_pytorch: low nibble first, value =
// FP4_VALUES[nibble] * 2^(scale-127)); routing replay as in quantization.py:593-636 (softmax over
// the K selected logits, stable sort by expert id); top-k routing as in HF GptOssTopKRouter.
#include "common.h"
#include "host_utils.h"
#include "mxfp4.cuh"
#include "sm100.cuh"

namespace af3 {

// ------------------------------------ MXFP4 ------------------------------------------
// One thread per 4 packed bytes (8 values, 16 output bytes): loads and stores of a warp are
// contiguous (128 B in, 512 B out); the 4 threads of one 32-element block share its scale.
__global__ void mxfp4_dequant_kernel(const uint32_t* __restrict__ words,
                                     const uint8_t* __restrict__ scales, uint4* __restrict__ out,
                                     int64_t n_words) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_words;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t w = __ldg(words + i);
    const uint32_t s = __ldg(scales + (i >> 2));
    out[i] = e2m1x8_to_bf16x8(w, e8m0_to_bf16_bits(s));
  }
}

void mxfp4_dequant(torch::Tensor blocks, torch::Tensor scales, torch::Tensor out) {
  AF3_CHECK(blocks.is_cuda() && blocks.scalar_type() == torch::kUInt8, "blocks must be uint8 CUDA");
  AF3_CHECK(scales.scalar_type() == torch::kUInt8, "scales must be uint8");
  AF3_CHECK(blocks.is_contiguous() && scales.is_contiguous() && out.is_contiguous(),
            "mxfp4_dequant needs contiguous tensors");
  AF3_CHECK(blocks.size(-1) == 16, "blocks last dim must be 16");
  const int64_t n = scales.numel();
  AF3_CHECK(blocks.numel() == n * 16 && out.numel() == n * 32, "mxfp4 shape mismatch");
  AF3_CHECK(out.scalar_type() == torch::kBFloat16, "out must be bf16");
  AF3_CHECK(reinterpret_cast<uintptr_t>(blocks.data_ptr()) % 4 == 0 &&
                reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
            "mxfp4_dequant needs 4-byte aligned blocks and 16-byte aligned out");
  const c10::cuda::CUDAGuard guard(blocks.device());
  if (n == 0) return;
  const int threads = 256;
  const int64_t n_words = n * 4;
  const int64_t grid = std::min<int64_t>((n_words + threads - 1) / threads, (int64_t)num_sms() * 32);
  mxfp4_dequant_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint32_t*>(blocks.data_ptr<uint8_t>()), scales.data_ptr<uint8_t>(),
      reinterpret_cast<uint4*>(out.data_ptr()), n_words);
  AF3_CUDA_CHECK(cudaGetLastError());
}

// MXFP4 -> bf16 of an expert stack whose experts are spread over the ranks of a node: expert e
// lives on rank e / experts_per_rank at local index e % experts_per_rank, in that rank's
// peer-mapped shard (plain loads over NVLink for the other ranks' experts, no TMA).  This is
// the all-gather of the sharded frozen experts fused with their dequantisation: the packed
// bytes cross NVLink once and only the bf16 result is written, to this GPU's own memory.
// Grid: (blocks over the words of one expert, experts).
__global__ void mxfp4_dequant_gather_kernel(const uint64_t* __restrict__ block_ptrs,
                                            const uint64_t* __restrict__ scale_ptrs,
                                            int experts_per_rank, int64_t words_per_expert,
                                            uint4* __restrict__ out) {
  const int e = blockIdx.y;
  const int r = e / experts_per_rank, le = e - r * experts_per_rank;
  const uint32_t* words = reinterpret_cast<const uint32_t*>(block_ptrs[r]) + le * words_per_expert;
  const uint8_t* scales = reinterpret_cast<const uint8_t*>(scale_ptrs[r]) + le * (words_per_expert / 4);
  uint4* dst = out + (int64_t)e * words_per_expert;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words_per_expert;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t w = __ldg(words + i);
    const uint32_t s = __ldg(scales + (i >> 2));
    dst[i] = e2m1x8_to_bf16x8(w, e8m0_to_bf16_bits(s));
  }
}

void mxfp4_dequant_gather(torch::Tensor block_ptrs, torch::Tensor scale_ptrs,
                          int64_t experts_per_rank, torch::Tensor out) {
  AF3_CHECK(block_ptrs.is_cuda() && block_ptrs.scalar_type() == torch::kInt64 &&
                scale_ptrs.is_cuda() && scale_ptrs.scalar_type() == torch::kInt64,
            "pointer tables must be int64 CUDA tensors");
  AF3_CHECK(block_ptrs.numel() == scale_ptrs.numel() && block_ptrs.numel() >= 1, "pointer tables");
  AF3_CHECK(out.is_cuda() && out.scalar_type() == torch::kBFloat16 && out.is_contiguous() &&
                out.dim() == 3, "out must be contiguous bf16 [E, N, K]");
  AF3_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out must be 16-byte aligned");
  const int64_t E = out.size(0), N = out.size(1), K = out.size(2);
  AF3_CHECK(K % 32 == 0, "K must be a multiple of 32");
  AF3_CHECK(experts_per_rank > 0 && E == experts_per_rank * block_ptrs.numel(),
            "experts must equal experts_per_rank x ranks");
  const c10::cuda::CUDAGuard guard(out.device());
  const int64_t words = N * K / 8;   // one 32-bit word = 8 e2m1 values
  if (E == 0 || words == 0) return;
  const int threads = 256;
  const int64_t per = std::max<int64_t>(1, std::min<int64_t>((words + threads - 1) / threads,
                                                              (int64_t)num_sms() * 32 / E + 1));
  mxfp4_dequant_gather_kernel<<<dim3((unsigned)per, (unsigned)E), threads, 0,
                                at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint64_t*>(block_ptrs.data_ptr<int64_t>()),
      reinterpret_cast<const uint64_t*>(scale_ptrs.data_ptr<int64_t>()), (int)experts_per_rank,
      words, reinterpret_cast<uint4*>(out.data_ptr()));
  AF3_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------ router -----------------------------------------
// One warp per token.  If `replay`, ids[t, :] are read; otherwise the top-K logits are
// selected (ties: lower expert id first, as torch.topk on CPU/CUDA for distinct values).
// gates[t, k] = softmax over the K chosen logits.
template <int KMAX>
__global__ void moe_route_kernel(const float* __restrict__ logits, int T, int E, int K,
                                 bool replay, int* __restrict__ ids, float* __restrict__ gates) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= T) return;
  const float* lrow = logits + (int64_t)warp * E;
  int sel[KMAX];
  float val[KMAX];
  if (replay) {
    for (int k = 0; k < K; ++k) {
      sel[k] = ids[(int64_t)warp * K + k];
      val[k] = lrow[sel[k]];
    }
  } else {
    // iterative arg-max over the row, K rounds
    for (int k = 0; k < K; ++k) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        bool taken = false;
        for (int j = 0; j < k; ++j) taken |= (sel[j] == e);
        const float x = lrow[e];
        if (!taken && (x > best || (x == best && e < bi))) { best = x; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffff, best, o);
        const int oi = __shfl_xor_sync(0xffffffff, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
      }
      sel[k] = bi;
      val[k] = best;
    }
  }
  if (lane == 0) {
    float m = -INFINITY;
    for (int k = 0; k < K; ++k) m = fmaxf(m, val[k]);
    float s = 0.f;
    float e[KMAX];
    for (int k = 0; k < K; ++k) { e[k] = __expf(val[k] - m); s += e[k]; }
    for (int k = 0; k < K; ++k) {
      gates[(int64_t)warp * K + k] = e[k] / s;
      if (!replay) ids[(int64_t)warp * K + k] = sel[k];
    }
  }
}

void moe_route(torch::Tensor logits, torch::Tensor ids, torch::Tensor gates, bool replay) {
  AF3_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kFloat32 && logits.is_contiguous(),
            "logits must be contiguous fp32 CUDA");
  AF3_CHECK(ids.scalar_type() == torch::kInt32 && ids.is_contiguous(), "ids must be int32");
  AF3_CHECK(gates.scalar_type() == torch::kFloat32 && gates.is_contiguous(), "gates must be fp32");
  const int T = (int)logits.size(0), E = (int)logits.size(1), K = (int)ids.size(1);
  AF3_CHECK(K >= 1 && K <= 8, "top-k must be in [1, 8]");
  const c10::cuda::CUDAGuard guard(logits.device());
  if (T == 0) return;
  const int threads = 256;
  const int grid = (T * 32 + threads - 1) / threads;
  moe_route_kernel<8><<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), T, E, K, replay, ids.data_ptr<int>(), gates.data_ptr<float>());
  AF3_CUDA_CHECK(cudaGetLastError());
}

// ------------------------- deterministic grouping by expert ---------------------------
constexpr int kChunk = 2048;
constexpr int kPad = 128;

// counts[c, e] = number of entries of chunk c routed to expert e
__global__ void moe_chunk_hist_kernel(const int* __restrict__ ids, int n, int E,
                                      int* __restrict__ counts) {
  extern __shared__ int sh[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int c = blockIdx.x;
  for (int i = c * kChunk + threadIdx.x; i < min(n, (c + 1) * kChunk); i += blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&sh[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) counts[(int64_t)c * E + e] = sh[e];
}

// Single block: per-expert exclusive scan over chunks -> chunk bases (in place), expert
// totals, 128-padded segment offsets [E+1].
__global__ void moe_scan_kernel(int* __restrict__ counts, int n_chunks, int E,
                                int* __restrict__ expert_counts, int* __restrict__ offsets) {
  extern __shared__ int tot[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int c = 0; c < n_chunks; ++c) {
      const int v = counts[(int64_t)c * E + e];
      counts[(int64_t)c * E + e] = run;
      run += v;
    }
    tot[e] = run;
    expert_counts[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = off;
      off += (tot[e] + kPad - 1) / kPad * kPad;
    }
    offsets[E] = off;
  }
}

// One warp per chunk walks it in order: stable rank within expert.
__global__ void moe_rank_kernel(const int* __restrict__ ids, int n, int E, int K,
                                const int* __restrict__ chunk_base,
                                const int* __restrict__ offsets, const float* __restrict__ gates,
                                int* __restrict__ dest, int* __restrict__ row_src,
                                float* __restrict__ row_gate) {
  extern __shared__ int run[];
  const int c = blockIdx.x;
  const int lane = threadIdx.x;
  for (int e = lane; e < E; e += 32) run[e] = chunk_base[(int64_t)c * E + e];
  __syncwarp();
  const int end = min(n, (c + 1) * kChunk);
  for (int base = c * kChunk; base < end; base += 32) {
    const int i = base + lane;
    const int e = (i < end) ? ids[i] : -1;
    const unsigned active = __ballot_sync(0xffffffff, i < end);
    const unsigned same = __match_any_sync(0xffffffff, e);
    const unsigned peers = same & active;
    const int rank = __popc(peers & ((1u << lane) - 1));
    int r0 = 0;
    if (i < end && e >= 0 && e < E) r0 = run[e];
    __syncwarp();
    if (i < end && e >= 0 && e < E) {
      const int row = offsets[e] + r0 + rank;
      dest[i] = row;
      row_src[row] = i / K;
      row_gate[row] = gates[i];
      // the highest-ranked lane of each expert group advances the running counter
      if ((peers >> lane) == 1u) run[e] = r0 + rank + 1;
    } else if (i < end) {
      dest[i] = -1;
    }
    __syncwarp();
  }
}

__global__ void fill_int_kernel(int* p, int64_t n, int v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// ids [T, K] int32, gates [T, K] fp32.  Outputs: offsets [E+1] (padded segment starts),
// expert_counts [E], dest [T*K] (row of each entry in the sorted buffer), row_src [R] (token
// of each sorted row, -1 for padding), row_gate [R].  R = capacity of the sorted buffer
// (>= T*K + E*127).  `scratch` int32 of at least n_chunks*E elements.
void moe_group(torch::Tensor ids, torch::Tensor gates, int64_t E, torch::Tensor offsets,
               torch::Tensor expert_counts, torch::Tensor dest, torch::Tensor row_src,
               torch::Tensor row_gate, torch::Tensor scratch) {
  const int n = (int)ids.numel();
  const int K = (int)ids.size(-1);
  const int n_chunks = (n + kChunk - 1) / kChunk;
  AF3_CHECK(scratch.numel() >= (int64_t)n_chunks * E, "moe_group scratch too small");
  AF3_CHECK(row_src.numel() >= (int64_t)n + E * (kPad - 1), "moe_group row capacity too small");
  AF3_CHECK(E <= 1024, "at most 1024 experts");
  const c10::cuda::CUDAGuard guard(ids.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  const int64_t R = row_src.numel();
  fill_int_kernel<<<std::min<int64_t>((R + 255) / 256, 4096), 256, 0, stream>>>(
      row_src.data_ptr<int>(), R, -1);
  AF3_CUDA_CHECK(cudaMemsetAsync(row_gate.data_ptr(), 0, R * sizeof(float), stream));
  if (n == 0) {
    AF3_CUDA_CHECK(cudaMemsetAsync(offsets.data_ptr(), 0, (E + 1) * sizeof(int), stream));
    AF3_CUDA_CHECK(cudaMemsetAsync(expert_counts.data_ptr(), 0, E * sizeof(int), stream));
    return;
  }
  moe_chunk_hist_kernel<<<n_chunks, 256, E * sizeof(int), stream>>>(ids.data_ptr<int>(), n, (int)E,
                                                                   scratch.data_ptr<int>());
  moe_scan_kernel<<<1, 256, E * sizeof(int), stream>>>(scratch.data_ptr<int>(), n_chunks, (int)E,
                                                       expert_counts.data_ptr<int>(),
                                                       offsets.data_ptr<int>());
  moe_rank_kernel<<<n_chunks, 32, E * sizeof(int), stream>>>(
      ids.data_ptr<int>(), n, (int)E, K, scratch.data_ptr<int>(), offsets.data_ptr<int>(),
      gates.data_ptr<float>(), dest.data_ptr<int>(), row_src.data_ptr<int>(),
      row_gate.data_ptr<float>());
  AF3_CUDA_CHECK(cudaGetLastError());
}

// --------------------------------- gather / combine ------------------------------------
// out[r, :] = scale[r] * x[src[r], :] (or 0 when src[r] < 0).  H multiple of 8.
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                   const int* __restrict__ src, const float* __restrict__ scale,
                                   __nv_bfloat16* __restrict__ out, int64_t ldo, int64_t R,
                                   int H, int zero_pad) {
  const int vec = H / 8;
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    const int s = src[r];
    const float sc = scale ? scale[r] : 1.f;
    uint4* o = reinterpret_cast<uint4*>(out + r * ldo);
    if (s < 0) {
      if (zero_pad)
        for (int j = threadIdx.x; j < vec; j += blockDim.x) o[j] = make_uint4(0, 0, 0, 0);
    } else {
      const uint4* xi = reinterpret_cast<const uint4*>(x + (int64_t)s * ldx);
      for (int j = threadIdx.x; j < vec; j += blockDim.x) {
        uint4 w = xi[j];
        if (scale) {
          __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float2 f = __bfloat1622float2(h[q]);
            h[q] = __floats2bfloat162_rn(f.x * sc, f.y * sc);
          }
        }
        o[j] = w;
      }
    }
  }
}

void gather_rows(torch::Tensor x, torch::Tensor src, c10::optional<torch::Tensor> scale,
                 torch::Tensor out, bool zero_pad) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(out, "out");
  const int H = (int)x.size(1);
  AF3_CHECK(H % 8 == 0 && out.size(1) == H, "gather_rows: H must match and be a multiple of 8");
  const int64_t R = src.numel();
  const c10::cuda::CUDAGuard guard(x.device());
  if (R == 0) return;
  const int grid = (int)std::min<int64_t>(R, (int64_t)num_sms() * 32);
  gather_rows_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), src.data_ptr<int>(),
      scale.has_value() ? scale->data_ptr<float>() : nullptr,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), R, H, zero_pad ? 1 : 0);
  AF3_CUDA_CHECK(cudaGetLastError());
}

// out[t, :] = sum_k y[dest[t*K + k], :] (+ residual[t, :]).  fp32 accumulation.
__global__ void combine_rows_kernel(const __nv_bfloat16* __restrict__ y, int64_t ldy,
                                    const int* __restrict__ dest, int K,
                                    const __nv_bfloat16* __restrict__ residual, int64_t ldr,
                                    __nv_bfloat16* __restrict__ out, int64_t ldo, int64_t T,
                                    int H) {
  const int vec = H / 8;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    for (int j = threadIdx.x; j < vec; j += blockDim.x) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (residual) {
        uint4 w = reinterpret_cast<const uint4*>(residual + t * ldr)[j];
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = __bfloat162float(h[q]);
      }
      for (int k = 0; k < K; ++k) {
        const int r = dest[t * K + k];
        if (r < 0) continue;
        uint4 w = reinterpret_cast<const uint4*>(y + (int64_t)r * ldy)[j];
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(h[q]);
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(out + t * ldo)[j] = o;
    }
  }
}

void combine_rows(torch::Tensor y, torch::Tensor dest, int64_t K,
                  c10::optional<torch::Tensor> residual, torch::Tensor out) {
  check_cuda_bf16(y, "y");
  check_cuda_bf16(out, "out");
  const int H = (int)out.size(1);
  AF3_CHECK(H % 8 == 0, "combine_rows: H must be a multiple of 8");
  const int64_t T = out.size(0);
  const c10::cuda::CUDAGuard guard(y.device());
  if (T == 0) return;
  const int grid = (int)std::min<int64_t>(T, (int64_t)num_sms() * 32);
  combine_rows_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), y.stride(0), dest.data_ptr<int>(),
      (int)K,
      residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr,
      residual.has_value() ? residual->stride(0) : 0,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), T, H);
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
