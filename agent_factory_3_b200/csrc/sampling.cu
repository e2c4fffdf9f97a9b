// Token sampling for the rollout engine (sm_100a), one CTA per request row of fp32 logits:
//   z = logits / temperature;  p = softmax(z)
//   token  = argmax_v (z_v + Gumbel_v)      (exact sampling from p: the Gumbel-max trick)
//            restricted to v with p_v >= min_p * p_max when min_p > 0
//   logprob = z_token - log sum exp z,  entropy = log sum exp z - E_p[z]
// temperature == 0 selects the argmax.  Gumbel noise comes from a counter-based hash of
// (seed, step, row, v) (SplitMix64 finaliser), so a request with a fixed sampling seed is
// reproducible.  Top-k / top-p truncation (which need a sort) is done by the caller.
#include "common.h"
#include "host_utils.h"

namespace af3 {

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__device__ __forceinline__ float uniform01(uint64_t h) {
  // 24 random bits -> (0, 1)
  return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

constexpr int kSampThreads = 1024;

template <typename T>
__device__ __forceinline__ T block_reduce(T v, T* sh, bool is_max) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    T w = __shfl_xor_sync(0xffffffff, v, o);
    v = is_max ? (w > v ? w : v) : v + w;
  }
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x / 32) ? sh[lane] : (is_max ? (T)-INFINITY : (T)0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      T w = __shfl_xor_sync(0xffffffff, v, o);
      v = is_max ? (w > v ? w : v) : v + w;
    }
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  T r = sh[0];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kSampThreads)
    sample_kernel(const float* __restrict__ logits, int64_t ld, int V,
                  const float* __restrict__ temperature, const float* __restrict__ min_p,
                  const int64_t* __restrict__ seeds, int64_t step, int* __restrict__ tokens,
                  float* __restrict__ logprobs, float* __restrict__ entropy) {
  __shared__ float shf[32];
  __shared__ float sbest[32];
  __shared__ int sidx[32];
  const int row = blockIdx.x;
  const float* z = logits + (int64_t)row * ld;
  const float T = temperature[row];
  const bool greedy = !(T > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / T;
  float mx = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) mx = fmaxf(mx, z[v] * inv_t);
  mx = block_reduce<float>(mx, shf, true);
  float se = 0.f, sze = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float zz = z[v] * inv_t;
    const float e = __expf(zz - mx);
    se += e;
    sze += e * zz;
  }
  se = block_reduce<float>(se, shf, false);
  sze = block_reduce<float>(sze, shf, false);
  const float logZ = mx + __logf(se);
  const float mp = min_p ? min_p[row] : 0.f;
  const float thresh = (mp > 0.f) ? mx + __logf(mp) : -INFINITY;  // p_v >= min_p * p_max
  const uint64_t key = mix64((uint64_t)seeds[row] ^ mix64((uint64_t)step * 0x100000001B3ull + row));
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float zz = z[v] * inv_t;
    if (zz < thresh) continue;
    float score = zz;
    if (!greedy) {
      const float u = uniform01(mix64(key + (uint64_t)v));
      score = zz - __logf(-__logf(u));  // + Gumbel(0, 1)
    }
    if (score > best || (score == best && v < bi)) { best = score; bi = v; }
  }
  // block argmax
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffff, best, o);
    const int oi = __shfl_xor_sync(0xffffffff, bi, o);
    if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
  }
  if (lane == 0) { sbest[warp] = best; sidx[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x / 32); ++w)
      if (sbest[w] > best || (sbest[w] == best && sidx[w] < bi)) { best = sbest[w]; bi = sidx[w]; }
    tokens[row] = bi;
    logprobs[row] = z[bi] * inv_t - logZ;
    entropy[row] = logZ - sze / se;
  }
}

void sample_tokens(torch::Tensor logits, torch::Tensor temperature, c10::optional<torch::Tensor> min_p,
                   torch::Tensor seeds, int64_t step, torch::Tensor tokens, torch::Tensor logprobs,
                   torch::Tensor entropy) {
  AF3_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kFloat32 && logits.stride(1) == 1,
            "logits must be fp32 CUDA with unit inner stride");
  const int B = (int)logits.size(0);
  const c10::cuda::CUDAGuard guard(logits.device());
  if (B == 0) return;
  sample_kernel<<<B, kSampThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.stride(0), (int)logits.size(1), temperature.data_ptr<float>(),
      min_p.has_value() ? min_p->data_ptr<float>() : nullptr, seeds.data_ptr<int64_t>(), step,
      tokens.data_ptr<int>(), logprobs.data_ptr<float>(), entropy.data_ptr<float>());
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
