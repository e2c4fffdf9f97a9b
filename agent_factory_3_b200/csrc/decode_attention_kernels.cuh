// Kernels of the paged decode attention, shared by the torch entry point and the
// allocation-free C entry point.  They live in an anonymous namespace, so every file
// that includes this header compiles its own copy.
//
// Paged decode attention for the rollout engine (sm_100a): one new query token per request,
// GQA (all q heads of a kv head handled together), learned sinks, optional sliding window,
// bf16 KV in fixed-size pages.  Decode attention reads every cached key/value once per step,
// so it is bound by HBM bandwidth; the kernel streams pages with 16-byte loads and keeps the
// q-head group in shared memory.
//
// Split-KV ("flash decoding"): grid = (chunks, kv_heads, requests).  A chunk is up to
// kChunkPages pages.  Within a CTA each warp takes 32 consecutive keys at a time:
//   scores: lane j owns key j and computes the G = Hq/Hkv dot products q_h . k_j
//   softmax: per-head online max / sum over the warp's keys (warp shuffles)
//   values: lane l owns dims 2l, 2l+1 and accumulates sum_j p_hj v_j[2l..2l+1]
// Partial (m, l, o) of each warp are merged in shared memory; the CTA writes its chunk's
// partial result, and a combine kernel merges the chunks and adds the sink to the denominator.
//
// KV layout (one layer): k_pages, v_pages [num_pages, page_size, Hkv, 64] bf16;
// page_table [B, max_pages] int32; seq_lens [B] (context length including the new token).

#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace af3 {
namespace dec {
namespace {

constexpr int kD = 64;
constexpr int kWarps = 4;
constexpr int kMaxG = 16;  // q heads per kv head
constexpr int kChunkPages = 16;

struct Params {
  const __nv_bfloat16* q;      // [B, Hq, 64] (ld_q elements between requests)
  int64_t ld_q;
  const __nv_bfloat16* kp;     // [pages, page_size, Hkv, 64]
  const __nv_bfloat16* vp;
  const int* page_table;       // [B, max_pages]
  int max_pages;
  const int* seq_lens;         // [B]
  float* part_o;               // [B, Hq, chunks, 64]
  float* part_ml;              // [B, Hq, chunks, 2]
  int page_size, hq, hkv, window, chunks;
  float scale_log2;
};

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int G>
__global__ void __launch_bounds__(kWarps * 32) decode_attn_kernel(const Params p) {
  const int chunk = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int L = p.seq_lens[b];
  const int pos = L - 1;  // position of the query token
  int k_lo = 0;
  if (p.window > 0) k_lo = max(0, pos - p.window + 1);
  const int tokens_per_chunk = kChunkPages * p.page_size;
  const int c_lo = max(k_lo, chunk * tokens_per_chunk);
  const int c_hi = min(L, (chunk + 1) * tokens_per_chunk);

  __shared__ float sq[G][kD];
  __shared__ float s_m[kWarps][G], s_l[kWarps][G];
  __shared__ float s_o[kWarps][G][kD];
  const __nv_bfloat16* qb = p.q + (int64_t)b * p.ld_q + (int64_t)g * G * kD;
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x)
    sq[i / kD][i % kD] = __bfloat162float(qb[i]) * p.scale_log2;
  __syncthreads();

  float m[G], l[G], o0[G], o1[G];
#pragma unroll
  for (int h = 0; h < G; ++h) { m[h] = -INFINITY; l[h] = 0.f; o0[h] = 0.f; o1[h] = 0.f; }
  const int* pt = p.page_table + (int64_t)b * p.max_pages;
  const int64_t tok_stride = (int64_t)p.hkv * kD;  // elements between tokens of a page

  for (int base = c_lo + warp * 32; base < c_hi; base += kWarps * 32) {
    const int kj = base + lane;
    const bool valid = kj < c_hi;
    float s[G];
    if (valid) {
      const int page = pt[kj / p.page_size];
      const __nv_bfloat16* krow = p.kp + ((int64_t)page * p.page_size + kj % p.page_size) * tok_stride + g * kD;
#pragma unroll
      for (int h = 0; h < G; ++h) s[h] = 0.f;
#pragma unroll
      for (int c = 0; c < kD / 8; ++c) {
        const uint4 w = reinterpret_cast<const uint4*>(krow)[c];
        const __nv_bfloat162* kv = reinterpret_cast<const __nv_bfloat162*>(&w);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(kv[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
#pragma unroll
          for (int e = 0; e < 8; ++e) s[h] = fmaf(sq[h][c * 8 + e], kf[e], s[h]);
        }
      }
    } else {
#pragma unroll
      for (int h = 0; h < G; ++h) s[h] = -INFINITY;
    }
    // online softmax per head over the warp's 32 keys
    float pr[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float mx = s[h];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
      const float mn = fmaxf(m[h], mx);
      const float mu = (mn == -INFINITY) ? 0.f : mn;
      const float a = ex2f(m[h] - mu);
      pr[h] = ex2f(s[h] - mu);
      float sum = pr[h];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffff, sum, o);
      l[h] = l[h] * a + sum;
      o0[h] *= a;
      o1[h] *= a;
      m[h] = mn;
    }
    // values: lane owns dims 2*lane, 2*lane+1.  The lane's words of all 32 keys are loaded
    // first (independent loads in flight together), then consumed from registers; the 32 keys
    // span at most two pages when a page holds >= 32 tokens.
    const int nk = min(32, c_hi - base);
    __nv_bfloat162 vreg[32];
    {
      const int pa = pt[base / p.page_size];
      const int pb = pt[min(base + 31, c_hi - 1) / p.page_size];
      const int first_page = base / p.page_size;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int kk = base + j;
        if (j < nk) {
          const int page = p.page_size >= 32 ? ((kk / p.page_size == first_page) ? pa : pb)
                                              : pt[kk / p.page_size];
          vreg[j] = reinterpret_cast<const __nv_bfloat162*>(
              p.vp + ((int64_t)page * p.page_size + kk % p.page_size) * tok_stride + g * kD)[lane];
        } else {
          vreg[j] = __floats2bfloat162_rn(0.f, 0.f);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j >= nk) break;
      const float2 vf = __bfloat1622float2(vreg[j]);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float ph = __shfl_sync(0xffffffff, pr[h], j);
        o0[h] = fmaf(ph, vf.x, o0[h]);
        o1[h] = fmaf(ph, vf.y, o1[h]);
      }
    }
  }
  // merge warps
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) { s_m[warp][h] = m[h]; s_l[warp][h] = l[h]; }
  }
#pragma unroll
  for (int h = 0; h < G; ++h) {
    s_o[warp][h][2 * lane] = o0[h];
    s_o[warp][h][2 * lane + 1] = o1[h];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int h = i / kD, d = i % kD;
    float mm = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, s_m[w][h]);
    const float mu = (mm == -INFINITY) ? 0.f : mm;
    float ll = 0.f, oo = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float a = ex2f(s_m[w][h] - mu);
      ll += s_l[w][h] * a;
      oo += s_o[w][h][d] * a;
    }
    const int hq = g * G + h;
    const int64_t idx = ((int64_t)b * p.hq + hq) * p.chunks + chunk;
    p.part_o[idx * kD + d] = oo;
    if (d == 0) {
      p.part_ml[idx * 2] = mm;
      p.part_ml[idx * 2 + 1] = ll;
    }
  }
}

// out[b, h] = sum_c o_c * 2^(m_c - M) / (sum_c l_c 2^(m_c - M) + 2^(sink*log2e - M))
__global__ void decode_combine_kernel(const float* __restrict__ part_o,
                                      const float* __restrict__ part_ml,
                                      const float* __restrict__ sinks, __nv_bfloat16* __restrict__ out,
                                      int64_t ld_out, int hq, int chunks, float* __restrict__ lse) {
  const int b = blockIdx.y, h = blockIdx.x, d = threadIdx.x;
  const int64_t base = ((int64_t)b * hq + h) * chunks;
  float M = sinks[h] * 1.4426950408889634f;
  for (int c = 0; c < chunks; ++c) M = fmaxf(M, part_ml[(base + c) * 2]);
  float den = ex2f(sinks[h] * 1.4426950408889634f - M), num = 0.f;
  for (int c = 0; c < chunks; ++c) {
    const float mc = part_ml[(base + c) * 2];
    if (mc == -INFINITY) continue;
    const float a = ex2f(mc - M);
    den += part_ml[(base + c) * 2 + 1] * a;
    num += part_o[(base + c) * kD + d] * a;
  }
  out[(int64_t)b * ld_out + h * kD + d] = __float2bfloat16(num / den);
  if (lse != nullptr && d == 0) lse[(int64_t)b * hq + h] = (M + __log2f(den)) * 0.6931471805599453f;
}

}  // namespace
}  // namespace dec
}  // namespace af3
