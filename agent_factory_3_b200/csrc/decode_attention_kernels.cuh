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

// ---------------------------------------------------------------------------------------
// Tensor-core variant for 8 q heads per kv head (gpt-oss): mma.sync m16n8k16 (bf16 in, fp32
// accumulate) with the head group as the M rows (rows 8-15 of the fragment stay zero).  Per warp
// and 32 keys: S = Q K^T is 4 key tiles x 4 head-dim steps = 16 MMAs, P V is 2 key steps x 8
// output-dim tiles = 16 MMAs, against ~3700 FMA instructions in the CUDA-core kernel above.
// Two consistent index permutations keep every load a contiguous 16 bytes:
//   * head dim in S: thread (group g, lane-in-group t) feeds k-step s with dims 16t + 4s + {0,1}
//     (fragment k = 2t, 2t+1) and 16t + 4s + {2,3} (k = 2t + 8, 2t + 9) of Q and of K, so it
//     loads dims [16t, 16t + 16) of its query row and of its key row;
//   * output dim in P V: column n of output tile i is dim 8n + i, so the B fragment of thread
//     (g, t) needs dims [8g, 8g + 8) of four value rows, and the thread's outputs are dims
//     16t + i and 16t + 8 + i.
// P reuses the S accumulator layout as the A operand (keys 16s + 2t + {0,1}, 16s + 8 + 2t + {0,1}).
__device__ __forceinline__ void mma_16816_bf16(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                               uint32_t b1) {
  // A rows 8-15 are zero: registers 1 and 3 of the A fragment are 0
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__global__ void __launch_bounds__(kWarps * 32) decode_attn_mma_kernel(const Params p) {
  constexpr int G = 8;
  const int chunk = blockIdx.x, gh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int grp = lane >> 2, tig = lane & 3;
  const int L = p.seq_lens[b];
  const int pos = L - 1;
  int k_lo = 0;
  if (p.window > 0) k_lo = max(0, pos - p.window + 1);
  const int tokens_per_chunk = kChunkPages * p.page_size;
  const int c_lo = max(k_lo, chunk * tokens_per_chunk);
  const int c_hi = min(L, (chunk + 1) * tokens_per_chunk);

  __shared__ float s_m[kWarps][G], s_l[kWarps][G];
  __shared__ float s_o[kWarps][G][kD];
  // query row grp of the group, dims [16 tig, 16 tig + 16)
  const uint4* qrow = reinterpret_cast<const uint4*>(
      p.q + (int64_t)b * p.ld_q + (int64_t)(gh * G + grp) * kD + 16 * tig);
  const uint4 qa = __ldg(qrow), qb = __ldg(qrow + 1);
  const uint32_t qr[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  float m = -INFINITY, l = 0.f;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const int* pt = p.page_table + (int64_t)b * p.max_pages;
  const int64_t tok_stride = (int64_t)p.hkv * kD;

  for (int base = c_lo + warp * 32; base < c_hi; base += kWarps * 32) {
    const int first = base / p.page_size;
    const int pa = pt[first];
    const int pb = pt[min(base + 31, c_hi - 1) / p.page_size];
    auto row = [&](const __nv_bfloat16* pages, int key) {
      const int kk = min(key, c_hi - 1);                      // clamp: masked below
      const int page = p.page_size >= 32 ? (kk / p.page_size == first ? pa : pb)
                                         : pt[kk / p.page_size];
      return pages + ((int64_t)page * p.page_size + kk % p.page_size) * tok_stride + gh * kD;
    };
    // ---- S = Q K^T for keys base + 8j + grp (B column = grp)
    float sacc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4* kr = reinterpret_cast<const uint4*>(row(p.kp, base + 8 * j + grp) + 16 * tig);
      const uint4 k0 = __ldg(kr), k1 = __ldg(kr + 1);
      const uint32_t kw[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
      sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
      for (int s = 0; s < 4; ++s) mma_16816_bf16(sacc[j], qr[2 * s], qr[2 * s + 1], kw[2 * s], kw[2 * s + 1]);
    }
    // ---- online softmax of head grp over keys base + 8j + 2 tig + e
    float sc[8];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = base + 8 * j + 2 * tig + e;
        sc[2 * j + e] = key < c_hi ? sacc[j][e] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, sc[2 * j + e]);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m, mx);
    const float mu = (mn == -INFINITY) ? 0.f : mn;
    const float a = ex2f(m - mu);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      sc[k] = ex2f(sc[k] - mu);
      sum += sc[k];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l = l * a + sum;
    m = mn;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= a;
      o[i][1] *= a;
    }
    // ---- O += P V, key steps of 16
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const uint32_t pa0 = pack2_bf16(sc[4 * t], sc[4 * t + 1]);
      const uint32_t pa2 = pack2_bf16(sc[4 * t + 2], sc[4 * t + 3]);
      const int k0 = base + 16 * t + 2 * tig;
      const uint4 va0 = __ldg(reinterpret_cast<const uint4*>(row(p.vp, k0) + 8 * grp));
      const uint4 va1 = __ldg(reinterpret_cast<const uint4*>(row(p.vp, k0 + 1) + 8 * grp));
      const uint4 vb0 = __ldg(reinterpret_cast<const uint4*>(row(p.vp, k0 + 8) + 8 * grp));
      const uint4 vb1 = __ldg(reinterpret_cast<const uint4*>(row(p.vp, k0 + 9) + 8 * grp));
      const uint32_t wa0[4] = {va0.x, va0.y, va0.z, va0.w}, wa1[4] = {va1.x, va1.y, va1.z, va1.w};
      const uint32_t wb0[4] = {vb0.x, vb0.y, vb0.z, vb0.w}, wb1[4] = {vb1.x, vb1.y, vb1.z, vb1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;    // high or low bf16 of each word
        const uint32_t b0 = __byte_perm(wa0[i >> 1], wa1[i >> 1], sel);
        const uint32_t b1 = __byte_perm(wb0[i >> 1], wb1[i >> 1], sel);
        mma_16816_bf16(o[i], pa0, pa2, b0, b1);
      }
    }
  }
  // merge warps (thread (grp, tig) holds dims 16 tig + i and 16 tig + 8 + i of head grp)
  if (tig == 0) {
    s_m[warp][grp] = m;
    s_l[warp][grp] = l;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s_o[warp][grp][16 * tig + i] = o[i][0];
    s_o[warp][grp][16 * tig + 8 + i] = o[i][1];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * kD; i += blockDim.x) {
    const int h = i / kD, d = i % kD;
    float mm = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, s_m[w][h]);
    const float mu2 = (mm == -INFINITY) ? 0.f : mm;
    float ll = 0.f, oo = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float a2 = ex2f(s_m[w][h] - mu2);
      ll += s_l[w][h] * a2;
      oo += s_o[w][h][d] * a2;
    }
    const int hq = gh * G + h;
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
