// Persistent warp-specialized tcgen05 GEMM for sm_100a.
//
//   C[M, N] = epilogue( A[M, K] * B[N, K]^T )      bf16 inputs, fp32 TMEM accumulation
//
// * A is K-major ([M, K] row-major) or MN-major ([K, M] row-major); B is K-major ([N, K])
//   or MN-major ([K, N]).  Operands are staged by TMA with 128-byte swizzle.
// * Grouped ("ragged M") mode: rows are split into G segments whose starts are multiples of
//   128 (expert segments of a routed MoE batch, padded on the device).  Segment g multiplies
//   by B[g] (a 3-D tensor map over [G, N, K] or [G, K, N]).  The tile list is derived on the
//   device from the segment offsets, so no host synchronisation is needed.
// * Grouped-K mode: the reduction runs over segment g's rows only and the output is C[g]
//   (weight gradients of per-expert LoRA factors).
// * FP8 variant (template flag F8): A and B are e4m3 bytes, K-major, and the MMA runs as
//   tcgen05 kind::f8f6f4 (32 K elements per instruction, twice the bf16 rate).  A stage still
//   holds 128-byte rows, now 128 K elements, so tiles, swizzle and descriptors are unchanged.
//   The epilogue multiplies the accumulator by a per-row scale of A (per-token quantisation)
//   and a per-group scale of B (per-expert weight scale) before everything else.
//
// Warp roles (256 threads): warp 0 = TMA producer, warp 1 = MMA issuer (one elected
// thread), warp 2 = TMEM allocator, warps 4..7 = epilogue (thread t owns accumulator row t;
// TMEM lane quarter = warp % 4).  The accumulator is double buffered in TMEM so the
// epilogue of tile i overlaps the main loop of tile i+1.
#pragma once
#include "sm100.cuh"

namespace af3 {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kGemmThreads = 256;
constexpr int kMaxGroups = 512;

enum SchedMode : int { kSchedPlain = 0, kSchedGroupedM = 1, kSchedGroupedK = 2 };

enum EpiKind : int {
  kEpiBf16 = 0,       // out_bf16 = alpha*acc + bias (+ residual aux)
  kEpiF32 = 1,        // out_f32 = alpha*acc + bias  (beta: += existing)
  kEpiSwiglu = 2,     // interleaved gate/up -> clamped SwiGLU (bf16 [M, N/2]); raw -> out2
  kEpiRowScale = 3,   // out_bf16 = row_scale[row] * (alpha*acc + bias)
  kEpiSwigluBwd = 4,  // acc = dL/dh; aux = raw gate_up -> out = dL/d(gate_up) (bf16 [M, 2N])
  kEpiLse = 5,        // per-row online log-sum-exp partials over this N tile (fused logprob)
  kEpiLogprobBwd = 6, // out_bf16 = dL/dlogits for this vocab chunk (fused logprob backward)
};

struct GemmArgs {
  int M, N, K;
  int K2;                    // dual-operand mode: extra reduction over (A2, B2), 0 = off
  int num_groups;
  const int* group_offsets;  // [G+1] (grouped modes)
  int band;                  // raster band (M tiles) for L2 reuse
  // epilogue
  void* out;
  int64_t ldo;
  int64_t out_group_stride;  // grouped-K: elements between C[g] and C[g+1]
  const float* bias;         // [G, N] fp32 or null
  int64_t bias_group_stride;
  const float* row_scale;    // [M] fp32 or null
  const __nv_bfloat16* aux;  // residual (kEpiBf16) or raw gate_up (kEpiSwigluBwd)
  int64_t ld_aux;
  void* out2;                // raw gate_up (kEpiSwiglu), optional
  int64_t ldo2;
  float alpha;
  float beta;                // kEpiF32: out = beta*out + ...
  float act_alpha, act_limit;
  // fused logprob (kEpiLse / kEpiLogprobBwd)
  const int* labels;         // [M] label ids (absolute vocabulary ids)
  int vocab_offset;          // vocabulary id of column 0 of this GEMM
  float* lse_part;           // [M, n_tiles, 3] (max, sumexp, sum z*exp) per tile
  float* label_logit;        // [M]
  const float* row_stats;    // backward: [M, 4] = (logZ, H, g_logprob, g_entropy)
  int n_tiles_total;
  int* err;                  // device error word
  // FP8 dequantisation scales (either may be null) and an optional bf16 term added to the
  // scaled accumulator before bias and epilogue (a second GEMM's result, e.g. the base output
  // of an FP8 pass under a bf16 LoRA pass)
  const float* a_scale;      // [M] per row of A
  const float* b_scale;      // [G] per group (per expert) of B
  const __nv_bfloat16* acc_add;
  int64_t ld_acc_add;
  int kx_shift;              // K-major x coordinate = k >> kx_shift (FP8 bytes described as
                             // 16-bit elements to the TMA unit: 1)
};

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 256) ? 4 : (BN >= 192 ? 5 : 6);
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = 1024 /*align*/ + STAGES * STAGE_BYTES + 1024 /*barriers*/ +
                                    (kMaxGroups + 2) * 4;
};

struct TileCoord {
  int g, m0, n0, k_begin, k_end;
};

// Tile enumeration shared by the producer, the MMA issuer and the epilogue.
// s_prefix[g] = number of tiles before group g (grouped modes).
template <int SCHED>
__device__ __forceinline__ bool get_tile(int t, const GemmArgs& a, int BN, const int* s_prefix,
                                         TileCoord& tc) {
  const int n_tiles = (a.N + BN - 1) / BN;
  if (SCHED == kSchedPlain) {
    const int m_tiles = (a.M + kBM - 1) / kBM;
    if (t >= m_tiles * n_tiles) return false;
    // banded raster: within a band of `band` M tiles, M varies fastest
    const int band = a.band;
    const int per_band = band * n_tiles;
    const int b = t / per_band;
    const int r = t - b * per_band;
    const int mb0 = b * band;
    const int bm = min(band, m_tiles - mb0);
    tc.g = 0;
    tc.m0 = (mb0 + r % bm) * kBM;
    tc.n0 = (r / bm) * BN;
    tc.k_begin = 0;
    tc.k_end = a.K;
    return true;
  }
  // grouped: binary search the prefix
  const int G = a.num_groups;
  if (t >= s_prefix[G]) return false;
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (s_prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int g = lo;
  const int local = t - s_prefix[g];
  tc.g = g;
  if (SCHED == kSchedGroupedK) {
    // grouped-K: tiles of the [M, N] output of group g; reduction over its rows
    const int m_tiles = (a.M + kBM - 1) / kBM;
    tc.m0 = (local % m_tiles) * kBM;
    tc.n0 = (local / m_tiles) * BN;
    tc.k_begin = a.group_offsets[g];
    tc.k_end = a.group_offsets[g + 1];
  } else {
    const int row0 = a.group_offsets[g];
    const int rows = a.group_offsets[g + 1] - row0;
    const int m_tiles = (rows + kBM - 1) / kBM;
    const int band = a.band;
    const int per_band = band * n_tiles;
    const int b = local / per_band;
    const int r = local - b * per_band;
    const int mb0 = b * band;
    const int bm = min(band, m_tiles - mb0);
    tc.m0 = row0 + (mb0 + r % bm) * kBM;
    tc.n0 = (r / bm) * BN;
    tc.k_begin = 0;
    tc.k_end = a.K;
  }
  return true;
}

// sigmoid through the fast reciprocal (__fdividef): the IEEE division would cost a
// multi-instruction sequence per element in the epilogue, which for e4m3 tiles (half the
// main-loop time of bf16) otherwise becomes the limiter
__device__ __forceinline__ float silu_clamped_fwd(float g, float u, float alpha, float limit) {
  const float gc = fminf(g, limit);
  const float uc = fminf(fmaxf(u, -limit), limit);
  const float s = __fdividef(1.0f, 1.0f + __expf(-alpha * gc));
  return gc * s * (uc + 1.0f);
}

__device__ __forceinline__ void silu_clamped_bwd(float dout, float g, float u, float alpha,
                                                 float limit, float& dg, float& du) {
  const float gc = fminf(g, limit);
  const float uc = fminf(fmaxf(u, -limit), limit);
  const float s = __fdividef(1.0f, 1.0f + __expf(-alpha * gc));
  const float glu = gc * s;
  du = (u >= -limit && u <= limit) ? dout * glu : 0.0f;
  const float dglu = dout * (uc + 1.0f);
  dg = (g <= limit) ? dglu * (s + gc * alpha * s * (1.0f - s)) : 0.0f;
}

// Epilogue state for the fused log-sum-exp (kept per thread = per row across chunks).
struct LseState {
  float m, s, t;
};

template <int EPI>
__device__ __forceinline__ void epi_chunk(const GemmArgs& a, int row, bool row_ok, int g,
                                          int col0, const uint32_t (&r)[32], LseState& st) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * a.alpha;
  const bool full = (col0 + 32 <= a.N);
  if (EPI == kEpiLse) {
    if (!row_ok) return;
    float cm = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full || col0 + j < a.N) cm = fmaxf(cm, v[j]);
    if (cm == -INFINITY) return;
    const float nm = fmaxf(st.m, cm);
    const float sc = (st.m == -INFINITY) ? 0.f : __expf(st.m - nm);
    float s = st.s * sc, t = st.t * sc;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (full || col0 + j < a.N) {
        const float e = __expf(v[j] - nm);
        s += e;
        t += e * v[j];
      }
    }
    st.m = nm; st.s = s; st.t = t;
    const int lab = a.labels[row] - a.vocab_offset;
    if (lab >= col0 && lab < col0 + 32 && lab < a.N) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j == lab - col0) a.label_logit[row] = v[j];
    }
    return;
  }
  if (!row_ok) return;
  if (a.a_scale != nullptr || a.b_scale != nullptr) {
    const float sc = (a.a_scale != nullptr ? a.a_scale[row] : 1.f) *
                     (a.b_scale != nullptr ? a.b_scale[g] : 1.f);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] *= sc;
  }
  if (a.acc_add != nullptr) {
    const __nv_bfloat16* ap = a.acc_add + (int64_t)row * a.ld_acc_add + col0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w = *reinterpret_cast<const uint4*>(ap + q * 8);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[q * 8 + e] += __bfloat162float(h[e]);
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < a.N) v[j] += __bfloat162float(ap[j]);
    }
  }
  if (a.bias != nullptr) {
    const float* bp = a.bias + (int64_t)g * a.bias_group_stride + col0;
    if (full && (reinterpret_cast<uintptr_t>(bp) & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(bp) + q);
        v[4 * q] += b4.x;
        v[4 * q + 1] += b4.y;
        v[4 * q + 2] += b4.z;
        v[4 * q + 3] += b4.w;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < a.N) v[j] += bp[j];
    }
  }
  if (EPI == kEpiBf16 || EPI == kEpiRowScale) {
    if (EPI == kEpiRowScale) {
      const float sc = a.row_scale[row];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= sc;
    }
    if (a.aux != nullptr) {
      const __nv_bfloat16* ap = a.aux + (int64_t)row * a.ld_aux + col0;
      if (full) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w = *reinterpret_cast<const uint4*>(ap + q * 8);
          const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[q * 8 + e] += __bfloat162float(h[e]);
        }
      } else {
        for (int j = 0; j < 32; ++j)
          if (col0 + j < a.N) v[j] += __bfloat162float(ap[j]);
      }
    }
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)row * a.ldo + col0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
        w.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
        w.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
        w.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
        *reinterpret_cast<uint4*>(op + q * 8) = w;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < a.N) op[j] = __float2bfloat16(v[j]);
    }
  } else if (EPI == kEpiF32) {
    float* op = reinterpret_cast<float*>(a.out) + (int64_t)g * a.out_group_stride +
                (int64_t)row * a.ldo + col0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 w = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
        if (a.beta != 0.f) {
          float4 o = *reinterpret_cast<float4*>(op + q * 4);
          w.x += a.beta * o.x; w.y += a.beta * o.y; w.z += a.beta * o.z; w.w += a.beta * o.w;
        }
        *reinterpret_cast<float4*>(op + q * 4) = w;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < a.N) op[j] = v[j] + (a.beta != 0.f ? a.beta * op[j] : 0.f);
    }
  } else if (EPI == kEpiSwiglu) {
    // columns (2j, 2j+1) = (gate, up); output column col0/2 + j
    if (a.out2 != nullptr) {
      __nv_bfloat16* rp =
          reinterpret_cast<__nv_bfloat16*>(a.out2) + (int64_t)row * a.ldo2 + col0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
        w.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
        w.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
        w.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
        *reinterpret_cast<uint4*>(rp + q * 8) = w;
      }
    }
    float h[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      // round to bf16 first so forward and recomputation see the stored values
      const float gq = __bfloat162float(__float2bfloat16(v[2 * j]));
      const float uq = __bfloat162float(__float2bfloat16(v[2 * j + 1]));
      h[j] = silu_clamped_fwd(gq, uq, a.act_alpha, a.act_limit);
    }
    __nv_bfloat16* op =
        reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)row * a.ldo + col0 / 2;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint4 w;
      w.x = pack_bf16x2(h[q * 8 + 0], h[q * 8 + 1]);
      w.y = pack_bf16x2(h[q * 8 + 2], h[q * 8 + 3]);
      w.z = pack_bf16x2(h[q * 8 + 4], h[q * 8 + 5]);
      w.w = pack_bf16x2(h[q * 8 + 6], h[q * 8 + 7]);
      *reinterpret_cast<uint4*>(op + q * 8) = w;
    }
  } else if (EPI == kEpiSwigluBwd) {
    // v[j] = dL/dh[row, col0+j]; aux = raw gate_up [row, 2*(col0+j) + {0,1}]
    const __nv_bfloat16* ap = a.aux + (int64_t)row * a.ld_aux + 2 * col0;
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)row * a.ldo + 2 * col0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint4 w = *reinterpret_cast<const uint4*>(ap + q * 8);
      const __nv_bfloat16* hh = reinterpret_cast<const __nv_bfloat16*>(&w);
      float d[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        silu_clamped_bwd(v[q * 4 + e], __bfloat162float(hh[2 * e]),
                         __bfloat162float(hh[2 * e + 1]), a.act_alpha, a.act_limit, d[2 * e],
                         d[2 * e + 1]);
      }
      uint4 o;
      o.x = pack_bf16x2(d[0], d[1]);
      o.y = pack_bf16x2(d[2], d[3]);
      o.z = pack_bf16x2(d[4], d[5]);
      o.w = pack_bf16x2(d[6], d[7]);
      *reinterpret_cast<uint4*>(op + q * 8) = o;
    }
  } else if (EPI == kEpiLogprobBwd) {
    // z = alpha*acc (alpha = 1/temperature); p = exp(z - logZ)
    // dz = g_lp*(1[v==y] - p) - g_H*p*(z - logZ + H);  dlogits = dz*alpha
    const float logZ = a.row_stats[row * 4 + 0];
    const float H = a.row_stats[row * 4 + 1];
    const float glp = a.row_stats[row * 4 + 2];
    const float gh = a.row_stats[row * 4 + 3];
    const int lab = a.labels[row] - a.vocab_offset;
    float d[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float p = __expf(v[j] - logZ);
      float dz = -glp * p - gh * p * (v[j] - logZ + H);
      if (col0 + j == lab) dz += glp;
      d[j] = (full || col0 + j < a.N) ? dz * a.alpha : 0.f;
    }
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(a.out) + (int64_t)row * a.ldo + col0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(d[q * 8 + 0], d[q * 8 + 1]);
        w.y = pack_bf16x2(d[q * 8 + 2], d[q * 8 + 3]);
        w.z = pack_bf16x2(d[q * 8 + 4], d[q * 8 + 5]);
        w.w = pack_bf16x2(d[q * 8 + 6], d[q * 8 + 7]);
        *reinterpret_cast<uint4*>(op + q * 8) = w;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < a.N) op[j] = __float2bfloat16(d[j]);
    }
  }
}

// DUAL: after the main K loop, K2 more columns are reduced from a second operand pair
// (A2, B2) with the same majors -- e.g. the LoRA branch [x | s*x*A^T] x [W | B]^T of a
// LoRA-adapted linear layer runs as one GEMM.
template <int BN, bool A_MN, bool B_MN, bool B_3D, int SCHED, int EPI, bool DUAL, bool F8 = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tma_a,
                      const __grid_constant__ CUtensorMap tma_b,
                      const __grid_constant__ CUtensorMap tma_a2,
                      const __grid_constant__ CUtensorMap tma_b2, const GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  static_assert(!F8 || (!A_MN && !B_MN && !DUAL), "FP8 operands are K-major, single pair");
  constexpr int KB = F8 ? 128 : kBK;   // K elements per stage (128 bytes per row either way)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* s_prefix = reinterpret_cast<int*>(smem + STAGES * Cfg::STAGE_BYTES + 1024);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  // ---- setup -------------------------------------------------------------------------
  const bool grouped = (SCHED != kSchedPlain);
  if (grouped) {
    // tiles per group -> prefix (one warp; G <= kMaxGroups)
    const int n_tiles = (args.N + BN - 1) / BN;
    if (warp == 3) {
      int carry = 0;
      for (int base = 0; base < args.num_groups; base += 32) {
        const int g = base + lane;
        int cnt = 0;
        if (g < args.num_groups) {
          if (SCHED == kSchedGroupedK) {
            const int m_tiles = (args.M + kBM - 1) / kBM;
            const int kr = args.group_offsets[g + 1] - args.group_offsets[g];
            cnt = kr > 0 ? m_tiles * n_tiles : 0;
          } else {
            const int rows = args.group_offsets[g + 1] - args.group_offsets[g];
            cnt = ((rows + kBM - 1) / kBM) * n_tiles;
          }
        }
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          int y = __shfl_up_sync(0xffffffff, incl, o);
          if (lane >= o) incl += y;
        }
        if (g < args.num_groups) s_prefix[g] = carry + incl - cnt;
        carry += __shfl_sync(0xffffffff, incl, 31);
      }
      if (lane == 0) s_prefix[args.num_groups] = carry;
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    if (DUAL) {
      tma_prefetch_desc(&tma_a2);
      tma_prefetch_desc(&tma_b2);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int* prefix = grouped ? s_prefix : nullptr;

  if (warp == 0) {
    // ================================ TMA producer ====================================
    if (elect_one_sync()) {
      int stage = 0;
      uint32_t phase = 0;
      TileCoord tc;
      for (int t = blockIdx.x; get_tile<SCHED>(t, args, BN, prefix, tc); t += gridDim.x) {
        const int nk1 = (tc.k_end - tc.k_begin + KB - 1) / KB;
        const int nk = nk1 + (DUAL ? (args.K2 + kBK - 1) / kBK : 0);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, args.err, abort_flag)) goto producer_done;
          uint8_t* sa = tiles + stage * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          const bool second = DUAL && kb >= nk1;
          const CUtensorMap* ma = second ? &tma_a2 : &tma_a;
          const CUtensorMap* mb = second ? &tma_b2 : &tma_b;
          const int k = second ? (kb - nk1) * kBK : tc.k_begin + kb * KB;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          const int kx = F8 ? (k >> args.kx_shift) : k;
          if (!A_MN) {
            tma_load_2d(sa, ma, &full_bar[stage], kx, tc.m0);
          } else {
#pragma unroll
            for (int c = 0; c < kBM / 64; ++c)
              tma_load_2d(sa + c * 8192, ma, &full_bar[stage], tc.m0 + c * 64, k);
          }
          if (!B_MN) {
            if (B_3D) tma_load_3d(sb, mb, &full_bar[stage], kx, tc.n0, tc.g);
            else tma_load_2d(sb, mb, &full_bar[stage], kx, tc.n0);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) {
              if (B_3D) tma_load_3d(sb + c * 8192, mb, &full_bar[stage], tc.n0 + c * 64, k, tc.g);
              else tma_load_2d(sb + c * 8192, mb, &full_bar[stage], tc.n0 + c * 64, k);
            }
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ================================ MMA issuer ======================================
    if (elect_one_sync()) {
      constexpr uint32_t idesc =
          F8 ? make_idesc_e4m3(kBM, BN) : make_idesc_bf16(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t tphase = 0;
      TileCoord tc;
      for (int t = blockIdx.x; get_tile<SCHED>(t, args, BN, prefix, tc); t += gridDim.x) {
        if (!mbar_wait(&tempty_bar[buf], tphase ^ 1, args.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        uint32_t accum = 0;
        bool ok = true;
        const int nk = (tc.k_end - tc.k_begin + KB - 1) / KB +
                       (DUAL ? (args.K2 + kBK - 1) / kBK : 0);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, args.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(tiles + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_smem_desc(sa + kk * 2048, 8192, 1024, kLayoutSW128)
                                     : make_smem_desc(sa + kk * 32, 16, 1024, kLayoutSW128);
            const uint64_t bd = B_MN ? make_smem_desc(sb + kk * 2048, 8192, 1024, kLayoutSW128)
                                     : make_smem_desc(sb + kk * 32, 16, 1024, kLayoutSW128);
            if (F8) umma_f8(d_tmem, ad, bd, idesc, accum);
            else umma_f16(d_tmem, ad, bd, idesc, accum);
            accum = 1;
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[buf]);
        if (++buf == 2) { buf = 0; tphase ^= 1; }
      }
    }
  } else if (warp >= 4) {
    // ================================ epilogue ========================================
    const int q = warp & 3;  // TMEM lane quarter
    const int row_in_tile = q * 32 + lane;
    int buf = 0;
    uint32_t tphase = 0;
    TileCoord tc;
    for (int t = blockIdx.x; get_tile<SCHED>(t, args, BN, prefix, tc); t += gridDim.x) {
      if (!mbar_wait(&tfull_bar[buf], tphase, args.err, abort_flag)) break;
      tc_fence_after();
      const int row = tc.m0 + row_in_tile;
      const bool row_ok = (SCHED == kSchedGroupedM)
                              ? (row < args.group_offsets[tc.g + 1])
                              : (row < args.M);
      LseState st{-INFINITY, 0.f, 0.f};
      GemmArgs la = args;
      if (EPI == kEpiLse || EPI == kEpiLogprobBwd) la.N = args.N;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN + c;
        tmem_ld_32x32b_x32(taddr, r);
        tmem_ld_wait();
        if (tc.n0 + c < args.N) epi_chunk<EPI>(la, row, row_ok, tc.g, tc.n0 + c, r, st);
      }
      if (EPI == kEpiLse && row_ok) {
        float* p = args.lse_part + ((int64_t)row * args.n_tiles_total + tc.n0 / BN) * 3;
        p[0] = st.m; p[1] = st.s; p[2] = st.t;
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[buf]);
      if (++buf == 2) { buf = 0; tphase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace af3
