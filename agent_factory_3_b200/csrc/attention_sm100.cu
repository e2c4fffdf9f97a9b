// Flash attention forward for gpt-oss on sm_100a: causal GQA over packed variable-length
// sequences, optional sliding window, learned per-head sinks, head_dim 64.
//
// One CTA per (q head, span of up to 256 query rows).  The span is two 128-row tiles A and B
// that share every K/V block loaded by TMA; each tile has its own softmax warpgroup, so the
// tensor core works on one tile while the other tile's softmax runs.
//   warp 0      TMA: Q_A, Q_B once, then K_j (K-major) and V_j (MN-major, two 64-key boxes)
//               into a 3-stage ring
//   warp 1      tcgen05 issuer.  S_X(j+1) = Q_X K_{j+1}^T (M=128, N=128, K=64, both operands
//               in shared memory) is issued as soon as the softmax of tile X has copied S_X(j)
//               out of TMEM, i.e. while that softmax still runs; O_X += P_X(j) V_j (M=128,
//               N=64, K=128) reads P straight from TMEM (A operand in tensor memory) and is
//               issued when the softmax has stored P_X(j).
//   warps 4-7   softmax of tile A, warps 8-11 softmax of tile B: thread t owns query row t.
//               It reads S with tcgen05.ld, applies the causal / window / sequence masks,
//               keeps a reference max m (log2 domain) that only moves when a block's max
//               exceeds it by more than 2^8 (then O in TMEM and the row sum are rescaled
//               once), computes P = 2^(s*scale*log2e - m), adds P into a row sum held in
//               registers and stores P as bf16 pairs into its TMEM lane (tcgen05.st).  The
//               scaling and row sums run as packed fp32x2 instructions.  Optionally
//               (AF3_ATTN_POLY=2..8) a share of the 2^x evaluations of unmasked blocks runs on
//               the FMA pipe (cubic minimax polynomial after range reduction, relative error
//               7.5e-5, far below bf16's 2^-9) instead of the MUFU unit; measured slower on
//               B200, so it is off by default.
//   The sink logit joins the denominator at the end: l += 2^(sink*log2e - m).
//   Outputs: O (bf16) and the natural-log LSE per (head, query), sink included.
//
// TMEM columns: S[A] 0..127, S[B] 128..255, P[A] 256..319, P[B] 320..383 (bf16 pairs),
//               O[A] 384..447, O[B] 448..511.
//
// Reference semantics: HF transformers eager_attention_forward for gpt-oss (sinks appended to
// the logits, softmax, sink column dropped; models/gpt_oss in transformers); sliding window:
// key j visible from query i iff i - j < window.
#include <cstdlib>
#include <string>

#include "common.h"
#include "host_utils.h"
#include "sm100.cuh"

namespace af3 {

constexpr int kFwdThreads = 384;
constexpr int kHD = 64;  // head dim
constexpr int kBQ = 128;
constexpr int kBKV = 128;
constexpr int kKVStages = 3;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f;  // reference max moves only when exceeded by 2^8
constexpr uint32_t kColS = 0, kColP = 256, kColO = 384;
// Measured on B200 (32k causal, 64q/8kv, cvt packing): 0 -> 826, 2 -> 706, 4 -> 647,
// 6 -> 584, 8 -> 519 TFLOP/s.  The kernel is bound by softmax issue and latency, not by the MUFU unit, so moving
// exponentials to the FMA pipe only adds instructions; the polynomial path stays selectable.
constexpr int kDefaultPoly = 0;

struct AttnFwdSmem {
  // all tiles 1024-aligned
  static constexpr int Q = 0;                                  // 2 x 16 KB (A, B)
  static constexpr int K = Q + 2 * kBQ * kHD * 2;              // 3 x 16 KB
  static constexpr int V = K + kKVStages * kBKV * kHD * 2;     // 3 x 16 KB
  static constexpr int BAR = V + kKVStages * kBKV * kHD * 2;
  static constexpr int TOTAL = BAR + 1024;
};

struct AttnParams {
  const int* tiles;  // [n, 3] (seq_start, q_start, q_end), q_end - q_start <= 256
  const float* sinks;
  __nv_bfloat16* out;
  int64_t ld_out;
  float* lse;  // [Hq, T]
  int T, hq, hkv, window;
  float scale_log2;  // softmax scale * log2(e)
  int* err;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------ packed fp32x2 arithmetic --------------------------------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// bf16 pair of two non-negative finite floats (P values).  INT_PACK rounds on the integer
// pipe (add half an ulp, keep the upper halves with one byte permute: round-half-up, which
// differs from round-to-nearest-even only on exact ties), so the packing does not compete
// with the exponentials for the conversion unit; otherwise one cvt.rn.bf16x2.f32.
template <bool INT_PACK>
__device__ __forceinline__ uint32_t bf16x2_of(float lo, float hi) {
  uint32_t r;
  if constexpr (INT_PACK) {
    const uint32_t a = __float_as_uint(lo) + 0x8000u, b = __float_as_uint(hi) + 0x8000u;
    asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(r) : "r"(a), "r"(b));
  } else {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  }
  return r;
}

// 2^x for a pair on the FMA pipe.  x = n + f with n = rint(x) (adding 1.5 * 2^23 leaves n in
// the low mantissa bits), f in [-0.5, 0.5]; 2^f by a cubic fitted to minimise the relative
// error on that interval (Remez exchange, max relative error 7.5e-5); 2^n is added to the
// exponent field.  x is clamped to >= -125 so the exponent cannot wrap; callers only pass
// finite x <= 8 (unmasked blocks).
__device__ __forceinline__ void exp2_poly_x2(uint64_t x2, float& r0, float& r1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  float x0, x1;
  f2_unpack(x2, x0, x1);
  x0 = fmaxf(x0, -125.f);
  x1 = fmaxf(x1, -125.f);
  const uint64_t xx = f2_pack(x0, x1);
  const uint64_t t = f2_add(xx, f2_pack(kMagic, kMagic));
  const uint64_t nf = f2_add(t, f2_pack(-kMagic, -kMagic));
  const uint64_t fr = f2_fma(nf, f2_pack(-1.f, -1.f), xx);
  uint64_t p = f2_fma(f2_pack(0.05517167f, 0.05517167f), fr, f2_pack(0.24261113f, 0.24261113f));
  p = f2_fma(p, fr, f2_pack(0.69326097f, 0.69326097f));
  p = f2_fma(p, fr, f2_pack(0.99992806f, 0.99992806f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  r0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  r1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// Key-block range of one 128-row query tile inside the CTA's span.
struct FwdTile {
  int q0, q1;    // query rows [q0, q1); empty when q1 <= q0
  int jlo, jhi;  // key blocks [jlo, jhi) relative to the span's first key
};

__device__ __forceinline__ FwdTile fwd_tile(int q0, int q1, int seq0, int kv_lo, int window) {
  FwdTile t{q0, q1, 0, 0};
  if (q1 > q0) {
    const int lo = window > 0 ? max(seq0, q0 - window + 1) : seq0;
    t.jlo = (lo - kv_lo) / kBKV;
    t.jhi = (q1 - 1 - kv_lo) / kBKV + 1;
  }
  return t;
}

// MMA-issuer state of one tile.
struct FwdIssue {
  int jlo, jhi;   // key blocks of the tile
  int n_s, n_pv;  // S / PV blocks issued so far
};

// S_X(j) = Q_X K_j^T into TMEM S[X].  The S buffer must have been read by the softmax of the
// tile's previous block (s_free).
template <int X>
__device__ __forceinline__ bool fwd_issue_s(FwdIssue& t, int j, uint32_t tmem, uint32_t sq,
                                            uint32_t sk0, uint64_t* s_free, uint64_t* s_full,
                                            int* err, volatile int* abort_flag) {
  if (j < t.jlo || j >= t.jhi) return true;
  if (t.n_s > 0 && !mbar_wait(&s_free[X], (t.n_s - 1) & 1, err, abort_flag)) return false;
  tc_fence_after();
  constexpr uint32_t idesc_s = make_idesc_bf16(kBQ, kBKV, false, false);
  const uint32_t q = sq + X * kBQ * kHD * 2;
  const uint32_t k = sk0 + (j % kKVStages) * kBKV * kHD * 2;
#pragma unroll
  for (int kk = 0; kk < kHD / 16; ++kk) {
    umma_f16(tmem + kColS + X * kBKV, make_smem_desc(q + kk * 32, 16, 1024, kLayoutSW128),
             make_smem_desc(k + kk * 32, 16, 1024, kLayoutSW128), idesc_s, kk > 0);
  }
  umma_commit(&s_full[X]);
  ++t.n_s;
  return true;
}

// O_X += P_X(j) V_j with P read from TMEM (two bf16 per column, row = lane).
template <int X>
__device__ __forceinline__ bool fwd_issue_pv(FwdIssue& t, int j, uint32_t tmem, uint32_t sv0,
                                             uint64_t* p_full, uint64_t* o_ready, int* err,
                                             volatile int* abort_flag) {
  if (j < t.jlo || j >= t.jhi) return true;
  if (!mbar_wait(&p_full[X], t.n_pv & 1, err, abort_flag)) return false;
  tc_fence_after();
  constexpr uint32_t idesc_o = make_idesc_bf16(kBQ, kHD, false, true);
  const uint32_t v = sv0 + (j % kKVStages) * kBKV * kHD * 2;
  const uint32_t first = t.n_pv > 0 ? 1u : 0u;
#pragma unroll
  for (int kk = 0; kk < kBKV / 16; ++kk) {
    const uint64_t bd = make_smem_desc(v + (kk / 4) * 8192 + (kk % 4) * 2048, 8192, 1024, kLayoutSW128);
    umma_f16_tmem_a(tmem + kColO + X * kHD, tmem + kColP + X * 64 + kk * 8, bd, idesc_o,
                    kk > 0 ? 1u : first);
  }
  umma_commit(&o_ready[X]);
  ++t.n_pv;
  return true;
}

// POLY: number of the sixteen 8-column groups of a 128-key block whose exponentials run on
// the FMA pipe in unmasked blocks (0 = all on the MUFU unit).
template <int POLY, bool INT_PACK>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tma_qk,
                    const __grid_constant__ CUtensorMap tma_v, const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AttnFwdSmem::BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;    // [3]
  uint64_t* kv_empty = bars + 4;   // [3]
  uint64_t* s_full = bars + 7;     // [2] per tile: S in TMEM
  uint64_t* s_free = bars + 9;     // [2] S copied out of TMEM by the softmax
  uint64_t* p_full = bars + 11;    // [2] P stored in TMEM (O rescaled if needed)
  uint64_t* o_ready = bars + 13;   // [2] PV complete: P buffer free, O stable
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int h = blockIdx.x;
  const int span = blockIdx.y;
  const int seq0 = p.tiles[span * 3 + 0];
  const int qs0 = p.tiles[span * 3 + 1];
  const int qs1 = p.tiles[span * 3 + 2];
  if (qs1 <= qs0) return;
  const int kvh = h / (p.hq / p.hkv);
  const int kv_lo = p.window > 0 ? max(seq0, qs0 - p.window + 1) : seq0;
  const int nb = (qs1 - kv_lo + kBKV - 1) / kBKV;
  const FwdTile tl[2] = {fwd_tile(qs0, min(qs1, qs0 + kBQ), seq0, kv_lo, p.window),
                         fwd_tile(qs0 + kBQ, qs1, seq0, kv_lo, p.window)};
  const bool has_b = tl[1].q1 > tl[1].q0;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_qk);
    tma_prefetch_desc(&tma_v);
    mbar_init(q_full, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], 4);    // one arrive per softmax warp
      mbar_init(&p_full[x], 4);
      mbar_init(&o_ready[x], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // register split (launch: 384 x 168): control warps 128 x 96 + softmax 256 x 200 = 63488 <= 64512
  if (warp < 4) {
    setmaxnreg_dec<96>();
    if (warp == 0) {
      if (elect_one_sync()) {
        mbar_arrive_expect_tx(q_full, (has_b ? 2 : 1) * kBQ * kHD * 2);
        tma_load_2d(smem + AttnFwdSmem::Q, &tma_qk, q_full, h * kHD, qs0);
        if (has_b) tma_load_2d(smem + AttnFwdSmem::Q + kBQ * kHD * 2, &tma_qk, q_full, h * kHD, qs0 + kBQ);
        for (int j = 0; j < nb; ++j) {
          const int s = j % kKVStages;
          if (!mbar_wait(&kv_empty[s], ((j / kKVStages) & 1) ^ 1, p.err, abort_flag)) break;
          const int k0 = kv_lo + j * kBKV;
          mbar_arrive_expect_tx(&kv_full[s], 2 * kBKV * kHD * 2);
          tma_load_2d(smem + AttnFwdSmem::K + s * kBKV * kHD * 2, &tma_qk, &kv_full[s],
                      (p.hq + kvh) * kHD, k0);
          uint8_t* vb = smem + AttnFwdSmem::V + s * kBKV * kHD * 2;
          tma_load_2d(vb, &tma_v, &kv_full[s], (p.hq + p.hkv + kvh) * kHD, k0);
          tma_load_2d(vb + 8192, &tma_v, &kv_full[s], (p.hq + p.hkv + kvh) * kHD, k0 + 64);
        }
      }
    } else if (warp == 1) {
      if (elect_one_sync()) {
        const uint32_t sq = smem_u32(smem + AttnFwdSmem::Q);
        const uint32_t sk0 = smem_u32(smem + AttnFwdSmem::K);
        const uint32_t sv0 = smem_u32(smem + AttnFwdSmem::V);
        FwdIssue a{tl[0].jlo, tl[0].jhi, 0, 0}, b{tl[1].jlo, tl[1].jhi, 0, 0};
        bool ok = mbar_wait(q_full, 0, p.err, abort_flag) &&
                  mbar_wait(&kv_full[0], 0, p.err, abort_flag);
        ok = ok && fwd_issue_s<0>(a, 0, tmem, sq, sk0, s_free, s_full, p.err, abort_flag) &&
             fwd_issue_s<1>(b, 0, tmem, sq, sk0, s_free, s_full, p.err, abort_flag);
        for (int j = 0; ok && j < nb; ++j) {
          const bool next = j + 1 < nb;
          if (next)
            ok = mbar_wait(&kv_full[(j + 1) % kKVStages], ((j + 1) / kKVStages) & 1, p.err,
                           abort_flag);
          // S of the next block runs while the softmax of this block is still working
          if (ok && next)
            ok = fwd_issue_s<0>(a, j + 1, tmem, sq, sk0, s_free, s_full, p.err, abort_flag);
          ok = ok && fwd_issue_pv<0>(a, j, tmem, sv0, p_full, o_ready, p.err, abort_flag);
          if (ok && next)
            ok = fwd_issue_s<1>(b, j + 1, tmem, sq, sk0, s_free, s_full, p.err, abort_flag);
          ok = ok && fwd_issue_pv<1>(b, j, tmem, sv0, p_full, o_ready, p.err, abort_flag);
          umma_commit(&kv_empty[j % kKVStages]);
        }
      }
    }
  } else {
    setmaxnreg_inc<200>();
    const int x = (warp - 4) >> 2;  // tile owned by this warpgroup
    const FwdTile t = x ? tl[1] : tl[0];
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int qi = t.q0 + row;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + kColS + x * kBKV;
    const uint32_t p_addr = tmem + lane_base + kColP + x * 64;
    const uint32_t o_addr = tmem + lane_base + kColO + x * kHD;
    const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
    float m_ref = -INFINITY;
    float l_run = 0.f;  // row sum of P relative to m_ref
    int c = 0;
    bool ok = true;
    for (int j = t.jlo; j < t.jhi; ++j, ++c) {
      if (!mbar_wait(&s_full[x], c & 1, p.err, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float sv[kBKV];
      {
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld_32x32b_x32(s_addr, r0);
        tmem_ld_32x32b_x32(s_addr + 32, r1);
        tmem_ld_32x32b_x32(s_addr + 64, r2);
        tmem_ld_32x32b_x32(s_addr + 96, r3);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          sv[e] = __uint_as_float(r0[e]);
          sv[32 + e] = __uint_as_float(r1[e]);
          sv[64 + e] = __uint_as_float(r2[e]);
          sv[96 + e] = __uint_as_float(r3[e]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[x]);   // the MMA may overwrite S with block j+1
      const int k0 = kv_lo + j * kBKV;
      const bool need_mask = (k0 + kBKV - 1 > t.q0) || (k0 < seq0) ||
                             (p.window > 0 && t.q0 + kBQ - 1 - k0 >= p.window);
      if (need_mask) {
#pragma unroll
        for (int cc = 0; cc < kBKV; ++cc) {
          const int kj = k0 + cc;
          const bool vis = kj <= qi && kj >= seq0 && (p.window == 0 || qi - kj < p.window);
          if (!vis) sv[cc] = -INFINITY;
        }
      }
      float mxp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mxp[u] = fmaxf(sv[u], sv[8 + u]);
#pragma unroll
      for (int cc = 16; cc < kBKV; cc += 16) {
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = fmax3(mxp[u], sv[cc + u], sv[cc + 8 + u]);
      }
      const float mraw = fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]),
                               fmaxf(mxp[6], mxp[7]));
      const float cand = mraw * p.scale_log2;
      const bool resc = cand > m_ref + kRescaleLog2;  // false while both are -inf
      float alpha = 1.f;
      if (resc) {
        alpha = ex2(m_ref - cand);  // m_ref = -inf -> 0
        m_ref = cand;
      }
      const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
      const uint64_t negm2 = f2_pack(-m_use, -m_use);
      // P = 2^(s * scale - m) as bf16 pairs; the row sum accumulates in two packed lanes
      uint32_t pk[kBKV / 2];
      uint64_t rs2[4] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f), f2_pack(0.f, 0.f),
                         f2_pack(0.f, 0.f)};   // four chains: no serial add dependency
#pragma unroll
      for (int c8 = 0; c8 < kBKV / 8; ++c8) {
        const bool poly = POLY > 0 && ((c8 * POLY) % 16) < POLY;
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const uint64_t x2 = f2_fma(f2_pack(sv[c8 * 8 + e], sv[c8 * 8 + e + 1]), scale2, negm2);
          float e0, e1;
          if (poly && !need_mask) {
            exp2_poly_x2(x2, e0, e1);
          } else {
            float x0, x1;
            f2_unpack(x2, x0, x1);
            e0 = ex2(x0);
            e1 = ex2(x1);
          }
          rs2[e / 2] = f2_add(rs2[e / 2], f2_pack(e0, e1));
          pk[c8 * 4 + e / 2] = bf16x2_of<INT_PACK>(e0, e1);
        }
      }
      const uint64_t rsa = f2_add(f2_add(rs2[0], rs2[1]), f2_add(rs2[2], rs2[3]));
      float rs0, rs1;
      f2_unpack(rsa, rs0, rs1);
      l_run = l_run * alpha + (rs0 + rs1);
      // PV of the previous block must be complete before P is overwritten or O rescaled
      if (c > 0) {
        if (!mbar_wait(&o_ready[x], (c - 1) & 1, p.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, resc)) {
#pragma unroll
          for (int h32 = 0; h32 < kHD / 32; ++h32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(o_addr + h32 * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st_32x32b_x32(o_addr + h32 * 32, r);
          }
        }
      }
      {
        uint32_t w0[32], w1[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          w0[e] = pk[e];
          w1[e] = pk[32 + e];
        }
        tmem_st_32x32b_x32(p_addr, w0);
        tmem_st_32x32b_x32(p_addr + 32, w1);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    if (ok && c > 0) {
      if (mbar_wait(&o_ready[x], (c - 1) & 1, p.err, abort_flag)) {
        tc_fence_after();
        uint32_t o0[32], o1[32];
        tmem_ld_32x32b_x32(o_addr, o0);
        tmem_ld_32x32b_x32(o_addr + 32, o1);
        tmem_ld_wait();
        if (qi < t.q1) {
          // the sink joins the max: a row whose scores all lie far below the sink would
          // otherwise overflow 2^(sink - m)
          const float m_use = (m_ref == -INFINITY) ? -INFINITY : m_ref;
          const float sk = p.sinks[h] * kLog2e;
          const float m_fin = fmaxf(m_use, sk);
          const float a = ex2(m_use - m_fin);  // m_use = -inf -> 0 (O and l are 0 then)
          const float l_tot = l_run * a + ex2(sk - m_fin);
          const float inv = a / l_tot;
          __nv_bfloat16* orow = p.out + (int64_t)qi * p.ld_out + h * kHD;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o0[c8 * 8 + 0]) * inv, __uint_as_float(o0[c8 * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o0[c8 * 8 + 2]) * inv, __uint_as_float(o0[c8 * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o0[c8 * 8 + 4]) * inv, __uint_as_float(o0[c8 * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o0[c8 * 8 + 6]) * inv, __uint_as_float(o0[c8 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c8 * 8) = w;
          }
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o1[c8 * 8 + 0]) * inv, __uint_as_float(o1[c8 * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o1[c8 * 8 + 2]) * inv, __uint_as_float(o1[c8 * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o1[c8 * 8 + 4]) * inv, __uint_as_float(o1[c8 * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o1[c8 * 8 + 6]) * inv, __uint_as_float(o1[c8 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + 32 + c8 * 8) = w;
          }
          p.lse[(int64_t)h * p.T + qi] = (m_fin + __log2f(l_tot)) * kLn2;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

void attn_fwd(torch::Tensor qkv, torch::Tensor sinks, torch::Tensor tiles, torch::Tensor cu,
              torch::Tensor out, torch::Tensor lse, int64_t hq, int64_t hkv, int64_t d,
              int64_t window, double scale) {
  check_cuda_bf16(qkv, "qkv");
  AF3_CHECK(d == kHD, "attention kernel is built for head_dim 64");
  AF3_CHECK(qkv.size(1) == (hq + 2 * hkv) * d && qkv.stride(1) == 1, "qkv layout");
  AF3_CHECK(hq % hkv == 0, "hq must be a multiple of hkv");
  AF3_CHECK(sinks.scalar_type() == torch::kFloat32, "sinks must be fp32");
  const int64_t T = qkv.size(0);
  const int64_t n_tiles = tiles.size(0);
  const c10::cuda::CUDAGuard guard(qkv.device());
  if (T == 0 || n_tiles == 0) return;
  const uint64_t dims[2] = {(uint64_t)qkv.size(1), (uint64_t)T};
  const uint64_t strides[1] = {(uint64_t)qkv.stride(0) * 2};
  const uint32_t box_qk[2] = {64, 128};
  const uint32_t box_v[2] = {64, 64};
  CUtensorMap tqk = make_tmap(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides,
                              box_qk, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tv = make_tmap(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides,
                             box_v, CU_TENSOR_MAP_SWIZZLE_128B);
  AttnParams p;
  p.tiles = tiles.data_ptr<int>();
  p.sinks = sinks.data_ptr<float>();
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ld_out = out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.T = (int)T;
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.window = (int)window;
  p.scale_log2 = (float)scale * kLog2e;
  p.err = device_error_ptr();
  const int smem = AttnFwdSmem::TOTAL + 1024;
  // share of the exponentials on the FMA pipe (8-column groups out of 16), AF3_ATTN_POLY;
  // P packing with cvt (default) or on the integer pipe (AF3_ATTN_PACK=int).  Measured on
  // B200 (32k causal, 64q/8kv): cvt 10.5 ms, int 11.4 ms.
  static const int poly = [] {
    const char* e = std::getenv("AF3_ATTN_POLY");
    const int v = e ? std::atoi(e) : kDefaultPoly;
    return (v == 0 || v == 4) ? v : kDefaultPoly;
  }();
  static const bool int_pack = [] {
    const char* e = std::getenv("AF3_ATTN_PACK");
    return e && std::string(e) == "int";
  }();
  static bool attr[64][4] = {};
  int dev;
  AF3_CUDA_CHECK(cudaGetDevice(&dev));
  auto kern = poly == 0 ? (int_pack ? attn_fwd_kernel<0, true> : attn_fwd_kernel<0, false>)
                        : (int_pack ? attn_fwd_kernel<4, true> : attn_fwd_kernel<4, false>);
  const int ai = (poly ? 2 : 0) + (int_pack ? 1 : 0);
  if (!attr[dev][ai]) {
    AF3_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev][ai] = true;
  }
  dim3 grid((unsigned)hq, (unsigned)n_tiles);
  kern<<<grid, kFwdThreads, smem, at::cuda::getCurrentCUDAStream()>>>(tqk, tv, p);
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
