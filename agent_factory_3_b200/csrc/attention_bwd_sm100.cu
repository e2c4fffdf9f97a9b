// Flash-attention backward for gpt-oss on sm_100a (causal GQA, packed varlen, sliding
// window, learned sinks, head_dim 64).
//
// One CTA per (128-key tile, kv head).  It keeps K and V of its key tile on chip and loops
// over every q head of the kv group and every 128-query block that can see the tile, in two
// 64-query halves per block:
//   S^T  = K Q^T        (tcgen05, M=128 keys, N=64 queries per half, K=64)  TMEM cols   0..127
//   dP^T = V dO^T       (same shape)                                        TMEM cols 128..255
//   P^T  = 2^(S^T * scale*log2e - lse2[q]),  dS^T = P^T * (dP^T - D[q])   (softmax warps,
//          thread = key row; written back as bf16 pairs over the S^T / dP^T columns they
//          were computed from, and dS^T also into 128B-swizzled shared memory)
//   dV  += P^T dO       (A = P^T from TMEM, B = dO as MN-major)        TMEM cols 256..319
//   dK  += dS^T Q       (A = dS^T from TMEM, B = Q as MN-major)        TMEM cols 320..383
//   dQ   = dS K         (A = dS^T read as MN-major from shared memory, B = K as MN-major)
//                                                                      TMEM cols 384..447
// K and V are the A operands of S^T / dP^T and sit in TMEM too (cols 448..479, 480..511,
// copied there once per CTA).  With N = 64, an MMA that reads both operands from shared memory
// needs 6 KB per 32 tensor cycles, more than the 128 B per cycle that shared memory delivers.
// So every product except dQ takes its A operand from TMEM and reads only its 2 KB B slice
// from shared memory.
// The eight softmax warps work on one half at a time (warp quarter = 32 key rows, warps 4-7
// the first 32 queries of the half, warps 12-15 the other 32); while they compute one half,
// the tensor core runs dV / dK of the other half and the next block's S^T / dP^T of it.
// dQ of each block is added to an fp32 buffer by warps 8-11: each warp stages its 32 rows,
// scaled, as two [32 x 32] 128B-swizzled boxes in its 4 KB share of V's shared memory (unused
// once V is in TMEM) and issues a TMA reduce-add per box, so the L2 adds whole lines.  dK and
// dV are complete at the end of the CTA (all q heads of the group were visited) and are written
// once as bf16 -- no atomics.  A prologue kernel computes D = rowsum(dO * O) and the
// sink gradient d(sink_h) = -sum_i exp(sink_h - lse_h(i)) * D_h(i); an epilogue kernel
// converts dQ to bf16.
#include "common.h"
#include "host_utils.h"
#include "sm100.cuh"

namespace af3 {
namespace attnb {

constexpr int kThreads = 512;
constexpr int kHD = 64;
constexpr int kB = 128;  // keys per CTA tile, queries per block
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kColDQ = 384;  // dQ accumulator (64 columns, one block at a time)
constexpr int kColK = 448;   // K as bf16 pairs: the A operand of S^T
constexpr int kColV = 480;   // V as bf16 pairs: the A operand of dP^T

struct Smem {
  static constexpr int K = 0;                         // 16 KB  [128 keys x 64] K-major
  static constexpr int V = K + kB * kHD * 2;          // 16 KB
  static constexpr int QDO = V + kB * kHD * 2;        // 2 stages x (Q 16 KB + dO 16 KB)
  static constexpr int DST = QDO + 2 * 2 * kB * kHD * 2;  // 2 x 32 KB dS^T (double buffered)
  static constexpr int LD = DST + 2 * kB * kB * 2;    // 2 stages x (lse2 512 B + D 512 B)
  static constexpr int BAR = LD + 2 * 2 * kB * 4;
  static constexpr int TOTAL = BAR + 1024;            // 163 KB
};

struct Params {
  const int* tiles;   // [n, 4] (seq_start, seq_end, k_start, k_end)
  const float* lse;   // [Hq, T] natural log
  const float* Dd;    // [Hq, T]
  float* dq;          // [T, Hq*64] fp32 accumulator
  __nv_bfloat16* dqkv;
  int64_t ld_dqkv;
  int T, hq, hkv, window;
  float scale, scale_log2;
  int* err;
};

// Bounded wait whose result is the same on every lane of the warp (a lane that timed out makes
// the whole warp give up), so the per-warp arrives after __syncwarp never diverge.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* err,
                                               volatile int* abort_flag) {
  const bool ok = mbar_wait(bar, parity, err, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// element (row, 8*c8 .. 8*c8+7) of a [128 rows x 128 cols] bf16 K-major SW128 tile made of
// two 64-column blocks of 16 KB (shared-window address)
__device__ __forceinline__ void store_sw128(uint32_t base, int row, int c8, uint32_t a, uint32_t b,
                                            uint32_t c, uint32_t d) {
  const int blk = c8 >> 3, ch = (c8 & 7) ^ (row & 7);
  st_shared_v4(base + blk * 16384 + row * 128 + ch * 16, a, b, c, d);
}

// bf16 pairs of 8 consecutive values
__device__ __forceinline__ void pack8(const float* v, uint32_t& a, uint32_t& b, uint32_t& c,
                                      uint32_t& d) {
  a = pack_bf16x2(v[0], v[1]);
  b = pack_bf16x2(v[2], v[3]);
  c = pack_bf16x2(v[4], v[5]);
  d = pack_bf16x2(v[6], v[7]);
}

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
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_of(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// P^T and dS^T of one key row over 16 query columns starting at c, as bf16 pairs (packed
// fp32x2 arithmetic).  -lse2 (log2 domain, negated so that it is the FMA's addend as loaded)
// and D of the block's queries are in shared memory at lds (-lse2[128] then D[128]); every
// lane reads the same addresses, so the 16-byte loads are broadcasts.
template <bool MASK>
__device__ __forceinline__ void softmax_grad16(const uint32_t (&sv)[16], const uint32_t (&dv)[16],
                                               const float* lds, int c, float scale_log2, int key,
                                               int qb, int k1, int q_end, int window,
                                               uint32_t (&pp)[8], uint32_t (&dd)[8]) {
  const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
#pragma unroll
  for (int e4 = 0; e4 < 4; ++e4) {
    const float4 l4 = *reinterpret_cast<const float4*>(lds + c + e4 * 4);
    const float4 d4 = *reinterpret_cast<const float4*>(lds + kB + c + e4 * 4);
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int e = e4 * 4 + h2 * 2;
      const float la = h2 ? l4.z : l4.x, lb = h2 ? l4.w : l4.y;
      const float da = h2 ? d4.z : d4.x, db = h2 ? d4.w : d4.y;
      float t0, t1;
      f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), sc2,
                       f2_pack(la, lb)), t0, t1);
      float p0 = ex2(t0), p1 = ex2(t1);
      if (MASK) {
        const int q0 = qb + c + e, q1 = q0 + 1;
        const bool v0 = key < k1 && key <= q0 && q0 < q_end && (window == 0 || q0 - key < window);
        const bool v1 = key < k1 && key <= q1 && q1 < q_end && (window == 0 || q1 - key < window);
        p0 = v0 ? p0 : 0.f;
        p1 = v1 ? p1 : 0.f;
      }
      float s0, s1;
      f2_unpack(f2_mul(f2_pack(p0, p1),
                       f2_sub(f2_pack(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])),
                              f2_pack(da, db))), s0, s1);
      pp[e / 2] = bf16x2_of(p0, p1);
      dd[e / 2] = bf16x2_of(s0, s1);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tma_qkv,
                    const __grid_constant__ CUtensorMap tma_do,
                    const __grid_constant__ CUtensorMap tma_dq, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the 128B-swizzled tiles need a 1024-aligned base; the launch adds 1 KB of slack for it
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* ld_full = bars + 5;    // [2]
  uint64_t* ld_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;     // [2] per query half
  uint64_t* p_full = bars + 13;    // [2] per query half: P^T / dS^T of the half written
  uint64_t* mma_done = bars + 15;  // [2] dS^T buffer b consumed
  uint64_t* dq_full = bars + 17;   // [2]
  uint64_t* dq_empty = bars + 19;  // [2]
  uint64_t* final_done = bars + 21;
  uint64_t* kv_tmem = bars + 22;   // K and V copied into TMEM
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 23);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = blockIdx.x;  // kv head
  const int tile = blockIdx.y;
  const int seq1 = p.tiles[tile * 4 + 1];
  const int k0 = p.tiles[tile * 4 + 2];
  const int k1 = p.tiles[tile * 4 + 3];
  if (k1 <= k0) return;
  const int rep = p.hq / p.hkv;
  int q_end = seq1;
  if (p.window > 0) q_end = min(seq1, k1 - 1 + p.window);
  const int nqb = (q_end - k0 + kB - 1) / kB;
  const int n_it = rep * nqb;  // (q head, query block) pairs

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_qkv);
    tma_prefetch_desc(&tma_do);
    tma_prefetch_desc(&tma_dq);
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&qdo_full[s], 1);
      mbar_init(&qdo_empty[s], 1);
      // consumer-side barriers take one arrive per warp (lane 0 after __syncwarp), not one per
      // thread: hundreds of per-thread arrives per block serialise on the barrier word
      mbar_init(&ld_full[s], 1);
      mbar_init(&ld_empty[s], 8);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 8);
      mbar_init(&mma_done[s], 1);
      mbar_init(&dq_full[s], 1);   // only [0] is used
      mbar_init(&dq_empty[s], 4);  // only [0] is used: one dQ accumulator
    }
    mbar_init(final_done, 1);
    mbar_init(kv_tmem, 8);
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

  if (warp == 0) {
    // ------------------------------- TMA producer ------------------------------------
    if (elect_one_sync()) {
      mbar_arrive_expect_tx(kv_full, 2 * kB * kHD * 2);
      tma_load_2d(smem + Smem::K, &tma_qkv, kv_full, (p.hq + g) * kHD, k0);
      tma_load_2d(smem + Smem::V, &tma_qkv, kv_full, (p.hq + p.hkv + g) * kHD, k0);
      for (int it = 0; it < n_it; ++it) {
        const int s = it & 1;
        if (!mbar_wait(&qdo_empty[s], ((it >> 1) & 1) ^ 1, p.err, abort_flag)) break;
        const int h = g * rep + it / nqb;
        const int qb = k0 + (it % nqb) * kB;
        uint8_t* q = smem + Smem::QDO + s * 2 * kB * kHD * 2;
        mbar_arrive_expect_tx(&qdo_full[s], 2 * kB * kHD * 2);
        tma_load_2d(q, &tma_qkv, &qdo_full[s], h * kHD, qb);
        tma_load_2d(q + kB * kHD * 2, &tma_do, &qdo_full[s], h * kHD, qb);
      }
    }
  } else if (warp == 3) {
    // ---------------------- lse / D loader (plain loads) -----------------------------
    for (int it = 0; it < n_it; ++it) {
      const int s = it & 1;
      if (!mbar_wait_warp(&ld_empty[s], ((it >> 1) & 1) ^ 1, p.err, abort_flag)) break;
      const int h = g * rep + it / nqb;
      const int qb = k0 + (it % nqb) * kB;
      float* dst = reinterpret_cast<float*>(smem + Smem::LD + s * 2 * kB * 4);
      // all eight loads are in flight together (one memory latency per block, not four)
      float lv[4], dv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int qi = qb + lane + 32 * k;
        const bool ok = qi < p.T;
        lv[k] = ok ? __ldg(p.lse + (int64_t)h * p.T + qi) * -kLog2e : -INFINITY;
        dv[k] = ok ? __ldg(p.Dd + (int64_t)h * p.T + qi) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        dst[lane + 32 * k] = lv[k];
        dst[kB + lane + 32 * k] = dv[k];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ld_full[s]);
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer --------------------------------------
    // Work goes in half-steps u = 2*it + hf (block it, query half hf).  For each u, once the
    // softmax has written P^T / dS^T of the half into TMEM (over the S^T / dP^T columns it
    // read): dV += P^T dO_hf and dK += dS^T Q_hf (A from TMEM), then S^T / dP^T of the same
    // half of block it+1 into the same columns; after half 1, dQ of block it.  The tensor pipe
    // runs one CTA's MMAs in issue order, so S(u+2) overwrites the columns only after
    // dV / dK(u) read them.
    if (elect_one_sync()) {
      constexpr uint32_t id_s = make_idesc_bf16(kB, kB / 2, false, false);  // S^T, dP^T halves
      constexpr uint32_t id_kv = make_idesc_bf16(kB, kHD, false, true);     // dV, dK
      constexpr uint32_t id_q = make_idesc_bf16(kB, kHD, true, true);       // dQ
      const uint32_t sK = smem_u32(smem + Smem::K);
      const uint32_t sDS = smem_u32(smem + Smem::DST);
      auto issue_s = [&](int it, int hf) {
        const uint32_t sQ = smem_u32(smem + Smem::QDO + (it & 1) * 2 * kB * kHD * 2);
        const uint32_t sDO = sQ + kB * kHD * 2;
        // queries hf*64 .. hf*64+63 start 64 rows (8 KB, swizzle-atom aligned) in
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk) {
          umma_f16_tmem_a(tmem + hf * 64, tmem + kColK + kk * 8,
                          make_smem_desc(sQ + hf * 8192 + kk * 32, 16, 1024, kLayoutSW128),
                          id_s, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < kHD / 16; ++kk) {
          umma_f16_tmem_a(tmem + 128 + hf * 64, tmem + kColV + kk * 8,
                          make_smem_desc(sDO + hf * 8192 + kk * 32, 16, 1024, kLayoutSW128),
                          id_s, kk > 0);
        }
        umma_commit(&s_full[hf]);
      };
      bool ok = mbar_wait(kv_tmem, 0, p.err, abort_flag);
      tc_fence_after();
      if (ok && n_it > 0) {
        ok = mbar_wait(&qdo_full[0], 0, p.err, abort_flag);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          issue_s(0, 1);
        }
      }
      for (int it = 0; ok && it < n_it; ++it) {
        const int s = it & 1;
        const uint32_t sQ = smem_u32(smem + Smem::QDO + s * 2 * kB * kHD * 2);
        const uint32_t sDO = sQ + kB * kHD * 2;
        for (int hf = 0; hf < 2 && ok; ++hf) {
          if (!mbar_wait(&p_full[hf], it & 1, p.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // queries hf*64 + 16*kk .. +15: P^T / dS^T pairs at column (kk/2)*32 + (kk%2)*8
            // of the half (each softmax warp writes its 32 queries over its own S columns)
            const uint32_t col = hf * 64 + (kk >> 1) * 32 + (kk & 1) * 8;
            const uint64_t b_do = make_smem_desc(sDO + (hf * 4 + kk) * 2048, 8192, 1024, kLayoutSW128);
            const uint64_t b_q = make_smem_desc(sQ + (hf * 4 + kk) * 2048, 8192, 1024, kLayoutSW128);
            const uint32_t acc = (it > 0 || hf > 0 || kk > 0) ? 1u : 0u;
            umma_f16_tmem_a(tmem + 256, tmem + col, b_do, id_kv, acc);
            umma_f16_tmem_a(tmem + 320, tmem + 128 + col, b_q, id_kv, acc);
          }
          if (it + 1 < n_it) {
            if (hf == 0) {
              if (!mbar_wait(&qdo_full[(it + 1) & 1], ((it + 1) >> 1) & 1, p.err, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            issue_s(it + 1, hf);
          }
        }
        if (!ok) break;
        // dQ of block it: reduction over the 128 keys, A = dS (M = queries) read from dS^T in
        // shared memory as MN-major; the drain has read the previous block's dQ out of TMEM
        if (!mbar_wait(&dq_empty[0], (it & 1) ^ 1, p.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t sDSb = sDS + s * kB * kB * 2;
#pragma unroll
        for (int kk = 0; kk < kB / 16; ++kk) {
          const uint64_t a = make_smem_desc(sDSb + kk * 2048, 16384, 1024, kLayoutSW128);
          const uint64_t b = make_smem_desc(sK + kk * 2048, 8192, 1024, kLayoutSW128);
          umma_f16(tmem + kColDQ, a, b, id_q, kk > 0);
        }
        umma_commit(&mma_done[s]);
        umma_commit(&dq_full[0]);
        umma_commit(&qdo_empty[s]);
      }
      if (ok) umma_commit(final_done);
    }
  } else if (warp >= 8 && warp < 12) {
    // ------------- dQ drain (TMEM -> swizzled smem -> TMA reduce-add into fp32) -------------
    const int qd = warp & 3;
    const uint32_t lb = (uint32_t)(qd * 32) << 16;
    for (int j = 0; j < n_it; ++j) {
      if (!mbar_wait_warp(&dq_full[0], j & 1, p.err, abort_flag)) break;
      tc_fence_after();
      const int h = g * rep + j / nqb;
      const int q0 = k0 + (j % nqb) * kB + qd * 32;  // first query row of this warp
      uint32_t v0[32], v1[32];
      tmem_ld_32x32b_x32(tmem + lb + kColDQ, v0);
      tmem_ld_32x32b_x32(tmem + lb + kColDQ + 32, v1);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_empty[0]);
      // rows past q_end hold exact zeros (their P is masked), so only whole-warp tails skip
      if (q0 < q_end) {
        uint8_t* stage = smem + Smem::V + qd * 4096;
        const uint32_t sw = smem_u32(stage) + lane * 128;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          // the TMA has read the previous box out of this warp's staging area
          if (lane == 0) bulk_wait_read();
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t* v = half ? v1 : v0;
            st_shared_v4(sw + ((c ^ (lane & 7)) * 16),
                         __float_as_uint(__uint_as_float(v[4 * c]) * p.scale),
                         __float_as_uint(__uint_as_float(v[4 * c + 1]) * p.scale),
                         __float_as_uint(__uint_as_float(v[4 * c + 2]) * p.scale),
                         __float_as_uint(__uint_as_float(v[4 * c + 3]) * p.scale));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(&tma_dq, stage, h * kHD + half * 32, q0);
            bulk_commit();
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  } else if (warp >= 4) {
    // ------ softmax gradient: key rows of quarter qd, query columns cg*32.. of each half ------
    const int cg = warp >= 12 ? 1 : 0;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // key row of S^T
    const uint32_t lb = (uint32_t)(qd * 32) << 16;
    const int key = k0 + r;
    bool ok = mbar_wait_warp(kv_full, 0, p.err, abort_flag);
    if (ok) {
      // row r of K (warps 4-7) or V (warps 12-15), 128B-swizzled in shared memory, as 32
      // bf16 pairs into this row's TMEM lane: the A operand layout of the S^T / dP^T MMAs
      const uint8_t* row = smem + (cg ? Smem::V : Smem::K) + r * 128;
      uint32_t w[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(row + ((c ^ (r & 7)) * 16));
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
      tmem_st_32x32b_x32(tmem + lb + (cg ? kColV : kColK), w);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(kv_tmem);
    }
    for (int it = 0; it < n_it && ok; ++it) {
      const int s = it & 1;
      // dS^T buffer s is free once the MMAs of block it-2 (its previous user) completed
      if (it >= 2 && !mbar_wait_warp(&mma_done[s], ((it >> 1) & 1) ^ 1, p.err, abort_flag)) {
        ok = false;
        break;
      }
      if (!mbar_wait_warp(&ld_full[s], (it >> 1) & 1, p.err, abort_flag)) { ok = false; break; }
      const float* lds = reinterpret_cast<const float*>(smem + Smem::LD + s * 2 * kB * 4);  // lse2, D
      const int qb = k0 + (it % nqb) * kB;
      const uint32_t ds = smem_u32(smem + Smem::DST + s * kB * kB * 2);
      for (int hf = 0; hf < 2; ++hf) {
        if (!mbar_wait_warp(&s_full[hf], it & 1, p.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const int c0 = hf * 64 + cg * 32;      // first query column of this warp
        const uint32_t col = tmem + lb + c0;   // its S^T columns; dP^T 128 columns on
        uint32_t sA[16], dA[16], sB[16], dB[16];
        tmem_ld_32x32b_x16(col, sA);
        tmem_ld_32x32b_x16(col + 128, dA);
        tmem_ld_32x32b_x16(col + 16, sB);
        tmem_ld_32x32b_x16(col + 128 + 16, dB);
        tmem_ld_wait();
        uint32_t p0[8], d0[8], p1[8], d1[8];
        const bool vis0 = key < k1 && key <= qb + c0 && qb + c0 + 15 < q_end &&
                          (p.window == 0 || qb + c0 + 15 - key < p.window);
        const bool vis1 = key < k1 && key <= qb + c0 + 16 && qb + c0 + 31 < q_end &&
                          (p.window == 0 || qb + c0 + 31 - key < p.window);
        if (vis0)
          softmax_grad16<false>(sA, dA, lds, c0, p.scale_log2, key, qb, k1, q_end, p.window, p0, d0);
        else
          softmax_grad16<true>(sA, dA, lds, c0, p.scale_log2, key, qb, k1, q_end, p.window, p0, d0);
        if (vis1)
          softmax_grad16<false>(sB, dB, lds, c0 + 16, p.scale_log2, key, qb, k1, q_end, p.window, p1, d1);
        else
          softmax_grad16<true>(sB, dB, lds, c0 + 16, p.scale_log2, key, qb, k1, q_end, p.window, p1, d1);
        // P^T / dS^T of the 32 queries as bf16 pairs over this warp's first 16 S^T / dP^T
        // columns (already read): the TMEM A operands of the dV / dK MMAs
        uint32_t wp[16], wd[16];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          wp[e] = p0[e];
          wp[8 + e] = p1[e];
          wd[e] = d0[e];
          wd[8 + e] = d1[e];
        }
        tmem_st_32x32b_x16(col, wp);
        tmem_st_32x32b_x16(col + 128, wd);
        // dS^T in shared memory: the A operand of the dQ MMA
        store_sw128(ds, r, c0 / 8, d0[0], d0[1], d0[2], d0[3]);
        store_sw128(ds, r, c0 / 8 + 1, d0[4], d0[5], d0[6], d0[7]);
        store_sw128(ds, r, c0 / 8 + 2, d1[0], d1[1], d1[2], d1[3]);
        store_sw128(ds, r, c0 / 8 + 3, d1[4], d1[5], d1[6], d1[7]);
        tmem_st_wait();
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[hf]);
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&ld_empty[s]);
    }
    if (ok && mbar_wait(final_done, 0, p.err, abort_flag)) {
      // warps 4-7 write dV, warps 12-15 write dK
      tc_fence_after();
      uint32_t a0[32], a1[32];
      tmem_ld_32x32b_x32(tmem + lb + 256 + cg * 64, a0);
      tmem_ld_32x32b_x32(tmem + lb + 288 + cg * 64, a1);
      tmem_ld_wait();
      if (key < k1) {
        const float sc = cg ? p.scale : 1.f;
        __nv_bfloat16* dst = p.dqkv + (int64_t)key * p.ld_dqkv + (p.hq + (cg ? 0 : p.hkv) + g) * kHD;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float t[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) t[e] = __uint_as_float(a0[c8 * 8 + e]) * sc;
          uint4 w;
          pack8(t, w.x, w.y, w.z, w.w);
          reinterpret_cast<uint4*>(dst)[c8] = w;
#pragma unroll
          for (int e = 0; e < 8; ++e) t[e] = __uint_as_float(a1[c8 * 8 + e]) * sc;
          pack8(t, w.x, w.y, w.z, w.w);
          reinterpret_cast<uint4*>(dst)[4 + c8] = w;
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

// D[h, i] = sum_d dO[i, h, d] * O[i, h, d]; dsink[h] -= exp(sink_h - lse[h, i]) * D[h, i].
// One block per kPreRows rows; warp w takes heads w, w + 8, ... and walks the block's rows
// (head_dim 64 = 2 elements per lane), summing its sink-gradient terms in a register: one
// atomic per (block, head) instead of one per (row, head), which serialised on the hq words.
constexpr int kPreRows = 64;
__global__ void __launch_bounds__(256)
    attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ out, int64_t ld_out,
                        const __nv_bfloat16* __restrict__ dout, int64_t ld_dout,
                        const float* __restrict__ lse, const float* __restrict__ sinks,
                        float* __restrict__ Dd, float* __restrict__ dsink, int T, int hq) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t r0 = (int64_t)blockIdx.x * kPreRows;
  const int rows = T - r0 < kPreRows ? (int)(T - r0) : kPreRows;
  for (int h = warp; h < hq; h += 8) {
    const float sk = sinks[h];
    float acc = 0.f;
#pragma unroll 4
    for (int k = 0; k < rows; ++k) {
      const int64_t i = r0 + k;
      const __nv_bfloat162 o =
          reinterpret_cast<const __nv_bfloat162*>(out + i * ld_out + h * kHD)[lane];
      const __nv_bfloat162 d =
          reinterpret_cast<const __nv_bfloat162*>(dout + i * ld_dout + h * kHD)[lane];
      const float2 of = __bfloat1622float2(o), df = __bfloat1622float2(d);
      float s = of.x * df.x + of.y * df.y;
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) s += __shfl_xor_sync(0xffffffff, s, m);
      if (lane == 0) {
        Dd[(int64_t)h * T + i] = s;
        acc -= __expf(sk - lse[(int64_t)h * T + i]) * s;
      }
    }
    if (lane == 0) atomicAdd(&dsink[h], acc);
  }
}

// dqkv[:, q part] = bf16(dq)
__global__ void attn_bwd_post_kernel(const float* __restrict__ dq, __nv_bfloat16* __restrict__ dqkv,
                                     int64_t ld, int64_t T, int qcols) {
  const int64_t n = T * qcols / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(dq)[i];
    const int64_t row = (i * 4) / qcols, col = (i * 4) % qcols;
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(dqkv + row * ld + col);
    o[0] = __floats2bfloat162_rn(v.x, v.y);
    o[1] = __floats2bfloat162_rn(v.z, v.w);
  }
}

}  // namespace attnb

void attn_bwd(torch::Tensor qkv, torch::Tensor sinks, torch::Tensor kv_tiles, torch::Tensor cu,
              torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor dqkv,
              torch::Tensor dsinks, int64_t hq, int64_t hkv, int64_t d, int64_t window,
              double scale) {
  using namespace attnb;
  check_cuda_bf16(qkv, "qkv");
  check_cuda_bf16(dout, "dout");
  check_cuda_bf16(dqkv, "dqkv");
  AF3_CHECK(d == kHD, "attention backward is built for head_dim 64");
  AF3_CHECK(dout.stride(1) == 1 && out.stride(1) == 1 && dqkv.stride(1) == 1, "unit inner strides");
  AF3_CHECK(kv_tiles.size(1) == 4, "kv_tiles must be [n, 4]");
  const int64_t T = qkv.size(0);
  const int64_t n_tiles = kv_tiles.size(0);
  const c10::cuda::CUDAGuard guard(qkv.device());
  if (T == 0 || n_tiles == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto Dd = torch::empty({hq, T}, qkv.options().dtype(torch::kFloat32));
  auto dq = torch::zeros({T, hq * kHD}, qkv.options().dtype(torch::kFloat32));
  {
    attn_bwd_pre_kernel<<<(unsigned)((T + kPreRows - 1) / kPreRows), 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), out.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
        lse.data_ptr<float>(), sinks.data_ptr<float>(), Dd.data_ptr<float>(),
        dsinks.data_ptr<float>(), (int)T, (int)hq);
    AF3_CUDA_CHECK(cudaGetLastError());
  }
  const uint64_t dims[2] = {(uint64_t)qkv.size(1), (uint64_t)T};
  const uint64_t strides[1] = {(uint64_t)qkv.stride(0) * 2};
  const uint32_t box[2] = {64, 128};
  CUtensorMap tq = make_tmap(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides,
                             box, CU_TENSOR_MAP_SWIZZLE_128B);
  const uint64_t ddims[2] = {(uint64_t)dout.size(1), (uint64_t)T};
  const uint64_t dstrides[1] = {(uint64_t)dout.stride(0) * 2};
  CUtensorMap tdo = make_tmap(dout.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ddims,
                              dstrides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  // dQ accumulator: fp32 [T, hq*64]; boxes of 32 rows x 32 columns (128 B, the swizzle span)
  const uint64_t qdims[2] = {(uint64_t)(hq * kHD), (uint64_t)T};
  const uint64_t qstrides[1] = {(uint64_t)(hq * kHD * 4)};
  const uint32_t qbox[2] = {32, 32};
  CUtensorMap tdq = make_tmap(dq.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, qdims, qstrides,
                              qbox, CU_TENSOR_MAP_SWIZZLE_128B);
  Params p;
  p.tiles = kv_tiles.data_ptr<int>();
  p.lse = lse.data_ptr<float>();
  p.Dd = Dd.data_ptr<float>();
  p.dq = dq.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.ld_dqkv = dqkv.stride(0);
  p.T = (int)T;
  p.hq = (int)hq;
  p.hkv = (int)hkv;
  p.window = (int)window;
  p.scale = (float)scale;
  p.scale_log2 = (float)scale * kLog2e;
  p.err = device_error_ptr();
  const int smem = Smem::TOTAL + 1024;
  static bool attr[64] = {};
  int dev;
  AF3_CUDA_CHECK(cudaGetDevice(&dev));
  if (!attr[dev]) {
    AF3_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  dim3 grid((unsigned)hkv, (unsigned)n_tiles);
  attn_bwd_kernel<<<grid, kThreads, smem, stream>>>(tq, tdo, tdq, p);
  AF3_CUDA_CHECK(cudaGetLastError());
  const int64_t n4 = T * hq * kHD / 4;
  attn_bwd_post_kernel<<<std::min<int64_t>((n4 + 255) / 256, num_sms() * 16), 256, 0, stream>>>(
      dq.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), dqkv.stride(0), T,
      (int)(hq * kHD));
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
