// MXFP4 MoE expert GEMM for small token counts per expert (rollout decode), sm_100a.
//
// For every expert e with n_e routed rows (rows [offsets[e], offsets[e] + counts[e]) of the
// expert-sorted activations X):
//     Y[rows, f] = epilogue( sum_k W_e[f, k] * X[rows, k] + bias[e, f] )
// with W_e stored as MXFP4 (blocks [E, N, K/32, 16] u8 e2m1 pairs, scales [E, N, K/32] u8).
//
// "Swap-AB": the tensor-core M dimension runs over 128 weight rows (output features) and N over
// the few tokens of the expert (BN = 16..128), so a decode batch with a handful of tokens per
// expert does not pad every expert to 128 token rows, and only experts that received tokens
// are read.  The kernel is bound by reading the packed weights (4.25 bits per weight).
//
// The tile runs in f16: e2m1 -> f16 is one hardware conversion per byte, every e2m1 value times
// a block scale 2^(s-127) with s in [104, 140] is an exact f16 number, and bf16 activations in
// the f16 range convert exactly -- so the products are those of the bf16 dequantised weights.
// The host checks the scale range once per weight tensor and uses the dequantise path
// otherwise; it also converts the token rows to f16 once (a small kernel) so that TMA can feed
// them to the tensor core unchanged.
//
// The converted weight tile never touches shared memory: the tensor core reads its A operand
// from tensor memory (tcgen05.mma with A in TMEM, two f16 per 32-bit column, row = TMEM lane),
// and each converter thread owns one TMEM lane, so it stores its row with tcgen05.st.  Shared
// memory carries only the packed 4-bit bytes and the token tile; a design that staged the f16
// tile in shared memory spent 16 KB of writes and 16 KB of MMA reads per 4 KB of packed
// weights and was bound by shared-memory bandwidth.
//
// Warp roles (1024 threads, persistent CTAs over tiles (expert, 128-feature tile, token tile)):
//   warp 0      TMA: packed weight rows [128 x 32 bytes] per 64-wide K block into a 32-stage
//               ring (128 KB in flight per SM: above the latency x bandwidth product of HBM)
//   warp 3      TMA: the f16 token tile [BN x 64] per K block into its own ring; each tile's
//               e8m0 scales (one contiguous block) by a bulk copy into a double buffer.  With
//               LoRA, ceil(r/64) more K blocks follow: the rows' x A_e^T * scale as the token
//               tile and the expert's LoRA up-projection rows as the weight tile (loaded by
//               the converters), so the low-rank term accumulates into the same TMEM tile
//   warp 1      tcgen05.mma (kind::f16, A from TMEM, M=128, N=BN, K=16 x 4 per block) into a
//               double-buffered TMEM accumulator
//   warps 4-27  converters, six groups of four warps; group g converts the K blocks
//               it = g (mod 6), so six blocks are in flight and the conversion latency of one
//               overlaps the others (the converters are issue-bound: more of them keep the
//               schedulers busier).  Thread (warp % 4, lane) owns weight row 32 (warp % 4) +
//               lane: 32 packed bytes -> 64 f16 -> 32 TMEM columns of a 6- or 12-stage ring
//   warps 28-31 epilogue: thread t owns feature row t; bias, then clamped SwiGLU (gate / up are
//               interleaved rows 2i / 2i+1, partner taken with a lane shuffle) or a per-row
//               router-gate scale; bf16 stores of Y[token, feature]
#include "common.h"
#include "host_utils.h"
#include "mxfp4.cuh"
#include "sm100.cuh"

namespace af3 {
namespace mxm {

constexpr int kThreads = 1024;
constexpr int kGroups = 6;          // converter groups of four warps (warps 4-27)
constexpr int kEpiWarp = 4 + 4 * kGroups;   // warps 28-31: epilogue
constexpr int kMaxScaleCols = 96;   // K / 32 <= 96 (K <= 3072)
constexpr int kBM = 128;    // weight rows per tile
constexpr int kBK = 64;     // K per pipeline stage (one 128-byte f16 swizzle row)
constexpr int kPackStages = 32;   // packed-weight stages (TMA: latency x bandwidth)
constexpr int kMaxExperts = 512;
constexpr int kTmemCols = 512;    // [0, 2 BN) accumulators, [kACol, 512) A stages

enum Epi : int { kSwiglu = 0, kRowScale = 1 };

struct Params {
  int N, K, E;                // W_e is [N, K]; N output features
  int K2;                     // LoRA rank (0 = none): extra K blocks from (lora_b, xa)
  const __nv_bfloat16* lora_b;  // [E, N, K2] bf16
  const int* offsets;         // [E+1] segment starts of the sorted rows
  const int* counts;          // [E] rows per expert
  const uint8_t* scales;      // [E, N, K/32]
  const float* bias;          // [E, N] or null
  const float* row_scale;     // [R] (kRowScale)
  __nv_bfloat16* out;         // kSwiglu: [R, N/2]; kRowScale: [R, N]
  int64_t ldo;
  float act_alpha, act_limit;
  int* err;
  int int_cvt;                // 1: integer e2m1 -> f16 conversion (scales <= 128), 0: cvt
};

template <int BN>
struct Cfg {
  static constexpr int PACK = kBM * kBK / 2;        // 4 KB packed fp4
  static constexpr int X = BN * kBK * 2;            // f16 token tile (SW128)
  static constexpr int X_STAGES = BN <= 32 ? 16 : (BN == 64 ? 8 : 4);   // TMA-filled ring
  static constexpr int X_RING = 0;
  static constexpr int PACK_RING = X_RING + X_STAGES * X;
  static constexpr int BARS = PACK_RING + kPackStages * PACK;
  // converted-weight stages in TMEM (32 columns each): two per converter group when the
  // accumulators leave room, else one
  static constexpr int A_STAGES = BN <= 64 ? 2 * kGroups : kGroups;
  static constexpr int ACOL = kTmemCols - A_STAGES * 32;
  static constexpr int BAR_BYTES = 2048;
  // expert tile prefix, padded so the scale buffers after it stay 128-byte aligned (the bulk
  // copy that fills them needs a 16-byte aligned destination)
  static constexpr int PREFIX = ((kMaxExperts + 1) * 4 + 127) / 128 * 128;
  static constexpr int SCALES = kBM * kMaxScaleCols;   // one tile's e8m0 scales
  static constexpr int SMEM = 1024 + BARS + BAR_BYTES + PREFIX + 2 * SCALES;   // double-buffered
  static_assert((BARS + BAR_BYTES + PREFIX) % 16 == 0 && SCALES % 16 == 0, "bulk copy alignment");
  static_assert((2 * A_STAGES + 2 * X_STAGES + 2 * kPackStages + 8) * 8 + 8 <= BAR_BYTES,
                "barrier area");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(2 * BN <= ACOL, "accumulators overlap the A stages");
};

struct Tile {
  int e, f0, n0, n_valid, row0;
};

// Tile t -> (expert, feature tile, token tile).  Token tiles of one (expert, feature tile)
// are consecutive, so CTAs running them at the same time share the weight tile through L2.
// prefix[e] = tiles before expert e.
template <int BN>
__device__ __forceinline__ bool tile_of(int t, const Params& p, const int* prefix, Tile& tile) {
  if (t >= prefix[p.E]) return false;
  int lo = 0, hi = p.E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int e = lo, local = t - prefix[e];
  const int cnt = p.counts[e];
  const int nt = (cnt + BN - 1) / BN;
  tile.e = e;
  tile.n0 = (local % nt) * BN;
  tile.f0 = (local / nt) * kBM;
  tile.n_valid = min(BN, cnt - tile.n0);
  tile.row0 = p.offsets[e] + tile.n0;
  return true;
}

__device__ __forceinline__ float silu_clamped(float g, float u, float alpha, float limit) {
  const float gc = fminf(g, limit);
  const float uc = fminf(fmaxf(u, -limit), limit);
  return gc / (1.0f + __expf(-alpha * gc)) * (uc + 1.0f);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    moe_mxfp4_kernel(const __grid_constant__ CUtensorMap tma_w,   // [E][N][K/2] bytes
                     const __grid_constant__ CUtensorMap tma_x,   // [R][K] f16
                     const __grid_constant__ CUtensorMap tma_x2,  // [R][r] f16 (x A^T s)
                     const Params p) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BARS);
  uint64_t* a_full = bars;                                   // [A_STAGES] converters done
  uint64_t* a_empty = a_full + C::A_STAGES;                  // [A_STAGES] MMA done
  uint64_t* x_full = a_empty + C::A_STAGES;                  // [X_STAGES] TMA landed
  uint64_t* x_empty = x_full + C::X_STAGES;                  // [X_STAGES] MMA done
  uint64_t* pack_full = x_empty + C::X_STAGES;               // [kPackStages] TMA landed
  uint64_t* pack_empty = pack_full + kPackStages;            // [kPackStages] converters read
  uint64_t* acc_full = pack_empty + kPackStages;             // [2]
  uint64_t* acc_empty = acc_full + 2;                        // [2]
  uint64_t* sc_full = acc_empty + 2;                         // [2] tile scales landed
  uint64_t* sc_empty = sc_full + 2;                          // [2] converters done with them
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* prefix = reinterpret_cast<int*>(smem + C::BARS + C::BAR_BYTES);
  uint8_t* tile_scales = smem + C::BARS + C::BAR_BYTES + C::PREFIX;   // [2][SCALES]

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ft = (p.N + kBM - 1) / kBM;
  const int kb_w = p.K / kBK;                          // MXFP4 blocks
  const int kb_n = kb_w + (p.K2 + kBK - 1) / kBK;      // + LoRA blocks

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_w);
    tma_prefetch_desc(&tma_x);
    if (p.K2 > 0) tma_prefetch_desc(&tma_x2);
    for (int s = 0; s < C::A_STAGES; ++s) {
      mbar_init(&a_full[s], 4);   // the four warps of the converting group
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < C::X_STAGES; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < kPackStages; ++s) {
      mbar_init(&pack_full[s], 1);
      mbar_init(&pack_empty[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
      mbar_init(&sc_full[b], 1);
      mbar_init(&sc_empty[b], 4 * kGroups);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2 && lane == 0) {
    int acc = 0;
    for (int e = 0; e < p.E; ++e) {
      prefix[e] = acc;
      acc += ((p.counts[e] + BN - 1) / BN) * ft;
    }
    prefix[p.E] = acc;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------ TMA producer: packed weights ----------------------------
    if (elect_one_sync()) {
      int ip = 0;
      bool ok = true;
      Tile tl;
      for (int t = blockIdx.x; ok && tile_of<BN>(t, p, prefix, tl); t += gridDim.x) {
        for (int kb = 0; kb < kb_w; ++kb, ++ip) {
          const int s = ip % kPackStages;
          if (!mbar_wait(&pack_empty[s], ((ip / kPackStages) & 1) ^ 1, p.err, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&pack_full[s], C::PACK);
          tma_load_3d(smem + C::PACK_RING + s * C::PACK, &tma_w, &pack_full[s], kb * (kBK / 2),
                      tl.f0, tl.e);
        }
      }
    }
  } else if (warp == 3) {
    // ------------------- TMA producer: token tiles (and x A^T s), scales ----------------
    if (elect_one_sync()) {
      int ix = 0, tc = 0;
      bool ok = true;
      Tile tl;
      const int kblk = p.K / 32;
      for (int t = blockIdx.x; ok && tile_of<BN>(t, p, prefix, tl); t += gridDim.x, ++tc) {
        // the tile's e8m0 scales: rows f0.. of expert e are one contiguous block
        const int b = tc & 1;
        if (!mbar_wait(&sc_empty[b], ((tc >> 1) & 1) ^ 1, p.err, abort_flag)) break;
        const uint32_t bytes = (uint32_t)(min(kBM, p.N - tl.f0) * kblk);
        mbar_arrive_expect_tx(&sc_full[b], bytes);
        bulk_load(tile_scales + b * C::SCALES, p.scales + ((int64_t)tl.e * p.N + tl.f0) * kblk,
                  bytes, &sc_full[b]);
        for (int kb = 0; kb < kb_n; ++kb, ++ix) {
          const int s = ix % C::X_STAGES;
          if (!mbar_wait(&x_empty[s], ((ix / C::X_STAGES) & 1) ^ 1, p.err, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&x_full[s], C::X);
          uint8_t* dst = smem + C::X_RING + s * C::X;
          if (kb < kb_w) tma_load_2d(dst, &tma_x, &x_full[s], kb * kBK, tl.row0);
          else tma_load_2d(dst, &tma_x2, &x_full[s], (kb - kb_w) * kBK, tl.row0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer --------------------------------------
    if (elect_one_sync()) {
      constexpr uint32_t idesc = make_idesc_f16(kBM, BN, false, false);
      int it = 0, tc = 0;
      bool ok = true;
      Tile tl;
      for (int t = blockIdx.x; ok && tile_of<BN>(t, p, prefix, tl); t += gridDim.x, ++tc) {
        const int b = tc & 1;
        if (!mbar_wait(&acc_empty[b], ((tc >> 1) & 1) ^ 1, p.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * BN;
        for (int kb = 0; kb < kb_n; ++kb, ++it) {
          const int sa = it % C::A_STAGES, sx = it % C::X_STAGES;
          if (!mbar_wait(&a_full[sa], (it / C::A_STAGES) & 1, p.err, abort_flag) ||
              !mbar_wait(&x_full[sx], (it / C::X_STAGES) & 1, p.err, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = tmem + C::ACOL + sa * 32;
          const uint32_t x0 = smem_u32(smem + C::X_RING + sx * C::X);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            umma_f16_tmem_a(d, a0 + kk * 8, make_smem_desc(x0 + kk * 32, 16, 1024, kLayoutSW128),
                            idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&a_empty[sa]);
          umma_commit(&x_empty[sx]);
        }
        if (ok) umma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= 4 && warp < kEpiWarp) {
    // ------------------------- MXFP4 -> f16 converters --------------------------------
    const int g = (warp - 4) >> 2;             // group: converts the K blocks it = g (mod kGroups)
    const int q = warp & 3;                    // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;               // weight row of the tile = TMEM lane
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int kblk = p.K / 32;
    int it_base = 0, ip_base = 0, tc = 0;   // blocks / packed blocks of the earlier tiles
    bool ok = true;
    Tile tl;
    for (int t = blockIdx.x; ok && tile_of<BN>(t, p, prefix, tl); t += gridDim.x, ++tc) {
      const int b = tc & 1;
      if (!mbar_wait(&sc_full[b], (tc >> 1) & 1, p.err, abort_flag)) break;
      const uint8_t* my_scales = tile_scales + b * C::SCALES + r * kblk;
      const int f = tl.f0 + r;
      const bool row_ok = f < p.N;
      // this group's blocks of the tile: global block index it = g (mod kGroups)
      for (int kb = ((g - it_base) % kGroups + kGroups) % kGroups; kb < kb_n; kb += kGroups) {
        const int it = it_base + kb;
        const int ip = ip_base + kb;            // packed-ring index (MXFP4 blocks only)
        const bool mx = kb < kb_w;
        const int sa = it % C::A_STAGES;
        // the TMEM stage is free once the MMA of the block A_STAGES earlier has finished
        if (!mbar_wait(&a_empty[sa], ((it / C::A_STAGES) & 1) ^ 1, p.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ta = tmem + lane_base + C::ACOL + sa * 32;
        uint32_t v[16];
        if (mx) {
          // 32 packed bytes (64 values) of row r: two scale blocks -> 32 TMEM columns
          const int ps = ip % kPackStages;
          if (!mbar_wait(&pack_full[ps], (ip / kPackStages) & 1, p.err, abort_flag)) { ok = false; break; }
          const uint4* src = reinterpret_cast<const uint4*>(smem + C::PACK_RING + ps * C::PACK + r * 32);
          const uint4 w0 = src[0], w1 = src[1];
          __syncwarp();                        // the warp's packed bytes are in registers
          if (lane == 0) mbar_arrive(&pack_empty[ps]);
          const uint32_t r0 = row_ok ? my_scales[2 * kb] : 127u;
          const uint32_t r1 = row_ok ? my_scales[2 * kb + 1] : 127u;
          if (p.int_cvt) {
            e2m1x32_to_f16x32_int(w0, e8m0_to_f16x2_int_scale(r0), v);
            tmem_st_32x32b_x16(ta, v);
            e2m1x32_to_f16x32_int(w1, e8m0_to_f16x2_int_scale(r1), v);
            tmem_st_32x32b_x16(ta + 16, v);
          } else {
            e2m1x32_to_f16x32(w0, e8m0_to_f16_bits(r0), v);
            tmem_st_32x32b_x16(ta, v);
            e2m1x32_to_f16x32(w1, e8m0_to_f16_bits(r1), v);
            tmem_st_32x32b_x16(ta + 16, v);
          }
        } else {
          // LoRA block: row f of B_e (bf16, K2 wide) -> f16; zeros past K2 and past N
          const int k2 = (kb - kb_w) * kBK;
          const __nv_bfloat16* src = p.lora_b + ((int64_t)tl.e * p.N + (row_ok ? f : 0)) * p.K2;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int k = k2 + h * 32 + j * 8;
              uint4 c = make_uint4(0, 0, 0, 0);
              if (row_ok && k < p.K2) c = bf16x8_to_f16x8(__ldg(reinterpret_cast<const uint4*>(src + k)));
              v[4 * j] = c.x;
              v[4 * j + 1] = c.y;
              v[4 * j + 2] = c.z;
              v[4 * j + 3] = c.w;
            }
            tmem_st_32x32b_x16(ta + 16 * h, v);
          }
        }
        tmem_st_wait();                        // this thread's TMEM stores have landed
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
      }
      it_base += kb_n;
      ip_base += kb_w;
      __syncwarp();                            // this warp is done with the tile's scales
      if (ok && lane == 0) mbar_arrive(&sc_empty[b]);
    }
  } else if (warp >= kEpiWarp) {
    // ------------------------------------ epilogue -------------------------------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int tc = 0;
    Tile tl;
    for (int t = blockIdx.x; tile_of<BN>(t, p, prefix, tl); t += gridDim.x, ++tc) {
      const int b = tc & 1;
      if (!mbar_wait(&acc_full[b], (tc >> 1) & 1, p.err, abort_flag)) break;
      tc_fence_after();
      const int f = tl.f0 + r;
      const float bias = (p.bias != nullptr && f < p.N) ? p.bias[(int64_t)tl.e * p.N + f] : 0.f;
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(tmem + lane_base + b * BN + c0, v);
        tmem_ld_wait();
        if (c0 + 16 >= BN) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float y = __uint_as_float(v[j]) + bias;
          const int n = c0 + j;
          const int64_t row = tl.row0 + n;
          if (EPI == kSwiglu) {
            // rows 2i (gate) and 2i+1 (up) sit in neighbouring lanes; round to bf16 first,
            // as the training epilogue does
            const float mine = __bfloat162float(__float2bfloat16(y));
            const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
            if ((r & 1) == 0 && n < tl.n_valid && f < p.N)
              p.out[row * p.ldo + f / 2] =
                  __float2bfloat16(silu_clamped(mine, other, p.act_alpha, p.act_limit));
          } else {
            if (n < tl.n_valid && f < p.N)
              p.out[row * p.ldo + f] = __float2bfloat16(p.row_scale[row] * y);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace mxm
}  // namespace af3

namespace af3 {
namespace mxm {

// Token rows bf16 -> contiguous f16 for the kernel's TMA (the tensor core reads both operands
// of kind::f16 as f16).  Only the rows the experts own are converted: rows
// [offsets[e], offsets[e] + counts[e]) for each expert e (block y = expert); the padding rows of
// the segments stay uninitialised -- they only ever feed token columns the epilogue drops.
__global__ void rows_bf16_to_f16_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                        uint4* __restrict__ y, int c8,
                                        const int* __restrict__ offsets,
                                        const int* __restrict__ counts) {
  const int e = blockIdx.y;
  const int64_t r0 = offsets[e];
  const int64_t n = (int64_t)counts[e] * c8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = r0 + i / c8, c = i % c8;
    y[row * c8 + c] = bf16x8_to_f16x8(__ldg(reinterpret_cast<const uint4*>(x + row * ldx) + c));
  }
}

torch::Tensor rows_to_f16(const torch::Tensor& x, const torch::Tensor& offsets,
                          const torch::Tensor& counts, cudaStream_t stream) {
  AF3_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(1) % 8 == 0 && (x.stride(0) * 2) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
            "token rows must be [R, C] with C % 8 == 0 and 16-byte aligned rows");
  auto y = torch::empty({x.size(0), x.size(1)}, x.options().dtype(torch::kHalf));
  const int E = (int)counts.numel();
  if (x.size(0) == 0 || E == 0) return y;
  // rows per expert are few in decode: a handful of blocks per expert covers them
  rows_bf16_to_f16_kernel<<<dim3(4, (unsigned)E), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
      reinterpret_cast<uint4*>(y.data_ptr()), (int)(x.size(1) / 8), offsets.data_ptr<int>(),
      counts.data_ptr<int>());
  AF3_CUDA_CHECK(cudaGetLastError());
  return y;
}

template <int BN, int EPI>
void launch(const CUtensorMap& tw, const CUtensorMap& tx, const CUtensorMap& tx2, const Params& p,
            cudaStream_t stream) {
  static bool attr[64] = {};
  int dev;
  AF3_CUDA_CHECK(cudaGetDevice(&dev));
  const int smem = Cfg<BN>::SMEM;
  if (!attr[dev]) {
    AF3_CUDA_CHECK(cudaFuncSetAttribute(moe_mxfp4_kernel<BN, EPI>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  moe_mxfp4_kernel<BN, EPI><<<num_sms(), kThreads, smem, stream>>>(tw, tx, tx2, p);
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace mxm

// Y = epilogue(X_sorted W_e^T + b_e) for MXFP4 expert weights; see the file comment.
//   x       bf16 [R, K] expert-sorted rows; offsets [E+1], counts [E] int32 (device)
//   blocks  uint8 [E, N, K/32, 16], scales uint8 [E, N, K/32], bias fp32 [E, N] (optional)
//   epi 0   clamped SwiGLU over interleaved (gate, up) rows -> out bf16 [R, N/2]
//   epi 1   row_scale[r] * (...) -> out bf16 [R, N]
//   bn      token tile (16, 32, 64 or 128): ~ the largest number of rows per expert
//   lora_b  optional bf16 [E, N, r] and xa bf16 [R, r] (= x A_e^T * scale): adds xa B_e^T
//   int_cvt 1: integer e2m1 -> f16 conversion, valid when every scale byte is <= 128 (the
//           caller checks); 0: the hardware cvt path (scales <= 140)
void moe_mxfp4_gemm(torch::Tensor x, torch::Tensor blocks, torch::Tensor scales,
                    c10::optional<torch::Tensor> bias, torch::Tensor offsets, torch::Tensor counts,
                    int64_t epi, c10::optional<torch::Tensor> row_scale, torch::Tensor out,
                    double act_alpha, double act_limit, int64_t bn,
                    c10::optional<torch::Tensor> lora_b, c10::optional<torch::Tensor> xa,
                    int64_t int_cvt) {
  using namespace mxm;
  check_cuda_bf16(x, "x");
  check_cuda_bf16(out, "out");
  AF3_CHECK(blocks.scalar_type() == torch::kUInt8 && scales.scalar_type() == torch::kUInt8,
            "blocks / scales must be uint8");
  AF3_CHECK(blocks.dim() == 4 && blocks.size(3) == 16 && blocks.is_contiguous() &&
                scales.is_contiguous(), "blocks must be contiguous [E, N, K/32, 16]");
  const int64_t E = blocks.size(0), N = blocks.size(1), K = blocks.size(2) * 32;
  AF3_CHECK(E <= kMaxExperts, "too many experts");
  AF3_CHECK(K % kBK == 0 && K / 32 <= kMaxScaleCols, "K must be a multiple of 64, at most 3072");
  // a tile's scales are fetched as one bulk copy: 16-byte aligned start and length
  AF3_CHECK((N * (K / 32)) % 16 == 0 && ((N % kBM) * (K / 32)) % 16 == 0 &&
                (kBM * (K / 32)) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(scales.data_ptr()) % 16 == 0,
            "scale rows must allow 16-byte aligned per-tile copies");
  AF3_CHECK(x.dim() == 2 && x.size(1) == K && x.stride(1) == 1, "x must be [R, K] with unit stride");
  AF3_CHECK(scales.numel() == E * N * (K / 32), "scales shape");
  AF3_CHECK(offsets.numel() == E + 1 && counts.numel() == E &&
                offsets.scalar_type() == torch::kInt32 && counts.scalar_type() == torch::kInt32,
            "offsets [E+1] / counts [E] int32");
  AF3_CHECK(epi == kSwiglu || epi == kRowScale, "epi must be 0 (swiglu) or 1 (row scale)");
  AF3_CHECK(out.stride(1) == 1 && out.size(0) == x.size(0) &&
                out.size(1) == (epi == kSwiglu ? N / 2 : N), "out shape");
  if (epi == kSwiglu) AF3_CHECK(N % 2 == 0, "SwiGLU needs an even N");
  if (epi == kRowScale)
    AF3_CHECK(row_scale.has_value() && row_scale->scalar_type() == torch::kFloat32 &&
                  row_scale->numel() >= x.size(0), "row_scale fp32 [R] required");
  if (bias.has_value())
    AF3_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() == E * N &&
                  bias->is_contiguous(), "bias must be contiguous fp32 [E, N]");
  const c10::cuda::CUDAGuard guard(x.device());
  if (x.size(0) == 0) return;
  const uint64_t wd[3] = {(uint64_t)(K / 2), (uint64_t)N, (uint64_t)E};
  const uint64_t ws[2] = {(uint64_t)(K / 2), (uint64_t)(N * K / 2)};
  const uint32_t wb[3] = {kBK / 2, kBM, 1};
  const CUtensorMap tw = make_tmap(blocks.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, wd, ws, wb,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
  auto stream = at::cuda::getCurrentCUDAStream();
  const torch::Tensor x16 = rows_to_f16(x, offsets, counts, stream);
  const uint64_t xd[2] = {(uint64_t)K, (uint64_t)x.size(0)};
  const uint64_t xs[1] = {(uint64_t)K * 2};
  const uint32_t xb[2] = {kBK, (uint32_t)bn};
  const CUtensorMap tx = make_tmap(x16.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xd, xs, xb,
                                   CU_TENSOR_MAP_SWIZZLE_128B);
  int64_t r = 0;
  CUtensorMap tx2 = tx;  // unused without LoRA
  torch::Tensor xa16;     // keeps the converted xa alive until the launch is queued
  if (lora_b.has_value()) {
    AF3_CHECK(xa.has_value(), "xa is required with lora_b");
    check_cuda_bf16(*lora_b, "lora_b");
    check_cuda_bf16(*xa, "xa");
    r = lora_b->size(2);
    AF3_CHECK(lora_b->dim() == 3 && lora_b->size(0) == E && lora_b->size(1) == N &&
                  lora_b->is_contiguous() && (r * 2) % 16 == 0, "lora_b must be [E, N, r], r % 8 == 0");
    AF3_CHECK(xa->dim() == 2 && xa->size(0) == x.size(0) && xa->size(1) == r && xa->stride(1) == 1,
              "xa must be [R, r]");
    xa16 = rows_to_f16(*xa, offsets, counts, stream);
    const uint64_t ad[2] = {(uint64_t)r, (uint64_t)x.size(0)};
    const uint64_t as[1] = {(uint64_t)r * 2};
    tx2 = make_tmap(xa16.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ad, as, xb,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  }
  Params p;
  p.K2 = (int)r;
  p.lora_b = lora_b.has_value() ? reinterpret_cast<const __nv_bfloat16*>(lora_b->data_ptr()) : nullptr;
  p.N = (int)N;
  p.K = (int)K;
  p.E = (int)E;
  p.offsets = offsets.data_ptr<int>();
  p.counts = counts.data_ptr<int>();
  p.scales = scales.data_ptr<uint8_t>();
  p.bias = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  p.row_scale = row_scale.has_value() ? row_scale->data_ptr<float>() : nullptr;
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldo = out.stride(0);
  p.act_alpha = (float)act_alpha;
  p.act_limit = (float)act_limit;
  p.err = device_error_ptr();
  p.int_cvt = int_cvt ? 1 : 0;
#define AF3_MXM(B)                                                                  \
  case B:                                                                           \
    if (epi == kSwiglu) launch<B, kSwiglu>(tw, tx, tx2, p, stream);                 \
    else launch<B, kRowScale>(tw, tx, tx2, p, stream);                              \
    break;
  switch (bn) {
    AF3_MXM(16)
    AF3_MXM(32)
    AF3_MXM(64)
    AF3_MXM(128)
    default: AF3_CHECK(false, "bn must be 16, 32, 64 or 128");
  }
#undef AF3_MXM
}

}  // namespace af3
