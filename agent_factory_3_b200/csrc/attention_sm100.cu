// Flash attention for gpt-oss on sm_100a: causal GQA over packed variable-length sequences,
// optional sliding window, learned per-head sinks, head_dim 64.
//
// Forward, one CTA per (128-query tile, q head):
//   warp 0   TMA: Q tile once, then K_j (K-major) and V_j (MN-major, two 64-key boxes)
//            into a 3-stage ring
//   warp 1   tcgen05 issuer: S_j = Q K_j^T into TMEM S[j%2] (M=128, N=128, K=64), and one
//            block later O_j = P_j V_j into TMEM O[j%2] (M=128, N=64, K=128)
//   warps 4-7 softmax: thread t owns query row t; reads S_j with tcgen05.ld, applies the
//            causal / window / sequence masks, online max and row sum in the log2 domain,
//            writes P_j (bf16) into 128B-swizzled shared memory for the PV MMA, and
//            accumulates O = O * 2^(m_old - m_new) + O_j in registers.
//   The sink logit joins the denominator at the end: l += 2^(sink*log2e - m).
//   Outputs: O (bf16) and the natural-log LSE per (head, query), sink included.
//
// Backward, one CTA per (128-key tile, q head): recomputes S^T = K Q^T and P^T, computes
// dP^T = V dO^T, dS^T = P^T (dP^T - D), accumulates dV += P^T dO and dK += dS^T Q in TMEM,
// and reduces dQ += dS K into an fp32 buffer with bulk tensor reduce-add.  dK/dV of the
// q heads sharing a kv head are summed with fp32 atomics.  d(sink_h) = -sum_i p_sink(i) D_i.
//
// Reference semantics: HF transformers eager_attention_forward for gpt-oss (sinks appended to
// the logits, softmax, sink column dropped); sliding window: key j visible from query i iff
// i - j < window.
#include "common.h"
#include "host_utils.h"
#include "sm100.cuh"

namespace af3 {

constexpr int kAttnThreads = 256;
constexpr int kHD = 64;  // head dim
constexpr int kBQ = 128;
constexpr int kBKV = 128;
constexpr int kKVStages = 3;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct AttnFwdSmem {
  // all tiles 1024-aligned
  static constexpr int Q = 0;                                  // 16 KB
  static constexpr int K = Q + kBQ * kHD * 2;                  // 3 x 16 KB
  static constexpr int V = K + kKVStages * kBKV * kHD * 2;     // 3 x 16 KB
  static constexpr int P = V + kKVStages * kBKV * kHD * 2;     // 2 x 32 KB
  static constexpr int BAR = P + 2 * kBQ * kBKV * 2;
  static constexpr int TOTAL = BAR + 1024;
};

struct AttnParams {
  const int* tiles;  // [n, 3] (seq_start, q_start, q_end)
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

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tma_qk,
                    const __grid_constant__ CUtensorMap tma_v, const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AttnFwdSmem::BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;    // [3]
  uint64_t* kv_empty = bars + 4;   // [3]
  uint64_t* s_full = bars + 7;     // [2]
  uint64_t* s_empty = bars + 9;    // [2]
  uint64_t* p_full = bars + 11;    // [2]
  uint64_t* o_full = bars + 13;    // [2]
  uint64_t* o_empty = bars + 15;   // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int h = blockIdx.x;
  const int tile = blockIdx.y;
  const int seq0 = p.tiles[tile * 3 + 0];
  const int q0 = p.tiles[tile * 3 + 1];
  const int q1 = p.tiles[tile * 3 + 2];
  if (q1 <= q0) return;
  const int kvh = h / (p.hq / p.hkv);
  int kv_lo = seq0;
  if (p.window > 0) kv_lo = max(seq0, q0 - p.window + 1);
  const int nb = (q1 - kv_lo + kBKV - 1) / kBKV;

  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_qk);
    tma_prefetch_desc(&tma_v);
    mbar_init(q_full, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 128);
      mbar_init(&p_full[b], 128);
      mbar_init(&o_full[b], 1);
      mbar_init(&o_empty[b], 128);
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
  // TMEM columns: S[0] 0..127, S[1] 128..255, O[0] 256..319, O[1] 320..383

  if (warp == 0) {
    if (elect_one_sync()) {
      mbar_arrive_expect_tx(q_full, kBQ * kHD * 2);
      tma_load_2d(smem + AttnFwdSmem::Q, &tma_qk, q_full, h * kHD, q0);
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
      constexpr uint32_t idesc_s = make_idesc_bf16(kBQ, kBKV, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(kBQ, kHD, false, true);
      const uint32_t sq = smem_u32(smem + AttnFwdSmem::Q);
      bool ok = mbar_wait(q_full, 0, p.err, abort_flag);
      for (int j = 0; ok && j <= nb; ++j) {
        if (j < nb) {
          const int s = j % kKVStages;
          if (!mbar_wait(&kv_full[s], (j / kKVStages) & 1, p.err, abort_flag)) break;
          if (!mbar_wait(&s_empty[j & 1], ((j >> 1) & 1) ^ 1, p.err, abort_flag)) break;
          tc_fence_after();
          const uint32_t sk = smem_u32(smem + AttnFwdSmem::K + s * kBKV * kHD * 2);
#pragma unroll
          for (int kk = 0; kk < kHD / 16; ++kk) {
            umma_f16(tmem + (j & 1) * kBKV, make_smem_desc(sq + kk * 32, 16, 1024, kLayoutSW128),
                     make_smem_desc(sk + kk * 32, 16, 1024, kLayoutSW128), idesc_s, kk > 0);
          }
          umma_commit(&s_full[j & 1]);
        }
        if (j >= 1) {
          const int i = j - 1;
          const int s = i % kKVStages;
          if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, p.err, abort_flag)) break;
          if (!mbar_wait(&o_empty[i & 1], ((i >> 1) & 1) ^ 1, p.err, abort_flag)) break;
          tc_fence_after();
          const uint32_t sp = smem_u32(smem + AttnFwdSmem::P + (i & 1) * kBQ * kBKV * 2);
          const uint32_t sv = smem_u32(smem + AttnFwdSmem::V + s * kBKV * kHD * 2);
#pragma unroll
          for (int kk = 0; kk < kBKV / 16; ++kk) {
            const uint64_t ad =
                make_smem_desc(sp + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024, kLayoutSW128);
            const uint64_t bd =
                make_smem_desc(sv + (kk / 4) * 8192 + (kk % 4) * 2048, 8192, 1024, kLayoutSW128);
            umma_f16(tmem + 256 + (i & 1) * kHD, ad, bd, idesc_o, kk > 0);
          }
          umma_commit(&o_full[i & 1]);
          umma_commit(&kv_empty[s]);
        }
      }
    }
  } else if (warp >= 4) {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int qi = q0 + row;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float o_acc[kHD];
#pragma unroll
    for (int d = 0; d < kHD; ++d) o_acc[d] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, m_acc = -INFINITY;
    float m_hist[2] = {-INFINITY, -INFINITY};
    uint8_t* pbase = smem + AttnFwdSmem::P;
    bool ok = true;
    for (int j = 0; j <= nb && ok; ++j) {
      if (j < nb) {
        if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        float sv[kBKV];
        {
          uint32_t r0[32], r1[32], r2[32], r3[32];
          const uint32_t ta = tmem + lane_base + (j & 1) * kBKV;
          tmem_ld_32x32b_x32(ta, r0);
          tmem_ld_32x32b_x32(ta + 32, r1);
          tmem_ld_32x32b_x32(ta + 64, r2);
          tmem_ld_32x32b_x32(ta + 96, r3);
          tmem_ld_wait();
          // raw scores; the softmax scale is applied inside the exp2 argument (one FFMA)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            sv[e] = __uint_as_float(r0[e]);
            sv[32 + e] = __uint_as_float(r1[e]);
            sv[64 + e] = __uint_as_float(r2[e]);
            sv[96 + e] = __uint_as_float(r3[e]);
          }
        }
        tc_fence_before();
        mbar_arrive(&s_empty[j & 1]);
        // masks
        const int k0 = kv_lo + j * kBKV;
        const bool need_mask = (k0 + kBKV - 1 > q0) || (k0 < seq0) ||
                               (p.window > 0 && q0 + kBQ - 1 - k0 >= p.window);
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < kBKV; ++c) {
            const int kj = k0 + c;
            const bool vis = kj <= qi && kj >= seq0 && (p.window == 0 || qi - kj < p.window);
            if (!vis) sv[c] = -INFINITY;
          }
        }
        // row max as a tree of independent chains (raw score units)
        float mxp[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) mxp[t] = sv[t];
#pragma unroll
        for (int c = 8; c < kBKV; c += 8) {
#pragma unroll
          for (int t = 0; t < 8; ++t) mxp[t] = fmaxf(mxp[t], sv[c + t]);
        }
        float mraw = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                           fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
        const float mx = fmaxf(m_run, mraw * p.scale_log2);
        const float m_use = (mx == -INFINITY) ? 0.f : mx;
        const float alpha = ex2(m_run - m_use);  // m_run = -inf -> 0
        float rsp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        // P_j -> shared memory (bf16, 128B swizzle, two 64-key column blocks)
        uint8_t* prow = pbase + (j & 1) * kBQ * kBKV * 2 + row * 128;
#pragma unroll
        for (int c8 = 0; c8 < kBKV / 8; ++c8) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            pv[e] = ex2(fmaf(sv[c8 * 8 + e], p.scale_log2, -m_use));
            rsp[e] += pv[e];
          }
          uint4 w;
          w.x = pack_bf16x2(pv[0], pv[1]);
          w.y = pack_bf16x2(pv[2], pv[3]);
          w.z = pack_bf16x2(pv[4], pv[5]);
          w.w = pack_bf16x2(pv[6], pv[7]);
          const int blk = c8 >> 3, ch = (c8 & 7) ^ (row & 7);
          *reinterpret_cast<uint4*>(prow + blk * 16384 + ch * 16) = w;
        }
        const float rs = ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
        l_run = l_run * alpha + rs;
        m_run = mx;
        m_hist[j & 1] = m_use;
        fence_proxy_async_smem();
        mbar_arrive(&p_full[j & 1]);
      }
      if (j >= 1) {
        const int i = j - 1;
        if (!mbar_wait(&o_full[i & 1], (i >> 1) & 1, p.err, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const float mi = m_hist[i & 1];
        const float sc = (m_acc == -INFINITY) ? 0.f : ex2(m_acc - mi);
#pragma unroll
        for (int c = 0; c < kHD / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_base + 256 + (i & 1) * kHD + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e)
            o_acc[c * 32 + e] = o_acc[c * 32 + e] * sc + __uint_as_float(r[e]);
        }
        m_acc = mi;
        tc_fence_before();
        mbar_arrive(&o_empty[i & 1]);
      }
    }
    if (ok && qi < q1) {
      // o_acc is relative to m_acc (= last block's m_use); l_run relative to m_run
      const float m_fin = (m_run == -INFINITY) ? 0.f : m_run;
      const float sink = p.sinks[h] * kLog2e;
      const float l_tot = l_run + ex2(sink - m_fin);
      const float inv = 1.f / l_tot;
      const float osc = ex2(m_acc - m_fin) * inv;
      __nv_bfloat16* orow = p.out + (int64_t)qi * p.ld_out + h * kHD;
#pragma unroll
      for (int c8 = 0; c8 < kHD / 8; ++c8) {
        uint4 w;
        w.x = pack_bf16x2(o_acc[c8 * 8 + 0] * osc, o_acc[c8 * 8 + 1] * osc);
        w.y = pack_bf16x2(o_acc[c8 * 8 + 2] * osc, o_acc[c8 * 8 + 3] * osc);
        w.z = pack_bf16x2(o_acc[c8 * 8 + 4] * osc, o_acc[c8 * 8 + 5] * osc);
        w.w = pack_bf16x2(o_acc[c8 * 8 + 6] * osc, o_acc[c8 * 8 + 7] * osc);
        *reinterpret_cast<uint4*>(orow + c8 * 8) = w;
      }
      p.lse[(int64_t)h * p.T + qi] = (m_fin + __log2f(l_tot)) * kLn2;
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
  static bool attr[64] = {};
  int dev;
  AF3_CUDA_CHECK(cudaGetDevice(&dev));
  if (!attr[dev]) {
    AF3_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  dim3 grid((unsigned)hq, (unsigned)n_tiles);
  attn_fwd_kernel<<<grid, kAttnThreads, smem, at::cuda::getCurrentCUDAStream()>>>(tqk, tv, p);
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
