// Tensor-parallel all-reduce over NVLink peer memory for the rollout engine (sm_100a), fused
// with the residual add and the RMSNorm that follows it.
//
// In the engine's tensor-parallel decode every rank holds a slice of the attention heads and of
// the experts; after the attention output projection and after the MoE combine, each rank has a
// partial [T, H] sum that must be added over ranks (the reference's rollout engine does this with
// NCCL / a custom all-reduce inside sglang).  Here every rank writes its partial straight into a
// buffer that all ranks have mapped (CUDA IPC; the GEMM / combine kernels take it as their output),
// and ONE kernel per reduction then
//   1. signals its arrival to every rank (release store of the call's epoch into each rank's flag
//      array over NVLink) and waits until all ranks have arrived (acquire loads of its own flags;
//      bounded by a time limit, after which it records an error and returns);
//   2. reads the T x H partials of all ranks over NVLink (16-byte loads, rank order fixed so every
//      rank computes bit-identical sums), adds the residual in fp32, rounds to bf16 -> x;
//   3. RMSNorm of x with the next layer's weight -> xn (one block per row, block reduction).
// Two buffer sets alternate between calls: a rank can only overwrite set s (two calls later)
// after every rank has arrived at the call in between, i.e. after all ranks finished reading s.
#include <cstring>

#include <torch/extension.h>

#include "common.h"
#include "host_utils.h"
#include "sm100.cuh"

namespace af3 {
namespace tpar {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 384;         // H / 8 <= 2 * kThreads  (H <= 6144)
constexpr int kVecPerThread = 2;

struct Params {
  const __nv_bfloat16* bufs[kMaxRanks];   // each rank's partial [T, ld_buf] (peer mappings)
  uint32_t* flags[kMaxRanks];             // each rank's flag array [kMaxRanks] (peer mappings)
  int rank, world;
  uint32_t epoch;
  int64_t ld_buf;
  const __nv_bfloat16* residual;          // [T, ld_res] or null
  int64_t ld_res;
  const float* w;                         // [H] RMSNorm weight or null (no norm output)
  float eps;
  __nv_bfloat16* out_x;                   // [T, ld_out]
  __nv_bfloat16* out_n;                   // [T, ld_out] (when w)
  int64_t ld_out;
  int T, H;
  int* err;
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[2 * i] += __uint_as_float(w[i] << 16);
    acc[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__global__ void __launch_bounds__(kThreads) allreduce_residual_norm_kernel(const Params p) {
  __shared__ int s_ok;
  __shared__ float s_red[kThreads / 32];
  // 1. arrival: every block tells every rank (including itself) that this rank's partial is
  //    ready (the same epoch value, so the repeats are harmless, and no block depends on another
  //    block of this grid being scheduled).  The partial was written by earlier kernels of this
  //    stream, which finished before this one started; the system-scope fence + release store
  //    publish it to the peers.
  if (threadIdx.x < p.world) {
    __threadfence_system();
    st_release_sys(p.flags[threadIdx.x] + p.rank, p.epoch);
  }
  if (threadIdx.x == 0) {
    const uint32_t* mine = p.flags[p.rank];
    int ok = 1;
    const uint64_t t0 = now_ns();
    for (int j = 0; j < p.world && ok; ++j) {
      while ((int32_t)(ld_acquire_sys(mine + j) - p.epoch) < 0) {
        if (now_ns() - t0 > p.timeout_ns) {
          atomicCAS(p.err, 0, kErrPeerTimeout);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int nv = p.H / 8;
  for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
    float x[kVecPerThread][8];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < kVecPerThread; ++u) {
      const int c = threadIdx.x + u * kThreads;
#pragma unroll
      for (int i = 0; i < 8; ++i) x[u][i] = 0.f;
      if (c < nv) {
        if (p.residual != nullptr)
          add_bf16x8(x[u], __ldg(reinterpret_cast<const uint4*>(p.residual + t * p.ld_res) + c));
        for (int j = 0; j < p.world; ++j)
          add_bf16x8(x[u], __ldcg(reinterpret_cast<const uint4*>(p.bufs[j] + t * p.ld_buf) + c));
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          ow[i] = pack_bf16x2(x[u][2 * i], x[u][2 * i + 1]);
          // continue with the rounded values, as a norm of the stored bf16 x would
          x[u][2 * i] = __uint_as_float(ow[i] << 16);
          x[u][2 * i + 1] = __uint_as_float(ow[i] & 0xFFFF0000u);
          ss += x[u][2 * i] * x[u][2 * i] + x[u][2 * i + 1] * x[u][2 * i + 1];
        }
        reinterpret_cast<uint4*>(p.out_x + t * p.ld_out)[c] = o;
      }
    }
    if (p.w == nullptr) continue;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x / 32] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) tot += s_red[i];
    __syncthreads();   // s_red is reused by the next row
    const float rstd = rsqrtf(tot / (float)p.H + p.eps);
#pragma unroll
    for (int u = 0; u < kVecPerThread; ++u) {
      const int c = threadIdx.x + u * kThreads;
      if (c >= nv) continue;
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(p.w) + 2 * c);
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(p.w) + 2 * c + 1);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        ow[i] = pack_bf16x2(wv[2 * i] * (x[u][2 * i] * rstd), wv[2 * i + 1] * (x[u][2 * i + 1] * rstd));
      reinterpret_cast<uint4*>(p.out_n + t * p.ld_out)[c] = o;
    }
  }
}

}  // namespace tpar

namespace py = pybind11;

// A zeroed device buffer of `nbytes` from its own cudaMalloc (so its IPC handle covers exactly
// this buffer) and the 64-byte CUDA IPC handle that lets other processes map it.
std::tuple<torch::Tensor, py::bytes> symm_alloc(int64_t nbytes, int64_t device) {
  AF3_CHECK(nbytes > 0, "symm_alloc: nbytes must be positive");
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* ptr = nullptr;
  AF3_CUDA_CHECK(cudaMalloc(&ptr, (size_t)nbytes));
  AF3_CUDA_CHECK(cudaMemset(ptr, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  AF3_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  auto t = torch::from_blob(
      ptr, {nbytes}, [device](void* q) {
        const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
        cudaFree(q);
      },
      torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device));
  return {t, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

// Map another process's buffer into this process, accessible from the current device (peer
// access is enabled on first use).  Returns the device pointer.
int64_t ipc_open(py::bytes handle) {
  const std::string s = handle;
  AF3_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* ptr = nullptr;
  AF3_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

// Let kernels on the current device access memory of device `peer` in this process.
void enable_peer_access(int64_t peer) {
  int dev = 0;
  AF3_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev == (int)peer) return;
  int can = 0;
  AF3_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, dev, (int)peer));
  AF3_CHECK(can, "device cannot access the peer's memory");
  const cudaError_t e = cudaDeviceEnablePeerAccess((int)peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();   // clear the sticky-free "already enabled" status
    return;
  }
  AF3_CUDA_CHECK(e);
}

void ipc_close(int64_t ptr) {
  AF3_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

// dst (contiguous, current device) <- dst.nbytes() bytes at device address src (this GPU's
// memory or a peer mapping), one async copy on the current stream.
void copy_from_address(int64_t src, torch::Tensor dst) {
  AF3_CHECK(dst.is_cuda() && dst.is_contiguous(), "copy_from_address: dst must be contiguous CUDA");
  const c10::cuda::CUDAGuard guard(dst.device());
  const size_t n = dst.numel() * dst.element_size();
  if (n == 0) return;
  AF3_CUDA_CHECK(cudaMemcpyAsync(dst.data_ptr(), reinterpret_cast<const void*>(src), n,
                                 cudaMemcpyDefault, at::cuda::getCurrentCUDAStream()));
}

// x = residual + sum over ranks of the partials at bufs[j] (+ byte offset), and, with w,
// xn = RMSNorm(x) * w.  bufs / flags: one device address per rank (own + peer mappings).
void tp_allreduce_norm(std::vector<int64_t> bufs, std::vector<int64_t> flags, int64_t rank,
                       int64_t epoch, int64_t ld_buf, c10::optional<torch::Tensor> residual,
                       c10::optional<torch::Tensor> w, double eps, torch::Tensor out_x,
                       c10::optional<torch::Tensor> out_n, int64_t T, int64_t H,
                       double timeout_s) {
  using namespace tpar;
  const int world = (int)bufs.size();
  AF3_CHECK(world >= 1 && world <= kMaxRanks && (int)flags.size() == world, "1..8 ranks");
  AF3_CHECK(rank >= 0 && rank < world, "rank out of range");
  AF3_CHECK(H % 8 == 0 && H / 8 <= kThreads * kVecPerThread, "H must be a multiple of 8, <= 6144");
  check_cuda_bf16(out_x, "out_x");
  AF3_CHECK(out_x.stride(1) == 1 && out_x.size(0) >= T && out_x.size(1) == H, "out_x shape");
  AF3_CHECK(ld_buf % 8 == 0 && out_x.stride(0) % 8 == 0, "row strides must be multiples of 8");
  Params p{};
  for (int j = 0; j < world; ++j) {
    AF3_CHECK(bufs[j] % 16 == 0 && flags[j] % 4 == 0, "buffers must be 16-byte aligned");
    p.bufs[j] = reinterpret_cast<const __nv_bfloat16*>(bufs[j]);
    p.flags[j] = reinterpret_cast<uint32_t*>(flags[j]);
  }
  p.rank = (int)rank;
  p.world = world;
  p.epoch = (uint32_t)epoch;
  p.ld_buf = ld_buf;
  if (residual.has_value()) {
    check_cuda_bf16(*residual, "residual");
    AF3_CHECK(residual->stride(1) == 1 && residual->size(1) == H && residual->stride(0) % 8 == 0,
              "residual shape");
    p.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ld_res = residual->stride(0);
  }
  if (w.has_value()) {
    AF3_CHECK(w->scalar_type() == torch::kFloat32 && w->is_contiguous() && w->numel() == H,
              "norm weight must be fp32 [H]");
    AF3_CHECK(out_n.has_value(), "out_n is required with a norm weight");
    check_cuda_bf16(*out_n, "out_n");
    AF3_CHECK(out_n->stride(0) == out_x.stride(0) && out_n->stride(1) == 1, "out_n layout");
    p.w = w->data_ptr<float>();
    p.out_n = reinterpret_cast<__nv_bfloat16*>(out_n->data_ptr());
  }
  p.eps = (float)eps;
  p.out_x = reinterpret_cast<__nv_bfloat16*>(out_x.data_ptr());
  p.ld_out = out_x.stride(0);
  p.T = (int)T;
  p.H = (int)H;
  p.err = device_error_ptr();
  p.timeout_ns = (uint64_t)(timeout_s * 1e9);
  const c10::cuda::CUDAGuard guard(out_x.device());
  // at least one block even for T == 0 so the arrival is still signalled
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(T, (int64_t)num_sms() * 2));
  allreduce_residual_norm_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
