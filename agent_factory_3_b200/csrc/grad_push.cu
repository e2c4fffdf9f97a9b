// Reduce-scatter of the data-parallel LoRA gradient, overlapped with the backward pass.
//
// Every rank owns one contiguous shard of the flat fp32 gradient (the sharded AdamW state).
// Each rank has an "inbox" that all ranks have mapped (CUDA IPC): a 256-byte flag area, then
// one slot per source rank of the owner's shard size.  During the backward of the step's last
// microbatch, as soon as a parameter's gradient is final, the trainer copies its pieces into
// the owners' inboxes (slot = this rank) with the copy engines over NVLink, on a side stream,
// so the transfer overlaps the rest of the backward and takes no SM time.  At the end:
//   grad_signal : after this rank's last copy, publish the step's epoch into every owner's flag
//                 word for this rank (system-scope fence + release store over NVLink);
//   grad_reduce : wait (bounded) until every rank's epoch has arrived in this rank's flags, then
//                 sum the slots of the inbox in rank order (bit-identical on every run) into the
//                 local shard gradient and accumulate its sum of squares (the gradient norm).
// Reuse of an inbox by the next step is ordered by the collective that follows the optimizer
// step (the all-gather of the updated shards): no rank starts the next backward before every
// rank has finished its reduction.
#include <torch/extension.h>

#include "common.h"
#include "host_utils.h"
#include "sm100.cuh"

namespace af3 {
namespace gpush {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct SignalParams {
  uint32_t* flags[kMaxRanks];   // each owner's flag area (peer mappings; own for r == rank)
  int rank, world;
  uint32_t epoch;
};

__global__ void grad_signal_kernel(const SignalParams p) {
  if (threadIdx.x < p.world) {
    __threadfence_system();
    st_release_sys(p.flags[threadIdx.x] + p.rank, p.epoch);
  }
}

__global__ void __launch_bounds__(kThreads) grad_reduce_kernel(
    const float4* __restrict__ inbox, const uint32_t* flags, int world, uint32_t epoch,
    int64_t shard_vec, float4* __restrict__ out, float* __restrict__ sumsq, int* err,
    uint64_t timeout_ns) {
  __shared__ int s_ok;
  __shared__ float s_red[kThreads / 32];
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int j = 0; j < world && ok; ++j) {
      while ((int32_t)(ld_acquire_sys(flags + j) - epoch) < 0) {
        if (globaltimer_ns() - t0 > timeout_ns) {
          atomicCAS(err, 0, kErrPeerTimeout);
          ok = 0;
          break;
        }
        __nanosleep(256);
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  float ss = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < shard_vec;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = __ldcs(inbox + i);
    for (int j = 1; j < world; ++j) {
      const float4 b = __ldcs(inbox + (int64_t)j * shard_vec + i);
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    out[i] = a;
    ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) t += s_red[i];
    atomicAdd(sumsq, t);
  }
}

}  // namespace gpush

// Release-store `epoch` into every owner's flag word for this rank (after everything this
// stream did before, e.g. the copies into the owners' inboxes).
void grad_signal(std::vector<int64_t> flag_ptrs, int64_t rank, int64_t epoch) {
  using namespace gpush;
  const int world = (int)flag_ptrs.size();
  AF3_CHECK(world >= 1 && world <= kMaxRanks, "grad_signal: 1..8 ranks");
  AF3_CHECK(rank >= 0 && rank < world, "grad_signal: bad rank");
  SignalParams p{};
  for (int j = 0; j < world; ++j) p.flags[j] = reinterpret_cast<uint32_t*>(flag_ptrs[j]);
  p.rank = (int)rank;
  p.world = world;
  p.epoch = (uint32_t)epoch;
  grad_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  AF3_CUDA_CHECK(cudaGetLastError());
}

// out[i] = sum over j of inbox[j * S + i] (S = out.numel()), sumsq += sum of out^2, after every
// rank's flag in `flags` (this rank's flag area) has reached `epoch`.  On time-out the kernel
// writes nothing and records kErrPeerTimeout in the device error word.
void grad_reduce(int64_t inbox_ptr, int64_t flags_ptr, int64_t world, int64_t epoch,
                 torch::Tensor out, torch::Tensor sumsq, double timeout_s) {
  using namespace gpush;
  AF3_CHECK(out.is_cuda() && out.scalar_type() == torch::kFloat32 && out.is_contiguous(),
            "grad_reduce: out must be contiguous fp32 CUDA");
  AF3_CHECK(sumsq.is_cuda() && sumsq.scalar_type() == torch::kFloat32 && sumsq.numel() == 1,
            "grad_reduce: sumsq must be one fp32 element");
  AF3_CHECK(out.numel() % 4 == 0, "grad_reduce: shard size must be a multiple of 4");
  AF3_CHECK(inbox_ptr % 16 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
            "grad_reduce: 16-byte aligned buffers required");
  AF3_CHECK(world >= 1 && world <= kMaxRanks, "grad_reduce: 1..8 ranks");
  const c10::cuda::CUDAGuard guard(out.device());
  const int64_t vec = out.numel() / 4;
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((vec + kThreads - 1) / kThreads,
                                                              (int64_t)num_sms() * 8));
  grad_reduce_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(inbox_ptr), reinterpret_cast<const uint32_t*>(flags_ptr),
      (int)world, (uint32_t)epoch, vec, reinterpret_cast<float4*>(out.data_ptr()),
      sumsq.data_ptr<float>(), device_error_ptr(), (uint64_t)(timeout_s * 1e9));
  AF3_CUDA_CHECK(cudaGetLastError());
}

// Copy src (contiguous, current device) to the device address dst (own memory or a peer
// mapping) with one async copy on the current stream (copy engine over NVLink for a peer).
void copy_to_address(torch::Tensor src, int64_t dst) {
  AF3_CHECK(src.is_cuda() && src.is_contiguous(), "copy_to_address: src must be contiguous CUDA");
  const c10::cuda::CUDAGuard guard(src.device());
  const size_t n = src.numel() * src.element_size();
  if (n == 0) return;
  AF3_CUDA_CHECK(cudaMemcpyAsync(reinterpret_cast<void*>(dst), src.data_ptr(), n,
                                 cudaMemcpyDefault, at::cuda::getCurrentCUDAStream()));
}

}  // namespace af3
