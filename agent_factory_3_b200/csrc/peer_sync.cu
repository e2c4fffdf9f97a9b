// Trainer -> rollout-engine weight sync over NVLink in one kernel (sm_100a).
//
// The engine exports a flat bf16 staging buffer (CUDA IPC); the trainer maps it and this kernel
// reads the trainer's tensors (fp32 master copies or bf16), casts them to bf16 and stores them
// straight into the peer GPU's buffer at their layout offsets -- the cast is fused with the
// NVLink transfer, and nothing is staged on the trainer's GPU or the host.  The reference syncs
// through files on a shared filesystem plus an HTTP reload (trainer/sglang_controller.py).
//
// Work decomposition: the concatenation of all items is cut into 8-element vectors; a thread
// finds the item of its vector by binary search over the item prefix (in shared memory), loads
// 32 (fp32) or 16 (bf16) bytes and writes one 16-byte store to the peer.  Items must hold a
// multiple of 8 elements at 16-byte aligned offsets (the host checks).
#include "common.h"
#include "host_utils.h"
#include "sm100.cuh"

namespace af3 {
namespace psync {

constexpr int kMaxItems = 4096;

struct Item {
  const void* src;
  int64_t vec_begin;   // first 8-element vector of this item in the concatenation
  int64_t dst_off;     // element offset in the destination buffer
  int src_f32;
};

__global__ void __launch_bounds__(256) peer_cast_copy_kernel(const Item* __restrict__ items,
                                                             int n_items, int64_t n_vec,
                                                             __nv_bfloat16* __restrict__ dst) {
  __shared__ int64_t s_begin[kMaxItems + 1];
  for (int i = threadIdx.x; i < n_items; i += blockDim.x) s_begin[i] = items[i].vec_begin;
  if (threadIdx.x == 0) s_begin[n_items] = n_vec;
  __syncthreads();
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < n_vec;
       v += (int64_t)gridDim.x * blockDim.x) {
    int lo = 0, hi = n_items - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_begin[mid] <= v) lo = mid; else hi = mid - 1;
    }
    const Item it = items[lo];
    const int64_t k = v - it.vec_begin;   // vector index inside the item
    uint4 w;
    if (it.src_f32) {
      const float4* s = reinterpret_cast<const float4*>(it.src) + 2 * k;
      const float4 a = __ldg(s), b = __ldg(s + 1);
      w.x = pack_bf16x2(a.x, a.y);
      w.y = pack_bf16x2(a.z, a.w);
      w.z = pack_bf16x2(b.x, b.y);
      w.w = pack_bf16x2(b.z, b.w);
    } else {
      w = __ldg(reinterpret_cast<const uint4*>(it.src) + k);
    }
    *reinterpret_cast<uint4*>(dst + it.dst_off + 8 * k) = w;   // NVLink store to the peer
  }
}

}  // namespace psync

// dst_ptr: device address of a bf16 buffer of dst_numel elements (typically a peer GPU's staging
// buffer opened with ipc_open on the current device); srcs: tensors on the current device (fp32
// or bf16, contiguous, numel % 8 == 0); offsets: element offset of each source in dst
// (multiples of 8).
void peer_cast_copy(int64_t dst_ptr, int64_t dst_numel, std::vector<torch::Tensor> srcs,
                    std::vector<int64_t> offsets) {
  using namespace psync;
  AF3_CHECK(dst_ptr != 0 && dst_ptr % 16 == 0, "dst must be a 16-byte aligned device address");
  AF3_CHECK(srcs.size() == offsets.size(), "one offset per source");
  AF3_CHECK((int64_t)srcs.size() <= kMaxItems, "too many tensors for one sync");
  if (srcs.empty()) return;
  const auto dev = srcs[0].device();
  const c10::cuda::CUDAGuard guard(dev);
  std::vector<Item> items(srcs.size());
  int64_t nv = 0;
  for (size_t i = 0; i < srcs.size(); ++i) {
    const auto& t = srcs[i];
    AF3_CHECK(t.is_cuda() && t.device() == dev && t.is_contiguous(), "sources must be contiguous on one device");
    AF3_CHECK(t.scalar_type() == torch::kFloat32 || t.scalar_type() == torch::kBFloat16,
              "sources must be fp32 or bf16");
    AF3_CHECK(t.numel() % 8 == 0 && offsets[i] % 8 == 0, "sizes and offsets must be multiples of 8");
    AF3_CHECK(offsets[i] + t.numel() <= dst_numel, "source does not fit in dst");
    AF3_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "sources must be 16-byte aligned");
    items[i] = Item{t.data_ptr(), nv, offsets[i], t.scalar_type() == torch::kFloat32 ? 1 : 0};
    nv += t.numel() / 8;
  }
  if (nv == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  auto d_items = torch::empty({(int64_t)(items.size() * sizeof(Item))},
                              torch::TensorOptions().dtype(torch::kUInt8).device(dev));
  AF3_CUDA_CHECK(cudaMemcpyAsync(d_items.data_ptr(), items.data(), items.size() * sizeof(Item),
                                 cudaMemcpyHostToDevice, stream));
  const int threads = 256;
  const int64_t grid = std::min<int64_t>((nv + threads - 1) / threads, (int64_t)num_sms() * 8);
  peer_cast_copy_kernel<<<(unsigned)grid, threads, 0, stream>>>(
      reinterpret_cast<const Item*>(d_items.data_ptr()), (int)items.size(), nv,
      reinterpret_cast<__nv_bfloat16*>(dst_ptr));
  AF3_CUDA_CHECK(cudaGetLastError());
}

}  // namespace af3
