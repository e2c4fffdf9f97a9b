// Per-device error word.  Kernels whose waits are bounded record a non-zero code here
// instead of hanging; the Python layer checks it after suspicious launches and in tests.
#include <mutex>
#include <vector>

#include "common.h"
#include "host_utils.h"

namespace af3 {

int* device_error_ptr() {
  static std::mutex mu;
  static std::vector<int*> ptrs;
  int dev = 0;
  AF3_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if ((int)ptrs.size() <= dev) ptrs.resize(dev + 1, nullptr);
  if (ptrs[dev] == nullptr) {
    AF3_CUDA_CHECK(cudaMalloc(&ptrs[dev], sizeof(int)));
    AF3_CUDA_CHECK(cudaMemset(ptrs[dev], 0, sizeof(int)));
  }
  return ptrs[dev];
}

int64_t device_error_take() {
  int* p = device_error_ptr();
  int h = 0;
  auto stream = at::cuda::getCurrentCUDAStream();
  AF3_CUDA_CHECK(cudaMemcpyAsync(&h, p, sizeof(int), cudaMemcpyDeviceToHost, stream));
  AF3_CUDA_CHECK(cudaStreamSynchronize(stream));
  if (h != 0) AF3_CUDA_CHECK(cudaMemsetAsync(p, 0, sizeof(int), stream));
  return h;
}

}  // namespace af3
