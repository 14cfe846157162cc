// Device status word shared by every kernel with bounded waits.  Kernels write
// the first failure code (see DeviceStatus in sm100.cuh) instead of trapping;
// the host polls it with device_status() after a step and raises.
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <c10/cuda/CUDAException.h>
#include <mutex>
#include <vector>

namespace dmad {

int* device_status_ptr(int device) {
  static std::mutex mu;
  static std::vector<int*> ptrs;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)ptrs.size() <= device) ptrs.resize(device + 1, nullptr);
  if (ptrs[device] == nullptr) {
    int prev;
    C10_CUDA_CHECK(cudaGetDevice(&prev));
    C10_CUDA_CHECK(cudaSetDevice(device));
    C10_CUDA_CHECK(cudaMalloc(&ptrs[device], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(ptrs[device], 0, sizeof(int)));
    C10_CUDA_CHECK(cudaDeviceSynchronize());
    C10_CUDA_CHECK(cudaSetDevice(prev));
  }
  return ptrs[device];
}

// Returns the status code of `device` (synchronising with it) and optionally clears it.
int64_t device_status(int64_t device, bool reset) {
  int* p = device_status_ptr((int)device);
  int prev;
  C10_CUDA_CHECK(cudaGetDevice(&prev));
  C10_CUDA_CHECK(cudaSetDevice((int)device));
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  C10_CUDA_CHECK(cudaSetDevice(prev));
  return v;
}

}  // namespace dmad
