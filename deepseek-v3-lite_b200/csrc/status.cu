#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <cuda_runtime.h>

#include <mutex>

#include "status.h"

namespace dsv3 {

namespace {
constexpr int kMaxDevices = 64;
unsigned int* g_status[kMaxDevices] = {nullptr};
std::mutex g_mu;
}  // namespace

unsigned int* status_ptr() {
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_status[dev]) {
    C10_CUDA_CHECK(cudaMalloc(&g_status[dev], sizeof(unsigned int)));
    C10_CUDA_CHECK(cudaMemset(g_status[dev], 0, sizeof(unsigned int)));
  }
  return g_status[dev];
}

unsigned int status_read() {
  unsigned int v = 0;
  auto stream = at::cuda::getCurrentCUDAStream();
  C10_CUDA_CHECK(cudaMemcpyAsync(&v, status_ptr(), sizeof(v), cudaMemcpyDeviceToHost, stream));
  C10_CUDA_CHECK(cudaStreamSynchronize(stream));
  return v;
}

void status_reset() {
  C10_CUDA_CHECK(cudaMemsetAsync(status_ptr(), 0, sizeof(unsigned int), at::cuda::getCurrentCUDAStream()));
}

}  // namespace dsv3
