#include <cuda_runtime.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <mutex>
#include "status.h"

namespace mb {
static int* g_status[64] = {nullptr};
static std::mutex g_mu;

int* status_ptr(int device) {
  if (g_status[device]) return g_status[device];
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status[device]) {
    c10::cuda::CUDAGuard guard(device);
    int* p = nullptr;
    C10_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
    g_status[device] = p;
  }
  return g_status[device];
}

int read_and_clear_status(int device) {
  int* p = status_ptr(device);
  c10::cuda::CUDAGuard guard(device);
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) C10_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  return v;
}
}  // namespace mb
