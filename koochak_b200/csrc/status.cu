// Per-device status word shared by every bounded-wait kernel of the library.
//
// The word lives in a small cudaMalloc'd block that is allocated once per
// device on first use and never freed (it must outlive every kernel that may
// still hold its address). Kernels write a nonzero StatusCode with atomicCAS;
// the host reads and clears it at synchronisation points and raises.
#include "host_utils.h"

#include <mutex>

namespace kb {

static std::mutex g_status_mu;
static int* g_status[64] = {nullptr};

int* device_status_ptr(int device) {
  KB_CHECK(device >= 0 && device < 64, "device index out of range");
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (g_status[device] == nullptr) {
    int prev = 0;
    KB_CUDA_CHECK(cudaGetDevice(&prev));
    KB_CUDA_CHECK(cudaSetDevice(device));
    int* p = nullptr;
    KB_CUDA_CHECK(cudaMalloc(&p, 64));
    KB_CUDA_CHECK(cudaMemset(p, 0, 64));
    KB_CUDA_CHECK(cudaSetDevice(prev));
    g_status[device] = p;
  }
  return g_status[device];
}

int read_and_clear_status(int device) {
  int* p = device_status_ptr(device);
  int value = 0;
  KB_CUDA_CHECK(cudaMemcpy(&value, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (value != 0) KB_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  return value;
}

}  // namespace kb
