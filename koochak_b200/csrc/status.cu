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

std::tuple<int, long long, long long> read_debug_bounds_detail(int device) {
  int* p = device_status_ptr(device);
  long long words[3] = {0, 0, 0};  // [0]: status word and site; [1]: index; [2]: extent
  KB_CUDA_CHECK(cudaMemcpy(words, p, sizeof(words), cudaMemcpyDeviceToHost));
  KB_CUDA_CHECK(cudaMemset(reinterpret_cast<char*>(p) + 4, 0, sizeof(words) - 4));
  const int site = reinterpret_cast<const int*>(words)[1];
  return std::make_tuple(site, words[1], words[2]);
}

}  // namespace kb
