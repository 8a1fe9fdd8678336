// Host-side helpers shared by the koochak_b200 CUDA sources: tensor-map
// encoding through the driver entry point (no libcuda link needed), a small
// cache of encoded maps keyed by (pointer, shape, strides, box), the device
// status word, and argument checks that fail loudly.
#pragma once

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <tuple>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

namespace kb {

#define KB_CHECK(cond, msg)                                                      \
  do {                                                                           \
    if (!(cond)) throw std::runtime_error(std::string("koochak_b200: ") + (msg)); \
  } while (0)

#define KB_CUDA_CHECK(expr)                                                                       \
  do {                                                                                            \
    cudaError_t _e = (expr);                                                                      \
    if (_e != cudaSuccess)                                                                        \
      throw std::runtime_error(std::string("koochak_b200 CUDA error: ") + cudaGetErrorString(_e) + \
                               " at " + __FILE__ + ":" + std::to_string(__LINE__));               \
  } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  KB_CHECK(fn != nullptr, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  return fn;
}

inline CUtensorMapDataType tma_dtype(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case at::kHalf: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case at::kFloat: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    default: KB_CHECK(false, "unsupported TMA dtype");
  }
  return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

struct TmaKey {
  uint64_t ptr;
  int rank;
  int dtype;
  int swizzle;
  std::array<uint64_t, 5> dims;
  std::array<uint64_t, 4> strides;
  std::array<uint32_t, 5> box;
  bool operator==(const TmaKey& o) const {
    return ptr == o.ptr && rank == o.rank && dtype == o.dtype && swizzle == o.swizzle && dims == o.dims &&
           strides == o.strides && box == o.box;
  }
};
struct TmaKeyHash {
  size_t operator()(const TmaKey& k) const {
    uint64_t h = k.ptr * 0x9E3779B97F4A7C15ull ^ (uint64_t)k.rank ^ ((uint64_t)k.dtype << 8);
    for (auto d : k.dims) h = (h ^ d) * 0x100000001B3ull;
    for (auto s : k.strides) h = (h ^ s) * 0x100000001B3ull;
    for (auto b : k.box) h = (h ^ b) * 0x100000001B3ull;
    return static_cast<size_t>(h);
  }
};

// Encodes (or fetches from cache) a tiled tensor map. dims/box are innermost
// first; strides are the byte strides of dims 1..rank-1.
inline CUtensorMap make_tma(const void* base, at::ScalarType dtype, int rank, const uint64_t* dims,
                            const uint64_t* byte_strides, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  KB_CHECK((reinterpret_cast<uint64_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i) KB_CHECK(byte_strides[i] % 16 == 0, "TMA strides must be multiples of 16 bytes");
  TmaKey key{};
  key.ptr = reinterpret_cast<uint64_t>(base);
  key.rank = rank;
  key.dtype = static_cast<int>(dtype);
  key.swizzle = static_cast<int>(swizzle);
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) key.strides[i] = byte_strides[i];
  static std::mutex mu;
  static std::unordered_map<TmaKey, CUtensorMap, TmaKeyHash> cache;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) s[i] = byte_strides[i];
  CUresult r = encode_tiled_fn()(&map, tma_dtype(dtype), rank, const_cast<void*>(base), d, s, b, e,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, map);
  }
  return map;
}

// Host-side count of kernels launched by this library (a benchmark reads it
// before and after a timed region).
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> n{0};
  return n;
}

#define KB_LAUNCHED()                      \
  do {                                     \
    ::kb::launch_counter().fetch_add(1);   \
    KB_CUDA_CHECK(cudaGetLastError());     \
  } while (0)

// Device status word: one int per device, allocated once and kept alive for
// the life of the process. Kernels with bounded waits record timeouts here.
int* device_status_ptr(int device);
int read_and_clear_status(int device);
// Site, index and extent recorded with a kStatusDebugBounds failure (cleared on read).
std::tuple<int, long long, long long> read_debug_bounds_detail(int device);

// Elements a kernel may touch from ``t``'s data pointer to the end of its
// storage: the extent a KB_DEBUG_BOUNDS build checks indices against. The
// debug slack (0 unless a test sets it) is subtracted, so a test can declare
// a buffer shorter than it is and see the check fire without any access
// leaving the real allocation.
inline std::atomic<long long>& debug_extent_slack() {
  static std::atomic<long long> n{0};
  return n;
}

inline long long declared_extent(const at::Tensor& t) {
  const long long es = (long long)t.element_size();
  const long long total = (long long)t.storage().nbytes() / es - (long long)t.storage_offset();
  return total - debug_extent_slack().load();
}

inline long long declared_extent_bytes(const at::Tensor& t) { return declared_extent(t) * (long long)t.element_size(); }

inline int num_sms(int device) {
  static int cached[64] = {0};
  if (device >= 0 && device < 64 && cached[device]) return cached[device];
  int n = 0;
  KB_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  if (device >= 0 && device < 64) cached[device] = n;
  return n;
}

// SMs kept free of the kernels that occupy a whole SM for their lifetime
// (persistent GEMM and attention), so that kernels running beside them --
// the data-parallel gradient reductions overlapped with backward -- always
// find SMs to run on instead of waiting for a persistent grid to drain.
// Set from Python around the overlapped region; 0 (the default) uses every SM.
inline std::atomic<int>& sm_reserve() {
  static std::atomic<int> n{0};
  return n;
}

// SMs available to a persistent kernel: all of them less the reserve, kept
// even so that CTA pairs (cta_group::2) still tile it, and at least 2.
inline int compute_sms(int device) {
  const int n = num_sms(device) - sm_reserve().load();
  return std::max(2, n & ~1);
}

inline void check_cuda_tensor(const at::Tensor& t, const char* name) {
  KB_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
}

}  // namespace kb
