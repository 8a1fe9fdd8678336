// Single-node gradient synchronisation over NVLink / NVSwitch, fused with the
// gradient gate.
//
// (replaces the DDP bucket all-reduce and the gradient gate of the reference:
//  koochak/loop.py:705-723 and 1612-1637, koochak/optim/grad_clip.py:47-73)
//
// Every rank owns one symmetric workspace (same size and layout on every GPU,
// each mapped into every peer's address space):
//
//   flags  [kMaxRanks] u32            arrival slot per source rank, written by that rank
//   stats  [2][n_tensors + 1] f32     per-tensor sum of squares + found_inf
//                                     (two copies, alternating per step)
//   data   bucket buffers, fp32 gradients
//
// Arrival protocol. Every launch of this file's kernels carries an epoch, the
// same increasing sequence on every rank (ranks issue the same launches in the
// same order). At its start a kernel publishes "rank r reached epoch e" into
// slot r of every peer (st.release.sys) and waits until every slot of its own
// array holds at least e (ld.acquire.sys, bounded). Because each rank's
// kernels run in order on one stream, seeing epoch e from a peer means the
// peer's kernels of every earlier epoch have finished. So:
//   * a bucket kernel only waits for "every rank has produced this bucket";
//     the peers' previous bucket kernels (which read this rank's memory and
//     wrote into it) are then complete too, so no closing barrier is needed;
//   * the last launch of a step (gate_seal_kernel) waits for every rank's
//     last bucket kernel, after which the statistics and all reduced values
//     are complete on every GPU.
// The protocol depends neither on the grid size nor on which block arrives
// first, so ranks may launch the same bucket with different grids.
//
// grad_sync_kernel, per bucket, on a side stream while backward runs: for each
// chunk (start, length, tensor, mode) of this rank's part of the bucket:
//     v = sum over ranks (P2P loads from every peer, or one
//         multimem.ld_reduce through the NVSwitch) * (inv_scale / W)
//     found_inf |= !isfinite(v);  sumsq[tensor] += v^2
//     mode 0: v is written to every rank (all-reduce of a replicated tensor);
//     mode 1: v is written to this rank only (reduction to the owner of a
//             sharded tensor: a Muon matrix's owner, or this rank's shard of a
//             tensor whose optimizer update is sharded),
// and the chunk's sum of squares / found flag is added into every rank's stats.
//
// Every flag wait is bounded by a %globaltimer budget; a wait that runs out
// records kStatusTimeoutPeer in the device status word and the kernel returns
// (the host raises). No TMA and no cluster multicast: plain and multimem
// loads/stores only.
#include "host_utils.h"
#include "sm100.cuh"

#include <torch/extension.h>

namespace kb {

constexpr int kMaxRanks = 8;
constexpr int kMaxCommBlocks = 148;
constexpr int kCommThreads = 512;

struct SyncArgs {
  unsigned long long base[kMaxRanks];  // each rank's workspace base (mapped here)
  unsigned long long mc_base;          // multicast mapping of the workspace, or 0
  long long flags_off;                 // bytes
  long long stats_off;                 // bytes, start of this step's stats copy
  long long data_off;                  // bytes, start of this bucket
  int world, rank;
  unsigned int epoch;
  unsigned long long timeout_ns;
  const float* scale;                  // GradScaler scale (device scalar) or null
  float divisor;                       // world size for averaging
  const long long* chunks;             // [n_chunks][4]: start (elements), length, tensor id, mode
  int n_chunks;
  int n_tensors;
  int* status;
  long long ws_bytes;                  // KB_DEBUG_BOUNDS: declared workspace size (bytes)
};

__device__ __forceinline__ void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

template <typename T>
__device__ __forceinline__ T* at_rank(const SyncArgs& a, int r, long long off) {
  return reinterpret_cast<T*>(a.base[r] + off);
}

// Publishes this rank's arrival at `epoch` to every peer (from every block:
// the stores are idempotent, and no block then depends on another being
// resident) and waits, bounded, until every rank has arrived. Returns false
// (status recorded) when a peer did not arrive in time.
__device__ bool arrive_and_wait(const SyncArgs& a, uint32_t epoch, volatile int* fail) {
  __syncthreads();
  const int t = threadIdx.x;
  if (t < a.world) st_release_sys(at_rank<uint32_t>(a, t, a.flags_off) + a.rank, epoch);
  if (t < a.world) {
    const uint32_t* slot = at_rank<uint32_t>(a, a.rank, a.flags_off) + t;
    const unsigned long long start = global_timer_ns();
    while ((int)(ld_acquire_sys(slot) - epoch) < 0) {
      if (*fail) break;
      if (global_timer_ns() - start > a.timeout_ns) {
        atomicCAS(a.status, 0, (int)kStatusTimeoutPeer);
        *fail = 1;
        break;
      }
      __nanosleep(128);
    }
  }
  __syncthreads();
  return *fail == 0;
}

__device__ __forceinline__ float4 mm_ld_reduce_f32x4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void mm_st_f32x4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float mm_ld_reduce_f32(const float* mc) {
  float v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(v) : "l"(mc) : "memory");
  return v;
}

__device__ __forceinline__ void mm_st_f32(float* mc, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}

__device__ __forceinline__ bool finite4(float4 v) {
  return isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

// Sum over ranks of float4 element i of the region at byte offset `off`.
template <bool MULTIMEM>
__device__ __forceinline__ float4 gather_sum4(const SyncArgs& a, long long off, int i) {
  if constexpr (MULTIMEM) {
    return mm_ld_reduce_f32x4(reinterpret_cast<const float*>(a.mc_base + off) + 4 * i);
  } else {
    float4 v = __ldcg(at_rank<const float4>(a, 0, off) + i);
    for (int r = 1; r < a.world; ++r) v = add4(v, __ldcg(at_rank<const float4>(a, r, off) + i));
    return v;
  }
}

template <bool MULTIMEM>
__device__ __forceinline__ void put4(const SyncArgs& a, long long off, int i, float4 v, bool everywhere) {
  if (!everywhere) {
    __stcg(at_rank<float4>(a, a.rank, off) + i, v);
  } else if constexpr (MULTIMEM) {
    mm_st_f32x4(reinterpret_cast<float*>(a.mc_base + off) + 4 * i, v);
  } else {
    for (int r = 0; r < a.world; ++r) __stcg(at_rank<float4>(a, r, off) + i, v);
  }
}

template <bool MULTIMEM>
__global__ void __launch_bounds__(kCommThreads) grad_sync_kernel(const SyncArgs a) {
  __shared__ volatile int fail;
  __shared__ float red[kCommThreads / 32];
  __shared__ int red_bad[kCommThreads / 32];
  if (threadIdx.x == 0) fail = 0;
  if (!arrive_and_wait(a, a.epoch, &fail)) return;
  // Peers wrote the bucket through their own (unicast) mappings; order those
  // writes before loads through the multicast alias.
  if constexpr (MULTIMEM) asm volatile("fence.proxy.alias;" ::: "memory");

  const float mul = (a.scale ? 1.f / *a.scale : 1.f) / a.divisor;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int c = blockIdx.x; c < a.n_chunks; c += gridDim.x) {
    const long long* row = a.chunks + 4 * c;
    const long long start = row[0];
    const int len = (int)row[1];
    const int tid = (int)row[2];
    const bool everywhere = row[3] == 0;
    float ss = 0.f;
    bool bad = false;
    const long long off = a.data_off + start * 4;  // bytes; start is a multiple of 4 elements
    if (!debug_bounds_ok(a.status, kSiteCommChunk, off + 4LL * len - 1, a.ws_bytes) ||
        !debug_bounds_ok(a.status, kSiteCommChunk, tid, a.n_tensors))
      continue;  // the same decision in every thread of the block
    const int n4 = len >> 2;
    // kUnroll float4 per thread per pass, every rank's loads issued before
    // the first use, so each thread keeps kUnroll * world loads in flight.
    constexpr int kUnroll = 4;
    const int stride = blockDim.x;
    int i0 = threadIdx.x;
    for (; i0 + (kUnroll - 1) * stride < n4; i0 += kUnroll * stride) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = gather_sum4<MULTIMEM>(a, off, i0 + u * stride);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        float4 x = v[u];
        x.x *= mul; x.y *= mul; x.z *= mul; x.w *= mul;
        bad |= !finite4(x);
        ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
        put4<MULTIMEM>(a, off, i0 + u * stride, x, everywhere);
      }
    }
    for (int i = i0; i < n4; i += stride) {
      float4 x = gather_sum4<MULTIMEM>(a, off, i);
      x.x *= mul; x.y *= mul; x.z *= mul; x.w *= mul;
      bad |= !finite4(x);
      ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
      put4<MULTIMEM>(a, off, i, x, everywhere);
    }
    for (int i = 4 * n4 + threadIdx.x; i < len; i += stride) {  // ragged tail (< 4 elements)
      float v;
      if constexpr (MULTIMEM) {
        v = mm_ld_reduce_f32(reinterpret_cast<const float*>(a.mc_base + off) + i);
      } else {
        v = 0.f;
        for (int r = 0; r < a.world; ++r) v += __ldcg(at_rank<const float>(a, r, off) + i);
      }
      v *= mul;
      bad |= !isfinite(v);
      ss += v * v;
      if (!everywhere) {
        __stcg(at_rank<float>(a, a.rank, off) + i, v);
      } else if constexpr (MULTIMEM) {
        mm_st_f32(reinterpret_cast<float*>(a.mc_base + off) + i, v);
      } else {
        for (int r = 0; r < a.world; ++r) __stcg(at_rank<float>(a, r, off) + i, v);
      }
    }
    ss = warp_sum(ss);
    const int any_bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
      red[warp] = ss;
      red_bad[warp] = any_bad;
    }
    __syncthreads();
    if (threadIdx.x < a.world) {
      float tot = 0.f;
      int b = 0;
      for (int w = 0; w < kCommThreads / 32; ++w) {
        tot += red[w];
        b |= red_bad[w];
      }
      float* stats = at_rank<float>(a, threadIdx.x, a.stats_off);
      atomicAdd(stats + tid, tot);
      if (b) atomicExch(stats + a.n_tensors, 1.f);
    }
    __syncthreads();
  }
  // Make this thread's remote stores and atomics visible system-wide before the
  // kernel ends: a peer that sees a later epoch from this rank reads them.
  if constexpr (MULTIMEM) asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
}

// Arrival-only launch: start-up, the optimizer's parameter publication, and the
// tests of the bounded wait.
__global__ void __launch_bounds__(kCommThreads) comm_barrier_kernel(const SyncArgs a) {
  __shared__ volatile int fail;
  if (threadIdx.x == 0) fail = 0;
  arrive_and_wait(a, a.epoch, &fail);
}

// norm = sqrt(sum_t (sqrt(sumsq_t))^2 in fp64); coef = min(1, max_norm / (norm + 1e-6)).
// out = [norm, coef, found_inf, device status word]
__device__ void gate_values(const float* __restrict__ stats, int n_tensors, float max_norm, int clip,
                            const int* __restrict__ status, float* __restrict__ out) {
  double acc = 0.0;
  for (int t = 0; t < n_tensors; ++t) {
    const double nt = (double)sqrtf(stats[t]);
    acc += nt * nt;
  }
  const double norm = sqrt(acc);
  out[0] = (float)norm;
  out[1] = clip ? (float)fmin(1.0, (double)max_norm / (norm + 1e-6)) : 1.f;
  out[2] = stats[n_tensors];
  out[3] = (float)*status;
}

__global__ void gate_from_stats_kernel(const float* __restrict__ stats, int n_tensors, float max_norm, int clip,
                                       const int* __restrict__ status, float* __restrict__ out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  gate_values(stats, n_tensors, max_norm, clip, status, out);
}

// Last launch of a step: wait until every rank's bucket kernels have finished
// (their reduced values and statistics are then in place on every GPU), then
// form the gate from this rank's complete statistics.
__global__ void __launch_bounds__(32) gate_seal_kernel(const SyncArgs a, float max_norm, int clip,
                                                       float* __restrict__ out) {
  __shared__ volatile int fail;
  if (threadIdx.x == 0) fail = 0;
  arrive_and_wait(a, a.epoch, &fail);
  if (threadIdx.x == 0) gate_values(at_rank<const float>(a, a.rank, a.stats_off), a.n_tensors, max_norm, clip,
                                    a.status, out);
}

// ---------------------------------------------------------------------- host

static SyncArgs make_args(const std::vector<int64_t>& bases, int64_t mc_base, int64_t flags_off, int64_t stats_off,
                          int64_t data_off, int64_t rank, int64_t epoch, double timeout_s, int device) {
  SyncArgs a;
  std::memset(&a, 0, sizeof(a));
  const int world = (int)bases.size();
  KB_CHECK(world >= 1 && world <= kMaxRanks, "comm: world size must be 1..8");
  KB_CHECK(rank >= 0 && rank < world, "comm: bad rank");
  for (int r = 0; r < world; ++r) {
    KB_CHECK(bases[r] != 0 && bases[r] % 16 == 0, "comm: workspace bases must be 16-byte aligned");
    a.base[r] = (unsigned long long)bases[r];
  }
  KB_CHECK(flags_off % 16 == 0 && stats_off % 16 == 0 && data_off % 16 == 0, "comm: offsets must be 16-byte aligned");
  KB_CHECK(mc_base % 16 == 0, "comm: multicast base must be 16-byte aligned");
  a.mc_base = (unsigned long long)mc_base;
  a.flags_off = flags_off;
  a.stats_off = stats_off;
  a.data_off = data_off;
  a.world = world;
  a.rank = (int)rank;
  a.epoch = (unsigned int)epoch;
  a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  a.divisor = (float)world;
  a.status = device_status_ptr(device);
  return a;
}

void comm_grad_sync(const std::vector<int64_t>& bases, int64_t mc_base, int64_t flags_off, int64_t stats_off,
                    int64_t data_off, const at::Tensor& chunks, int64_t n_tensors, int64_t rank, int64_t epoch,
                    const c10::optional<at::Tensor>& scale, int64_t blocks, double timeout_s, int64_t ws_bytes) {
  check_cuda_tensor(chunks, "chunks");
  KB_CHECK(chunks.scalar_type() == at::kLong && chunks.is_contiguous() && chunks.dim() == 2 && chunks.size(1) == 4,
           "comm: chunks must be int64 [n, 4]");
  KB_CHECK(blocks >= 1 && blocks <= kMaxCommBlocks, "comm: blocks must be 1..148");
  const c10::cuda::CUDAGuard guard(chunks.device());
  const int dev = chunks.get_device();
  SyncArgs a = make_args(bases, mc_base, flags_off, stats_off, data_off, rank, epoch, timeout_s, dev);
  a.chunks = reinterpret_cast<const long long*>(chunks.data_ptr<int64_t>());
  a.n_chunks = (int)chunks.size(0);
  a.n_tensors = (int)n_tensors;
  a.ws_bytes = ws_bytes > 0 ? ws_bytes - 4 * debug_extent_slack().load() : (long long)INT64_MAX;
  if (scale.has_value() && scale->defined()) {
    KB_CHECK(scale->scalar_type() == at::kFloat && scale->numel() == 1, "comm: scale must be an fp32 scalar");
    a.scale = scale->data_ptr<float>();
  }
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream().stream();
  if (mc_base != 0) {
    grad_sync_kernel<true><<<(unsigned)blocks, kCommThreads, 0, stream>>>(a);
  } else {
    grad_sync_kernel<false><<<(unsigned)blocks, kCommThreads, 0, stream>>>(a);
  }
  KB_LAUNCHED();
}

void comm_barrier(const std::vector<int64_t>& bases, int64_t flags_off, int64_t rank, int64_t epoch, int64_t blocks,
                  double timeout_s, int64_t device) {
  KB_CHECK(blocks >= 1 && blocks <= kMaxCommBlocks, "comm: blocks must be 1..148");
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  SyncArgs a = make_args(bases, 0, flags_off, 0, 0, rank, epoch, timeout_s, (int)device);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream().stream();
  comm_barrier_kernel<<<(unsigned)blocks, kCommThreads, 0, stream>>>(a);
  KB_LAUNCHED();
}

void comm_gate_seal(const std::vector<int64_t>& bases, int64_t flags_off, int64_t stats_off, int64_t n_tensors,
                    int64_t rank, int64_t epoch, double timeout_s, double max_norm, bool clip, at::Tensor& out) {
  check_cuda_tensor(out, "out");
  KB_CHECK(out.scalar_type() == at::kFloat && out.numel() >= 4 && out.is_contiguous(), "gate: out must be fp32 [4]");
  const c10::cuda::CUDAGuard guard(out.device());
  SyncArgs a = make_args(bases, 0, flags_off, stats_off, 0, rank, epoch, timeout_s, out.get_device());
  a.n_tensors = (int)n_tensors;
  gate_seal_kernel<<<1, 32, 0, c10::cuda::getCurrentCUDAStream().stream()>>>(a, (float)max_norm, clip ? 1 : 0,
                                                                             out.data_ptr<float>());
  KB_LAUNCHED();
}

void gate_from_stats(const at::Tensor& stats, int64_t n_tensors, double max_norm, bool clip, at::Tensor& out) {
  check_cuda_tensor(stats, "stats");
  KB_CHECK(stats.scalar_type() == at::kFloat && stats.numel() >= n_tensors + 1, "gate: stats too small");
  KB_CHECK(out.scalar_type() == at::kFloat && out.numel() >= 4, "gate: out must be fp32 [4]");
  const c10::cuda::CUDAGuard guard(stats.device());
  gate_from_stats_kernel<<<1, 32, 0, c10::cuda::getCurrentCUDAStream().stream()>>>(
      stats.data_ptr<float>(), (int)n_tensors, (float)max_norm, clip ? 1 : 0, device_status_ptr(stats.get_device()),
      out.data_ptr<float>());
  KB_LAUNCHED();
}

void register_comm_ops(pybind11::module& m) {
  m.def("comm_grad_sync", &comm_grad_sync,
        "fused bucket reduction (+unscale, finite flag, sumsq); per chunk to every rank or to this rank only",
        pybind11::arg("bases"), pybind11::arg("mc_base"), pybind11::arg("flags_off"), pybind11::arg("stats_off"),
        pybind11::arg("data_off"), pybind11::arg("chunks"), pybind11::arg("n_tensors"), pybind11::arg("rank"),
        pybind11::arg("epoch"), pybind11::arg("scale"), pybind11::arg("blocks"), pybind11::arg("timeout_s"),
        pybind11::arg("ws_bytes") = 0);
  m.def("comm_barrier", &comm_barrier, "cross-GPU arrival barrier with a bounded wait", pybind11::arg("bases"),
        pybind11::arg("flags_off"), pybind11::arg("rank"), pybind11::arg("epoch"), pybind11::arg("blocks"),
        pybind11::arg("timeout_s"), pybind11::arg("device"));
  m.def("comm_gate_seal", &comm_gate_seal,
        "wait for every rank's bucket kernels, then norm / clip coefficient / found_inf from the statistics",
        pybind11::arg("bases"), pybind11::arg("flags_off"), pybind11::arg("stats_off"), pybind11::arg("n_tensors"),
        pybind11::arg("rank"), pybind11::arg("epoch"), pybind11::arg("timeout_s"), pybind11::arg("max_norm"),
        pybind11::arg("clip"), pybind11::arg("out"));
  m.def("gate_from_stats", &gate_from_stats, "norm / clip coefficient / found_inf from fused statistics");
  m.attr("comm_max_blocks") = kMaxCommBlocks;
  m.attr("comm_max_ranks") = kMaxRanks;
}

}  // namespace kb
