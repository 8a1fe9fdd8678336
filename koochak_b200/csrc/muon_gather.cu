// Sharded Muon: the parameter update of the owning rank, fused with the
// all-gather of the updated parameter to every rank of the node.
//
// (replaces, for the native distributed Muon path, the per-rank update plus
//  the padded parameter all-gather of the reference:
//  koochak/optim/muon.py:256-277, MuonWithAuxAdam.step)
//
// Every Muon matrix of a parameter group lives in one symmetric fp32 slab: the
// same offset on every GPU, each rank's slab mapped into every peer (and, with
// NVSwitch multicast, one multicast alias of the whole slab). The rank that
// owns a matrix runs momentum and Newton-Schulz on it; this kernel then forms
//
//   p_new = p * (1 - lr * wd) - lr * scale * U        (U = X or X^T)
//
// and stores p_new into every rank's copy in the same pass: one
// `multimem.st.v4.f32` through the switch when a multicast alias exists,
// otherwise one 16-byte P2P store per rank. The owner's bf16 compute copy is
// written too. Peers learn that the stores have landed from a bounded flag
// barrier launched after the last bucket (comm.cu: comm_barrier); the fence at
// the end of every thread orders its remote stores before that release.
//
// The math is the same expression, in the same order, as muon_epilogue_kernel
// (optim.cu), so a sharded step is bit-identical to a single-GPU step.
//
// adam_shard_gather_kernel is the same idea for the aux-Adam parameters
// (reference koochak/optim/muon.py:289-333, replicated there): after the
// gradient sync reduced each Adam tensor's per-rank shard into that rank only
// (a reduce-scatter), each rank runs AdamW on its own shard -- clip
// coefficient applied on read, moments, bias correction, decoupled weight
// decay, the same expression as adamw_kernel (optim.cu) -- and stores the new
// parameter values into every rank's copy. Moment tensors are kept full-size
// on every rank but only the shard's elements are updated there; a
// checkpoint gathers them (optim/muon.py).
//
// Every parameter handed to these kernels must lie inside the local slab: the
// host checks [ptr, ptr + bytes) against the slab's extent, because every
// store to a peer lands at the same offset of that peer's slab.
// No TMA and no cluster multicast: plain and multimem stores only.
#include "host_utils.h"
#include "step_guard.h"
#include "sm100.cuh"

#include <torch/extension.h>

#include <cmath>
#include <vector>

namespace kb {

namespace {

constexpr int kGatherMats = 64;
constexpr int kGatherRanks = 8;

struct GatherMats {
  int R, C;                            // parameter shape (rows, cols); C % 4 == 0
  int world;
  float* p[kGatherMats];               // this rank's copy (inside the slab)
  __nv_bfloat16* shadow[kGatherMats];  // bf16 compute copy on this rank, or null
  long long delta[kGatherRanks];       // bytes from this rank's slab to rank r's
  long long mc_delta;                  // bytes from this rank's slab to the multicast alias (0: none)
  const float* skip;                   // device skip flag (step_guard.h) or null
};

__device__ __forceinline__ void mm_st_v4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

template <typename T>
__device__ __forceinline__ T* shifted(T* p, long long bytes) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p) + bytes);
}

// One CTA per 32 x 32 block of one matrix; a thread owns 4 consecutive columns
// of one row, so every store is 16 bytes and a warp covers 4 full 128-byte rows.
template <bool MULTIMEM>
__global__ void __launch_bounds__(256)
    muon_update_gather_kernel(const __grid_constant__ GatherMats mm, const __nv_bfloat16* __restrict__ X, float lr,
                              float wd, float scale, int transpose, const float* __restrict__ row_scale) {
  if (step_skipped(mm.skip)) return;
  const int i = blockIdx.z;
  const int R = mm.R, C = mm.C;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const __nv_bfloat16* x = X + (long long)i * R * C;
  __shared__ float tile[32][33];
  if (transpose) {
    // X is [C, R]: read coalesced along R, tile[c - c0][r - r0].
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + ty + 8 * k, r = r0 + tx;
      tile[ty + 8 * k][tx] = (r < R && c < C) ? __bfloat162float(x[(long long)c * R + r]) : 0.f;
    }
    __syncthreads();
  }
  const int row = threadIdx.x >> 3, col = (threadIdx.x & 7) * 4;
  const int r = r0 + row, c = c0 + col;
  if (r < R && c < C) {  // C % 4 == 0: the whole 4-vector is in range
    const long long idx = (long long)r * C + c;
    float u[4];
    if (transpose) {
#pragma unroll
      for (int j = 0; j < 4; ++j) u[j] = tile[col + j][row];
    } else {
      const uint2 raw = *reinterpret_cast<const uint2*>(x + idx);
      const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
      const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
      u[0] = __low2float(lo);
      u[1] = __high2float(lo);
      u[2] = __low2float(hi);
      u[3] = __high2float(hi);
    }
    float* p = mm.p[i] + idx;
    const float4 old = *reinterpret_cast<const float4*>(p);
    const float decay = 1.f - lr * wd;
    const float f = row_scale ? row_scale[(long long)i * R + r] : scale;
    float4 pn;
    pn.x = old.x * decay - lr * (f * u[0]);
    pn.y = old.y * decay - lr * (f * u[1]);
    pn.z = old.z * decay - lr * (f * u[2]);
    pn.w = old.w * decay - lr * (f * u[3]);
    if constexpr (MULTIMEM) {
      mm_st_v4(shifted(p, mm.mc_delta), pn);
    } else {
      for (int q = 0; q < mm.world; ++q) __stcg(shifted(reinterpret_cast<float4*>(p), mm.delta[q]), pn);
    }
    if (__nv_bfloat16* sh = mm.shadow[i]) {
      __nv_bfloat162 a = __floats2bfloat162_rn(pn.x, pn.y);
      __nv_bfloat162 b = __floats2bfloat162_rn(pn.z, pn.w);
      uint2 packed;
      packed.x = *reinterpret_cast<uint32_t*>(&a);
      packed.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(sh + idx) = packed;
    }
  }
  if constexpr (MULTIMEM) asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
}

// Matrices already in their wide orientation (no transpose): one contiguous
// index for every operand, so a CTA takes 4096 consecutive elements, four
// float4 per thread with all loads issued first. Same expression as above.
constexpr int kGatherFlatVecs = 4;
constexpr int kGatherFlatPerCta = 256 * kGatherFlatVecs;  // float4 per CTA

template <bool MULTIMEM>
__global__ void __launch_bounds__(256)
    muon_update_gather_flat_kernel(const __grid_constant__ GatherMats mm, const __nv_bfloat16* __restrict__ X,
                                   float lr, float wd, float scale, const float* __restrict__ row_scale) {
  if (step_skipped(mm.skip)) return;
  const int i = blockIdx.y;
  const long long n4 = (long long)mm.R * mm.C / 4;
  float4* p = reinterpret_cast<float4*>(mm.p[i]);
  uint2* sh = reinterpret_cast<uint2*>(mm.shadow[i]);
  const uint2* x = reinterpret_cast<const uint2*>(X + (long long)i * mm.R * mm.C);
  const long long j0 = (long long)blockIdx.x * kGatherFlatPerCta + threadIdx.x;
  const float decay = 1.f - lr * wd;
  float4 pv[kGatherFlatVecs];
  uint2 xv[kGatherFlatVecs];
#pragma unroll
  for (int k = 0; k < kGatherFlatVecs; ++k) {
    const long long j = j0 + k * 256;
    if (j < n4) {
      pv[k] = p[j];
      xv[k] = x[j];
    }
  }
#pragma unroll
  for (int k = 0; k < kGatherFlatVecs; ++k) {
    const long long j = j0 + k * 256;
    if (j < n4) {
      const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&xv[k].x);
      const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&xv[k].y);
      const float f = row_scale ? row_scale[(long long)i * mm.R + (4 * j) / mm.C] : scale;  // C % 4 == 0
      float4 pn;
      pn.x = pv[k].x * decay - lr * (f * __low2float(lo));
      pn.y = pv[k].y * decay - lr * (f * __high2float(lo));
      pn.z = pv[k].z * decay - lr * (f * __low2float(hi));
      pn.w = pv[k].w * decay - lr * (f * __high2float(hi));
      if constexpr (MULTIMEM) {
        mm_st_v4(shifted(reinterpret_cast<float*>(p + j), mm.mc_delta), pn);
      } else {
        for (int q = 0; q < mm.world; ++q) __stcg(shifted(p + j, mm.delta[q]), pn);
      }
      if (sh) {
        __nv_bfloat162 a = __floats2bfloat162_rn(pn.x, pn.y);
        __nv_bfloat162 b = __floats2bfloat162_rn(pn.z, pn.w);
        uint2 packed;
        packed.x = *reinterpret_cast<uint32_t*>(&a);
        packed.y = *reinterpret_cast<uint32_t*>(&b);
        sh[j] = packed;
      }
    }
  }
  if constexpr (MULTIMEM) asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
}

}  // namespace

// params: this rank's owned matrices (views into the symmetric slab), all [R, C]
// fp32; X: bf16 [n, r, c] orthogonalised updates (r, c = C, R when transpose).
// bases: every rank's slab base address; mc_base: multicast alias or 0.
void muon_update_gather(const std::vector<at::Tensor>& params, const at::Tensor& X,
                        const std::vector<at::Tensor>& shadow, double lr, double wd, double scale, bool transpose,
                        const std::vector<int64_t>& bases, int64_t mc_base, int64_t rank, int64_t slab_bytes,
                        const c10::optional<at::Tensor>& row_scale) {
  const size_t n = params.size();
  if (n == 0) return;
  const int world = (int)bases.size();
  KB_CHECK(world >= 1 && world <= kGatherRanks, "muon_update_gather: world size must be 1..8");
  KB_CHECK(rank >= 0 && rank < world, "muon_update_gather: bad rank");
  KB_CHECK(shadow.empty() || shadow.size() == n, "muon_update_gather: shadow list length");
  const c10::cuda::CUDAGuard guard(params[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const int R = (int)params[0].size(0);
  const int C = (int)(params[0].numel() / R);
  KB_CHECK(C % 4 == 0, "muon_update_gather: column count must be a multiple of 4");
  KB_CHECK(X.scalar_type() == at::kBFloat16 && X.is_contiguous() && X.numel() >= (int64_t)n * R * C,
           "muon_update_gather: X must be contiguous bf16 [n, R*C]");
  KB_CHECK(reinterpret_cast<uintptr_t>(X.data_ptr()) % 8 == 0, "muon_update_gather: X must be 8-byte aligned");
  const float* rs_all = nullptr;
  if (row_scale.has_value() && row_scale->defined()) {
    KB_CHECK(row_scale->scalar_type() == at::kFloat && row_scale->is_contiguous() &&
                 row_scale->numel() >= (int64_t)n * R,
             "muon_update_gather: row_scale must be fp32 [n, rows]");
    rs_all = row_scale->data_ptr<float>();
  }
  for (int q = 0; q < world; ++q) KB_CHECK(bases[q] != 0 && bases[q] % 16 == 0, "muon_update_gather: bad slab base");
  KB_CHECK(mc_base % 16 == 0, "muon_update_gather: multicast base must be 16-byte aligned");
  for (size_t base = 0; base < n; base += kGatherMats) {
    const int count = (int)std::min<size_t>(kGatherMats, n - base);
    GatherMats mm{};
    mm.skip = step_skip_ptr();
    mm.R = R;
    mm.C = C;
    mm.world = world;
    for (int q = 0; q < world; ++q) mm.delta[q] = bases[q] - bases[rank];
    mm.mc_delta = mc_base ? mc_base - bases[rank] : 0;
    for (int j = 0; j < count; ++j) {
      const at::Tensor& p = params[base + j];
      KB_CHECK(p.scalar_type() == at::kFloat && p.is_contiguous() && p.numel() == (int64_t)R * C,
               "muon_update_gather: same-shape fp32 contiguous matrices required");
      const int64_t addr = reinterpret_cast<int64_t>(p.data_ptr());
      KB_CHECK(addr % 16 == 0 && addr >= bases[rank] && addr + 4 * (int64_t)R * C <= bases[rank] + slab_bytes,
               "muon_update_gather: parameter must lie in the local slab");
      mm.p[j] = p.data_ptr<float>();
      const at::Tensor* sh = shadow.empty() ? nullptr : &shadow[base + j];
      mm.shadow[j] = (sh && sh->numel() == (int64_t)R * C && sh->scalar_type() == at::kBFloat16 &&
                      sh->is_contiguous() && reinterpret_cast<uintptr_t>(sh->data_ptr()) % 8 == 0)
                         ? reinterpret_cast<__nv_bfloat16*>(sh->data_ptr())
                         : nullptr;
      KB_CHECK(sh == nullptr || sh->numel() == 0 || mm.shadow[j] != nullptr,
               "muon_update_gather: shadow must be a contiguous 8-byte aligned bf16 copy of the parameter");
    }
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()) + (int64_t)base * R * C;
    const float* rs = rs_all ? rs_all + (int64_t)base * R : nullptr;
    if (!transpose) {  // C % 4 == 0, params 16-byte and X / shadows 8-byte aligned (checked above)
      const long long n4 = (long long)R * C / 4;
      dim3 fgrid((unsigned)((n4 + kGatherFlatPerCta - 1) / kGatherFlatPerCta), count);
      if (mc_base != 0) {
        muon_update_gather_flat_kernel<true><<<fgrid, 256, 0, s>>>(mm, xb, (float)lr, (float)wd, (float)scale, rs);
      } else {
        muon_update_gather_flat_kernel<false><<<fgrid, 256, 0, s>>>(mm, xb, (float)lr, (float)wd, (float)scale, rs);
      }
      KB_LAUNCHED();
      continue;
    }
    dim3 grid((C + 31) / 32, (R + 31) / 32, count);
    if (mc_base != 0) {
      muon_update_gather_kernel<true><<<grid, 256, 0, s>>>(mm, xb, (float)lr, (float)wd, (float)scale, transpose, rs);
    } else {
      muon_update_gather_kernel<false><<<grid, 256, 0, s>>>(mm, xb, (float)lr, (float)wd, (float)scale, transpose,
                                                           rs);
    }
    KB_LAUNCHED();
  }
}


// ------------------------------------------------------------ sharded AdamW

namespace {

constexpr int kShardT = 64;             // tensors per launch
constexpr int kShardChunk = 4096;       // elements per work item (a multiple of 4)

struct AdamShard {
  int n, world;
  float* p[kShardT];          // this rank's copy (inside the slab)
  const float* g[kShardT];    // reduced gradient, indexed like p (valid on [lo, hi))
  float* m[kShardT];
  float* v[kShardT];
  long long lo[kShardT];      // shard [lo, hi) of tensor i, lo % 4 == 0
  long long hi[kShardT];
  long long first[kShardT + 1];  // prefix sum of work items per tensor
  float bc1[kShardT], bc2[kShardT];
  long long delta[kGatherRanks];
  long long mc_delta;
  long long ext[kShardT];     // KB_DEBUG_BOUNDS: elements every tensor of i is declared to hold
  int* status;
};

template <bool MULTIMEM>
__device__ __forceinline__ void publish4(const AdamShard& a, float* p, float4 v) {
  if constexpr (MULTIMEM) {
    mm_st_v4(shifted(p, a.mc_delta), v);
  } else {
    for (int q = 0; q < a.world; ++q) __stcg(shifted(reinterpret_cast<float4*>(p), a.delta[q]), v);
  }
}

template <bool MULTIMEM>
__device__ __forceinline__ void publish1(const AdamShard& a, float* p, float v) {
  if constexpr (MULTIMEM) {
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(shifted(p, a.mc_delta)), "f"(v) : "memory");
  } else {
    for (int q = 0; q < a.world; ++q) __stcg(shifted(p, a.delta[q]), v);
  }
}

__device__ __forceinline__ float adam_elem(float p, float g, float& m, float& v, float b1, float b2, float inv_bc1,
                                           float inv_bc2, float eps, float lr, float decay) {
  m = m + (1.f - b1) * (g - m);
  v = v + (1.f - b2) * (g * g - v);
  const float upd = (m * inv_bc1) / (sqrtf(v * inv_bc2) + eps);
  return p * decay - lr * upd;
}

template <bool MULTIMEM>
__global__ void __launch_bounds__(256)
    adam_shard_gather_kernel(const __grid_constant__ AdamShard a, const float* __restrict__ coef_ptr, float lr,
                             float b1, float b2, float eps, float wd, int skip_ptr_valid,
                             const float* __restrict__ skip_ptr) {
  // A step that the gradient gate marked non-finite (GradScaler overflow) is skipped on the device.
  if (skip_ptr_valid && *skip_ptr != 0.f) return;
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  const float decay = 1.f - lr * wd;
  const long long total = a.first[a.n];
  for (long long w = blockIdx.x; w < total; w += gridDim.x) {
    int i = 0;
    while (a.first[i + 1] <= w) ++i;
    const long long s0 = a.lo[i] + (w - a.first[i]) * kShardChunk;
    const long long s1 = min(a.hi[i], s0 + kShardChunk);
    if (!debug_bounds_ok(a.status, kSiteAdamShard, s1 - 1, a.ext[i])) continue;  // uniform over the block
    const float inv_bc1 = 1.f / a.bc1[i], inv_bc2 = 1.f / a.bc2[i];
    float* p = a.p[i];
    const float* g = a.g[i];
    float* m = a.m[i];
    float* v = a.v[i];
    const long long n4 = (s1 - s0) >> 2;
    for (long long k = threadIdx.x; k < n4; k += blockDim.x) {
      const long long j = s0 + 4 * k;
      const float4 pv = *reinterpret_cast<const float4*>(p + j);
      const float4 gv = *reinterpret_cast<const float4*>(g + j);
      float4 mv = *reinterpret_cast<const float4*>(m + j);
      float4 vv = *reinterpret_cast<const float4*>(v + j);
      float4 pn;
      pn.x = adam_elem(pv.x, gv.x * coef, mv.x, vv.x, b1, b2, inv_bc1, inv_bc2, eps, lr, decay);
      pn.y = adam_elem(pv.y, gv.y * coef, mv.y, vv.y, b1, b2, inv_bc1, inv_bc2, eps, lr, decay);
      pn.z = adam_elem(pv.z, gv.z * coef, mv.z, vv.z, b1, b2, inv_bc1, inv_bc2, eps, lr, decay);
      pn.w = adam_elem(pv.w, gv.w * coef, mv.w, vv.w, b1, b2, inv_bc1, inv_bc2, eps, lr, decay);
      *reinterpret_cast<float4*>(m + j) = mv;
      *reinterpret_cast<float4*>(v + j) = vv;
      publish4<MULTIMEM>(a, p + j, pn);
    }
    for (long long j = s0 + 4 * n4 + threadIdx.x; j < s1; j += blockDim.x) {  // ragged end of a tensor
      float mj = m[j], vj = v[j];
      const float pn = adam_elem(p[j], g[j] * coef, mj, vj, b1, b2, inv_bc1, inv_bc2, eps, lr, decay);
      m[j] = mj;
      v[j] = vj;
      publish1<MULTIMEM>(a, p + j, pn);
    }
  }
  if constexpr (MULTIMEM) asm volatile("fence.proxy.alias;" ::: "memory");
  __threadfence_system();
}

}  // namespace

// params / grads / exp_avg / exp_avg_sq: full-size fp32 tensors (params inside
// the local slab); lo / hi: this rank's shard of each; steps: Adam step count
// per tensor (after increment); coef: clip coefficient (device scalar) or
// None; skip: a device fp32 flag (non-zero: skip the update) or None.
void adam_shard_gather(const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& grads,
                       const std::vector<at::Tensor>& exp_avg, const std::vector<at::Tensor>& exp_avg_sq,
                       const std::vector<int64_t>& lo, const std::vector<int64_t>& hi,
                       const std::vector<int64_t>& steps, const c10::optional<at::Tensor>& coef,
                       const c10::optional<at::Tensor>& skip, double lr, double beta1, double beta2, double eps,
                       double weight_decay, const std::vector<int64_t>& bases, int64_t mc_base, int64_t rank,
                       int64_t slab_bytes) {
  const size_t n = params.size();
  KB_CHECK(grads.size() == n && exp_avg.size() == n && exp_avg_sq.size() == n && lo.size() == n && hi.size() == n &&
               steps.size() == n,
           "adam_shard_gather: list lengths differ");
  if (n == 0) return;
  const int world = (int)bases.size();
  KB_CHECK(world >= 1 && world <= kGatherRanks, "adam_shard_gather: world size must be 1..8");
  KB_CHECK(rank >= 0 && rank < world, "adam_shard_gather: bad rank");
  for (int q = 0; q < world; ++q) KB_CHECK(bases[q] != 0 && bases[q] % 16 == 0, "adam_shard_gather: bad slab base");
  KB_CHECK(mc_base % 16 == 0, "adam_shard_gather: multicast base must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(params[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const float* cp = (coef.has_value() && coef->defined()) ? coef->data_ptr<float>() : nullptr;
  // An explicit flag, else the one of the step being enqueued (step_guard.h).
  const float* sp = (skip.has_value() && skip->defined()) ? skip->data_ptr<float>() : step_skip_ptr();
  for (size_t base = 0; base < n; base += kShardT) {
    const int count = (int)std::min<size_t>(kShardT, n - base);
    AdamShard a{};
    a.n = count;
    a.world = world;
    for (int q = 0; q < world; ++q) a.delta[q] = bases[q] - bases[rank];
    a.mc_delta = mc_base ? mc_base - bases[rank] : 0;
    a.status = device_status_ptr(params[0].get_device());
    a.first[0] = 0;
    for (int j = 0; j < count; ++j) {
      const size_t k = base + j;
      const at::Tensor& p = params[k];
      KB_CHECK(p.scalar_type() == at::kFloat && p.is_contiguous() && grads[k].scalar_type() == at::kFloat &&
                   grads[k].is_contiguous() && exp_avg[k].is_contiguous() && exp_avg_sq[k].is_contiguous() &&
                   grads[k].numel() == p.numel() && exp_avg[k].numel() == p.numel() &&
                   exp_avg_sq[k].numel() == p.numel(),
               "adam_shard_gather: full-size fp32 contiguous tensors required");
      KB_CHECK(lo[k] >= 0 && lo[k] <= hi[k] && hi[k] <= p.numel() && lo[k] % 4 == 0,
               "adam_shard_gather: shard bounds out of range (lo must be a multiple of 4)");
      const int64_t addr = reinterpret_cast<int64_t>(p.data_ptr());
      KB_CHECK(addr % 16 == 0 && addr >= bases[rank] && addr + 4 * p.numel() <= bases[rank] + slab_bytes,
               "adam_shard_gather: parameter must lie in the local slab");
      for (const at::Tensor* t : {&grads[k], &exp_avg[k], &exp_avg_sq[k]})
        KB_CHECK(reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0, "adam_shard_gather: 16-byte alignment required");
      a.p[j] = p.data_ptr<float>();
      a.g[j] = grads[k].data_ptr<float>();
      a.m[j] = exp_avg[k].data_ptr<float>();
      a.v[j] = exp_avg_sq[k].data_ptr<float>();
      a.lo[j] = lo[k];
      a.hi[j] = hi[k];
      a.ext[j] = std::min({declared_extent(p), declared_extent(grads[k]), declared_extent(exp_avg[k]),
                           declared_extent(exp_avg_sq[k])});
      a.first[j + 1] = a.first[j] + (hi[k] - lo[k] + kShardChunk - 1) / kShardChunk;
      a.bc1[j] = (float)(1.0 - std::pow(beta1, (double)steps[k]));
      a.bc2[j] = (float)(1.0 - std::pow(beta2, (double)steps[k]));
    }
    if (a.first[count] == 0) continue;
    const int grid = (int)std::min<long long>(a.first[count], 4LL * num_sms(params[0].get_device()));
    if (mc_base != 0) {
      adam_shard_gather_kernel<true><<<grid, 256, 0, s>>>(a, cp, (float)lr, (float)beta1, (float)beta2, (float)eps,
                                                         (float)weight_decay, sp != nullptr, sp);
    } else {
      adam_shard_gather_kernel<false><<<grid, 256, 0, s>>>(a, cp, (float)lr, (float)beta1, (float)beta2, (float)eps,
                                                          (float)weight_decay, sp != nullptr, sp);
    }
    KB_LAUNCHED();
  }
}

void register_muon_gather_ops(pybind11::module& m) {
  m.def("muon_update_gather", &muon_update_gather,
        "owner's Muon update written into every rank's parameter copy (P2P or multimem stores)", pybind11::arg("params"),
        pybind11::arg("X"), pybind11::arg("shadow"), pybind11::arg("lr"), pybind11::arg("wd"), pybind11::arg("scale"),
        pybind11::arg("transpose"), pybind11::arg("bases"), pybind11::arg("mc_base"), pybind11::arg("rank"),
        pybind11::arg("slab_bytes"), pybind11::arg("row_scale") = pybind11::none());
  m.def("adam_shard_gather", &adam_shard_gather,
        "AdamW on this rank's shard of each tensor, new values written into every rank's copy (P2P or multimem)");
}

}  // namespace kb
