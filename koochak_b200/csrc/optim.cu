// Optimizer-side kernels for sm_100a.
//
//  * grad_stats: one pass over every gradient that (optionally) unscales it in
//    place (GradScaler), flags any non-finite entry, and accumulates per-tensor
//    sums of squares in fp64; a one-thread finalize turns them into the global
//    L2 norm and the clip coefficient min(1, max_norm / (norm + 1e-6)) on the
//    device, so the host needs one small read per step.
//  * adamw_step: the Adam update of the aux-Adam groups (bias-corrected,
//    decoupled weight decay) with the clip coefficient applied on read, and
//    optionally the EMA update of the new parameter and its bf16 shadow copy,
//    all in one pass.
//  * muon_prologue / muon_scale / muon_epilogue: the per-matrix parts of Muon
//    around the Newton-Schulz GEMMs (momentum + Nesterov + bf16 cast with an
//    optional transpose + Frobenius sum of squares; normalisation; parameter
//    update with weight decay, fused EMA and bf16 shadow).
//  * ema_update: shadow = d * shadow + (1 - d) * param for a tensor list.
//  * normuon_row_scale: NorMuon's per-row second moments and update scales.
//  * hyperball_project: each matrix scaled back to its radius after a step.
//
// Tensor lists are passed by value in the kernel parameter block (<= 32 KB)
// together with a block table, so a call is one launch and no host-to-device
// copy.
#include "host_utils.h"
#include "step_guard.h"
#include "sm100.cuh"

#include <torch/extension.h>

#include <cmath>
#include <vector>

namespace kb {

constexpr int kChunk = 8192;      // elements per block-table entry
constexpr int kMaxT = 96;         // tensors per launch
constexpr int kMaxBlocks = 1024;  // block-table entries per launch

struct BlockTable {
  int n_blocks;
  int tensor[kMaxBlocks];
  int chunk[kMaxBlocks];
};

template <typename F>
static void for_each_launch(const std::vector<int64_t>& numels, F&& launch) {
  // Splits the tensor list into launches that respect kMaxT and kMaxBlocks.
  size_t t = 0;
  int64_t chunk_in_t = 0;
  while (t < numels.size()) {
    std::vector<int> tensors;
    BlockTable bt;
    bt.n_blocks = 0;
    while (t < numels.size() && (int)tensors.size() < kMaxT && bt.n_blocks < kMaxBlocks) {
      const int64_t nch = (numels[t] + kChunk - 1) / kChunk;
      if (tensors.empty() || tensors.back() != (int)t) tensors.push_back((int)t);
      const int local = (int)tensors.size() - 1;
      while (chunk_in_t < nch && bt.n_blocks < kMaxBlocks) {
        bt.tensor[bt.n_blocks] = local;
        bt.chunk[bt.n_blocks] = (int)chunk_in_t;
        ++bt.n_blocks;
        ++chunk_in_t;
      }
      if (chunk_in_t >= nch) {
        ++t;
        chunk_in_t = 0;
      }
    }
    if (bt.n_blocks > 0) launch(tensors, bt);
  }
}

// ------------------------------------------------------------ grad stats

struct GradStatsArgs {
  int n;
  float* g[kMaxT];
  long long numel[kMaxT];
  int global_index[kMaxT];  // index into the per-tensor accumulator array
};

__global__ void __launch_bounds__(256)
    grad_stats_kernel(const __grid_constant__ GradStatsArgs a, const __grid_constant__ BlockTable bt,
                      const float* __restrict__ inv_scale, double* __restrict__ sumsq, int* __restrict__ nonfinite) {
  const int ti = bt.tensor[blockIdx.x];
  float* g = a.g[ti];
  const long long n = a.numel[ti];
  const long long start = (long long)bt.chunk[blockIdx.x] * kChunk;
  const long long end = min(n, start + kChunk);
  const float s = inv_scale ? *inv_scale : 1.f;
  float acc = 0.f;
  bool bad = false;
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
    float x = g[i];
    if (inv_scale) {
      x *= s;
      g[i] = x;
    }
    bad |= !isfinite(x);
    acc += x * x;
  }
  acc = warp_sum(acc);
  __shared__ float red[8];
  __shared__ int any_bad;
  if (threadIdx.x == 0) any_bad = 0;
  __syncthreads();
  if (bad) any_bad = 1;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    atomicAdd(&sumsq[a.global_index[ti]], (double)t);
    if (any_bad) atomicExch(nonfinite, 1);
  }
}

// out[0] = global norm, out[1] = clip coefficient, out[2] = non-finite flag (0/1)
__global__ void grad_stats_finalize_kernel(const double* __restrict__ sumsq, int n, const int* __restrict__ nonfinite,
                                           float max_norm, int clip, float* __restrict__ out,
                                           float* __restrict__ per_tensor_norm) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double total = 0.0;
  for (int i = 0; i < n; ++i) {
    const double v = sumsq[i];
    // Per-tensor norms are rounded to fp32 first, as a foreach norm would.
    const float nt = (float)sqrt(v);
    if (per_tensor_norm) per_tensor_norm[i] = nt;
    total += (double)nt * (double)nt;
  }
  const double norm = sqrt(total);
  float coef = 1.f;
  if (clip) {
    const double c = (double)max_norm / (norm + 1e-6);
    coef = (float)(c < 1.0 ? c : 1.0);
  }
  out[0] = (float)norm;
  out[1] = coef;
  out[2] = (*nonfinite || !isfinite(norm)) ? 1.f : 0.f;
}

// grads: fp32 tensors. scratch: fp64 [n] + int flag (caller supplies, zeroed here).
// out: fp32 [3] as above. per_tensor: optional fp32 [n].
void grad_stats(const std::vector<at::Tensor>& grads, const c10::optional<at::Tensor>& inv_scale, double max_norm,
                bool clip, at::Tensor& scratch, at::Tensor& out, const c10::optional<at::Tensor>& per_tensor) {
  KB_CHECK(!grads.empty(), "grad_stats: empty gradient list");
  const int n = (int)grads.size();
  KB_CHECK(scratch.scalar_type() == at::kDouble && scratch.numel() >= n + 1, "grad_stats: scratch must be fp64 [n+1]");
  const c10::cuda::CUDAGuard guard(grads[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  double* sumsq = scratch.data_ptr<double>();
  int* flag = reinterpret_cast<int*>(sumsq + n);
  KB_CUDA_CHECK(cudaMemsetAsync(sumsq, 0, (n + 1) * sizeof(double), s));
  std::vector<int64_t> numels;
  for (auto& g : grads) {
    KB_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && g.is_cuda(), "grad_stats: fp32 contiguous CUDA grads");
    numels.push_back(g.numel());
  }
  const float* isp = (inv_scale.has_value() && inv_scale->defined()) ? inv_scale->data_ptr<float>() : nullptr;
  int base = 0;
  for_each_launch(numels, [&](const std::vector<int>& tensors, const BlockTable& bt) {
    GradStatsArgs a{};
    a.n = (int)tensors.size();
    for (int i = 0; i < a.n; ++i) {
      const int gi = tensors[i];
      a.g[i] = grads[gi].data_ptr<float>();
      a.numel[i] = grads[gi].numel();
      a.global_index[i] = gi;
    }
    grad_stats_kernel<<<bt.n_blocks, 256, 0, s>>>(a, bt, isp, sumsq, flag);
    KB_LAUNCHED();
    base += a.n;
  });
  float* ptn = (per_tensor.has_value() && per_tensor->defined()) ? per_tensor->data_ptr<float>() : nullptr;
  grad_stats_finalize_kernel<<<1, 32, 0, s>>>(sumsq, n, flag, (float)max_norm, clip ? 1 : 0, out.data_ptr<float>(), ptn);
  KB_LAUNCHED();
}

// ------------------------------------------------------------ AdamW

struct AdamArgs {
  int n;
  float* p[kMaxT];
  const float* g[kMaxT];
  float* m[kMaxT];
  float* v[kMaxT];
  float* ema[kMaxT];       // may be null
  void* shadow[kMaxT];     // bf16 copy, may be null
  long long numel[kMaxT];
  float bc1[kMaxT];        // 1 - beta1^step
  float bc2[kMaxT];        // 1 - beta2^step
  const float* skip;       // device skip flag (step_guard.h) or null
};

__global__ void __launch_bounds__(256)
    adamw_kernel(const __grid_constant__ AdamArgs a, const __grid_constant__ BlockTable bt,
                 const float* __restrict__ coef_ptr, float lr, float beta1, float beta2, float eps, float wd,
                 float ema_decay) {
  if (step_skipped(a.skip)) return;
  const int ti = bt.tensor[blockIdx.x];
  const long long n = a.numel[ti];
  const long long start = (long long)bt.chunk[blockIdx.x] * kChunk;
  const long long end = min(n, start + kChunk);
  float* p = a.p[ti];
  const float* g = a.g[ti];
  float* m = a.m[ti];
  float* v = a.v[ti];
  float* e = a.ema[ti];
  __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(a.shadow[ti]);
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  const float inv_bc1 = 1.f / a.bc1[ti];
  const float inv_bc2 = 1.f / a.bc2[ti];
  const float decay = 1.f - lr * wd;
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float gi = g[i] * coef;
    float mi = m[i];
    float vi = v[i];
    mi = mi + (1.f - beta1) * (gi - mi);
    vi = vi + (1.f - beta2) * (gi * gi - vi);
    m[i] = mi;
    v[i] = vi;
    const float upd = (mi * inv_bc1) / (sqrtf(vi * inv_bc2) + eps);
    const float pn = p[i] * decay - lr * upd;
    p[i] = pn;
    if (e) e[i] = e[i] * ema_decay + (1.f - ema_decay) * pn;
    if (sh) sh[i] = __float2bfloat16_rn(pn);
  }
}

void adamw_step(const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& grads,
                const std::vector<at::Tensor>& exp_avg, const std::vector<at::Tensor>& exp_avg_sq,
                const std::vector<int64_t>& steps, const std::vector<at::Tensor>& ema,
                const std::vector<at::Tensor>& shadow, const c10::optional<at::Tensor>& coef, double lr, double beta1,
                double beta2, double eps, double weight_decay, double ema_decay) {
  const size_t n = params.size();
  KB_CHECK(grads.size() == n && exp_avg.size() == n && exp_avg_sq.size() == n && steps.size() == n,
           "adamw_step: list lengths differ");
  KB_CHECK(ema.empty() || ema.size() == n, "adamw_step: ema list length");
  KB_CHECK(shadow.empty() || shadow.size() == n, "adamw_step: shadow list length");
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(params[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  std::vector<int64_t> numels;
  for (size_t i = 0; i < n; ++i) {
    KB_CHECK(params[i].scalar_type() == at::kFloat && params[i].is_contiguous() && grads[i].is_contiguous() &&
                 grads[i].scalar_type() == at::kFloat && exp_avg[i].is_contiguous() && exp_avg_sq[i].is_contiguous(),
             "adamw_step: fp32 contiguous tensors required");
    numels.push_back(params[i].numel());
  }
  const float* cp = (coef.has_value() && coef->defined()) ? coef->data_ptr<float>() : nullptr;
  for_each_launch(numels, [&](const std::vector<int>& tensors, const BlockTable& bt) {
    AdamArgs a{};
    a.skip = step_skip_ptr();
    a.n = (int)tensors.size();
    for (int i = 0; i < a.n; ++i) {
      const int k = tensors[i];
      a.p[i] = params[k].data_ptr<float>();
      a.g[i] = grads[k].data_ptr<float>();
      a.m[i] = exp_avg[k].data_ptr<float>();
      a.v[i] = exp_avg_sq[k].data_ptr<float>();
      a.ema[i] = (ema.empty() || ema[k].numel() == 0) ? nullptr : ema[k].data_ptr<float>();
      a.shadow[i] = (shadow.empty() || shadow[k].numel() == 0) ? nullptr : shadow[k].data_ptr();
      a.numel[i] = params[k].numel();
      a.bc1[i] = (float)(1.0 - std::pow(beta1, (double)steps[k]));
      a.bc2[i] = (float)(1.0 - std::pow(beta2, (double)steps[k]));
    }
    adamw_kernel<<<bt.n_blocks, 256, 0, s>>>(a, bt, cp, (float)lr, (float)beta1, (float)beta2, (float)eps,
                                             (float)weight_decay, (float)ema_decay);
    KB_LAUNCHED();
  });
}

// ------------------------------------------------------------ EMA

struct EmaArgs {
  int n;
  float* shadow[kMaxT];
  const float* param[kMaxT];
  long long numel[kMaxT];
};

__global__ void __launch_bounds__(256) ema_kernel(const __grid_constant__ EmaArgs a, const __grid_constant__ BlockTable bt,
                                                  float d) {
  const int ti = bt.tensor[blockIdx.x];
  const long long n = a.numel[ti];
  const long long start = (long long)bt.chunk[blockIdx.x] * kChunk;
  const long long end = min(n, start + kChunk);
  float* sh = a.shadow[ti];
  const float* p = a.param[ti];
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) sh[i] = sh[i] * d + (1.f - d) * p[i];
}

void ema_update(const std::vector<at::Tensor>& shadow, const std::vector<at::Tensor>& params, double decay) {
  KB_CHECK(shadow.size() == params.size(), "ema_update: list lengths differ");
  if (shadow.empty()) return;
  const c10::cuda::CUDAGuard guard(shadow[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  std::vector<int64_t> numels;
  for (size_t i = 0; i < shadow.size(); ++i) {
    KB_CHECK(shadow[i].scalar_type() == at::kFloat && params[i].scalar_type() == at::kFloat &&
                 shadow[i].is_contiguous() && params[i].is_contiguous() && shadow[i].numel() == params[i].numel(),
             "ema_update: fp32 contiguous tensors of equal size required");
    numels.push_back(shadow[i].numel());
  }
  for_each_launch(numels, [&](const std::vector<int>& tensors, const BlockTable& bt) {
    EmaArgs a{};
    a.n = (int)tensors.size();
    for (int i = 0; i < a.n; ++i) {
      a.shadow[i] = shadow[tensors[i]].data_ptr<float>();
      a.param[i] = params[tensors[i]].data_ptr<float>();
      a.numel[i] = shadow[tensors[i]].numel();
    }
    ema_kernel<<<bt.n_blocks, 256, 0, s>>>(a, bt, (float)decay);
    KB_LAUNCHED();
  });
}

// ------------------------------------------------------------ Muon

constexpr int kMuonMax = 64;
struct MuonMats {
  int n;
  int R, C;  // parameter shape (rows, cols)
  const float* g[kMuonMax];
  float* mom[kMuonMax];
  float* p[kMuonMax];
  float* ema[kMuonMax];
  void* shadow[kMuonMax];
  const float* skip;  // device skip flag (step_guard.h) or null
};

// X[i] = bf16(nesterov(momentum update)) stored [R, C] or transposed [C, R];
// sumsq[i] += sum X^2 (of the bf16 values).
__global__ void __launch_bounds__(256)
    muon_prologue_kernel(const __grid_constant__ MuonMats mm, __nv_bfloat16* __restrict__ X, float* __restrict__ sumsq,
                         const float* __restrict__ coef_ptr, float beta, int nesterov, int transpose) {
  if (step_skipped(mm.skip)) return;
  const int i = blockIdx.z;
  const int R = mm.R, C = mm.C;
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  __shared__ float tile[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const float* g = mm.g[i];
  float* m = mm.mom[i];
  float local = 0.f;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = r0 + ty + 8 * k, c = c0 + tx;
    float u = 0.f;
    if (r < R && c < C) {
      const long long idx = (long long)r * C + c;
      const float gi = g[idx] * coef;
      float mi = m[idx];
      mi = mi + (1.f - beta) * (gi - mi);
      m[idx] = mi;
      u = nesterov ? gi + beta * (mi - gi) : mi;
      u = __bfloat162float(__float2bfloat16_rn(u));
      local += u * u;
      if (!transpose) X[(long long)i * R * C + idx] = __float2bfloat16_rn(u);
    }
    tile[ty + 8 * k][tx] = u;
  }
  if (transpose) {
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + ty + 8 * k, r = r0 + tx;  // output row = c, col = r
      if (r < R && c < C) X[(long long)i * R * C + (long long)c * R + r] = __float2bfloat16_rn(tile[tx][ty + 8 * k]);
    }
  }
  local = warp_sum(local);
  __shared__ float part[8];
  if (tx == 0) part[ty] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += part[k];
    atomicAdd(&sumsq[i], t);
  }
}

// X[i] *= 1 / (sqrt(sumsq[i]) + 1e-7)
__global__ void muon_scale_kernel(__nv_bfloat16* __restrict__ X, const float* __restrict__ sumsq, long long per_mat) {
  const int i = blockIdx.y;
  const float inv = 1.f / (sqrtf(sumsq[i]) + 1e-7f);
  __nv_bfloat16* x = X + (long long)i * per_mat;
  for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < per_mat; j += (long long)gridDim.x * blockDim.x)
    x[j] = __float2bfloat16_rn(__bfloat162float(x[j]) * inv);
}

// The same scaling, eight values (one 16-byte access) per thread; needs
// per_mat % 8 == 0 and a 16-byte aligned X.
__global__ void muon_scale_vec_kernel(__nv_bfloat16* __restrict__ X, const float* __restrict__ sumsq,
                                      long long per_mat) {
  const int i = blockIdx.y;
  const float inv = 1.f / (sqrtf(sumsq[i]) + 1e-7f);
  uint4* x = reinterpret_cast<uint4*>(X + (long long)i * per_mat);
  const long long n8 = per_mat >> 3;
  for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < n8; j += (long long)gridDim.x * blockDim.x) {
    uint4 q = x[j];
    __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&q);
#pragma unroll
    for (int t = 0; t < 8; ++t) e[t] = __float2bfloat16_rn(__bfloat162float(e[t]) * inv);
    x[j] = q;
  }
}

// p = p * (1 - lr*wd) - lr * scale * U  (U = X or X^T), then EMA and bf16 shadow.
__global__ void __launch_bounds__(256)
    muon_epilogue_kernel(const __grid_constant__ MuonMats mm, const __nv_bfloat16* __restrict__ X, float lr, float wd,
                         float scale, int transpose, float ema_decay, const float* __restrict__ row_scale) {
  if (step_skipped(mm.skip)) return;
  const int i = blockIdx.z;
  const int R = mm.R, C = mm.C;
  __shared__ float tile[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const __nv_bfloat16* x = X + (long long)i * R * C;
  if (transpose) {
    // X is [C, R]: read a 32x32 block coalesced along R, transpose through smem.
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + ty + 8 * k, r = r0 + tx;
      tile[ty + 8 * k][tx] = (r < R && c < C) ? __bfloat162float(x[(long long)c * R + r]) : 0.f;
    }
    __syncthreads();
  }
  float* p = mm.p[i];
  float* e = mm.ema[i];
  __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(mm.shadow[i]);
  const float decay = 1.f - lr * wd;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = r0 + ty + 8 * k, c = c0 + tx;
    if (r < R && c < C) {
      const long long idx = (long long)r * C + c;
      const float u = transpose ? tile[tx][ty + 8 * k] : __bfloat162float(x[idx]);
      const float f = row_scale ? row_scale[(long long)i * R + r] : scale;
      const float pn = p[idx] * decay - lr * (f * u);
      p[idx] = pn;
      if (e) e[idx] = e[idx] * ema_decay + (1.f - ema_decay) * pn;
      if (sh) sh[idx] = __float2bfloat16_rn(pn);
    }
  }
}

// Flat variants for matrices already in their wide orientation (no
// transpose): every operand shares one contiguous index, so a CTA takes 4096
// consecutive elements, four float4 per thread with all loads issued before
// the first use (the tiled kernels above keep one 4-byte load per thread in
// flight). Same expressions as the tiled kernels.
constexpr int kFlatVecs = 4;                  // float4 per thread
constexpr int kFlatVecsPerCta = 256 * kFlatVecs;

__device__ __forceinline__ uint2 pack_bf16x4(float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 r;
  r.x = *reinterpret_cast<uint32_t*>(&lo);
  r.y = *reinterpret_cast<uint32_t*>(&hi);
  return r;
}

__device__ __forceinline__ float4 unpack_bf16x4(uint2 r) {
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&r.x);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&r.y);
  return make_float4(__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi));
}

__global__ void __launch_bounds__(256)
    muon_prologue_flat_kernel(const __grid_constant__ MuonMats mm, __nv_bfloat16* __restrict__ X,
                              float* __restrict__ sumsq, const float* __restrict__ coef_ptr, float beta, int nesterov) {
  if (step_skipped(mm.skip)) return;
  const int i = blockIdx.y;
  const long long n4 = (long long)mm.R * mm.C / 4;
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  const float4* g = reinterpret_cast<const float4*>(mm.g[i]);
  float4* m = reinterpret_cast<float4*>(mm.mom[i]);
  uint2* x = reinterpret_cast<uint2*>(X + (long long)i * mm.R * mm.C);
  const long long j0 = (long long)blockIdx.x * kFlatVecsPerCta + threadIdx.x;
  float4 gv[kFlatVecs], mv[kFlatVecs];
#pragma unroll
  for (int k = 0; k < kFlatVecs; ++k) {
    const long long j = j0 + k * 256;
    if (j < n4) {
      gv[k] = g[j];
      mv[k] = m[j];
    }
  }
  float local = 0.f;
#pragma unroll
  for (int k = 0; k < kFlatVecs; ++k) {
    const long long j = j0 + k * 256;
    if (j < n4) {
      float gi[4] = {gv[k].x * coef, gv[k].y * coef, gv[k].z * coef, gv[k].w * coef};
      float mi[4] = {mv[k].x, mv[k].y, mv[k].z, mv[k].w};
      float u[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        mi[e] = mi[e] + (1.f - beta) * (gi[e] - mi[e]);
        const float t = nesterov ? gi[e] + beta * (mi[e] - gi[e]) : mi[e];
        u[e] = __bfloat162float(__float2bfloat16_rn(t));
        local += u[e] * u[e];
      }
      m[j] = make_float4(mi[0], mi[1], mi[2], mi[3]);
      x[j] = pack_bf16x4(u[0], u[1], u[2], u[3]);
    }
  }
  local = warp_sum(local);
  __shared__ float part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += part[k];
    atomicAdd(&sumsq[i], t);
  }
}

__global__ void __launch_bounds__(256)
    muon_epilogue_flat_kernel(const __grid_constant__ MuonMats mm, const __nv_bfloat16* __restrict__ X, float lr,
                              float wd, float scale, float ema_decay, const float* __restrict__ row_scale) {
  if (step_skipped(mm.skip)) return;
  const int i = blockIdx.y;
  const long long n4 = (long long)mm.R * mm.C / 4;
  float4* p = reinterpret_cast<float4*>(mm.p[i]);
  float4* e = reinterpret_cast<float4*>(mm.ema[i]);
  uint2* sh = reinterpret_cast<uint2*>(mm.shadow[i]);
  const uint2* x = reinterpret_cast<const uint2*>(X + (long long)i * mm.R * mm.C);
  const long long j0 = (long long)blockIdx.x * kFlatVecsPerCta + threadIdx.x;
  const float decay = 1.f - lr * wd;
  float4 pv[kFlatVecs];
  uint2 xv[kFlatVecs];
#pragma unroll
  for (int k = 0; k < kFlatVecs; ++k) {
    const long long j = j0 + k * 256;
    if (j < n4) {
      pv[k] = p[j];
      xv[k] = x[j];
    }
  }
#pragma unroll
  for (int k = 0; k < kFlatVecs; ++k) {
    const long long j = j0 + k * 256;
    if (j < n4) {
      const float4 u = unpack_bf16x4(xv[k]);
      // C % 4 == 0 on this path, so a float4 never straddles two rows.
      const float f = row_scale ? row_scale[(long long)i * mm.R + (4 * j) / mm.C] : scale;
      float4 pn;
      pn.x = pv[k].x * decay - lr * (f * u.x);
      pn.y = pv[k].y * decay - lr * (f * u.y);
      pn.z = pv[k].z * decay - lr * (f * u.z);
      pn.w = pv[k].w * decay - lr * (f * u.w);
      p[j] = pn;
      if (e) {
        const float4 ev = e[j];
        e[j] = make_float4(ev.x * ema_decay + (1.f - ema_decay) * pn.x, ev.y * ema_decay + (1.f - ema_decay) * pn.y,
                           ev.z * ema_decay + (1.f - ema_decay) * pn.z, ev.w * ema_decay + (1.f - ema_decay) * pn.w);
      }
      if (sh) sh[j] = pack_bf16x4(pn.x, pn.y, pn.z, pn.w);
    }
  }
}

static bool aligned(const void* ptr, uintptr_t a) { return ptr == nullptr || reinterpret_cast<uintptr_t>(ptr) % a == 0; }

static MuonMats make_mats(const std::vector<at::Tensor>& grads, const std::vector<at::Tensor>& moms,
                          const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& ema,
                          const std::vector<at::Tensor>& shadow, size_t base, int count) {
  MuonMats mm{};
  mm.skip = step_skip_ptr();
  mm.n = count;
  const auto& p0 = params.empty() ? grads[base] : params[base];
  mm.R = (int)p0.size(0);
  mm.C = (int)(p0.numel() / p0.size(0));
  for (int j = 0; j < count; ++j) {
    const size_t k = base + j;
    if (!grads.empty()) mm.g[j] = grads[k].data_ptr<float>();
    if (!moms.empty()) mm.mom[j] = moms[k].data_ptr<float>();
    if (!params.empty()) mm.p[j] = params[k].data_ptr<float>();
    mm.ema[j] = (ema.empty() || ema[k].numel() == 0) ? nullptr : ema[k].data_ptr<float>();
    mm.shadow[j] = (shadow.empty() || shadow[k].numel() == 0) ? nullptr : shadow[k].data_ptr();
  }
  return mm;
}

// X: bf16 [n, r, c] workspace (r <= c after the optional transpose), sumsq: fp32 [n] scratch.
void muon_prologue(const std::vector<at::Tensor>& grads, const std::vector<at::Tensor>& moms, at::Tensor& X,
                   at::Tensor& sumsq, const c10::optional<at::Tensor>& coef, double beta, bool nesterov, bool transpose) {
  const size_t n = grads.size();
  KB_CHECK(n > 0 && moms.size() == n, "muon_prologue: list lengths");
  const c10::cuda::CUDAGuard guard(grads[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const int R = (int)grads[0].size(0);
  const int C = (int)(grads[0].numel() / R);
  for (size_t i = 0; i < n; ++i)
    KB_CHECK(grads[i].is_contiguous() && moms[i].is_contiguous() && grads[i].numel() == (int64_t)R * C &&
                 grads[i].scalar_type() == at::kFloat,
             "muon_prologue: same-shape fp32 contiguous matrices required");
  KB_CHECK(X.scalar_type() == at::kBFloat16 && X.numel() >= (int64_t)n * R * C, "muon_prologue: X too small");
  KB_CUDA_CHECK(cudaMemsetAsync(sumsq.data_ptr<float>(), 0, n * sizeof(float), s));
  const float* cp = (coef.has_value() && coef->defined()) ? coef->data_ptr<float>() : nullptr;
  for (size_t base = 0; base < n; base += kMuonMax) {
    const int count = (int)std::min<size_t>(kMuonMax, n - base);
    MuonMats mm = make_mats(grads, moms, {}, {}, {}, base, count);
    __nv_bfloat16* xb = (__nv_bfloat16*)X.data_ptr() + (int64_t)base * R * C;
    bool flat = !transpose && ((int64_t)R * C) % 4 == 0 && aligned(xb, 8);
    for (int j = 0; j < count && flat; ++j) flat = aligned(mm.g[j], 16) && aligned(mm.mom[j], 16);
    if (flat) {
      const long long n4 = (long long)R * C / 4;
      dim3 grid((unsigned)((n4 + kFlatVecsPerCta - 1) / kFlatVecsPerCta), count);
      muon_prologue_flat_kernel<<<grid, 256, 0, s>>>(mm, xb, sumsq.data_ptr<float>() + base, cp, (float)beta,
                                                     nesterov ? 1 : 0);
    } else {
      dim3 grid((C + 31) / 32, (R + 31) / 32, count);
      muon_prologue_kernel<<<grid, 256, 0, s>>>(mm, xb, sumsq.data_ptr<float>() + base, cp, (float)beta,
                                                nesterov ? 1 : 0, transpose ? 1 : 0);
    }
    KB_LAUNCHED();
  }
}

void muon_scale(at::Tensor& X, const at::Tensor& sumsq, int64_t n) {
  const c10::cuda::CUDAGuard guard(X.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const long long per = X.numel() / X.size(0);
  const bool vec = per % 8 == 0 && (reinterpret_cast<uintptr_t>(X.data_ptr()) & 15) == 0;
  const long long work = vec ? per / 8 : per;
  dim3 grid((unsigned)std::max<long long>(1, std::min<long long>((work + 255) / 256, 256)), (unsigned)n);
  if (vec)
    muon_scale_vec_kernel<<<grid, 256, 0, s>>>((__nv_bfloat16*)X.data_ptr(), sumsq.data_ptr<float>(), per);
  else
    muon_scale_kernel<<<grid, 256, 0, s>>>((__nv_bfloat16*)X.data_ptr(), sumsq.data_ptr<float>(), per);
  KB_LAUNCHED();
}

void muon_epilogue(const std::vector<at::Tensor>& params, const at::Tensor& X, const std::vector<at::Tensor>& ema,
                   const std::vector<at::Tensor>& shadow, double lr, double wd, double scale, bool transpose,
                   double ema_decay, const c10::optional<at::Tensor>& row_scale) {
  const size_t n = params.size();
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(params[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const int R = (int)params[0].size(0);
  const int C = (int)(params[0].numel() / R);
  const float* rs_all = nullptr;
  if (row_scale.has_value() && row_scale->defined()) {
    KB_CHECK(row_scale->scalar_type() == at::kFloat && row_scale->is_contiguous() &&
                 row_scale->numel() >= (int64_t)n * R,
             "muon_epilogue: row_scale must be fp32 [n, rows]");
    rs_all = row_scale->data_ptr<float>();
  }
  for (size_t base = 0; base < n; base += kMuonMax) {
    const int count = (int)std::min<size_t>(kMuonMax, n - base);
    MuonMats mm = make_mats({}, {}, params, ema, shadow, base, count);
    const __nv_bfloat16* xb = (const __nv_bfloat16*)X.data_ptr() + (int64_t)base * R * C;
    const float* rs = rs_all ? rs_all + (int64_t)base * R : nullptr;
    bool flat = !transpose && ((int64_t)R * C) % 4 == 0 && aligned(xb, 8);
    for (int j = 0; j < count && flat; ++j)
      flat = aligned(mm.p[j], 16) && aligned(mm.ema[j], 16) && aligned(mm.shadow[j], 8);
    if (flat) {
      const long long n4 = (long long)R * C / 4;
      dim3 grid((unsigned)((n4 + kFlatVecsPerCta - 1) / kFlatVecsPerCta), count);
      muon_epilogue_flat_kernel<<<grid, 256, 0, s>>>(mm, xb, (float)lr, (float)wd, (float)scale, (float)ema_decay,
                                                     rs);
    } else {
      dim3 grid((C + 31) / 32, (R + 31) / 32, count);
      muon_epilogue_kernel<<<grid, 256, 0, s>>>(mm, xb, (float)lr, (float)wd, (float)scale, transpose ? 1 : 0,
                                                (float)ema_decay, rs);
    }
    KB_LAUNCHED();
  }
}

// ------------------------------------------------------------ NorMuon
//
// NorMuon rescales the orthogonalised update U (rows x cols in the
// parameter's own orientation; X holds U transposed when rows > cols) row by
// row (reference koochak/optim/muon.py:56-74):
//   v_r = mean_c U[r, c]^2,  m2_r <- m2_r + (1 - beta2) (v_r - m2_r)
//   A   = U / (sqrt(m2_r) + 1e-10),  B = A * |U| / (|A| + 1e-10),
//   final update = B * sqrt(max(1, rows / cols)).
// normuon_row_stats: per matrix, the row sums of squares of U.
// normuon_finish:    per matrix (one CTA), the m2 update and one factor per
//                    row, 1/(sqrt(m2_r)+1e-10) * |U|/(|A|+1e-10) *
//                    sqrt(max(1, rows/cols)), which the Muon update kernels
//                    apply in place of the scalar Muon scale.

// Non-transposed: a warp per row of X (contiguous). Transposed (X = U^T,
// [cols, rows]): a thread per U row = X column, walking the X rows, so a warp
// reads 32 consecutive columns of one X row at a time.
__global__ void __launch_bounds__(256)
    normuon_row_stats_kernel(const __nv_bfloat16* __restrict__ X, int R, int C, int transpose,
                             float* __restrict__ rowsq) {
  const int i = blockIdx.y;
  const __nv_bfloat16* x = X + (long long)i * R * C;
  float* out = rowsq + (long long)i * R;
  if (!transpose) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < R; r += gridDim.x * warps) {
      const __nv_bfloat16* row = x + (long long)r * C;
      float acc = 0.f;
      for (int c = lane; c < C; c += 32) {
        const float u = __bfloat162float(row[c]);
        acc += u * u;
      }
      acc = warp_sum(acc);
      if (lane == 0) out[r] = acc;
    }
    return;
  }
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < R; r += gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int c = 0; c < C; ++c) {
      const float u = __bfloat162float(x[(long long)c * R + r]);
      acc += u * u;
    }
    out[r] = acc;
  }
}

constexpr int kNormuonThreads = 512;

struct NormuonMoments {
  float* m[kMuonMax];  // each matrix's second-moment buffer (R values)
  const float* skip;   // device skip flag (step_guard.h) or null
};

__global__ void __launch_bounds__(kNormuonThreads)
    normuon_finish_kernel(const float* __restrict__ rowsq, int R, int C, float beta2,
                          const __grid_constant__ NormuonMoments m2, float* __restrict__ row_scale) {
  if (step_skipped(m2.skip)) return;
  const int i = blockIdx.x;
  const float* sq = rowsq + (long long)i * R;
  float* m = m2.m[i];
  float* scale = row_scale + (long long)i * R;
  __shared__ float red[2][kNormuonThreads / 32];
  float total = 0.f, rescaled = 0.f;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const float v = sq[r] / (float)C;
    const float mr = m[r] + (1.f - beta2) * (v - m[r]);
    m[r] = mr;
    const float inv = 1.f / (sqrtf(mr) + 1e-10f);
    scale[r] = inv;
    total += sq[r];
    rescaled += sq[r] * inv * inv;
  }
  total = warp_sum(total);
  rescaled = warp_sum(rescaled);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    red[0][warp] = total;
    red[1][warp] = rescaled;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    float a = lane < kNormuonThreads / 32 ? red[0][lane] : 0.f;
    float b = lane < kNormuonThreads / 32 ? red[1][lane] : 0.f;
    a = warp_sum(a);
    b = warp_sum(b);
    if (lane == 0) {
      red[0][0] = a;
      red[1][0] = b;
    }
  }
  __syncthreads();
  const float ratio = sqrtf(red[0][0]) / (sqrtf(red[1][0]) + 1e-10f);
  const float shape = sqrtf(fmaxf(1.f, (float)R / (float)C));
  for (int r = threadIdx.x; r < R; r += blockDim.x) scale[r] = scale[r] * ratio * shape;
}

// X: bf16 [n, r, c] orthogonalised batch (U^T when transpose); R, C: the
// parameter shape; second_moments: n fp32 tensors of R values (updated in
// place); rowsq, row_scale: fp32 [n, R] scratch / output.
void normuon_row_scale(const at::Tensor& X, int64_t R, int64_t C, bool transpose,
                       const std::vector<at::Tensor>& second_moments, double beta2, at::Tensor& rowsq,
                       at::Tensor& row_scale) {
  const int64_t n = (int64_t)second_moments.size();
  if (n == 0) return;
  KB_CHECK(X.scalar_type() == at::kBFloat16 && X.is_contiguous() && X.numel() >= n * R * C,
           "normuon_row_scale: X must be contiguous bf16 [n, R*C]");
  KB_CHECK(rowsq.scalar_type() == at::kFloat && rowsq.numel() >= n * R && row_scale.scalar_type() == at::kFloat &&
               row_scale.numel() >= n * R,
           "normuon_row_scale: rowsq / row_scale must be fp32 [n, R]");
  for (int64_t i = 0; i < n; ++i) {
    const at::Tensor& m = second_moments[i];
    KB_CHECK(m.scalar_type() == at::kFloat && m.is_contiguous() && m.numel() == R,
             "normuon_row_scale: second moments must be contiguous fp32 with one value per row");
  }
  const c10::cuda::CUDAGuard guard(X.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const int grid = transpose ? (int)std::min<int64_t>((R + 255) / 256, 64) : (int)std::min<int64_t>((R + 7) / 8, 128);
  normuon_row_stats_kernel<<<dim3(grid, (unsigned)n), 256, 0, s>>>((const __nv_bfloat16*)X.data_ptr(), (int)R, (int)C,
                                                                   transpose ? 1 : 0, rowsq.data_ptr<float>());
  KB_LAUNCHED();
  for (int64_t base = 0; base < n; base += kMuonMax) {
    const int count = (int)std::min<int64_t>(kMuonMax, n - base);
    NormuonMoments mom{};
    mom.skip = step_skip_ptr();
    for (int j = 0; j < count; ++j) mom.m[j] = second_moments[base + j].data_ptr<float>();
    normuon_finish_kernel<<<(unsigned)count, kNormuonThreads, 0, s>>>(rowsq.data_ptr<float>() + base * R, (int)R,
                                                                      (int)C, (float)beta2, mom,
                                                                      row_scale.data_ptr<float>() + base * R);
    KB_LAUNCHED();
  }
}

// ------------------------------------------------------------ hyperball projection
//
// After the inner optimizer's step, each listed matrix is pulled back to its
// radius r (reference koochak/optim/muon.py:158-168):
//   s = r / max(|p|, eps)            (sphere)
//   s = min(1, r / max(|p|, eps))    (ball)
//   p <- p * s   (and its bf16 copy, when the model keeps one)
// Two launches for any number of matrices: per-tensor sums of squares
// (atomics into an fp64 accumulator), then the scaling pass, which forms s
// from the finished sum itself.

struct ProjectArgs {
  int n;
  float* p[kMaxT];
  void* shadow[kMaxT];   // bf16 copy or null
  long long numel[kMaxT];
  int index[kMaxT];      // slot of the tensor in the sums / radii arrays
  const float* skip;     // device skip flag (step_guard.h) or null
};

__global__ void __launch_bounds__(256)
    tensor_sumsq_kernel(const __grid_constant__ ProjectArgs a, const __grid_constant__ BlockTable bt,
                        double* __restrict__ sumsq) {
  const int ti = bt.tensor[blockIdx.x];
  const long long n = a.numel[ti];
  const long long start = (long long)bt.chunk[blockIdx.x] * kChunk;
  const long long end = min(n, start + kChunk);
  const float* p = a.p[ti];
  float acc = 0.f;
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) acc += p[i] * p[i];
  acc = warp_sum(acc);
  __shared__ float part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int k = 0; k < 8; ++k) t += part[k];
    atomicAdd(sumsq + a.index[ti], t);
  }
}

__global__ void __launch_bounds__(256)
    project_radius_kernel(const __grid_constant__ ProjectArgs a, const __grid_constant__ BlockTable bt,
                          const double* __restrict__ sumsq, const float* __restrict__ radii, float eps, int ball) {
  if (step_skipped(a.skip)) return;
  const int ti = bt.tensor[blockIdx.x];
  const long long n = a.numel[ti];
  const long long start = (long long)bt.chunk[blockIdx.x] * kChunk;
  const long long end = min(n, start + kChunk);
  const int slot = a.index[ti];
  const float norm = (float)sqrt(sumsq[slot]);
  float s = radii[slot] / fmaxf(norm, eps);
  if (ball) s = fminf(s, 1.f);
  float* p = a.p[ti];
  __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(a.shadow[ti]);
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float v = p[i] * s;
    p[i] = v;
    if (sh) sh[i] = __float2bfloat16_rn(v);
  }
}

// params: fp32 contiguous matrices; radii: fp32 [n] on the same device;
// shadow: bf16 copies or empty placeholders (possibly an empty list).
void hyperball_project(const std::vector<at::Tensor>& params, const at::Tensor& radii,
                       const std::vector<at::Tensor>& shadow, double eps, bool ball) {
  const size_t n = params.size();
  if (n == 0) return;
  KB_CHECK(radii.scalar_type() == at::kFloat && radii.is_contiguous() && radii.numel() == (int64_t)n,
           "hyperball_project: radii must be fp32 [n]");
  KB_CHECK(shadow.empty() || shadow.size() == n, "hyperball_project: shadow list length");
  const c10::cuda::CUDAGuard guard(params[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  std::vector<int64_t> numels;
  for (const auto& p : params) {
    KB_CHECK(p.scalar_type() == at::kFloat && p.is_contiguous() && p.is_cuda(),
             "hyperball_project: fp32 contiguous CUDA tensors required");
    numels.push_back(p.numel());
  }
  at::Tensor sums = at::zeros({(int64_t)n}, params[0].options().dtype(at::kDouble));
  auto fill = [&](const std::vector<int>& tensors) {
    ProjectArgs a{};
    a.skip = step_skip_ptr();
    a.n = (int)tensors.size();
    for (int j = 0; j < a.n; ++j) {
      const int k = tensors[j];
      a.p[j] = params[k].data_ptr<float>();
      const bool has = !shadow.empty() && shadow[k].numel() == params[k].numel();
      a.shadow[j] = has ? shadow[k].data_ptr() : nullptr;
      a.numel[j] = params[k].numel();
      a.index[j] = k;
    }
    return a;
  };
  for_each_launch(numels, [&](const std::vector<int>& tensors, const BlockTable& bt) {
    tensor_sumsq_kernel<<<bt.n_blocks, 256, 0, s>>>(fill(tensors), bt, sums.data_ptr<double>());
    KB_LAUNCHED();
  });
  for_each_launch(numels, [&](const std::vector<int>& tensors, const BlockTable& bt) {
    project_radius_kernel<<<bt.n_blocks, 256, 0, s>>>(fill(tensors), bt, sums.data_ptr<double>(),
                                                      radii.data_ptr<float>(), (float)eps, ball ? 1 : 0);
    KB_LAUNCHED();
  });
}

static const float* g_step_skip = nullptr;
const float* step_skip_ptr() { return g_step_skip; }
void set_step_skip_ptr(const float* p) { g_step_skip = p; }

// Python: set (a one-element fp32 CUDA tensor, kept alive by the caller for the
// step) or clear (None) the device skip flag of the optimizer step being enqueued.
static void set_step_skip(const c10::optional<at::Tensor>& flag) {
  if (!flag.has_value() || !flag->defined()) {
    g_step_skip = nullptr;
    return;
  }
  KB_CHECK(flag->is_cuda() && flag->scalar_type() == at::kFloat && flag->numel() >= 1,
           "step skip flag must be a CUDA fp32 tensor");
  g_step_skip = flag->data_ptr<float>();
}

void register_optim_ops(pybind11::module& m) {
  m.def("set_step_skip", &set_step_skip,
        "device flag (non-zero: skip) read by the optimizer kernels of the step being enqueued; None clears it",
        pybind11::arg("flag"));
  m.def("grad_stats", &grad_stats);
  m.def("adamw_step", &adamw_step);
  m.def("ema_update", &ema_update);
  m.def("muon_prologue", &muon_prologue);
  m.def("muon_scale", &muon_scale);
  m.def("muon_epilogue", &muon_epilogue, "Muon parameter update (scalar or per-row scale), EMA and bf16 copy",
        pybind11::arg("params"), pybind11::arg("X"), pybind11::arg("ema"), pybind11::arg("shadow"), pybind11::arg("lr"),
        pybind11::arg("wd"), pybind11::arg("scale"), pybind11::arg("transpose"), pybind11::arg("ema_decay"),
        pybind11::arg("row_scale") = pybind11::none());
  m.def("normuon_row_scale", &normuon_row_scale, "NorMuon second-moment update and per-row update scales");
  m.def("hyperball_project", &hyperball_project, "scale each matrix back to its radius (sphere or ball)");
}

}  // namespace kb
