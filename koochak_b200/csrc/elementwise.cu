// Memory-bound kernels for sm_100a: token+position embedding (fwd/bwd),
// fused softmax cross-entropy (fwd saves the log-sum-exp; bwd overwrites the
// logits with their gradient in place), bias gradients (column sums), a
// multi-tensor fp32 -> bf16/fp16 cast, SwiGLU and rotary embedding.
#include "host_utils.h"
#include "sm100.cuh"

#include <torch/extension.h>

#include <type_traits>
#include <vector>

namespace kb {

// ------------------------------------------------------------ embedding

// out[t, :] = wte[idx[t], :] + wpe[t % S, :]   (fp32 out; wpe optional)
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ wte,
                                     const float* __restrict__ wpe, float* __restrict__ out, int T, int S, int C,
                                     int V, int* status) {
  const int t = blockIdx.x;
  if (t >= T) return;
  int64_t tok = idx[t];
  if (tok < 0 || tok >= V) {
    record_status(status, kStatusBadArgs);
    tok = 0;
  }
  const float4* we = reinterpret_cast<const float4*>(wte + tok * (int64_t)C);
  const float4* pe = wpe ? reinterpret_cast<const float4*>(wpe + (int64_t)(t % S) * C) : nullptr;
  float4* o = reinterpret_cast<float4*>(out + (int64_t)t * C);
  for (int i = threadIdx.x; i < C / 4; i += blockDim.x) {
    float4 a = we[i];
    if (pe) {
      const float4 b = pe[i];
      a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
    o[i] = a;
  }
}

// dwte[idx[t]] += dout[t];  dwpe[t % S] += dout[t]   (fp32 atomics)
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ dout,
                                     float* __restrict__ dwte, float* __restrict__ dwpe, int T, int S, int C, int V) {
  const int t = blockIdx.x;
  if (t >= T) return;
  int64_t tok = idx[t];
  if (tok < 0 || tok >= V) return;
  const float* g = dout + (int64_t)t * C;
  float* dw = dwte + tok * (int64_t)C;
  float* dp = dwpe ? dwpe + (int64_t)(t % S) * C : nullptr;
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    const float v = g[i];
    atomicAdd(dw + i, v);
    if (dp) atomicAdd(dp + i, v);
  }
}

void embedding_forward(const at::Tensor& idx, const at::Tensor& wte, const c10::optional<at::Tensor>& wpe,
                       at::Tensor& out, int64_t seq_len) {
  check_cuda_tensor(idx, "idx");
  KB_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous(), "idx must be contiguous int64");
  KB_CHECK(wte.scalar_type() == at::kFloat && wte.is_contiguous() && out.scalar_type() == at::kFloat, "fp32 tables");
  const int C = (int)wte.size(1);
  KB_CHECK(C % 4 == 0, "embedding width must be a multiple of 4");
  const int T = (int)idx.numel();
  const c10::cuda::CUDAGuard guard(idx.device());
  const float* pe = (wpe.has_value() && wpe->defined()) ? wpe->data_ptr<float>() : nullptr;
  embedding_fwd_kernel<<<T, 128, 0, c10::cuda::getCurrentCUDAStream().stream()>>>(
      idx.data_ptr<int64_t>(), wte.data_ptr<float>(), pe, out.data_ptr<float>(), T, (int)seq_len, C,
      (int)wte.size(0), device_status_ptr(idx.get_device()));
  KB_LAUNCHED();
}

void embedding_backward(const at::Tensor& idx, const at::Tensor& dout, at::Tensor& dwte,
                        const c10::optional<at::Tensor>& dwpe, int64_t seq_len) {
  const int C = (int)dwte.size(1);
  const int T = (int)idx.numel();
  KB_CHECK(dout.scalar_type() == at::kFloat && dout.is_contiguous(), "dout must be contiguous fp32");
  const c10::cuda::CUDAGuard guard(idx.device());
  float* dp = (dwpe.has_value() && dwpe->defined()) ? dwpe->data_ptr<float>() : nullptr;
  embedding_bwd_kernel<<<T, 256, 0, c10::cuda::getCurrentCUDAStream().stream()>>>(
      idx.data_ptr<int64_t>(), dout.data_ptr<float>(), dwte.data_ptr<float>(), dp, T, (int)seq_len, C,
      (int)dwte.size(0));
  KB_LAUNCHED();
}

// ------------------------------------------------------------ cross-entropy

// Per row: lse = log(sum exp(z)), loss = lse - z[target] (0 for ignored rows).
// One CTA per row, logits in bf16/fp16/fp32 with row stride ld, V valid columns.
template <typename T>
__device__ __forceinline__ void online_add8(const T* p, float& m, float& s) {
  const uint4 q = *reinterpret_cast<const uint4*>(p);
  const T* e = reinterpret_cast<const T*>(&q);
  float v[8];
  float lm = -INFINITY;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = to_f32<T>(e[j]);
    lm = fmaxf(lm, v[j]);
  }
  if (lm > m) {
    s *= __expf(m - lm);
    m = lm;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) s += __expf(v[j] - m);
}

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
  m = mm;
}

// Per row: lse = log(sum exp(z)), loss = lse - z[target] (0 for ignored rows).
// One CTA per row; 16-byte vector loads when the row is 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(256) ce_fwd_kernel(const T* __restrict__ logits, const int64_t* __restrict__ tgt,
                                                     float* __restrict__ loss, float* __restrict__ lse_out, int V,
                                                     long long ld, int64_t ignore_index) {
  const int row = blockIdx.x;
  const T* z = logits + (long long)row * ld;
  float m = -INFINITY, s = 0.f;
  constexpr int VEC = 16 / sizeof(T);
  const bool aligned = (reinterpret_cast<uintptr_t>(z) & 15) == 0;
  int done = 0;
  if (aligned && VEC == 8) {
    const int nvec = V / 8;
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) online_add8<T>(z + 8 * i, m, s);
    done = nvec * 8;
  }
  for (int i = done + threadIdx.x; i < V; i += blockDim.x) {
    const float v = to_f32<T>(z[i]);
    if (v > m) {
      s = s * __expf(m - v) + 1.f;
      m = v;
    } else {
      s += __expf(v - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[32], ss[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const float l = m + logf(s);
      lse_out[row] = l;
      const int64_t t = tgt[row];
      if (t == ignore_index || t < 0 || t >= V) loss[row] = 0.f;
      else loss[row] = l - to_f32<T>(z[t]);
    }
  }
}

// dz = (softmax(z) - onehot(target)) * scale_row, written over z in place.
// scale_row = grad_scale for counted rows, 0 for ignored rows.
template <typename T>
__global__ void __launch_bounds__(256) ce_bwd_kernel(T* __restrict__ logits, const int64_t* __restrict__ tgt,
                                                     const float* __restrict__ lse, const float* __restrict__ gscale,
                                                     int V, long long ld, int64_t ignore_index) {
  const int row = blockIdx.x;
  T* z = logits + (long long)row * ld;
  const int64_t t = tgt[row];
  const bool ignored = (t == ignore_index || t < 0 || t >= V);
  const float g = ignored ? 0.f : gscale[0];
  const float l = lse[row];
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(z) & 15) == 0 && sizeof(T) == 2) {
    const int nvec = V / 8;
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
      uint4 q = *reinterpret_cast<const uint4*>(z + 8 * i);
      T* e = reinterpret_cast<T*>(&q);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = 8 * i + j;
        const float p = __expf(to_f32<T>(e[j]) - l);
        e[j] = from_f32<T>((p - (col == t ? 1.f : 0.f)) * g);
      }
      *reinterpret_cast<uint4*>(z + 8 * i) = q;
    }
    done = nvec * 8;
  }
  for (int i = done + threadIdx.x; i < V; i += blockDim.x) {
    const float p = __expf(to_f32<T>(z[i]) - l);
    z[i] = from_f32<T>((p - (i == t ? 1.f : 0.f)) * g);
  }
}

void cross_entropy_forward(const at::Tensor& logits, const at::Tensor& target, at::Tensor& loss, at::Tensor& lse,
                           int64_t V, int64_t ignore_index) {
  check_cuda_tensor(logits, "logits");
  KB_CHECK(logits.stride(-1) == 1, "logits must have unit inner stride");
  const int rows = (int)target.numel();
  const long long ld = logits.stride(-2);
  const c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  if (rows == 0) return;
  switch (logits.scalar_type()) {
    case at::kBFloat16:
      ce_fwd_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>((const __nv_bfloat16*)logits.data_ptr(),
                                                        target.data_ptr<int64_t>(), loss.data_ptr<float>(),
                                                        lse.data_ptr<float>(), (int)V, ld, ignore_index);
      break;
    case at::kHalf:
      ce_fwd_kernel<__half><<<rows, 256, 0, s>>>((const __half*)logits.data_ptr(), target.data_ptr<int64_t>(),
                                                 loss.data_ptr<float>(), lse.data_ptr<float>(), (int)V, ld,
                                                 ignore_index);
      break;
    case at::kFloat:
      ce_fwd_kernel<float><<<rows, 256, 0, s>>>(logits.data_ptr<float>(), target.data_ptr<int64_t>(),
                                                loss.data_ptr<float>(), lse.data_ptr<float>(), (int)V, ld, ignore_index);
      break;
    default: KB_CHECK(false, "cross_entropy: unsupported dtype");
  }
  KB_LAUNCHED();
}

void cross_entropy_backward(at::Tensor& logits, const at::Tensor& target, const at::Tensor& lse,
                            const at::Tensor& gscale, int64_t V, int64_t ignore_index) {
  const int rows = (int)target.numel();
  const long long ld = logits.stride(-2);
  const c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  if (rows == 0) return;
  KB_CHECK(gscale.scalar_type() == at::kFloat && gscale.is_cuda(), "gscale must be a CUDA fp32 scalar");
  switch (logits.scalar_type()) {
    case at::kBFloat16:
      ce_bwd_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>((__nv_bfloat16*)logits.data_ptr(), target.data_ptr<int64_t>(),
                                                        lse.data_ptr<float>(), gscale.data_ptr<float>(), (int)V, ld,
                                                        ignore_index);
      break;
    case at::kHalf:
      ce_bwd_kernel<__half><<<rows, 256, 0, s>>>((__half*)logits.data_ptr(), target.data_ptr<int64_t>(),
                                                 lse.data_ptr<float>(), gscale.data_ptr<float>(), (int)V, ld,
                                                 ignore_index);
      break;
    case at::kFloat:
      ce_bwd_kernel<float><<<rows, 256, 0, s>>>(logits.data_ptr<float>(), target.data_ptr<int64_t>(),
                                                lse.data_ptr<float>(), gscale.data_ptr<float>(), (int)V, ld,
                                                ignore_index);
      break;
    default: KB_CHECK(false, "cross_entropy: unsupported dtype");
  }
  KB_LAUNCHED();
}

// ------------------------------------------------------------ bias gradient

// out[n] = sum_m g[m, n] (or out[n] += it), in two deterministic passes:
// CTAs of 256 columns (32 threads x 8 columns, 16-byte loads) x 8 row groups
// sum a slice of rows each and write one partial row; a second kernel sums
// the partial rows. No atomics, so no zero-fill launch before it and the same
// result on every run; each thread keeps four row loads in flight.
template <typename T>
__global__ void __launch_bounds__(256) bias_grad_partial_kernel(const T* __restrict__ g, float* __restrict__ part,
                                                                int M, int N, int rows_per_cta) {
  const int cg = threadIdx.x & 31, rg = threadIdx.x >> 5;
  const int col0 = blockIdx.x * 256 + cg * 8;
  const int r0 = blockIdx.y * rows_per_cta;
  const int r1 = min(M, r0 + rows_per_cta);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const bool vec = (col0 + 8 <= N) && (N % 8 == 0) && sizeof(T) == 2;
  if (vec) {
    int r = r0 + rg;
    for (; r + 24 < r1; r += 32) {
      uint4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = *reinterpret_cast<const uint4*>(g + (long long)(r + 8 * u) * N + col0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const T* e = reinterpret_cast<const T*>(&q[u]);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += to_f32<T>(e[j]);
      }
    }
    for (; r < r1; r += 8) {
      const uint4 q = *reinterpret_cast<const uint4*>(g + (long long)r * N + col0);
      const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += to_f32<T>(e[j]);
    }
  } else {
    for (int r = r0 + rg; r < r1; r += 8) {
      const T* p = g + (long long)r * N + col0;
      for (int j = 0; j < 8; ++j)
        if (col0 + j < N) acc[j] += to_f32<T>(p[j]);
    }
  }
  __shared__ float red[8][257];
#pragma unroll
  for (int j = 0; j < 8; ++j) red[rg][cg * 8 + j] = acc[j];
  __syncthreads();
  const int c = threadIdx.x;  // 256 columns, one per thread
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) t += red[k][c];
  if (blockIdx.x * 256 + c < N) part[(long long)blockIdx.y * N + blockIdx.x * 256 + c] = t;
}

// out[n] (+)= sum_r part[r, n]: 32 columns per CTA, 16 warps over the rows, four loads in flight each.
__global__ void __launch_bounds__(512) bias_grad_finish_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                               int R, int N, int accumulate) {
  const int lane = threadIdx.x & 31, rg = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (col < N) {
    int r = rg;
    for (; r + 48 < R; r += 64) {
      s0 += part[(long long)r * N + col];
      s1 += part[(long long)(r + 16) * N + col];
      s2 += part[(long long)(r + 32) * N + col];
      s3 += part[(long long)(r + 48) * N + col];
    }
    for (; r < R; r += 16) s0 += part[(long long)r * N + col];
  }
  __shared__ float red[16][33];
  red[rg][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (rg == 0 && col < N) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) t += red[k][lane];
    out[col] = accumulate ? out[col] + t : t;
  }
}

// out = column sums of g (accumulate: out += them).
void bias_grad(const at::Tensor& g, at::Tensor& out, bool accumulate) {
  KB_CHECK(g.is_contiguous() && out.scalar_type() == at::kFloat, "bias_grad: contiguous g, fp32 out");
  const int N = (int)g.size(-1);
  const int M = (int)(g.numel() / N);
  KB_CHECK(out.numel() == N && out.is_contiguous(), "bias_grad: out must be fp32 [N]");
  const c10::cuda::CUDAGuard guard(g.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const int col_blocks = (N + 255) / 256;
  const int target_ctas = num_sms(g.get_device()) * 4;
  int row_blocks = std::max(1, std::min((M + 63) / 64, target_ctas / std::max(1, col_blocks)));
  const int rows_per = (M + row_blocks - 1) / row_blocks;
  row_blocks = (M + rows_per - 1) / rows_per;
  at::Tensor part = at::empty({row_blocks, N}, g.options().dtype(at::kFloat));
  dim3 grid(col_blocks, row_blocks);
  if (g.scalar_type() == at::kBFloat16)
    bias_grad_partial_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)g.data_ptr(),
                                                                 part.data_ptr<float>(), M, N, rows_per);
  else if (g.scalar_type() == at::kHalf)
    bias_grad_partial_kernel<__half><<<grid, 256, 0, s>>>((const __half*)g.data_ptr(), part.data_ptr<float>(), M, N,
                                                          rows_per);
  else
    bias_grad_partial_kernel<float><<<grid, 256, 0, s>>>(g.data_ptr<float>(), part.data_ptr<float>(), M, N, rows_per);
  KB_LAUNCHED();
  bias_grad_finish_kernel<<<(N + 31) / 32, 512, 0, s>>>(part.data_ptr<float>(), out.data_ptr<float>(), row_blocks, N,
                                                        accumulate ? 1 : 0);
  KB_LAUNCHED();
}

// ------------------------------------------------------------ multi-tensor cast

constexpr int kCastMaxTensors = 128;
struct CastArgs {
  int n;
  const float* src[kCastMaxTensors];
  void* dst[kCastMaxTensors];
  long long start[kCastMaxTensors + 1];  // cumulative element offsets
};

template <typename TOut>
__global__ void cast_multi_kernel(const __grid_constant__ CastArgs a) {
  // Each CTA walks its share of every tensor with 4-wide loads (tensors are
  // 16-byte aligned allocations; the tail is scalar).
  for (int ti = 0; ti < a.n; ++ti) {
    const long long n = a.start[ti + 1] - a.start[ti];
    const float* src = a.src[ti];
    TOut* dst = reinterpret_cast<TOut*>(a.dst[ti]);
    const long long n4 = ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 7) == 0)
                             ? n / 4 : 0;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
      const float4 v = reinterpret_cast<const float4*>(src)[i];
      uint2 o;
      if constexpr (sizeof(TOut) == 2 && std::is_same<TOut, __nv_bfloat16>::value) {
        o.x = pack_bf16(v.x, v.y);
        o.y = pack_bf16(v.z, v.w);
      } else {
        o.x = pack_f16(v.x, v.y);
        o.y = pack_f16(v.z, v.w);
      }
      reinterpret_cast<uint2*>(dst)[i] = o;
    }
    for (long long i = n4 * 4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
      dst[i] = from_f32<TOut>(src[i]);
  }
}

void cast_multi(const std::vector<at::Tensor>& src, const std::vector<at::Tensor>& dst) {
  KB_CHECK(src.size() == dst.size(), "cast_multi: list lengths differ");
  if (src.empty()) return;
  const c10::cuda::CUDAGuard guard(src[0].device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const auto out_t = dst[0].scalar_type();
  for (size_t base = 0; base < src.size(); base += kCastMaxTensors) {
    CastArgs a{};
    a.n = (int)std::min<size_t>(kCastMaxTensors, src.size() - base);
    a.start[0] = 0;
    for (int i = 0; i < a.n; ++i) {
      const auto& x = src[base + i];
      const auto& y = dst[base + i];
      KB_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && y.is_contiguous() && x.numel() == y.numel() &&
                   y.scalar_type() == out_t,
               "cast_multi: fp32 contiguous sources and matching contiguous destinations required");
      a.src[i] = x.data_ptr<float>();
      a.dst[i] = y.data_ptr();
      a.start[i + 1] = a.start[i] + x.numel();
    }
    if (a.start[a.n] == 0) continue;
    const int blocks = (int)std::min<long long>((a.start[a.n] / 4 + 255) / 256 + 1, num_sms(src[0].get_device()) * 8LL);
    if (out_t == at::kBFloat16) cast_multi_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(a);
    else if (out_t == at::kHalf) cast_multi_kernel<__half><<<blocks, 256, 0, s>>>(a);
    else KB_CHECK(false, "cast_multi: destination must be bf16 or fp16");
    KB_LAUNCHED();
  }
}

// ------------------------------------------------------------ SwiGLU

// h[m, j] = silu(gu[m, j]) * gu[m, F + j]  (gate and up packed side by side)
// Eight consecutive values (one 16-byte access for 16-bit types, two for fp32)
// to and from fp32 registers. The address must be 16-byte aligned.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 q = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = to_f32<T>(e[i]);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 q;
    T* e = reinterpret_cast<T*>(&q);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint4*>(p) = q;
  }
}

template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ h, long long M, int F) {
  const long long total = M * F;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / F;
    const int j = (int)(i - m * F);
    const float g = to_f32<T>(gu[m * 2 * F + j]);
    const float u = to_f32<T>(gu[m * 2 * F + F + j]);
    const float sg = g / (1.f + __expf(-g));
    h[i] = from_f32<T>(sg * u);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ gu, const T* __restrict__ dh, T* __restrict__ dgu,
                                  long long M, int F) {
  const long long total = M * F;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / F;
    const int j = (int)(i - m * F);
    const float g = to_f32<T>(gu[m * 2 * F + j]);
    const float u = to_f32<T>(gu[m * 2 * F + F + j]);
    const float d = to_f32<T>(dh[i]);
    const float sig = 1.f / (1.f + __expf(-g));
    const float silu = g * sig;
    dgu[m * 2 * F + j] = from_f32<T>(d * u * (sig + silu * (1.f - sig)));
    dgu[m * 2 * F + F + j] = from_f32<T>(d * silu);
  }
}

// Vectorised SwiGLU: one thread per 8 consecutive outputs of a row (F % 8 == 0
// and 16-byte aligned rows), so every access is 16 bytes wide and the index
// arithmetic runs once per 8 values. The arithmetic per value is the scalar
// kernels'.
// Vectorised forms: a thread owns eight consecutive columns of the gate and
// up halves (16-byte loads for 16-bit types) at column j = 8 * (x index) and
// walks rows m = blockIdx.y, += gridDim.y, two rows per step with every load
// issued first. The 2-D grid needs no 64-bit division per element group, and
// the sigmoid uses the fast reciprocal (__fdividef, __expf): the kernels were
// instruction bound before at these byte counts.
template <typename T>
__global__ void __launch_bounds__(256)
    swiglu_fwd_vec_kernel(const T* __restrict__ gu, T* __restrict__ h, long long M, int F) {
  const int j = (blockIdx.x * 256 + threadIdx.x) * 8;
  if (j >= F) return;
  const long long step = gridDim.y;
  for (long long m = blockIdx.y; m < M; m += 2 * step) {
    const bool two = m + step < M;
    float g[2][8], u[2][8];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (q == 1 && !two) break;
      const T* row = gu + (m + q * step) * 2 * F;
      load8<T>(row + j, g[q]);
      load8<T>(row + F + j, u[q]);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (q == 1 && !two) break;
      float o[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) o[t] = __fdividef(g[q][t], 1.f + __expf(-g[q][t])) * u[q][t];
      store8<T>(h + (m + q * step) * F + j, o);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
    swiglu_bwd_vec_kernel(const T* __restrict__ gu, const T* __restrict__ dh, T* __restrict__ dgu, long long M,
                          int F) {
  const int j = (blockIdx.x * 256 + threadIdx.x) * 8;
  if (j >= F) return;
  const long long step = gridDim.y;
  for (long long m = blockIdx.y; m < M; m += 2 * step) {
    const bool two = m + step < M;
    float g[2][8], u[2][8], d[2][8];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (q == 1 && !two) break;
      const T* row = gu + (m + q * step) * 2 * F;
      load8<T>(row + j, g[q]);
      load8<T>(row + F + j, u[q]);
      load8<T>(dh + (m + q * step) * F + j, d[q]);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (q == 1 && !two) break;
      float dg[8], du[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float sig = __fdividef(1.f, 1.f + __expf(-g[q][t]));
        const float silu = g[q][t] * sig;
        dg[t] = d[q][t] * u[q][t] * (sig + silu * (1.f - sig));
        du[t] = d[q][t] * silu;
      }
      T* out = dgu + (m + q * step) * 2 * F;
      store8<T>(out + j, dg);
      store8<T>(out + F + j, du);
    }
  }
}

// 2-D grid of the vectorised kernels: column blocks of 256 x 8 columns, rows spread over about 16 CTAs per SM.
static dim3 swiglu_vec_grid(long long M, int F, int dev) {
  const int xb = (F / 8 + 255) / 256;
  const long long yb = std::max<long long>(1, std::min<long long>(M, (long long)num_sms(dev) * 16 / xb));
  return dim3(xb, (unsigned)yb);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

void swiglu_forward(const at::Tensor& gu, at::Tensor& h) {
  const int F = (int)h.size(-1);
  const long long M = h.numel() / F;
  const c10::cuda::CUDAGuard guard(gu.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  KB_CHECK(gu.scalar_type() == h.scalar_type(), "swiglu dtype mismatch");
  const bool vec = F % 8 == 0 && aligned16(gu.data_ptr()) && aligned16(h.data_ptr());
  const long long work = vec ? M * (F / 8) : M * F;
  const int blocks = (int)std::max<long long>(1, std::min<long long>((work + 255) / 256, num_sms(gu.get_device()) * 16LL));
  const dim3 vgrid = vec ? swiglu_vec_grid(M, F, gu.get_device()) : dim3(1);
  if (gu.scalar_type() == at::kBFloat16) {
    auto* in = (const __nv_bfloat16*)gu.data_ptr();
    auto* out = (__nv_bfloat16*)h.data_ptr();
    if (vec) swiglu_fwd_vec_kernel<<<vgrid, 256, 0, s>>>(in, out, M, F);
    else swiglu_fwd_kernel<<<blocks, 256, 0, s>>>(in, out, M, F);
  } else if (gu.scalar_type() == at::kHalf) {
    auto* in = (const __half*)gu.data_ptr();
    auto* out = (__half*)h.data_ptr();
    if (vec) swiglu_fwd_vec_kernel<<<vgrid, 256, 0, s>>>(in, out, M, F);
    else swiglu_fwd_kernel<<<blocks, 256, 0, s>>>(in, out, M, F);
  } else {
    if (vec) swiglu_fwd_vec_kernel<float><<<vgrid, 256, 0, s>>>(gu.data_ptr<float>(), h.data_ptr<float>(), M, F);
    else swiglu_fwd_kernel<float><<<blocks, 256, 0, s>>>(gu.data_ptr<float>(), h.data_ptr<float>(), M, F);
  }
  KB_LAUNCHED();
}

void swiglu_backward(const at::Tensor& gu, const at::Tensor& dh, at::Tensor& dgu) {
  const int F = (int)dh.size(-1);
  const long long M = dh.numel() / F;
  const c10::cuda::CUDAGuard guard(gu.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const bool vec = F % 8 == 0 && aligned16(gu.data_ptr()) && aligned16(dh.data_ptr()) && aligned16(dgu.data_ptr());
  const long long work = vec ? M * (F / 8) : M * F;
  const int blocks = (int)std::max<long long>(1, std::min<long long>((work + 255) / 256, num_sms(gu.get_device()) * 16LL));
  const dim3 vgrid = vec ? swiglu_vec_grid(M, F, gu.get_device()) : dim3(1);
  if (gu.scalar_type() == at::kBFloat16) {
    auto* g = (const __nv_bfloat16*)gu.data_ptr();
    auto* d = (const __nv_bfloat16*)dh.data_ptr();
    auto* o = (__nv_bfloat16*)dgu.data_ptr();
    if (vec) swiglu_bwd_vec_kernel<<<vgrid, 256, 0, s>>>(g, d, o, M, F);
    else swiglu_bwd_kernel<<<blocks, 256, 0, s>>>(g, d, o, M, F);
  } else if (gu.scalar_type() == at::kHalf) {
    auto* g = (const __half*)gu.data_ptr();
    auto* d = (const __half*)dh.data_ptr();
    auto* o = (__half*)dgu.data_ptr();
    if (vec) swiglu_bwd_vec_kernel<<<vgrid, 256, 0, s>>>(g, d, o, M, F);
    else swiglu_bwd_kernel<<<blocks, 256, 0, s>>>(g, d, o, M, F);
  } else {
    if (vec)
      swiglu_bwd_vec_kernel<float><<<vgrid, 256, 0, s>>>(gu.data_ptr<float>(), dh.data_ptr<float>(),
                                                          dgu.data_ptr<float>(), M, F);
    else
      swiglu_bwd_kernel<float><<<blocks, 256, 0, s>>>(gu.data_ptr<float>(), dh.data_ptr<float>(),
                                                      dgu.data_ptr<float>(), M, F);
  }
  KB_LAUNCHED();
}

// ------------------------------------------------------------ rotary embedding

// In place on x[B, S, H, D] (row stride given), rotate-half convention:
// x1' = x1*cos - x2*sin ; x2' = x2*cos + x1*sin with x1 = x[..., :D/2].
// inverse=1 applies the transpose rotation (used for the backward pass).
template <typename T>
__global__ void rope_kernel(T* __restrict__ x, const float* __restrict__ cosb, const float* __restrict__ sinb,
                            long long tokens, int S, int H, int D, long long row_stride, int inverse) {
  const int half = D / 2;
  const long long total = tokens * H * half;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const long long th = i / half;
    const int h = (int)(th % H);
    const long long t = th / H;
    const int pos = (int)(t % S);
    T* p = x + t * row_stride + (long long)h * D;
    const float c = cosb[(long long)pos * half + j];
    const float sn = inverse ? -sinb[(long long)pos * half + j] : sinb[(long long)pos * half + j];
    const float a = to_f32<T>(p[j]);
    const float b = to_f32<T>(p[j + half]);
    p[j] = from_f32<T>(a * c - b * sn);
    p[j + half] = from_f32<T>(b * c + a * sn);
  }
}

// Vectorised RoPE: one thread per 8 consecutive pairs (x1[j..j+8), x2[j..j+8))
// of one head of one token, with 16-byte accesses to x and to the fp32
// cos/sin rows. Requires D % 16 == 0 and 16-byte aligned heads; the
// arithmetic per pair is the scalar kernel's.
template <typename T>
__global__ void __launch_bounds__(256)
    rope_vec_kernel(T* __restrict__ x, const float* __restrict__ cosb, const float* __restrict__ sinb,
                    long long tokens, int S, int H, int D, long long row_stride, int inverse) {
  const int half = D >> 1, groups = half >> 3;
  const long long total = tokens * H * groups;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < total;
       v += (long long)gridDim.x * blockDim.x) {
    const int gq = (int)(v % groups);
    const long long th = v / groups;
    const int h = (int)(th % H);
    const long long t = th / H;
    const int pos = (int)(t % S);
    T* p = x + t * row_stride + (long long)h * D + gq * 8;
    const float* cp = cosb + (long long)pos * half + gq * 8;
    const float* sp = sinb + (long long)pos * half + gq * 8;
    float a[8], b[8], c[8], sn[8], o1[8], o2[8];
    load8<T>(p, a);
    load8<T>(p + half, b);
    load8<float>(cp, c);
    load8<float>(sp, sn);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float si = inverse ? -sn[i] : sn[i];
      o1[i] = a[i] * c[i] - b[i] * si;
      o2[i] = b[i] * c[i] + a[i] * si;
    }
    store8<T>(p, o1);
    store8<T>(p + half, o2);
  }
}

void rope_apply(at::Tensor& x, const at::Tensor& cosb, const at::Tensor& sinb, int64_t S, int64_t H, int64_t D,
                bool inverse) {
  KB_CHECK(x.dim() == 4 && x.stride(-1) == 1 && x.stride(-2) == D, "rope: x must be [B, S, H, D] with dense heads");
  KB_CHECK(x.stride(0) == S * x.stride(1), "rope: tokens must be evenly strided");
  KB_CHECK(cosb.is_contiguous() && sinb.is_contiguous() && cosb.scalar_type() == at::kFloat &&
               sinb.scalar_type() == at::kFloat && cosb.numel() >= S * (D / 2) && sinb.numel() >= S * (D / 2),
           "rope: cos/sin must be contiguous fp32 [S, D/2]");
  const long long row_stride = x.stride(-3);
  const long long T = x.size(0) * x.size(1);
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const int es = (int)x.element_size();
  const bool vec = D % 16 == 0 && aligned16(x.data_ptr()) && (row_stride * es) % 16 == 0 &&
                   aligned16(cosb.data_ptr()) && aligned16(sinb.data_ptr());
  const long long work = vec ? T * H * (D / 16) : T * H * (D / 2);
  const int blocks = (int)std::max<long long>(1, std::min<long long>((work + 255) / 256, num_sms(x.get_device()) * 16LL));
  const float* c = cosb.data_ptr<float>();
  const float* sn = sinb.data_ptr<float>();
  if (x.scalar_type() == at::kBFloat16) {
    auto* p = (__nv_bfloat16*)x.data_ptr();
    if (vec) rope_vec_kernel<<<blocks, 256, 0, s>>>(p, c, sn, T, (int)S, (int)H, (int)D, row_stride, inverse);
    else rope_kernel<<<blocks, 256, 0, s>>>(p, c, sn, T, (int)S, (int)H, (int)D, row_stride, inverse);
  } else if (x.scalar_type() == at::kHalf) {
    auto* p = (__half*)x.data_ptr();
    if (vec) rope_vec_kernel<<<blocks, 256, 0, s>>>(p, c, sn, T, (int)S, (int)H, (int)D, row_stride, inverse);
    else rope_kernel<<<blocks, 256, 0, s>>>(p, c, sn, T, (int)S, (int)H, (int)D, row_stride, inverse);
  } else {
    float* p = x.data_ptr<float>();
    if (vec) rope_vec_kernel<<<blocks, 256, 0, s>>>(p, c, sn, T, (int)S, (int)H, (int)D, row_stride, inverse);
    else rope_kernel<<<blocks, 256, 0, s>>>(p, c, sn, T, (int)S, (int)H, (int)D, row_stride, inverse);
  }
  KB_LAUNCHED();
}

// ------------------------------------------------------------ patchify (ViT)

// images fp32 [B, C, H, W] -> patches [B * (H/P) * (W/P), C * P * P] in the
// 16-bit compute type; column order (c, py, px) matches a Conv2d weight
// [out, C, P, P] flattened, so the patch embedding is one GEMM. Each thread
// moves four horizontally adjacent pixels (one 16-byte load).
template <typename T>
__global__ void patchify_kernel(const float* __restrict__ img, T* __restrict__ out, int B, int C, int H, int W,
                                int P) {
  const int w4 = W >> 2, gh = H / P, gw = W / P;
  const long long total = (long long)B * C * H * w4;
  const long long cols = (long long)C * P * P;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    long long r = i;
    const int x = (int)(r % w4) * 4;
    r /= w4;
    const int y = (int)(r % H);
    r /= H;
    const int c = (int)(r % C);
    const int b = (int)(r / C);
    const float4 v = *reinterpret_cast<const float4*>(img + (((long long)b * C + c) * H + y) * W + x);
    const long long row = ((long long)b * gh + y / P) * gw + x / P;
    T* dst = out + row * cols + ((long long)c * P + y % P) * P + x % P;
    uint2 packed;
    if constexpr (std::is_same<T, __half>::value) {
      packed.x = pack_f16(v.x, v.y);
      packed.y = pack_f16(v.z, v.w);
    } else {
      packed.x = pack_bf16(v.x, v.y);
      packed.y = pack_bf16(v.z, v.w);
    }
    *reinterpret_cast<uint2*>(dst) = packed;
  }
}

void patchify(const at::Tensor& img, at::Tensor& out, int64_t patch) {
  check_cuda_tensor(img, "images");
  KB_CHECK(img.scalar_type() == at::kFloat && img.is_contiguous() && img.dim() == 4, "images must be fp32 NCHW");
  const int B = (int)img.size(0), C = (int)img.size(1), H = (int)img.size(2), W = (int)img.size(3);
  const int P = (int)patch;
  KB_CHECK(P % 4 == 0 && H % P == 0 && W % P == 0, "patch size must divide the image and be a multiple of 4");
  KB_CHECK(out.is_contiguous() && out.numel() == img.numel() &&
               (out.scalar_type() == at::kHalf || out.scalar_type() == at::kBFloat16),
           "patches must be contiguous fp16/bf16 with the image's element count");
  const c10::cuda::CUDAGuard guard(img.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream().stream();
  const long long total = img.numel() / 4;
  const int grid = (int)std::min<long long>((total + 255) / 256, (long long)num_sms(img.get_device()) * 16);
  if (out.scalar_type() == at::kHalf)
    patchify_kernel<__half><<<grid, 256, 0, stream>>>(img.data_ptr<float>(), (__half*)out.data_ptr(), B, C, H, W, P);
  else
    patchify_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(img.data_ptr<float>(), (__nv_bfloat16*)out.data_ptr(),
                                                             B, C, H, W, P);
  KB_LAUNCHED();
}

void register_elementwise_ops(pybind11::module& m) {
  m.def("embedding_forward", &embedding_forward);
  m.def("embedding_backward", &embedding_backward);
  m.def("cross_entropy_forward", &cross_entropy_forward);
  m.def("cross_entropy_backward", &cross_entropy_backward);
  m.def("bias_grad", &bias_grad, "out = column sums of g (accumulate: out += them); deterministic",
        pybind11::arg("g"), pybind11::arg("out"), pybind11::arg("accumulate") = false);
  m.def("cast_multi", &cast_multi);
  m.def("swiglu_forward", &swiglu_forward);
  m.def("swiglu_backward", &swiglu_backward);
  m.def("rope_apply", &rope_apply);
  m.def("patchify", &patchify);
}

}  // namespace kb
