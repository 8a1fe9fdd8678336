// LayerNorm and RMSNorm forward/backward for sm_100a.
//
// One warp owns one row; each lane keeps VPT values of the row in registers
// (rows up to 32*VPT wide, VPT chosen per call). Inputs may be fp32 (a
// residual stream kept in fp32, as autocast does) or bf16/fp16; the normalised
// output is written in the compute dtype for the next GEMM. Statistics are
// fp32 and saved for the backward pass.
//
// Backward writes dx (optionally adding an incoming residual gradient in the
// same pass) and accumulates dgamma/dbeta per CTA (in shared memory for rows up
// to 2560 wide, in registers beyond); a persistent grid keeps the partial
// buffer at (#CTAs x C) and a second kernel reduces it.
#include "host_utils.h"
#include "sm100.cuh"
#include "noalloc.h"

#include <torch/extension.h>

namespace kb {

constexpr int kNormWarps = 8;

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
  float4 q = *reinterpret_cast<const float4*>(p);
  v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  uint2 q = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&q);
  for (int i = 0; i < 4; ++i) v[i] = __bfloat162float(e[i]);
}
template <>
__device__ __forceinline__ void load4<__half>(const __half* p, float (&v)[4]) {
  uint2 q = *reinterpret_cast<const uint2*>(p);
  const __half* e = reinterpret_cast<const __half*>(&q);
  for (int i = 0; i < 4; ++i) v[i] = __half2float(e[i]);
}

template <typename T>
__device__ __forceinline__ void store4(T* p, const float (&v)[4]);
template <>
__device__ __forceinline__ void store4<float>(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[4]) {
  uint2 q;
  q.x = pack_bf16(v[0], v[1]);
  q.y = pack_bf16(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = q;
}
template <>
__device__ __forceinline__ void store4<__half>(__half* p, const float (&v)[4]) {
  uint2 q;
  q.x = pack_f16(v[0], v[1]);
  q.y = pack_f16(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = q;
}

// Column layout: lane l owns columns {4*l + 128*j + t : j < VPT/4, t < 4}.
template <int VPT, typename TIn, typename TOut, bool RMS>
__global__ void __launch_bounds__(32 * kNormWarps)
    norm_fwd_kernel(const TIn* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                    TOut* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out, int M, int C,
                    float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kNormWarps + warp;
  if (row >= M) return;
  const TIn* xr = x + (long long)row * C;
  float v[VPT];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < VPT / 4; ++j) {
    const int col = 4 * lane + 128 * j;
    float q[4] = {0.f, 0.f, 0.f, 0.f};
    if (col < C) load4<TIn>(xr + col, q);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[4 * j + t] = q[t];
      sum += q[t];
    }
  }
  float mean = 0.f;
  if (!RMS) mean = warp_sum(sum) / C;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT / 4; ++j) {
    const int col = 4 * lane + 128 * j;
    if (col < C) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float d = v[4 * j + t] - mean;
        ss += d * d;
      }
    }
  }
  const float var = warp_sum(ss) / C;
  const float rstd = rsqrtf(var + eps);
  if (lane == 0) {
    if (!RMS) mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
  TOut* yr = y + (long long)row * C;
#pragma unroll
  for (int j = 0; j < VPT / 4; ++j) {
    const int col = 4 * lane + 128 * j;
    if (col < C) {
      float wq[4], o[4];
      load4<float>(w + col, wq);
      float bq[4] = {0.f, 0.f, 0.f, 0.f};
      if (!RMS && b != nullptr) load4<float>(b + col, bq);
#pragma unroll
      for (int t = 0; t < 4; ++t) o[t] = (v[4 * j + t] - mean) * rstd * wq[t] + bq[t];
      store4<TOut>(yr + col, o);
    }
  }
}

// dx = rstd * (w*dy - mean(w*dy) - xhat*mean(w*dy*xhat))     (LayerNorm)
// dx = rstd * (w*dy - xhat*mean(w*dy*xhat))                   (RMSNorm)
//
// One warp per row. For rows of up to 1024 values every load of a row (x, dy
// and the residual gradient) is issued before the row's reductions, so each
// warp keeps a whole row in flight; wider rows read the residual gradient at
// the store (registers would spill otherwise). With SMEM_ACC the per-column
// sums for dw / db live in shared memory (one private row per warp) and the
// weights are read from shared memory, which keeps the kernel near 100
// registers (two CTAs, sixteen rows in flight, per SM); without it (very wide
// rows) the sums stay in registers.
template <int VPT, typename TIn, typename TG, typename TDx, bool RMS, bool SMEM_ACC>
__global__ void __launch_bounds__(32 * kNormWarps)
    norm_bwd_kernel(const TG* __restrict__ dy, const TIn* __restrict__ x, const float* __restrict__ w,
                    const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                    const TDx* __restrict__ dres, TDx* __restrict__ dx, TG* __restrict__ dx_lp,
                    float* __restrict__ dw_part, float* __restrict__ db_part, int M, int C) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Shared memory: [kNormWarps][C] dw sums, then (SMEM_ACC only) [kNormWarps][C]
  // db sums and [C] weights.
  extern __shared__ float red[];
  float* sdw = red + warp * C;
  float* sdb = red + (kNormWarps + warp) * C;
  float* sw = red + 2 * kNormWarps * C;
  constexpr bool kEarlyRes = VPT <= 32;
  float dw_acc[SMEM_ACC ? 1 : VPT];
  float db_acc[SMEM_ACC ? 1 : VPT];
  float wv[SMEM_ACC ? 1 : VPT];
  if constexpr (SMEM_ACC) {
    for (int c = lane; c < C; c += 32) {
      sdw[c] = 0.f;
      sdb[c] = 0.f;
    }
    for (int c = threadIdx.x; c < C; c += blockDim.x) sw[c] = w[c];
    __syncthreads();
  } else {
#pragma unroll
    for (int i = 0; i < VPT; ++i) dw_acc[i] = db_acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < VPT / 4; ++j) {
      const int col = 4 * lane + 128 * j;
      float q[4] = {0.f, 0.f, 0.f, 0.f};
      if (col < C) load4<float>(w + col, q);
#pragma unroll
      for (int t = 0; t < 4; ++t) wv[4 * j + t] = q[t];
    }
  }
  for (int row = blockIdx.x * kNormWarps + warp; row < M; row += gridDim.x * kNormWarps) {
    const TIn* xr = x + (long long)row * C;
    const TG* gr = dy + (long long)row * C;
    const TDx* drr = dres ? dres + (long long)row * C : nullptr;
    float xq[VPT], g[VPT], rq[kEarlyRes ? VPT : 4];
#pragma unroll
    for (int j = 0; j < VPT / 4; ++j) {
      const int col = 4 * lane + 128 * j;
      float a[4] = {0.f, 0.f, 0.f, 0.f}, b[4] = {0.f, 0.f, 0.f, 0.f}, r[4] = {0.f, 0.f, 0.f, 0.f};
      if (col < C) {
        load4<TIn>(xr + col, a);
        load4<TG>(gr + col, b);
        if (kEarlyRes && drr) load4<TDx>(drr + col, r);
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        xq[4 * j + t] = a[t];
        g[4 * j + t] = b[t];
        if constexpr (kEarlyRes) rq[4 * j + t] = r[t];
      }
    }
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < VPT / 4; ++j) {
      const int col = 4 * lane + 128 * j;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int i = 4 * j + t;
        xq[i] = (col < C) ? (xq[i] - mean) * rstd : 0.f;  // x-hat from here on
        float wi;
        if constexpr (SMEM_ACC) wi = (col < C) ? sw[col + t] : 0.f;
        else wi = wv[i];
        const float wg = wi * g[i];
        s1 += wg;
        s2 += wg * xq[i];
        if constexpr (!SMEM_ACC) {
          dw_acc[i] += g[i] * xq[i];
          db_acc[i] += g[i];
        }
      }
      if constexpr (SMEM_ACC) {
        if (col < C) {
          float4 a = *reinterpret_cast<float4*>(sdw + col);
          float4 b = *reinterpret_cast<float4*>(sdb + col);
          a.x += g[4 * j] * xq[4 * j];
          a.y += g[4 * j + 1] * xq[4 * j + 1];
          a.z += g[4 * j + 2] * xq[4 * j + 2];
          a.w += g[4 * j + 3] * xq[4 * j + 3];
          b.x += g[4 * j];
          b.y += g[4 * j + 1];
          b.z += g[4 * j + 2];
          b.w += g[4 * j + 3];
          *reinterpret_cast<float4*>(sdw + col) = a;
          *reinterpret_cast<float4*>(sdb + col) = b;
        }
      }
    }
    s1 = warp_sum(s1) / C;
    s2 = warp_sum(s2) / C;
    TDx* dxr = dx + (long long)row * C;
#pragma unroll
    for (int j = 0; j < VPT / 4; ++j) {
      const int col = 4 * lane + 128 * j;
      if (col < C) {
        float o[4];
        float late[4] = {0.f, 0.f, 0.f, 0.f};
        if (!kEarlyRes && drr) load4<TDx>(drr + col, late);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int i = 4 * j + t;
          float wi, r;
          if constexpr (SMEM_ACC) wi = sw[col + t];
          else wi = wv[i];
          if constexpr (kEarlyRes) r = rq[i];
          else r = late[t];
          o[t] = rstd * (wi * g[i] - (RMS ? 0.f : s1) - xq[i] * s2) + r;
        }
        store4<TDx>(dxr + col, o);
        if (dx_lp) store4<TG>(dx_lp + (long long)row * C + col, o);
      }
    }
  }
  if constexpr (SMEM_ACC) {
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      float a = 0.f, b = 0.f;
#pragma unroll
      for (int k = 0; k < kNormWarps; ++k) {
        a += red[k * C + c];
        b += red[(kNormWarps + k) * C + c];
      }
      dw_part[(long long)blockIdx.x * C + c] = a;
      if (!RMS && db_part != nullptr) db_part[(long long)blockIdx.x * C + c] = b;
    }
  } else {
    // Register sums -> one [kNormWarps][C] shared buffer: dw first, then db.
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      if (pass == 1 && (RMS || db_part == nullptr)) break;
      if (pass == 1) __syncthreads();
#pragma unroll
      for (int j = 0; j < VPT / 4; ++j) {
        const int col = 4 * lane + 128 * j;
        if (col < C) {
#pragma unroll
          for (int t = 0; t < 4; ++t) sdw[col + t] = pass == 0 ? dw_acc[4 * j + t] : db_acc[4 * j + t];
        }
      }
      __syncthreads();
      float* dst = pass == 0 ? dw_part : db_part;
      for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float a = 0.f;
#pragma unroll
        for (int k = 0; k < kNormWarps; ++k) a += red[k * C + c];
        dst[(long long)blockIdx.x * C + c] = a;
      }
    }
  }
}

// RMSNorm backward for wide rows (C a multiple of 256, above 1024 values):
//   dx = rstd * (w*dy - xhat * mean(w*dy*xhat)) + dres,  dw += dy * xhat.
// Two passes over each row instead of holding it in registers: the first
// reads x and dy and forms the row sum and the dw contributions (summed per
// warp in shared memory), the second re-reads x and dy -- the row was just
// read, so these come from L2 -- and writes dx (and its 16-bit copy). With a
// handful of registers per lane and 72 KB of shared memory per CTA at
// C = 2048, three CTAs (24 rows) are resident per SM, against one CTA of the
// register-resident kernel. Lane l owns columns [8 l + 256 k, 8 l + 256 k + 8).
template <typename TIn, typename TG, typename TDx>
__global__ void __launch_bounds__(32 * kNormWarps, 3)
    rms_bwd_wide_kernel(const TG* __restrict__ dy, const TIn* __restrict__ x, const float* __restrict__ w,
                        const float* __restrict__ rstd_in, const TDx* __restrict__ dres, TDx* __restrict__ dx,
                        TG* __restrict__ dx_lp, float* __restrict__ dw_part, int M, int C) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  extern __shared__ float red[];
  float* sdw = red + warp * C;         // [kNormWarps][C] per-warp dw sums
  float* sw = red + kNormWarps * C;    // [C] weights
  for (int c = lane * 4; c < C; c += 128) *reinterpret_cast<float4*>(sdw + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c = threadIdx.x * 4; c < C; c += blockDim.x * 4)
    *reinterpret_cast<float4*>(sw + c) = *reinterpret_cast<const float4*>(w + c);
  __syncthreads();
  const int chunks = C >> 8;
  for (int row = blockIdx.x * kNormWarps + warp; row < M; row += gridDim.x * kNormWarps) {
    const TIn* xr = x + (long long)row * C;
    const TG* gr = dy + (long long)row * C;
    const float rstd = rstd_in[row];
    float s2 = 0.f;
    // pass 1: two chunks in flight per step
    for (int k = 0; k < chunks; k += 2) {
      float xa[2][8], ga[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int col = ((k + u) << 8) + lane * 8;
        if (k + u < chunks) {
          load4<TIn>(xr + col, *reinterpret_cast<float(*)[4]>(&xa[u][0]));
          load4<TIn>(xr + col + 4, *reinterpret_cast<float(*)[4]>(&xa[u][4]));
          load4<TG>(gr + col, *reinterpret_cast<float(*)[4]>(&ga[u][0]));
          load4<TG>(gr + col + 4, *reinterpret_cast<float(*)[4]>(&ga[u][4]));
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (k + u >= chunks) break;
        const int col = ((k + u) << 8) + lane * 8;
        float dv[8], wv[8];
        *reinterpret_cast<float4*>(&dv[0]) = *reinterpret_cast<const float4*>(sdw + col);
        *reinterpret_cast<float4*>(&dv[4]) = *reinterpret_cast<const float4*>(sdw + col + 4);
        *reinterpret_cast<float4*>(&wv[0]) = *reinterpret_cast<const float4*>(sw + col);
        *reinterpret_cast<float4*>(&wv[4]) = *reinterpret_cast<const float4*>(sw + col + 4);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float xh = xa[u][t] * rstd;
          s2 += wv[t] * ga[u][t] * xh;
          dv[t] += ga[u][t] * xh;
        }
        *reinterpret_cast<float4*>(sdw + col) = *reinterpret_cast<const float4*>(&dv[0]);
        *reinterpret_cast<float4*>(sdw + col + 4) = *reinterpret_cast<const float4*>(&dv[4]);
      }
    }
    s2 = warp_sum(s2) / C;
    // pass 2
    const TDx* rr = dres ? dres + (long long)row * C : nullptr;
    TDx* dxr = dx + (long long)row * C;
    TG* lpr = dx_lp ? dx_lp + (long long)row * C : nullptr;
    // two chunks per step, every load of both issued before the first use
    for (int k = 0; k < chunks; k += 2) {
      float xa[2][8], ga[2][8], ra[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int col = ((k + u) << 8) + lane * 8;
#pragma unroll
        for (int t = 0; t < 8; ++t) ra[u][t] = 0.f;
        if (k + u < chunks) {
          load4<TIn>(xr + col, *reinterpret_cast<float(*)[4]>(&xa[u][0]));
          load4<TIn>(xr + col + 4, *reinterpret_cast<float(*)[4]>(&xa[u][4]));
          load4<TG>(gr + col, *reinterpret_cast<float(*)[4]>(&ga[u][0]));
          load4<TG>(gr + col + 4, *reinterpret_cast<float(*)[4]>(&ga[u][4]));
          if (rr) {
            load4<TDx>(rr + col, *reinterpret_cast<float(*)[4]>(&ra[u][0]));
            load4<TDx>(rr + col + 4, *reinterpret_cast<float(*)[4]>(&ra[u][4]));
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (k + u >= chunks) break;
        const int col = ((k + u) << 8) + lane * 8;
        float wv[8], o[8];
        *reinterpret_cast<float4*>(&wv[0]) = *reinterpret_cast<const float4*>(sw + col);
        *reinterpret_cast<float4*>(&wv[4]) = *reinterpret_cast<const float4*>(sw + col + 4);
#pragma unroll
        for (int t = 0; t < 8; ++t) o[t] = rstd * (wv[t] * ga[u][t] - xa[u][t] * rstd * s2) + ra[u][t];
        store4<TDx>(dxr + col, *reinterpret_cast<float(*)[4]>(&o[0]));
        store4<TDx>(dxr + col + 4, *reinterpret_cast<float(*)[4]>(&o[4]));
        if (lpr) {
          store4<TG>(lpr + col, *reinterpret_cast<float(*)[4]>(&o[0]));
          store4<TG>(lpr + col + 4, *reinterpret_cast<float(*)[4]>(&o[4]));
        }
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < kNormWarps; ++k) a += red[k * C + c];
    dw_part[(long long)blockIdx.x * C + c] = a;
  }
}

// LayerNorm / RMSNorm backward with rows staged in shared memory by 1-D bulk
// copies, for rows of C = NT * V (NT threads per CTA, V consecutive columns
// per thread): C = 768, 1024 (V = 4) and 2048, 3072, 4096 (NT = 256).
//
// The register/shared-memory kernels above issue their row loads from the
// threads and wait for them before the reductions; at C = 2048 that left the
// wide RMSNorm kernel latency bound at 37 % of DRAM bandwidth (ncu: 18
// long-scoreboard stalls per issued instruction). Here one thread per CTA
// keeps kRowStages rows (x, dy and the incoming residual gradient) in flight
// as bulk copies while all NT threads work on the oldest staged row: each
// thread owns V consecutive columns for the CTA's whole life, so its share of
// dgamma (and dbeta) stays in registers, and a row costs one block-wide sum
// (one barrier). x and dy are read from DRAM once; dx (+ the residual
// gradient) and its 16-bit copy are written once.
constexpr int kRowStages = 4;

template <int NT, int V, bool RMS, typename TIn, typename TG, typename TDx>
__global__ void __launch_bounds__(NT, (NT <= 192 ? 4 : 2))
    norm_bwd_staged_kernel(const TG* __restrict__ dy, const TIn* __restrict__ x, const float* __restrict__ w,
                           const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                           const TDx* __restrict__ dres, TDx* __restrict__ dx, TG* __restrict__ dx_lp,
                           float* __restrict__ dw_part, float* __restrict__ db_part, int M, int* status) {
  constexpr int C = NT * V;
  constexpr int NW = NT / 32;
  constexpr int kXB = C * (int)sizeof(TIn), kGB = C * (int)sizeof(TG), kRB = C * (int)sizeof(TDx);
  constexpr int kStage = kXB + kGB + kRB;
  extern __shared__ __align__(128) uint8_t smem_rows[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_rows + kRowStages * kStage);
  float2* red = reinterpret_cast<float2*>(full + kRowStages);  // [2][NW] per-warp partial sums, by row parity
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red + 2 * NW);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col = tid * V;
  const int nrows = blockIdx.x < M ? (M - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const uint32_t row_bytes = (uint32_t)(kXB + kGB + (dres ? kRB : 0));

  if (tid == 0) {
    for (int s = 0; s < kRowStages; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](int i) {  // thread 0: stage row i of this CTA
    const long long row = (long long)blockIdx.x + (long long)i * gridDim.x;
    uint8_t* st = smem_rows + (i % kRowStages) * kStage;
    uint64_t* bar = &full[i % kRowStages];
    mbar_arrive_expect_tx(bar, row_bytes);
    bulk_load_1d(st, x + row * C, kXB, bar);
    bulk_load_1d(st + kXB, dy + row * C, kGB, bar);
    if (dres) bulk_load_1d(st + kXB + kGB, dres + row * C, kRB, bar);
  };
  int issued = 0;
  if (tid == 0)
    for (; issued < min(kRowStages, nrows); ++issued) issue(issued);

  float wv[V], acc[V], accb[V];
#pragma unroll
  for (int j = 0; j < V; j += 4) {
    *reinterpret_cast<float4*>(&wv[j]) = *reinterpret_cast<const float4*>(w + col + j);
    *reinterpret_cast<float4*>(&acc[j]) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(&accb[j]) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  int done = 0;
  // Statistics one row ahead: their load latency hides behind a row.
  float rstd_next = nrows > 0 ? rstd_in[blockIdx.x] : 0.f;
  float mean_next = (!RMS && nrows > 0) ? mean_in[blockIdx.x] : 0.f;
  for (int i = 0; i < nrows; ++i) {
    const long long row = (long long)blockIdx.x + (long long)i * gridDim.x;
    const float rstd = rstd_next, mean = mean_next;
    if (i + 1 < nrows) {
      rstd_next = rstd_in[row + gridDim.x];
      if (!RMS) mean_next = mean_in[row + gridDim.x];
    }
    const uint8_t* st = smem_rows + (i % kRowStages) * kStage;
    const bool ok = mbar_wait(&full[i % kRowStages], (uint32_t)(i / kRowStages) & 1u, abort_flag, status,
                              kStatusTimeoutRowStage);
    float xh[V], gv[V], rv[V];
#pragma unroll
    for (int j = 0; j < V; j += 4) {
      if (ok) {
        load4<TIn>(reinterpret_cast<const TIn*>(st) + col + j, *reinterpret_cast<float(*)[4]>(&xh[j]));
        load4<TG>(reinterpret_cast<const TG*>(st + kXB) + col + j, *reinterpret_cast<float(*)[4]>(&gv[j]));
        if (dres) load4<TDx>(reinterpret_cast<const TDx*>(st + kXB + kGB) + col + j, *reinterpret_cast<float(*)[4]>(&rv[j]));
        else *reinterpret_cast<float4*>(&rv[j]) = make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        *reinterpret_cast<float4*>(&xh[j]) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(&gv[j]) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(&rv[j]) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      xh[j] = RMS ? xh[j] * rstd : (xh[j] - mean) * rstd;  // normalised x
      const float dxh = wv[j] * gv[j];
      s1 += dxh;
      s2 += dxh * xh[j];
      acc[j] += gv[j] * xh[j];
      if (!RMS) accb[j] += gv[j];
    }
    s2 = warp_sum(s2);
    if (!RMS) s1 = warp_sum(s1);
    if (lane == 0) red[(i & 1) * NW + warp] = make_float2(s1, s2);
    // Every thread has read its part of the stage (and written its partial sums);
    // all leave together when any wait ran out.
    if (!__syncthreads_and(ok)) break;
    if (tid == 0 && issued < nrows) issue(issued++);
    float t1 = 0.f, t2 = 0.f;
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      const float2 v = red[(i & 1) * NW + k];
      t1 += v.x;
      t2 += v.y;
    }
    t1 *= 1.0f / C;
    t2 *= 1.0f / C;
    float o[V];
#pragma unroll
    for (int j = 0; j < V; ++j)
      o[j] = rstd * (wv[j] * gv[j] - (RMS ? 0.f : t1) - xh[j] * t2) + rv[j];
    TDx* dxr = dx + row * C + col;
#pragma unroll
    for (int j = 0; j < V; j += 4) store4<TDx>(dxr + j, *reinterpret_cast<float(*)[4]>(&o[j]));
    if (dx_lp) {
      TG* lpr = dx_lp + row * C + col;
#pragma unroll
      for (int j = 0; j < V; j += 4) store4<TG>(lpr + j, *reinterpret_cast<float(*)[4]>(&o[j]));
    }
    ++done;
  }
  if (tid == 0) {
    // After an abort, wait (bounded) for the copies still landing in this CTA's shared memory.
    volatile int never = 0;
    for (int i = done; i < issued; ++i)
      if (!mbar_wait(&full[i % kRowStages], (uint32_t)(i / kRowStages) & 1u, &never, status, kStatusTimeoutDrain))
        break;
  }
#pragma unroll
  for (int j = 0; j < V; j += 4) {
    *reinterpret_cast<float4*>(dw_part + (long long)blockIdx.x * C + col + j) = *reinterpret_cast<const float4*>(&acc[j]);
    if (!RMS)
      *reinterpret_cast<float4*>(db_part + (long long)blockIdx.x * C + col + j) =
          *reinterpret_cast<const float4*>(&accb[j]);
  }
}

// Threads per CTA of the staged backward for a row width, or 0 where it does not apply.
static inline int norm_bwd_staged_threads(int C) {
  switch (C) {
    case 768: return 192;
    case 1024: case 2048: case 3072: case 4096: return 256;
    default: return 0;
  }
}

static inline int norm_bwd_staged_smem(int C, int in_bytes, int g_bytes) {
  const int nw = norm_bwd_staged_threads(C) / 32;
  return kRowStages * C * (2 * in_bytes + g_bytes) + kRowStages * 8 + 2 * nw * 8 + 16;
}

// CTAs of the staged backward (also sizes its share of the workspace).
static inline int norm_bwd_staged_grid(int M, int C, int dev) {
  if (!norm_bwd_staged_threads(C)) return 0;
  const int smem = norm_bwd_staged_smem(C, 4, 2);  // the largest case: fp32 x and dx, 16-bit dy
  const int cap = norm_bwd_staged_threads(C) <= 192 ? 4 : 2;
  const int per_sm = std::max(1, std::min(cap, (227 * 1024) / (smem + 1024)));
  return std::max(1, std::min(num_sms(dev) * per_sm, M));
}

static inline bool rms_bwd_wide(bool rms, int C) { return rms && C > 1024 && C % 256 == 0 && C <= 4096; }
static inline int rms_bwd_wide_smem(int C) { return (kNormWarps + 1) * C * (int)sizeof(float); }

// CTAs of the backward grid (persistent; the partial-sum workspace holds one
// row of C per CTA, two rows for LayerNorm's dgamma and dbeta).
static inline int norm_bwd_grid(int M, int C, bool rms, int dev) {
  const int per_sm = rms_bwd_wide(rms, C) ? std::max(1, (227 * 1024) / (rms_bwd_wide_smem(C) + 1024)) : 2;
  return std::max(1, std::min(num_sms(dev) * per_sm, (M + kNormWarps - 1) / kNormWarps));
}

// Whether norm_bwd_kernel keeps its column sums in shared memory for this row
// width, and the dynamic shared memory it then needs.
static inline bool norm_bwd_smem_acc(int C) { return C <= 2560; }
static inline int norm_bwd_smem_bytes(int C) {
  return (norm_bwd_smem_acc(C) ? (2 * kNormWarps + 1) : kNormWarps) * C * (int)sizeof(float);
}

// out[c] (+)= sum_r part[r, c]; a CTA owns 32 columns, 8 row groups per column.
__global__ void __launch_bounds__(256) column_reduce_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                            int R, int C, int accumulate) {
  const int col = blockIdx.x * 32 + (threadIdx.x & 31);
  const int rg = threadIdx.x >> 5;
  float s = 0.f;
  if (col < C)
    for (int r = rg; r < R; r += 8) s += part[(long long)r * C + col];
  __shared__ float red[8][33];
  red[rg][threadIdx.x & 31] = s;
  __syncthreads();
  if (rg == 0 && col < C) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][threadIdx.x & 31];
    out[col] = accumulate ? out[col] + t : t;
  }
}

// out[c] (+)= sum_r part[r, c] for one or two partial-sum buffers (blockIdx.y
// picks dgamma or dbeta), used by norm_backward: a CTA owns 32 columns and
// splits the rows over 16 warps, each keeping four independent loads in
// flight (the reduction above, one warp per eight rows with one load at a
// time, took about 20 us for 592 partial rows of 768 columns).
__global__ void __launch_bounds__(512) column_sum_kernel(const float* __restrict__ part0, float* __restrict__ out0,
                                                         const float* __restrict__ part1, float* __restrict__ out1,
                                                         int R, int C, int accumulate) {
  const float* part = blockIdx.y ? part1 : part0;
  float* out = blockIdx.y ? out1 : out0;
  const int lane = threadIdx.x & 31, rg = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (col < C) {
    int r = rg;
    for (; r + 48 < R; r += 64) {
      s0 += part[(long long)r * C + col];
      s1 += part[(long long)(r + 16) * C + col];
      s2 += part[(long long)(r + 32) * C + col];
      s3 += part[(long long)(r + 48) * C + col];
    }
    for (; r < R; r += 16) s0 += part[(long long)r * C + col];
  }
  __shared__ float red[16][33];
  red[rg][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (rg == 0 && col < C) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) t += red[k][lane];
    out[col] = accumulate ? out[col] + t : t;
  }
}

// ---------------------------------------------------------------------- host

template <typename F>
static void with_vpt(int C, F&& f) {
  if (C <= 256) f(std::integral_constant<int, 8>{});
  else if (C <= 512) f(std::integral_constant<int, 16>{});
  else if (C <= 768) f(std::integral_constant<int, 24>{});
  else if (C <= 1024) f(std::integral_constant<int, 32>{});
  else if (C <= 2048) f(std::integral_constant<int, 64>{});
  else if (C <= 4096) f(std::integral_constant<int, 128>{});
  else KB_CHECK(false, "norm: rows wider than 4096 are not supported");
}

template <typename F>
static void with_lp_type(at::ScalarType t, F&& f) {
  if (t == at::kBFloat16) f(__nv_bfloat16{});
  else if (t == at::kHalf) f(__half{});
  else KB_CHECK(false, "norm backward: dy must be bf16 or fp16");
}

template <typename F>
static void with_type(at::ScalarType t, F&& f) {
  if (t == at::kFloat) f(float{});
  else if (t == at::kBFloat16) f(__nv_bfloat16{});
  else if (t == at::kHalf) f(__half{});
  else KB_CHECK(false, "norm: unsupported dtype");
}

// y = norm(x) * w + b ; returns nothing, writes y, mean (LayerNorm only), rstd.
void norm_forward(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& b, at::Tensor& y,
                  const c10::optional<at::Tensor>& mean, at::Tensor& rstd, double eps, bool rms) {
  check_cuda_tensor(x, "x");
  KB_CHECK(x.is_contiguous() && y.is_contiguous(), "norm: x and y must be contiguous");
  const int C = (int)x.size(-1);
  const int M = (int)(x.numel() / C);
  KB_CHECK(C % 4 == 0, "norm: row width must be a multiple of 4");
  KB_CHECK(w.scalar_type() == at::kFloat && w.numel() == C, "norm: weight must be fp32 [C]");
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream().stream();
  const float* bp = (b.has_value() && b->defined()) ? b->data_ptr<float>() : nullptr;
  float* mp = (mean.has_value() && mean->defined()) ? mean->data_ptr<float>() : nullptr;
  KB_CHECK(rms || mp != nullptr, "LayerNorm needs a mean buffer");
  const int grid = (M + kNormWarps - 1) / kNormWarps;
  with_vpt(C, [&](auto vpt) {
    constexpr int V = decltype(vpt)::value;
    with_type(x.scalar_type(), [&](auto tin) {
      using TIn = decltype(tin);
      with_type(y.scalar_type(), [&](auto tout) {
        using TOut = decltype(tout);
        if (rms)
          norm_fwd_kernel<V, TIn, TOut, true><<<grid, 32 * kNormWarps, 0, stream>>>(
              (const TIn*)x.data_ptr(), w.data_ptr<float>(), nullptr, (TOut*)y.data_ptr(), nullptr,
              rstd.data_ptr<float>(), M, C, (float)eps);
        else
          norm_fwd_kernel<V, TIn, TOut, false><<<grid, 32 * kNormWarps, 0, stream>>>(
              (const TIn*)x.data_ptr(), w.data_ptr<float>(), bp, (TOut*)y.data_ptr(), mp, rstd.data_ptr<float>(), M,
              C, (float)eps);
      });
    });
  });
  KB_LAUNCHED();
}

// Writes dx (= norm backward + optional dres) and dw (and db for LayerNorm),
// accumulating into dw/db when `accumulate` is set. `workspace` is fp32 scratch
// of at least (2 * grid * C) elements, grid = min(#SMs * 4, ceil(M / 8)).
void norm_backward(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                   const c10::optional<at::Tensor>& mean, const at::Tensor& rstd, const c10::optional<at::Tensor>& dres,
                   at::Tensor& dx, at::Tensor& dw, const c10::optional<at::Tensor>& db, at::Tensor& workspace,
                   bool rms, bool accumulate, const c10::optional<at::Tensor>& dx_lp) {
  check_cuda_tensor(dy, "dy");
  KB_CHECK(dy.is_contiguous() && x.is_contiguous() && dx.is_contiguous(), "norm bwd: contiguous tensors required");
  const int C = (int)x.size(-1);
  const int M = (int)(x.numel() / C);
  const c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream().stream();
  const int dev = x.get_device();
  const int grid = norm_bwd_grid(M, C, rms, dev);
  // Rows of partial sums the workspace holds for dgamma (and as many for dbeta).
  const int ws_grid = std::max({norm_bwd_grid(M, C, true, dev), norm_bwd_grid(M, C, false, dev),
                                norm_bwd_staged_grid(M, C, dev)});
  KB_CHECK(workspace.scalar_type() == at::kFloat && workspace.numel() >= 2LL * ws_grid * C,
           "norm bwd: workspace too small");
  float* dw_part = workspace.data_ptr<float>();
  float* db_part = rms ? nullptr : dw_part + (long long)ws_grid * C;
  const float* mp = (mean.has_value() && mean->defined()) ? mean->data_ptr<float>() : nullptr;
  KB_CHECK(rms || mp, "LayerNorm backward needs mean");
  const bool has_res = dres.has_value() && dres->defined();
  KB_CHECK(dx.scalar_type() == x.scalar_type(), "norm bwd: dx must have the dtype of x");
  if (has_res) KB_CHECK(dres->scalar_type() == dx.scalar_type() && dres->is_contiguous(), "dres must match dx");
  const int smem = norm_bwd_smem_bytes(C);
  const bool sacc = norm_bwd_smem_acc(C);
  bool wide = rms_bwd_wide(rms, C);
  int reduce_rows = grid;  // rows of dw_part the column reduction sums
  bool staged = false;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool lp_given = dx_lp.has_value() && dx_lp->defined();
  if (norm_bwd_staged_threads(C) && (rms || mp != nullptr) && a16(x.data_ptr()) && a16(dy.data_ptr()) &&
      a16(dx.data_ptr()) && (!has_res || a16(dres->data_ptr())) && (!lp_given || a16(dx_lp->data_ptr())) &&
      a16(w.data_ptr())) {
    with_type(x.scalar_type(), [&](auto tin) {
      using TIn = decltype(tin);
      with_lp_type(dy.scalar_type(), [&](auto tg) {
        using TG = decltype(tg);
        using TDx = TIn;
        TG* lp = nullptr;
        if (lp_given) {
          KB_CHECK(dx_lp->scalar_type() == dy.scalar_type() && dx_lp->is_contiguous() && dx_lp->numel() == dx.numel(),
                   "dx_lp must be contiguous, of dy's dtype and dx's size");
          lp = (TG*)dx_lp->data_ptr();
        }
        const int g = std::min(norm_bwd_staged_grid(M, C, dev), ws_grid);
        const int sm = norm_bwd_staged_smem(C, (int)sizeof(TIn), (int)sizeof(TG));
        auto go = [&](auto nt_c, auto v_c, auto rms_c) {
          constexpr int NT = decltype(nt_c)::value;
          constexpr int V = decltype(v_c)::value;
          constexpr bool R = decltype(rms_c)::value;
          auto kern = norm_bwd_staged_kernel<NT, V, R, TIn, TG, TDx>;
          KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
          kern<<<g, NT, sm, stream>>>((const TG*)dy.data_ptr(), (const TIn*)x.data_ptr(), w.data_ptr<float>(),
                                      R ? nullptr : mp, rstd.data_ptr<float>(),
                                      has_res ? (const TDx*)dres->data_ptr() : nullptr, (TDx*)dx.data_ptr(), lp,
                                      dw_part, R ? nullptr : db_part, M, device_status_ptr(dev));
        };
        auto by_width = [&](auto rms_c) {
          switch (C) {
            case 768: go(std::integral_constant<int, 192>{}, std::integral_constant<int, 4>{}, rms_c); break;
            case 1024: go(std::integral_constant<int, 256>{}, std::integral_constant<int, 4>{}, rms_c); break;
            case 2048: go(std::integral_constant<int, 256>{}, std::integral_constant<int, 8>{}, rms_c); break;
            case 3072: go(std::integral_constant<int, 256>{}, std::integral_constant<int, 12>{}, rms_c); break;
            default: go(std::integral_constant<int, 256>{}, std::integral_constant<int, 16>{}, rms_c); break;
          }
        };
        if (rms) by_width(std::true_type{});
        else by_width(std::false_type{});
        reduce_rows = g;
      });
    });
    staged = true;
    wide = false;
  } else if (wide) {
    with_type(x.scalar_type(), [&](auto tin) {
      using TIn = decltype(tin);
      with_lp_type(dy.scalar_type(), [&](auto tg) {
        using TG = decltype(tg);
        using TDx = TIn;
        TG* lp = nullptr;
        if (dx_lp.has_value() && dx_lp->defined()) {
          KB_CHECK(dx_lp->scalar_type() == dy.scalar_type() && dx_lp->is_contiguous() && dx_lp->numel() == dx.numel(),
                   "dx_lp must be contiguous, of dy's dtype and dx's size");
          lp = (TG*)dx_lp->data_ptr();
        }
        const int wsmem = rms_bwd_wide_smem(C);
        auto kern = rms_bwd_wide_kernel<TIn, TG, TDx>;
        KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, wsmem));
        kern<<<grid, 32 * kNormWarps, wsmem, stream>>>((const TG*)dy.data_ptr(), (const TIn*)x.data_ptr(),
                                                       w.data_ptr<float>(), rstd.data_ptr<float>(),
                                                       has_res ? (const TDx*)dres->data_ptr() : nullptr,
                                                       (TDx*)dx.data_ptr(), lp, dw_part, M, C);
      });
    });
  }
  if (!wide && !staged) with_vpt(C, [&](auto vpt) {
    constexpr int V = decltype(vpt)::value;
    with_type(x.scalar_type(), [&](auto tin) {
      using TIn = decltype(tin);
      with_lp_type(dy.scalar_type(), [&](auto tg) {
        using TG = decltype(tg);
        using TDx = TIn;
        const TDx* rp = has_res ? (const TDx*)dres->data_ptr() : nullptr;
        TG* lp = nullptr;
        if (dx_lp.has_value() && dx_lp->defined()) {
          KB_CHECK(dx_lp->scalar_type() == dy.scalar_type() && dx_lp->is_contiguous() && dx_lp->numel() == dx.numel(),
                   "dx_lp must be contiguous, of dy's dtype and dx's size");
          lp = (TG*)dx_lp->data_ptr();
        }
        auto go = [&](auto rms_c, auto sacc_c) {
          constexpr bool R = decltype(rms_c)::value;
          constexpr bool SA = decltype(sacc_c)::value;
          auto kern = norm_bwd_kernel<V, TIn, TG, TDx, R, SA>;
          if (smem > 48 * 1024)
            KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
          kern<<<grid, 32 * kNormWarps, smem, stream>>>((const TG*)dy.data_ptr(), (const TIn*)x.data_ptr(),
                                                        w.data_ptr<float>(), R ? nullptr : mp, rstd.data_ptr<float>(),
                                                        rp, (TDx*)dx.data_ptr(), lp, dw_part, R ? nullptr : db_part,
                                                        M, C);
        };
        if (rms) {
          if (sacc) go(std::true_type{}, std::true_type{});
          else go(std::true_type{}, std::false_type{});
        } else {
          if (sacc) go(std::false_type{}, std::true_type{});
          else go(std::false_type{}, std::false_type{});
        }
      });
    });
  });
  KB_LAUNCHED();
  KB_CHECK(dw.scalar_type() == at::kFloat && dw.numel() == C, "dw must be fp32 [C]");
  const bool want_db = !rms && db.has_value() && db->defined();
  if (want_db) KB_CHECK(db->scalar_type() == at::kFloat && db->numel() == C, "db must be fp32 [C]");
  column_sum_kernel<<<dim3((C + 31) / 32, want_db ? 2 : 1), 512, 0, stream>>>(
      dw_part, dw.data_ptr<float>(), want_db ? db_part : nullptr, want_db ? db->data_ptr<float>() : nullptr,
      reduce_rows, C, accumulate);
  KB_LAUNCHED();
}

int64_t norm_backward_workspace_elems(int64_t M, int64_t C, int64_t device) {
  // Sized for the largest grid of the backward kernels (dgamma and dbeta halves).
  const int grid = std::max({norm_bwd_grid((int)M, (int)C, true, (int)device),
                             norm_bwd_grid((int)M, (int)C, false, (int)device),
                             norm_bwd_staged_grid((int)M, (int)C, (int)device)});
  return 2LL * grid * C;
}

// ---------------------------------------------------------------------------
// kb_layernorm_backward_noalloc: LayerNorm backward that allocates nothing.
//
// This entry point has no counterpart in the reference framework.
//
// The regular norm_backward above takes its partial-sum scratch from the
// caller (the Python layer allocates it through PyTorch's caching allocator).
// Some callers cannot allocate device memory at the point where they need
// this op: engines that own a fixed device-memory arena and forbid any other
// allocation, and plain C callers that link this library without PyTorch and
// therefore have no allocator to hand over. For them this variant keeps its
// scratch in a file-scope device array of fixed size:
//
//   * limit: kNoAllocScratchFloats fp32 values (4 MiB). A call needs
//     2 * grid * C values, where the grid is shrunk (down to one CTA) to fit;
//     rows wider than kNoAllocMaxC = 4096 are rejected with an error code.
//   * every GPU that loads this library holds the 4 MiB until process exit.
//   * all calls share the one array, which keeps the previous call's
//     contents; every partial that is read is first written in the same
//     call, so nothing has to start at zero. Calls whose kernels overlap on
//     the GPU (different streams, or concurrent host threads) race on the
//     array and must be serialised by the caller.
//   * the first call on each device resolves the array's device address with
//     cudaGetSymbolAddress (the host-side name of a __device__ array is not a
//     device address).
//   * the resolved address is remembered per device ordinal for the rest of
//     the process. It assumes the device is not reset in between: after a
//     cudaDeviceReset in the same process the remembered address is stale,
//     so do not use this entry point across a device reset.
//   * no cudaMalloc, cudaFree or allocating library routine is called.
//
// Types: dy bf16 [M, C]; x, w, mean, rstd, dx, dw, db fp32; all contiguous,
// x/dy/dx rows 16-byte aligned. dx = LayerNorm backward (no residual term);
// dw, db are overwritten. Returns 0 on success, or a cudaError_t value / -1
// (bad arguments) / -2 (row width over the limit).

constexpr long long kNoAllocScratchFloats = 1ll << 20;  // 4 MiB of fp32
constexpr int kNoAllocMaxC = 4096;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

static float* noalloc_scratch_ptr(int device, cudaError_t* err) {
  static std::mutex mu;
  static float* ptrs[64] = {nullptr};
  if (device < 0 || device >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[device] == nullptr) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // `device` is current here
    if (*err != cudaSuccess) return nullptr;
    ptrs[device] = static_cast<float*>(p);
  }
  *err = cudaSuccess;
  return ptrs[device];
}

extern "C" __attribute__((visibility("default"))) int kb_layernorm_backward_noalloc(
    const void* dy, const float* x, const float* w, const float* mean, const float* rstd, float* dx, float* dw,
    float* db, int M, int C, cudaStream_t stream) {
  if (dy == nullptr || x == nullptr || w == nullptr || mean == nullptr || rstd == nullptr || dx == nullptr ||
      dw == nullptr || db == nullptr || M <= 0 || C <= 0 || C % 4 != 0)
    return -1;
  if (C > kNoAllocMaxC) return -2;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return (int)err;
  float* scratch = noalloc_scratch_ptr(device, &err);
  if (scratch == nullptr) return (int)err;
  int sms = 0;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (err != cudaSuccess) return (int)err;
  long long grid = std::min<long long>((long long)sms * 2, (M + kNormWarps - 1) / kNormWarps);
  grid = std::min<long long>(grid, kNoAllocScratchFloats / (2LL * C));
  grid = std::max<long long>(grid, 1);
  float* dw_part = scratch;
  float* db_part = scratch + grid * C;
  const int smem = norm_bwd_smem_bytes(C);
  const bool sacc = norm_bwd_smem_acc(C);
  bool launched = false;
  cudaError_t setup = cudaSuccess;
  with_vpt(C, [&](auto vpt) {
    constexpr int V = decltype(vpt)::value;
    auto kern = sacc ? norm_bwd_kernel<V, float, __nv_bfloat16, float, false, true>
                     : norm_bwd_kernel<V, float, __nv_bfloat16, float, false, false>;
    if (smem > 48 * 1024) {
      setup = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (setup != cudaSuccess) return;
    }
    kern<<<(unsigned)grid, 32 * kNormWarps, smem, stream>>>(static_cast<const __nv_bfloat16*>(dy), x, w, mean, rstd,
                                                             nullptr, dx, nullptr, dw_part, db_part, M, C);
    launched = true;
  });
  if (setup != cudaSuccess) return (int)setup;  // the attribute call's own error
  if (!launched) return (int)cudaErrorInvalidConfiguration;  // no kernel instance for this row width
  err = cudaGetLastError();
  if (err != cudaSuccess) return (int)err;
  column_reduce_kernel<<<(C + 31) / 32, 256, 0, stream>>>(dw_part, dw, (int)grid, C, 0);
  column_reduce_kernel<<<(C + 31) / 32, 256, 0, stream>>>(db_part, db, (int)grid, C, 0);
  err = cudaGetLastError();
  return (int)err;
}

void register_norm_ops(pybind11::module& m) {
  m.def("norm_forward", &norm_forward, "LayerNorm/RMSNorm forward");
  m.def("norm_backward", &norm_backward, "LayerNorm/RMSNorm backward", pybind11::arg("dy"), pybind11::arg("x"),
        pybind11::arg("w"), pybind11::arg("mean"), pybind11::arg("rstd"), pybind11::arg("dres"), pybind11::arg("dx"),
        pybind11::arg("dw"), pybind11::arg("db"), pybind11::arg("workspace"), pybind11::arg("rms"),
        pybind11::arg("accumulate"), pybind11::arg("dx_lp") = pybind11::none());
  m.def("norm_backward_workspace_elems", &norm_backward_workspace_elems, "scratch size for norm_backward");
}

}  // namespace kb
