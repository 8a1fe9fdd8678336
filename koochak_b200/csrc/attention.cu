// Flash attention (forward + backward), bf16/fp16 in, fp32 softmax statistics.
//
// Layout: q, k, v, o are [B, S, H, D] views with an arbitrary token stride
// (so the fused QKV projection output [B, S, 3, H, D] is consumed in place and
// the output feeds the next GEMM without a transpose). Head dims 64 and 128,
// causal or not, any sequence length (tails masked).
//
// Tensor-core path: warp-level mma.sync m16n8k16 with ldmatrix fragments out
// of XOR-swizzled shared memory, cp.async double buffering. Forward keeps the
// running max/sum per query row (online softmax) and saves the natural-log
// LSE; backward recomputes P per tile, keeps dK/dV for a 64-key block in
// registers and accumulates dQ with fp32 atomics.
#include "host_utils.h"
#include "sm100.cuh"

#include <torch/extension.h>

namespace kb {

// ---------------------------------------------------------------- primitives

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <bool F16>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <bool F16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (F16) return pack_f16(a, b);
  else return pack_bf16(a, b);
}

// Byte offset of element (row, col) in a swizzled tile whose rows are ROWB bytes.
template <int ROWB>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  constexpr int CH = ROWB / 16;                 // 16-byte chunks per row
  constexpr int MASK = CH >= 8 ? 7 : CH - 1;    // keep the XOR inside the row
  const int chunk = (col >> 3) ^ (row & MASK);
  return row * ROWB + chunk * 16 + (col & 7) * 2;
}

// Copy a [ROWS, D] tile (row stride `ld` elements) into swizzled smem.
template <int ROWS, int D, int NT>
__device__ __forceinline__ void load_tile(uint8_t* smem, const uint16_t* g, long long ld, int row0, int nrows_valid,
                                          int tid) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
#pragma unroll
  for (int i = tid; i < ROWS * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const bool ok = (row0 + r) < nrows_valid;
    const uint16_t* src = g + (long long)(ok ? row0 + r : 0) * ld + c * 8;
    cp_async16(smem + swz<D * 2>(r, c * 8), src, ok);
  }
}

// ---------------------------------------------------------------- forward

constexpr int kFwdBM = 64;
constexpr int kFwdBN = 64;
constexpr int kFwdThreads = 128;

template <int D, bool CAUSAL, bool F16>
__global__ void __launch_bounds__(kFwdThreads)
    flash_fwd_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                     uint16_t* __restrict__ o, float* __restrict__ lse, int H, int Sq, int Sk, long long q_ld,
                     long long k_ld, long long v_ld, long long o_ld, long long q_bs, long long k_bs, long long v_bs,
                     long long o_bs, float scale_log2) {
  constexpr int ROWB = D * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kFwdBM * ROWB;            // 2 buffers
  uint8_t* sV = sK + 2 * kFwdBN * ROWB;        // 2 buffers
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int num_qb = (Sq + kFwdBM - 1) / kFwdBM;
  const int qb = CAUSAL ? (num_qb - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const uint16_t* qg = q + b * q_bs + (long long)h * D;
  const uint16_t* kg = k + b * k_bs + (long long)h * D;
  const uint16_t* vg = v + b * v_bs + (long long)h * D;
  const int q0 = qb * kFwdBM;
  int nkb = (Sk + kFwdBN - 1) / kFwdBN;
  if (CAUSAL) nkb = min(nkb, (q0 + kFwdBM - 1) / kFwdBN + 1);

  load_tile<kFwdBM, D, kFwdThreads>(sQ, qg, q_ld, q0, Sq, tid);
  load_tile<kFwdBN, D, kFwdThreads>(sK, kg, k_ld, 0, Sk, tid);
  load_tile<kFwdBN, D, kFwdThreads>(sV, vg, v_ld, 0, Sk, tid);
  cp_async_commit();

  float oacc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) oacc[i][j] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  uint32_t qf[D / 16][4];

  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_tile<kFwdBN, D, kFwdThreads>(sK + (buf ^ 1) * kFwdBN * ROWB, kg, k_ld, (j + 1) * kFwdBN, Sk, tid);
      load_tile<kFwdBN, D, kFwdThreads>(sV + (buf ^ 1) * kFwdBN * ROWB, vg, v_ld, (j + 1) * kFwdBN, Sk, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int row = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int col = kk * 16 + 8 * (lane >> 4);
        ldsm_x4(smem_u32(sQ) + swz<ROWB>(row, col), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const uint8_t* cK = sK + buf * kFwdBN * ROWB;
    const uint8_t* cV = sV + buf * kFwdBN * ROWB;
    // S = Q K^T   (16 x 64 per warp)
    float s[kFwdBN / 8][4];
#pragma unroll
    for (int i = 0; i < kFwdBN / 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < kFwdBN / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int n = np * 16 + (lane & 7) + 8 * (lane >> 4);
        const int kc = kk * 16 + 8 * ((lane >> 3) & 1);
        ldsm_x4(smem_u32(cK) + swz<ROWB>(n, kc), b0, b1, b2, b3);
        mma16816<F16>(s[2 * np], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816<F16>(s[2 * np + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // scale + mask
    const int k0 = j * kFwdBN;
    const int qrow0 = q0 + warp * 16 + g;
    const bool need_mask = (k0 + kFwdBN > Sk) || (CAUSAL && k0 + kFwdBN - 1 > q0);
#pragma unroll
    for (int nt = 0; nt < kFwdBN / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[nt][e] * scale_log2;
        if (need_mask) {
          const int kc = k0 + nt * 8 + 2 * t4 + (e & 1);
          const int qr = qrow0 + ((e >> 1) ? 8 : 0);
          if (kc >= Sk || (CAUSAL && kc > qr)) x = -INFINITY;
        }
        s[nt][e] = x;
      }
    }
    // online softmax
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < kFwdBN / 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * r], s[nt][2 * r + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_r[r], mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(m_r[r] - m_use);
      float rs = 0.f;
#pragma unroll
      for (int nt = 0; nt < kFwdBN / 8; ++nt) {
        const float p0 = exp2f(s[nt][2 * r] - m_use);
        const float p1 = exp2f(s[nt][2 * r + 1] - m_use);
        s[nt][2 * r] = p0;
        s[nt][2 * r + 1] = p1;
        rs += p0 + p1;
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      l_r[r] = l_r[r] * alpha + rs;
      m_r[r] = m_new;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        oacc[dt][2 * r] *= alpha;
        oacc[dt][2 * r + 1] *= alpha;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < kFwdBN / 16; ++kk) {
      const uint32_t a0 = pack2<F16>(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack2<F16>(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack2<F16>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack2<F16>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int kr = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int nc = np * 16 + 8 * (lane >> 4);
        ldsm_x4_t(smem_u32(cV) + swz<ROWB>(kr, nc), b0, b1, b2, b3);
        mma16816<F16>(oacc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816<F16>(oacc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
  // epilogue
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qr = q0 + warp * 16 + g + 8 * r;
    if (qr >= Sq) continue;
    const float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    uint16_t* orow = o + b * o_bs + (long long)qr * o_ld + (long long)h * D;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      const uint32_t packed = pack2<F16>(oacc[dt][2 * r] * inv, oacc[dt][2 * r + 1] * inv);
      *reinterpret_cast<uint32_t*>(orow + dt * 8 + 2 * t4) = packed;
    }
    if (t4 == 0) {
      const float l2 = (m_r[r] == -INFINITY) ? -INFINITY : (m_r[r] + log2f(l_r[r]));
      lse[(long long)bh * Sq + qr] = l2 * 0.6931471805599453f;
    }
  }
}

// ---------------------------------------------------------------- backward

// delta[b,h,s] = sum_d dO[b,s,h,d] * O[b,s,h,d], and the fp32 dQ accumulator
// row (b,s,h) set to zero. D/8 threads per row, 16-byte loads; rows in
// (b, s, h) order so that neighbouring threads read neighbouring memory.
template <bool F16, int D>
__global__ void flash_bwd_pre_kernel(const uint16_t* __restrict__ o, const uint16_t* __restrict__ dout,
                                     float* __restrict__ delta, float* __restrict__ acc, long long rows, int H, int S,
                                     long long o_ld, long long do_ld, long long o_bs, long long do_bs) {
  constexpr int TPR = D / 8;
  const long long gt = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long row = gt / TPR;
  const int part = (int)(gt % TPR);
  float sum = 0.f;
  const bool in = row < rows;
  long long b = 0, s = 0, h = 0;
  if (in) {
    b = row / ((long long)S * H);
    const long long rem = row - b * S * H;
    s = rem / H;
    h = rem - s * H;
    const uint4 x = *reinterpret_cast<const uint4*>(o + b * o_bs + s * o_ld + h * D + part * 8);
    const uint4 y = *reinterpret_cast<const uint4*>(dout + b * do_bs + s * do_ld + h * D + part * 8);
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a0, a1, c0, c1;
      if constexpr (F16) {
        const __half2 u = *reinterpret_cast<const __half2*>(&xs[i]);
        const __half2 w = *reinterpret_cast<const __half2*>(&ys[i]);
        a0 = __low2float(u); a1 = __high2float(u); c0 = __low2float(w); c1 = __high2float(w);
      } else {
        const __nv_bfloat162 u = *reinterpret_cast<const __nv_bfloat162*>(&xs[i]);
        const __nv_bfloat162 w = *reinterpret_cast<const __nv_bfloat162*>(&ys[i]);
        a0 = __low2float(u); a1 = __high2float(u); c0 = __low2float(w); c1 = __high2float(w);
      }
      sum += a0 * c0 + a1 * c1;
    }
    float4* ar = reinterpret_cast<float4*>(acc + row * D + part * 8);
    ar[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    ar[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (in && part == 0) delta[(b * H + h) * S + s] = sum;
}

constexpr int kBwdBN = 64;  // keys per CTA
constexpr int kBwdThreads = 128;

template <int D>
struct BwdCfg {
  static constexpr int BQ = (D <= 64) ? 64 : 32;  // queries per inner iteration
};

template <int D, bool CAUSAL, bool F16>
__global__ void __launch_bounds__(kBwdThreads)
    flash_bwd_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                     const uint16_t* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ delta,
                     float* __restrict__ dq_acc, uint16_t* __restrict__ dk, uint16_t* __restrict__ dv, int H, int Sq,
                     int Sk, long long q_ld, long long k_ld, long long v_ld, long long do_ld, long long dk_ld,
                     long long dv_ld, long long q_bs, long long k_bs, long long v_bs, long long do_bs, long long dk_bs,
                     long long dv_bs, float scale, float scale_log2) {
  constexpr int BQ = BwdCfg<D>::BQ;
  constexpr int ROWB = D * 2;
  constexpr int NQT = BQ / 8;  // query n-tiles in S^T
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sK = smem;
  uint8_t* sV = sK + kBwdBN * ROWB;
  uint8_t* sQ = sV + kBwdBN * ROWB;       // 2 buffers
  uint8_t* sDO = sQ + 2 * BQ * ROWB;      // 2 buffers
  uint8_t* sDS = sDO + 2 * BQ * ROWB;     // [64 keys][BQ] swizzled, rows of BQ*2 bytes
  float* sL = reinterpret_cast<float*>(sDS + kBwdBN * BQ * 2);  // 2 x BQ
  float* sD = sL + 2 * BQ;                                      // 2 x BQ

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int kb = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int k0 = kb * kBwdBN;
  const uint16_t* qg = q + b * q_bs + (long long)h * D;
  const uint16_t* kg = k + b * k_bs + (long long)h * D;
  const uint16_t* vg = v + b * v_bs + (long long)h * D;
  const uint16_t* dog = dout + b * do_bs + (long long)h * D;
  const float* lseg = lse + (long long)bh * Sq;
  const float* deltag = delta + (long long)bh * Sq;
  float* dqg = dq_acc + ((long long)b * Sq * H + h) * D;  // row stride H*D floats

  const int nqb = (Sq + BQ - 1) / BQ;
  const int qb_start = CAUSAL ? (k0 / BQ) : 0;

  load_tile<kBwdBN, D, kBwdThreads>(sK, kg, k_ld, k0, Sk, tid);
  load_tile<kBwdBN, D, kBwdThreads>(sV, vg, v_ld, k0, Sk, tid);
  auto load_q_block = [&](int qb, int buf) {
    load_tile<BQ, D, kBwdThreads>(sQ + buf * BQ * ROWB, qg, q_ld, qb * BQ, Sq, tid);
    load_tile<BQ, D, kBwdThreads>(sDO + buf * BQ * ROWB, dog, do_ld, qb * BQ, Sq, tid);
    for (int i = tid; i < BQ; i += kBwdThreads) {
      const int qr = qb * BQ + i;
      sL[buf * BQ + i] = (qr < Sq) ? lseg[qr] * 1.4426950408889634f : INFINITY;
      sD[buf * BQ + i] = (qr < Sq) ? deltag[qr] : 0.f;
    }
  };
  if (qb_start < nqb) load_q_block(qb_start, 0);
  cp_async_commit();

  float dk_acc[D / 8][4], dv_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      dk_acc[i][e] = 0.f;
      dv_acc[i][e] = 0.f;
    }

  const int key_row0 = warp * 16;  // this warp's keys within the block
  for (int qb = qb_start; qb < nqb; ++qb) {
    const int buf = (qb - qb_start) & 1;
    if (qb + 1 < nqb) load_q_block(qb + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint8_t* cQ = sQ + buf * BQ * ROWB;
    const uint8_t* cDO = sDO + buf * BQ * ROWB;
    const float* cL = sL + buf * BQ;
    const float* cD = sD + buf * BQ;
    const int q0 = qb * BQ;

    // S^T = K_w Q^T and dP^T = V_w dO^T   (16 keys x BQ queries)
    float st[NQT][4], dpt[NQT][4];
#pragma unroll
    for (int i = 0; i < NQT; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        st[i][e] = 0.f;
        dpt[i][e] = 0.f;
      }
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t ka0, ka1, ka2, ka3, va0, va1, va2, va3;
      const int row = key_row0 + (lane & 7) + 8 * ((lane >> 3) & 1);
      const int col = kk * 16 + 8 * (lane >> 4);
      ldsm_x4(smem_u32(sK) + swz<ROWB>(row, col), ka0, ka1, ka2, ka3);
      ldsm_x4(smem_u32(sV) + swz<ROWB>(row, col), va0, va1, va2, va3);
#pragma unroll
      for (int np = 0; np < BQ / 16; ++np) {
        uint32_t b0, b1, b2, b3, c0, c1, c2, c3;
        const int n = np * 16 + (lane & 7) + 8 * (lane >> 4);
        const int kc = kk * 16 + 8 * ((lane >> 3) & 1);
        ldsm_x4(smem_u32(cQ) + swz<ROWB>(n, kc), b0, b1, b2, b3);
        ldsm_x4(smem_u32(cDO) + swz<ROWB>(n, kc), c0, c1, c2, c3);
        mma16816<F16>(st[2 * np], ka0, ka1, ka2, ka3, b0, b1);
        mma16816<F16>(st[2 * np + 1], ka0, ka1, ka2, ka3, b2, b3);
        mma16816<F16>(dpt[2 * np], va0, va1, va2, va3, c0, c1);
        mma16816<F16>(dpt[2 * np + 1], va0, va1, va2, va3, c2, c3);
      }
    }
    // P^T and dS^T
#pragma unroll
    for (int nt = 0; nt < NQT; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = nt * 8 + 2 * t4 + (e & 1);
        const int key = k0 + key_row0 + g + ((e >> 1) ? 8 : 0);
        const int qr = q0 + qi;
        float p = exp2f(st[nt][e] * scale_log2 - cL[qi]);
        if (qr >= Sq || key >= Sk || (CAUSAL && key > qr)) p = 0.f;
        st[nt][e] = p;
        dpt[nt][e] = p * (dpt[nt][e] - cD[qi]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q     (k = queries)
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      const uint32_t pa0 = pack2<F16>(st[2 * kk][0], st[2 * kk][1]);
      const uint32_t pa1 = pack2<F16>(st[2 * kk][2], st[2 * kk][3]);
      const uint32_t pa2 = pack2<F16>(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      const uint32_t pa3 = pack2<F16>(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      const uint32_t sa0 = pack2<F16>(dpt[2 * kk][0], dpt[2 * kk][1]);
      const uint32_t sa1 = pack2<F16>(dpt[2 * kk][2], dpt[2 * kk][3]);
      const uint32_t sa2 = pack2<F16>(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      const uint32_t sa3 = pack2<F16>(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3, c0, c1, c2, c3;
        const int kr = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int nc = np * 16 + 8 * (lane >> 4);
        ldsm_x4_t(smem_u32(cDO) + swz<ROWB>(kr, nc), b0, b1, b2, b3);
        ldsm_x4_t(smem_u32(cQ) + swz<ROWB>(kr, nc), c0, c1, c2, c3);
        mma16816<F16>(dv_acc[2 * np], pa0, pa1, pa2, pa3, b0, b1);
        mma16816<F16>(dv_acc[2 * np + 1], pa0, pa1, pa2, pa3, b2, b3);
        mma16816<F16>(dk_acc[2 * np], sa0, sa1, sa2, sa3, c0, c1);
        mma16816<F16>(dk_acc[2 * np + 1], sa0, sa1, sa2, sa3, c2, c3);
      }
      // dS^T into shared memory for the dQ product: rows = keys, cols = queries
      const int kr0 = key_row0 + g;
      const int qc = kk * 16 + 2 * t4;
      *reinterpret_cast<uint32_t*>(sDS + swz<BQ * 2>(kr0, qc)) = sa0;
      *reinterpret_cast<uint32_t*>(sDS + swz<BQ * 2>(kr0 + 8, qc)) = sa1;
      *reinterpret_cast<uint32_t*>(sDS + swz<BQ * 2>(kr0, qc + 8)) = sa2;
      *reinterpret_cast<uint32_t*>(sDS + swz<BQ * 2>(kr0 + 8, qc + 8)) = sa3;
    }
    __syncthreads();
    // dQ[q, d] += scale * sum_key dS[q, key] K[key, d]
    {
      constexpr int RG = BQ / 16;          // query row groups
      constexpr int DS = 4 / RG;           // d splits per row group
      constexpr int DW = D / DS;           // d columns per warp
      const int rg = warp % RG, ds = warp / RG;
      float acc[DW / 8][4];
#pragma unroll
      for (int i = 0; i < DW / 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kBwdBN / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        // A = dS (rows q, k = key) from sDS [key][q] via transposed load
        const int kr = kk * 16 + (lane & 7) + 8 * (lane >> 4);
        const int qc = rg * 16 + 8 * ((lane >> 3) & 1);
        ldsm_x4_t(smem_u32(sDS) + swz<BQ * 2>(kr, qc), a0, a1, a2, a3);
#pragma unroll
        for (int np = 0; np < DW / 16; ++np) {
          uint32_t b0, b1, b2, b3;
          const int kr2 = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
          const int nc = ds * DW + np * 16 + 8 * (lane >> 4);
          ldsm_x4_t(smem_u32(sK) + swz<ROWB>(kr2, nc), b0, b1, b2, b3);
          mma16816<F16>(acc[2 * np], a0, a1, a2, a3, b0, b1);
          mma16816<F16>(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int qr = q0 + rg * 16 + g + 8 * r;
        if (qr >= Sq) continue;
        float* row = dqg + (long long)qr * H * D + ds * DW;
#pragma unroll
        for (int dt = 0; dt < DW / 8; ++dt) {
          atomicAdd(row + dt * 8 + 2 * t4, acc[dt][2 * r] * scale);
          atomicAdd(row + dt * 8 + 2 * t4 + 1, acc[dt][2 * r + 1] * scale);
        }
      }
    }
    __syncthreads();
  }
  // write dK (scaled) and dV for this warp's 16 keys
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = k0 + key_row0 + g + 8 * r;
    if (key >= Sk) continue;
    uint16_t* dkr = dk + b * dk_bs + (long long)key * dk_ld + (long long)h * D;
    uint16_t* dvr = dv + b * dv_bs + (long long)key * dv_ld + (long long)h * D;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      *reinterpret_cast<uint32_t*>(dkr + dt * 8 + 2 * t4) = pack2<F16>(dk_acc[dt][2 * r] * scale, dk_acc[dt][2 * r + 1] * scale);
      *reinterpret_cast<uint32_t*>(dvr + dt * 8 + 2 * t4) = pack2<F16>(dv_acc[dt][2 * r], dv_acc[dt][2 * r + 1]);
    }
  }
}

// dq[b,s,h,:] = 16-bit(dq_acc[b,s,h,:]), eight elements per thread.
template <bool F16>
__global__ void dq_convert_kernel(const float* __restrict__ acc, uint16_t* __restrict__ dq, long long nvec, int HD8,
                                  long long dq_ld, long long dq_bs, int S) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / HD8;
    const int c = (int)(i - r * HD8) * 8;
    const long long bb = r / S, s = r - bb * S;
    const float4 a0 = *reinterpret_cast<const float4*>(acc + i * 8);
    const float4 a1 = *reinterpret_cast<const float4*>(acc + i * 8 + 4);
    uint4 w;
    w.x = pack2<F16>(a0.x, a0.y);
    w.y = pack2<F16>(a0.z, a0.w);
    w.z = pack2<F16>(a1.x, a1.y);
    w.w = pack2<F16>(a1.z, a1.w);
    *reinterpret_cast<uint4*>(dq + bb * dq_bs + s * dq_ld + c) = w;
  }
}

// ---------------------------------------------------------------- host

static void check_bshd(const at::Tensor& t, const char* name, int64_t D) {
  KB_CHECK(t.dim() == 4, std::string(name) + " must be [B, S, H, D]");
  KB_CHECK(t.stride(3) == 1 && t.stride(2) == D, std::string(name) + " must have contiguous heads");
  KB_CHECK(t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kHalf, std::string(name) + " must be bf16/fp16");
  KB_CHECK((t.stride(1) * 2) % 16 == 0 && (t.stride(0) * 2) % 16 == 0 &&
               (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0,
           std::string(name) + " rows must be 16-byte aligned");
}

template <int D, bool CAUSAL, bool F16>
static void launch_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                       float scale, cudaStream_t s) {
  const int B = (int)q.size(0), Sq = (int)q.size(1), H = (int)q.size(2), Sk = (int)k.size(1);
  const int smem = (kFwdBM + 4 * kFwdBN) * D * 2;
  auto kern = flash_fwd_kernel<D, CAUSAL, F16>;
  static bool set = false;
  if (!set) {
    KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    set = true;
  }
  dim3 grid((Sq + kFwdBM - 1) / kFwdBM, B * H);
  kern<<<grid, kFwdThreads, smem, s>>>(
      (const uint16_t*)q.data_ptr(), (const uint16_t*)k.data_ptr(), (const uint16_t*)v.data_ptr(),
      (uint16_t*)o.data_ptr(), lse.data_ptr<float>(), H, Sq, Sk, q.stride(1), k.stride(1), v.stride(1), o.stride(1),
      q.stride(0), k.stride(0), v.stride(0), o.stride(0), scale * 1.4426950408889634f);
  KB_LAUNCHED();
}

bool flash_attention_backward_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                 const at::Tensor& dout, const at::Tensor& lse, const float* delta, float* dq_acc,
                                 at::Tensor& dk, at::Tensor& dv, double scale, bool causal, cudaStream_t s);
bool flash_attention_forward_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                                at::Tensor& lse, double scale, bool causal, cudaStream_t s);

// 0: tcgen05 forward where the shape allows it (default); 1: the mma.sync kernels.
static int g_attn_impl = 0;
void attention_set_impl(int64_t impl) { g_attn_impl = (int)impl; }
extern int g_attn_bwd_debug;
void attention_set_debug(int64_t bits) { g_attn_bwd_debug = (int)bits; }
extern long long* g_attn_bwd_trace;
void attention_set_trace(int64_t ptr) { g_attn_bwd_trace = reinterpret_cast<long long*>(ptr); }

void flash_attention_forward(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                             at::Tensor& lse, double scale, bool causal) {
  const int64_t D = q.size(3);
  check_bshd(q, "q", D);
  check_bshd(k, "k", D);
  check_bshd(v, "v", D);
  check_bshd(o, "o", D);
  KB_CHECK(D == 64 || D == 128, "head dim must be 64 or 128");
  KB_CHECK(!causal || q.size(1) == k.size(1), "causal attention needs equal query/key lengths");
  KB_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == q.size(0) * q.size(2) * q.size(1),
           "lse must be fp32 [B, H, S]");
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  if (g_attn_impl == 0 && flash_attention_forward_tc(q, k, v, o, lse, scale, causal, s)) return;
  const bool f16 = q.scalar_type() == at::kHalf;
  const float sc = (float)scale;
#define KB_FWD(DD, CC, FF) launch_fwd<DD, CC, FF>(q, k, v, o, lse, sc, s)
  if (D == 64) {
    if (causal) { if (f16) KB_FWD(64, true, true); else KB_FWD(64, true, false); }
    else { if (f16) KB_FWD(64, false, true); else KB_FWD(64, false, false); }
  } else {
    if (causal) { if (f16) KB_FWD(128, true, true); else KB_FWD(128, true, false); }
    else { if (f16) KB_FWD(128, false, true); else KB_FWD(128, false, false); }
  }
#undef KB_FWD
}

template <int D, bool CAUSAL, bool F16>
static void launch_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
                       const at::Tensor& lse, const at::Tensor& delta, at::Tensor& dq_acc, at::Tensor& dk,
                       at::Tensor& dv, float scale, cudaStream_t s) {
  constexpr int BQ = BwdCfg<D>::BQ;
  const int B = (int)q.size(0), Sq = (int)q.size(1), H = (int)q.size(2), Sk = (int)k.size(1);
  const int smem = 2 * kBwdBN * D * 2 + 4 * BQ * D * 2 + kBwdBN * BQ * 2 + 4 * BQ * 4;
  auto kern = flash_bwd_kernel<D, CAUSAL, F16>;
  static bool set = false;
  if (!set) {
    KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    set = true;
  }
  dim3 grid((Sk + kBwdBN - 1) / kBwdBN, B * H);
  kern<<<grid, kBwdThreads, smem, s>>>(
      (const uint16_t*)q.data_ptr(), (const uint16_t*)k.data_ptr(), (const uint16_t*)v.data_ptr(),
      (const uint16_t*)dout.data_ptr(), lse.data_ptr<float>(), delta.data_ptr<float>(), dq_acc.data_ptr<float>(),
      (uint16_t*)dk.data_ptr(), (uint16_t*)dv.data_ptr(), H, Sq, Sk, q.stride(1), k.stride(1), v.stride(1),
      dout.stride(1), dk.stride(1), dv.stride(1), q.stride(0), k.stride(0), v.stride(0), dout.stride(0), dk.stride(0),
      dv.stride(0), scale, scale * 1.4426950408889634f);
  KB_LAUNCHED();
}

// Computes dq, dk, dv. `workspace` is fp32 scratch of at least
// B*S*H*D + B*H*S elements (dQ accumulator + softmax delta).
void flash_attention_backward(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                              const at::Tensor& dout, const at::Tensor& lse, at::Tensor& dq, at::Tensor& dk,
                              at::Tensor& dv, at::Tensor& workspace, double scale, bool causal) {
  const int64_t D = q.size(3);
  for (auto* t : {&q, &k, &v, &o, &dout}) check_bshd(*t, "attention operand", D);
  check_bshd(dq, "dq", D);
  check_bshd(dk, "dk", D);
  check_bshd(dv, "dv", D);
  const int B = (int)q.size(0), Sq = (int)q.size(1), H = (int)q.size(2);
  const int64_t acc_elems = (int64_t)B * Sq * H * D;
  const int64_t delta_elems = (int64_t)B * H * Sq;
  KB_CHECK(workspace.scalar_type() == at::kFloat && workspace.numel() >= acc_elems + delta_elems,
           "attention backward workspace too small");
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t s = c10::cuda::getCurrentCUDAStream().stream();
  const bool f16 = q.scalar_type() == at::kHalf;
  float* acc = workspace.data_ptr<float>();
  float* delta = acc + acc_elems;
  at::Tensor acc_t = workspace.narrow(0, 0, acc_elems);
  at::Tensor delta_t = workspace.narrow(0, acc_elems, delta_elems);
  {
    // delta pre-pass; also zeroes the dQ accumulator.
    const long long rows = (long long)B * Sq * H;
    const long long threads = rows * (D / 8);
    const int blocks = (int)((threads + 255) / 256);
    const uint16_t* op = (const uint16_t*)o.data_ptr();
    const uint16_t* dp = (const uint16_t*)dout.data_ptr();
#define KB_PRE(FF, DD)                                                                                          \
  flash_bwd_pre_kernel<FF, DD><<<blocks, 256, 0, s>>>(op, dp, delta, acc, rows, H, Sq, o.stride(1), dout.stride(1), \
                                                      o.stride(0), dout.stride(0))
    if (D == 64) { if (f16) KB_PRE(true, 64); else KB_PRE(false, 64); }
    else { if (f16) KB_PRE(true, 128); else KB_PRE(false, 128); }
#undef KB_PRE
    KB_LAUNCHED();
  }
  const float sc = (float)scale;
#define KB_BWD(DD, CC, FF) launch_bwd<DD, CC, FF>(q, k, v, dout, lse, delta_t, acc_t, dk, dv, sc, s)
  if (g_attn_impl == 0 && flash_attention_backward_tc(q, k, v, dout, lse, delta, acc, dk, dv, scale, causal, s)) {
  } else if (D == 64) {
    if (causal) { if (f16) KB_BWD(64, true, true); else KB_BWD(64, true, false); }
    else { if (f16) KB_BWD(64, false, true); else KB_BWD(64, false, false); }
  } else {
    if (causal) { if (f16) KB_BWD(128, true, true); else KB_BWD(128, true, false); }
    else { if (f16) KB_BWD(128, false, true); else KB_BWD(128, false, false); }
  }
#undef KB_BWD
  const long long nvec = (long long)B * Sq * H * D / 8;
  const int blocks = (int)std::min<long long>((nvec + 255) / 256, num_sms(q.get_device()) * 16LL);
  if (f16)
    dq_convert_kernel<true><<<blocks, 256, 0, s>>>(acc, (uint16_t*)dq.data_ptr(), nvec, (int)(H * D / 8),
                                                   dq.stride(1), dq.stride(0), Sq);
  else
    dq_convert_kernel<false><<<blocks, 256, 0, s>>>(acc, (uint16_t*)dq.data_ptr(), nvec, (int)(H * D / 8),
                                                    dq.stride(1), dq.stride(0), Sq);
  KB_LAUNCHED();
}

void register_attention_ops(pybind11::module& m) {
  m.def("attention_set_debug", &attention_set_debug,
        "Diagnostics for the tcgen05 attention backward (bit 0: skip dQ reductions, bit 1: skip elementwise math)");
  m.def("attention_set_trace", &attention_set_trace,
        "Diagnostics: device address of an int64[168] buffer for clock64 stamps of one backward CTA (0 = off)");
  m.def("attention_set_impl", &attention_set_impl,
        "attention forward implementation: 0 = tcgen05 (default), 1 = mma.sync kernels");
  m.def("flash_attention_forward", &flash_attention_forward);
  m.def("flash_attention_backward", &flash_attention_backward);
}

}  // namespace kb
