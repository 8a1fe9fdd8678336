// Flash-attention forward on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// One CTA computes 256 query rows (two 128-row tiles t = 0, 1) of one
// (batch, head) against its keys, 128 keys per step. K and V tiles are loaded
// once per step and used by both query tiles. Roles (384 threads):
//   warp 0      TMA producer: Q (both tiles) once, then K_j / V_j into a ring
//               of 128-byte-swizzled stages (no multicast).
//   warp 1      TMEM owner and single-thread MMA issuer, per step j and tile t:
//                 S_t  = Q_t K_j^T        M=128, N=128, K=D   (A, B in smem)
//                 O_t += P_t V_j          M=128, N=D,   K=128 (A = P in TMEM)
//               The two tiles alternate, so the tensor cores work on one tile
//               while the softmax warps of the other run.
//   warps 4..11 softmax, four warps per tile, one thread per query row (its
//               TMEM lane). A thread reads its row of S_t (two passes: maximum,
//               then exponentials), writes P_t = exp2(S_t * scale*log2e - m)
//               as 16-bit pairs over the first half of S_t's columns, and keeps
//               the row's running sum l. O_t accumulates in TMEM; it is only
//               rescaled when the row maximum grows by more than 2^8 over the
//               maximum the exponentials were taken against (the rescale reads
//               and rewrites O_t in TMEM). Probabilities up to 2^8 are exact in
//               the 16-bit P, and O / l is unchanged by the choice of m.
// TMEM (512 columns): S_0, S_1 at columns 0 and 128; O_0, O_1 at 256 and 256+D.
// The S MMA of step j+1 for a tile is issued after the P V MMA of step j that
// reads P from the same columns; tcgen05 MMAs issued by one thread execute in
// order, and the completion of S_{j+1} (signalled by tcgen05.commit, which
// tracks every earlier MMA of the thread) also means that O_t holds P_j V_j.
//
// Every mbarrier wait is bounded (%globaltimer); a wait that runs out records
// a status code, raises the CTA abort flag, and the kernel drains its own
// copies and MMAs, frees TMEM and returns. The LSE written is the natural-log
// log-sum-exp of the scaled scores, as the backward kernels expect.
#include "host_utils.h"
#include "sm100.cuh"

#include <torch/extension.h>

namespace kb {

constexpr int kTcBM = 128;        // query rows per tile (two tiles per CTA)
constexpr int kTcBN = 128;        // keys per step
constexpr int kTcThreads = 384;   // warpgroup 0: producer, MMA (+2 idle); warpgroups 1, 2: softmax
// Register split (launch: 168 per thread): warpgroup 0 gives back down to 72,
// the softmax warpgroups take 216 (72*128 + 2*216*128 = 384*168).
constexpr int kTcRegsCtl = 72;
constexpr int kTcRegsSoftmax = 216;
constexpr float kRescaleLog2 = 8.f;

template <int D>
struct TcFwdCfg {
  static constexpr int kChunks = D / 64;                 // 64-wide (128-byte) column chunks of a row
  static constexpr int kTileBytes = kTcBN * D * 2;       // one Q, K or V tile
  static constexpr int kStages = D == 64 ? 4 : 2;        // K/V ring depth
  static constexpr int kQBufs = D == 64 ? 2 : 1;         // Q buffers (of two tiles): the next item's Q prefetches
  static constexpr int kSmemBytes = (2 * kQBufs + 2 * kStages) * kTileBytes + 1024 + 256;
  static constexpr int kOCol = 2 * kTcBN;                // TMEM column of O_0
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool F16>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  if constexpr (F16) return pack_f16(a, b);
  else return pack_bf16(a, b);
}

struct TcFwdArgs {
  uint16_t* o;
  float* lse;
  int B, H, Sq, Sk;
  long long o_ld, o_bs;
  float scale_log2;
  int* status;
};

// One softmax step of one row: reads S (128 columns at s_tm) into registers,
// updates the row's reference maximum m (scaled, log2 units) and sum l,
// writes P over S's first 64 columns, and rescales O when m moved (after P,
// when the scores no longer occupy registers; O is not read by the tensor
// cores until this step's P is published, and it holds every earlier P V
// product: the completion of this block's S MMA implies that of the previous
// P V MMA).
template <int D, bool MASK, bool F16>
__device__ __forceinline__ void softmax_step(uint32_t s_tm, uint32_t o_tm, int key0, int key_lim, float scale_log2,
                                             bool first, float& m, float& l) {
  uint32_t v0[64], v1[64];
  tmem_ld_32x32b_x64(s_tm, v0);
  tmem_ld_32x32b_x64(s_tm + 64, v1);
  tmem_wait_ld_dep64(v0);
  tmem_wait_ld_dep64(v1);
  if (MASK) {
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      if (key0 + i >= key_lim) v0[i] = __float_as_uint(-INFINITY);
      if (key0 + 64 + i >= key_lim) v1[i] = __float_as_uint(-INFINITY);
    }
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 64; i += 2) {
    mx0 = max3f(mx0, __uint_as_float(v0[i]), __uint_as_float(v0[i + 1]));
    mx1 = max3f(mx1, __uint_as_float(v1[i]), __uint_as_float(v1[i + 1]));
  }
  const float mxs = fmaxf(mx0, mx1) * scale_log2;
  const bool upd = mxs > m + kRescaleLog2;
  float factor = 1.f;
  if (upd) {
    factor = ex2_approx(m - mxs);  // 0 while m is -inf
    m = mxs;
  }
  l *= factor;
  // Masked scores are -inf here, so their exponentials are exactly 0.
  const float mneg = m == -INFINITY ? 0.f : -m;
  const float2 sc2 = make_float2(scale_log2, scale_log2), mn2 = make_float2(mneg, mneg);
  float2 rs0 = make_float2(0.f, 0.f), rs1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t* v = c < 2 ? &v0[32 * c] : &v1[32 * (c - 2)];
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float2 x0 = fma2(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), sc2, mn2);
      const float2 x1 = fma2(make_float2(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3])), sc2, mn2);
      const float2 p0 = make_float2(ex2_approx(x0.x), ex2_approx(x0.y));
      const float2 p1 = make_float2(ex2_approx(x1.x), ex2_approx(x1.y));
      rs0 = add2(rs0, p0);
      rs1 = add2(rs1, p1);
      pk[i / 2] = pack_pair<F16>(p0.x, p0.y);
      pk[i / 2 + 1] = pack_pair<F16>(p1.x, p1.y);
    }
    tmem_st_32x32b_x16(s_tm + 16 * c, pk);
  }
  if (!first && __any_sync(0xffffffffu, upd)) {
    // O_t (which holds every earlier P V product) takes the new reference.
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      uint32_t ov[32];
      tmem_ld_32x32b_x32(o_tm + 32 * c, ov);
      tmem_wait_ld_dep(ov);
#pragma unroll
      for (int t = 0; t < 32; ++t) ov[t] = __float_as_uint(__uint_as_float(ov[t]) * factor);
      tmem_st_32x32b_x32(o_tm + 32 * c, ov);
    }
  }
  tmem_wait_st();
  l += (rs0.x + rs0.y) + (rs1.x + rs1.y);
}

// Work item `idx` of a persistent CTA: a 256-row query block of one (batch,
// head). Causal items are ordered by decreasing cost (most key blocks first),
// so the static round-robin assignment over CTAs stays balanced.
struct TcItem {
  int b, h, bh, q0, n0, n1;  // n0 / n1: key blocks that query tile 0 / 1 needs (n0 <= n1)
};

template <bool CAUSAL>
__device__ __forceinline__ TcItem tc_item(int idx, int H, int BH, int Sq, int Sk) {
  const int num_qb = (Sq + 2 * kTcBM - 1) / (2 * kTcBM);
  TcItem it;
  const int qb = CAUSAL ? num_qb - 1 - idx / BH : idx / BH;
  it.bh = idx % BH;
  it.b = it.bh / H;
  it.h = it.bh % H;
  it.q0 = qb * 2 * kTcBM;
  const int nk = (Sk + kTcBN - 1) / kTcBN;
  it.n0 = CAUSAL ? min(nk, (it.q0 + kTcBM - 1) / kTcBN + 1) : nk;
  it.n1 = CAUSAL ? min(nk, (it.q0 + 2 * kTcBM - 1) / kTcBN + 1) : nk;
  return it;
}

template <int D, bool CAUSAL, bool F16>
__global__ void __launch_bounds__(kTcThreads, 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const TcFwdArgs a) {
  using Cfg = TcFwdCfg<D>;
  constexpr int ST = Cfg::kStages;
  constexpr int QB = Cfg::kQBufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                              // QB buffers of two tiles
  uint8_t* sK = sQ + QB * 2 * Cfg::kTileBytes;
  uint8_t* sV = sK + ST * Cfg::kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ST * Cfg::kTileBytes);
  uint64_t* q_full = bars;             // [QB]
  uint64_t* q_empty = q_full + QB;     // [QB]: every S MMA of the item that used the buffer is done
  uint64_t* k_full = q_empty + QB;     // [ST]
  uint64_t* v_full = k_full + ST;      // [ST]
  uint64_t* kv_empty = v_full + ST;    // [ST]
  uint64_t* s_full = kv_empty + ST;    // [2], per tile
  uint64_t* p_full = s_full + 2;       // [2], per tile (4 softmax warps arrive)
  uint64_t* o_done = p_full + 2;       // [2], per tile: the item's last P V product is complete
  uint64_t* o_empty = o_done + 2;      // [2], per tile: the epilogue has read O (4 warps arrive)
  uint64_t* drain = o_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = a.B * a.H;
  const int n_items = ((a.Sq + 2 * kTcBM - 1) / (2 * kTcBM)) * BH;

  if (threadIdx.x == 0) {
    for (int i = 0; i < QB; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) tmem_alloc(tmem_holder, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kTcRegsCtl));
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------------- producer
      uint32_t armed = 0, armed_par = 0, q_armed = 0, q_par = 0;
      bool ok = true;
      int kv_it = 0, n_it = 0;
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ++n_it) {
        const TcItem it = tc_item<CAUSAL>(idx, a.H, BH, a.Sq, a.Sk);
        const int qbuf = n_it % QB;
        const uint32_t qph = (n_it / QB) & 1;
        if (!mbar_wait(&q_empty[qbuf], qph ^ 1, abort_flag, a.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full[qbuf], 2 * Cfg::kTileBytes);
        q_armed |= 1u << qbuf;
        q_par = (q_par & ~(1u << qbuf)) | (qph << qbuf);
        uint8_t* q_dst = sQ + qbuf * 2 * Cfg::kTileBytes;
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int c = 0; c < Cfg::kChunks; ++c)
            tma_load_4d(&tq, &q_full[qbuf], q_dst + t * Cfg::kTileBytes + c * (kTcBM * 128), 64 * c,
                        it.q0 + t * kTcBM, it.h, it.b);
        for (int j = 0; j < it.n1; ++j, ++kv_it) {
          const int st = kv_it % ST;
          const uint32_t ph = (kv_it / ST) & 1;
          if (!mbar_wait(&kv_empty[st], ph ^ 1, abort_flag, a.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], Cfg::kTileBytes);
          mbar_arrive_expect_tx(&v_full[st], Cfg::kTileBytes);
          armed |= 1u << st;
          armed_par = (armed_par & ~(1u << st)) | (ph << st);
#pragma unroll
          for (int c = 0; c < Cfg::kChunks; ++c) {
            tma_load_4d(&tk, &k_full[st], sK + st * Cfg::kTileBytes + c * (kTcBN * 128), 64 * c, j * kTcBN, it.h,
                        it.b);
            tma_load_4d(&tv, &v_full[st], sV + st * Cfg::kTileBytes + c * (kTcBN * 128), 64 * c, j * kTcBN, it.h,
                        it.b);
          }
        }
      }
      // Every issued copy must land before the CTA may exit (the last arming
      // of each barrier is the newest phase, so waiting on it covers the rest).
      volatile int never = 0;
      for (int i = 0; i < QB; ++i)
        if (q_armed & (1u << i))
          if (!mbar_wait(&q_full[i], (q_par >> i) & 1u, &never, a.status, kStatusTimeoutDrain)) break;
      for (int s = 0; s < ST; ++s) {
        if (armed & (1u << s)) {
          const uint32_t ph = (armed_par >> s) & 1u;
          if (!mbar_wait(&k_full[s], ph, &never, a.status, kStatusTimeoutDrain)) break;
          if (!mbar_wait(&v_full[s], ph, &never, a.status, kStatusTimeoutDrain)) break;
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_s = idesc_f16(kTcBM, kTcBN, F16, false, false);
      constexpr uint32_t idesc_o = idesc_f16(kTcBM, D, F16, false, true);
      bool ok = true, issued = false;
      int kv_it = 0, n_it = 0;
      uint32_t p_cnt0 = 0, p_cnt1 = 0;
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ++n_it) {
        const TcItem it = tc_item<CAUSAL>(idx, a.H, BH, a.Sq, a.Sk);
        const int qbuf = n_it % QB;
        if (!mbar_wait(&q_full[qbuf], (n_it / QB) & 1, abort_flag, a.status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        const uint32_t q_base = smem_u32(sQ + qbuf * 2 * Cfg::kTileBytes);
        auto issue_s = [&](int kvi, int t) -> bool {
          const int st = kvi % ST;
          if (!mbar_wait(&k_full[st], (kvi / ST) & 1, abort_flag, a.status, kStatusTimeoutMma)) return false;
          tc_fence_after();
          const uint32_t q_addr = q_base + t * Cfg::kTileBytes;
          const uint32_t k_addr = smem_u32(sK + st * Cfg::kTileBytes);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (kTcBN * 128) + (kk & 3) * 32;  // chunk, then 32 B per K=16 step
            umma_f16_ss(tmem + t * kTcBN, sw128_desc(q_addr + off, 16, 1024), sw128_desc(k_addr + off, 16, 1024),
                        idesc_s, kk != 0 ? 1u : 0u);
          }
          umma_commit(&s_full[t]);
          issued = true;
          return true;
        };
        if (!issue_s(kv_it, 0) || !issue_s(kv_it, 1)) {
          ok = false;
          break;
        }
        if (it.n1 == 1) umma_commit(&q_empty[qbuf]);
        for (int j = 0; j < it.n1 && ok; ++j, ++kv_it) {
          const int st = kv_it % ST;
          if (!mbar_wait(&v_full[st], (kv_it / ST) & 1, abort_flag, a.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          const uint32_t v_addr = smem_u32(sV + st * Cfg::kTileBytes);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int n = t == 0 ? it.n0 : it.n1;
            if (j >= n || !ok) continue;
            uint32_t& p_cnt = t == 0 ? p_cnt0 : p_cnt1;
            if (!mbar_wait(&p_full[t], p_cnt & 1, abort_flag, a.status, kStatusTimeoutMma) ||
                (j == 0 && !mbar_wait(&o_empty[t], (n_it & 1) ^ 1, abort_flag, a.status, kStatusTimeoutMma))) {
              ok = false;
              break;
            }
            ++p_cnt;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kTcBN / 16; ++kk)
              umma_f16_ts(tmem + Cfg::kOCol + t * D, tmem + t * kTcBN + kk * 8,
                          sw128_desc(v_addr + kk * 2048, kTcBN * 128, 1024), idesc_o, (j | kk) != 0 ? 1u : 0u);
            if (j + 1 < n) {
              if (!issue_s(kv_it + 1, t)) {
                ok = false;
                break;
              }
              if (t == 1 && j + 2 == it.n1) umma_commit(&q_empty[qbuf]);
            } else {
              umma_commit(&o_done[t]);
            }
          }
          umma_commit(&kv_empty[st]);
        }
      }
      if (issued) {
        umma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, a.status, kStatusTimeoutDrain);
      }
    }
    tc_fence_before();
    named_bar_sync(1, kTcThreads);
    if (warp == 1) tmem_dealloc(tmem, 512);
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kTcRegsSoftmax));
    // ---------------------------------------------------------------- softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tm = tmem + lane_off + t * kTcBN;
    const uint32_t o_tm = tmem + lane_off + Cfg::kOCol + t * D;
    uint32_t s_cnt = 0;
    bool ok = true;
    int n_it = 0;
    for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ++n_it) {
      const TcItem it = tc_item<CAUSAL>(idx, a.H, BH, a.Sq, a.Sk);
      const int n = t == 0 ? it.n0 : it.n1;
      const int row_first = it.q0 + t * kTcBM;  // first query row of the tile
      const int qrow = row_first + r;
      const int key_lim = CAUSAL ? min(a.Sk, qrow + 1) : a.Sk;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j, ++s_cnt) {
        if (!mbar_wait(&s_full[t], s_cnt & 1, abort_flag, a.status, kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int key0 = j * kTcBN;
        const bool need_mask = (key0 + kTcBN > a.Sk) || (CAUSAL && key0 + kTcBN - 1 > row_first);
        if (need_mask) softmax_step<D, true, F16>(s_tm, o_tm, key0, key_lim, a.scale_log2, j == 0, m, l);
        else softmax_step<D, false, F16>(s_tm, o_tm, key0, key_lim, a.scale_log2, j == 0, m, l);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok || !mbar_wait(&o_done[t], n_it & 1, abort_flag, a.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint16_t* orow = a.o + (long long)it.b * a.o_bs + (long long)qrow * a.o_ld + (long long)it.h * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(o_tm + 32 * c, ov);
        tmem_wait_ld_dep(ov);
        if (qrow < a.Sq) {
#pragma unroll
          for (int d = 0; d < 32; d += 8) {
            uint4 w;
            w.x = pack_pair<F16>(__uint_as_float(ov[d]) * inv, __uint_as_float(ov[d + 1]) * inv);
            w.y = pack_pair<F16>(__uint_as_float(ov[d + 2]) * inv, __uint_as_float(ov[d + 3]) * inv);
            w.z = pack_pair<F16>(__uint_as_float(ov[d + 4]) * inv, __uint_as_float(ov[d + 5]) * inv);
            w.w = pack_pair<F16>(__uint_as_float(ov[d + 6]) * inv, __uint_as_float(ov[d + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + 32 * c + d) = w;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[t]);
      if (qrow < a.Sq) {
        const float l2 = (m == -INFINITY || l <= 0.f) ? -INFINITY : (m + log2f(l));
        a.lse[(long long)it.bh * a.Sq + qrow] = l2 * 0.6931471805599453f;
      }
    }
    if (!ok) *abort_flag = 1;
    tc_fence_before();
    named_bar_sync(1, kTcThreads);
  }
}

// --------------------------------------------------------------------- host

// 4-D view {D, S, H, B} of a [B, S, H, D] tensor, 128-row x 64-column boxes.
static CUtensorMap bshd_map(const at::Tensor& t) {
  const int64_t es = 2;
  uint64_t dims[4] = {(uint64_t)t.size(3), (uint64_t)t.size(1), (uint64_t)t.size(2), (uint64_t)t.size(0)};
  uint64_t strides[3] = {(uint64_t)(t.stride(1) * es), (uint64_t)(t.stride(2) * es), (uint64_t)(t.stride(0) * es)};
  uint32_t box[4] = {64, 128, 1, 1};
  return make_tma(t.data_ptr(), t.scalar_type(), 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D, bool CAUSAL, bool F16>
static void launch_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                          at::Tensor& lse, float scale, cudaStream_t s) {
  using Cfg = TcFwdCfg<D>;
  const int B = (int)q.size(0), Sq = (int)q.size(1), H = (int)q.size(2), Sk = (int)k.size(1);
  const CUtensorMap tq = bshd_map(q), tk = bshd_map(k), tv = bshd_map(v);
  TcFwdArgs args;
  args.o = (uint16_t*)o.data_ptr();
  args.lse = lse.data_ptr<float>();
  args.B = B;
  args.H = H;
  args.Sq = Sq;
  args.Sk = Sk;
  args.o_ld = o.stride(1);
  args.o_bs = o.stride(0);
  args.scale_log2 = scale * 1.4426950408889634f;
  args.status = device_status_ptr(q.get_device());
  auto kern = flash_fwd_tc_kernel<D, CAUSAL, F16>;
  static bool set = false;
  if (!set) {
    KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    set = true;
  }
  const long long items = (long long)((Sq + 2 * kTcBM - 1) / (2 * kTcBM)) * B * H;
  const int grid = (int)std::min<long long>(items, compute_sms(q.get_device()));
  kern<<<grid, kTcThreads, Cfg::kSmemBytes, s>>>(tq, tk, tv, args);
  KB_LAUNCHED();
}

// Runs the tcgen05 forward when the shape allows it; returns false otherwise.
bool flash_attention_forward_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                                at::Tensor& lse, double scale, bool causal, cudaStream_t s) {
  const int64_t D = q.size(3);
  if (D != 64 && D != 128) return false;
  if (k.size(1) > INT32_MAX / 2 || q.size(1) > INT32_MAX / 2) return false;
  const bool f16 = q.scalar_type() == at::kHalf;
  const float sc = (float)scale;
#define KB_TC(DD, CC, FF) launch_fwd_tc<DD, CC, FF>(q, k, v, o, lse, sc, s)
  if (D == 64) {
    if (causal) { if (f16) KB_TC(64, true, true); else KB_TC(64, true, false); }
    else { if (f16) KB_TC(64, false, true); else KB_TC(64, false, false); }
  } else {
    if (causal) { if (f16) KB_TC(128, true, true); else KB_TC(128, true, false); }
    else { if (f16) KB_TC(128, false, true); else KB_TC(128, false, false); }
  }
#undef KB_TC
  return true;
}

}  // namespace kb
