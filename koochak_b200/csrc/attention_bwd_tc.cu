// Flash-attention backward on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Persistent CTAs take 128-key blocks j of one (batch, head) as work items
// and walk the query blocks i that can see each (128 queries per step). Keys are the M dimension
// of the transposed products, so dK and dV accumulate in TMEM across the
// whole walk and are written once:
//   S^T  = K_j Q_i^T             M=128 keys,    N=128 queries, K=D
//   dP^T = V_j dO_i^T            M=128 keys,    N=128 queries, K=D
//   P^T  = exp2(S^T * scale*log2e - LSE_i*log2e)        (16-bit, over S^T)
//   dS^T = P^T * (dP^T - delta_i)                        (16-bit, over dP^T
//                                                          and into smem)
//   dV  += P^T dO_i              A = P^T from TMEM, B = dO_i (MN-major)
//   dK  += dS^T Q_i              A = dS^T from TMEM, B = Q_i (MN-major)
//   dQ_i = dS K_j                A = dS from smem (MN-major), B = K_j (MN-major)
// dQ_i is read out of TMEM and added to the fp32 dQ accumulator by TMA
// reductions (cp.reduce.async.bulk.tensor .add) from a shared-memory staging
// tile, or at D = 128 with vector reductions (red.global.add.v4.f32); the
// softmax scale is applied to dK and dQ on the way out. delta = rowsum(dO * O)
// comes from a pre-pass.
//
// Roles (512 threads): warp 0 producer (lane 0 issues TMA for K_j, V_j and
// the Q_i / dO_i ring; all lanes stage LSE_i and delta_i into shared memory),
// warp 1 TMEM owner + MMA issuer, warps 4..11 elementwise (one thread per key
// row = TMEM lane, two warps per row quarter splitting the 128 queries),
// warps 12..15 dQ readout (one thread per query row).
// The S^T MMA of step i+1 is issued after the dV / dK MMAs of step i that read
// P^T / dS^T from the same TMEM columns; tcgen05 MMAs issued by one thread
// execute in order. At D = 64 it also goes ahead of dQ_i (dS is double
// buffered in shared memory; the completion of S^T_{i+2} covers dQ_i), so
// step i+1's elementwise work overlaps dQ_i. At D = 128 dQ_i uses the upper
// score columns, so S^T_{i+1} waits until dQ_i has been read out; dQ_i is
// issued before dV / dK there, so that readout overlaps their MMAs.
//
// Every mbarrier wait is bounded; a wait that runs out records a status code,
// raises the CTA abort flag, and the kernel drains its copies and MMAs, frees
// TMEM and returns. Head dimensions 64 and 128 (the latter keeps dQ in the
// free halves of the score columns); other head sizes use the mma.sync kernel.
#include "host_utils.h"
#include "sm100.cuh"

#include <cstring>

#include <torch/extension.h>

namespace kb {

int g_attn_bwd_debug = 0;
long long* g_attn_bwd_trace = nullptr;

namespace {

constexpr int kBwBK = 128;
constexpr int kBwBQ = 128;
constexpr int kBwThreads = 512;
// Register split per warpgroup (launch: 128 per thread, so control + dQ
// readout + 2 x elementwise must stay within 4 x 128): the dQ path stages
// through shared memory at D = 64 and reduces from registers at D = 128; at
// D = 128 the elementwise warps hold 64 scores and 64 dP values at once.
template <int D>
struct BwRegs {
  static constexpr int kCtl = D == 64 ? 72 : 80;
  static constexpr int kDq = D == 64 ? 96 : 64;
  static constexpr int kMath = D == 64 ? 168 : 184;
  static_assert((kCtl + kDq + 2 * kMath) * 128 <= 65536, "register split exceeds the launch budget");
};

template <int D>
struct TcBwdCfg {
  static constexpr int kTile = 128 * D * 2;          // one K, V, Q or dO tile
  static constexpr int kStages = 2;                  // Q / dO / LSE / delta ring
  static constexpr int kDsBytes = kBwBK * kBwBQ * 2;  // dS tile (16-bit)
  static constexpr int kVecBytes = kBwBQ * 4;         // one LSE or delta block
  // dQ leaves through TMA reductions from an fp32 staging tile (128 B
  // swizzled, 32 columns per box) where shared memory allows (D = 64); at
  // D = 128 it leaves through vector reductions straight from registers
  // (staging it through the dS tile instead, in two halves, measured slower:
  // 554 us against 494 us on the Llama-style shape).
  static constexpr bool kDqTma = D == 64;
  static constexpr int kDqStageBytes = kDqTma ? kBwBQ * D * 4 : 0;
  // dS tiles: two at D = 64, where step i+1's elementwise work writes dS
  // while step i's dQ MMA may still read it; one at D = 128, where dQ of
  // step i completes before step i+1's scores exist.
  static constexpr int kDsBuffers = D == 64 ? 2 : 1;
  static constexpr int kNeeded =
      (2 + 2 * kStages) * kTile + kDsBuffers * kDsBytes + kDqStageBytes + 2 * kStages * kVecBytes + 256;
  // Room to align the tiles to 1024 bytes where it fits; at D = 128 the tiles
  // fill the 227 KB limit, and the kernel checks that its base is aligned.
  static constexpr int kSmemBytes = kNeeded + 1024 <= 232448 ? kNeeded + 1024 : 232448;
  static constexpr int kColDP = 128;
  static constexpr int kColDV = 256;
  static constexpr int kColDK = 256 + D;
  // dQ (128 queries x D): its own columns at D = 64; at D = 128 TMEM is full
  // (S^T, dP^T, dV, dK), so dQ takes the upper halves of the S^T and dP^T
  // columns, which are free once P^T / dS^T (16-bit) sit in the lower halves.
  static constexpr bool kDqInScores = D > 64;
  // Where the 16-bit P^T (in the S^T columns) and dS^T (in the dP^T columns)
  // of queries 64*half .. +63 go, relative to the region's first column:
  //  * D = 64: over the first 32 columns of the half's own 64 scores, so a
  //    warp never writes columns that the other half still has to read; the
  //    A operand is then two 32-column pieces (query steps kk < 4 and >= 4).
  //  * D = 128: contiguous over the first 64 columns (the upper 64 hold dQ).
  static constexpr bool kOwnRegion = !kDqInScores;
  __host__ __device__ static constexpr int p_col(int half) { return kOwnRegion ? 64 * half : 32 * half; }
  // TMEM column of the A operand for query step kk (16 queries = 8 columns).
  __host__ __device__ static constexpr int a_col(int kk) { return p_col(kk >> 2) + (kk & 3) * 8; }
  __host__ __device__ static constexpr int dq_col(int chunk64) {
    return kDqInScores ? (chunk64 == 0 ? 64 : 192) : 256 + 2 * D + 64 * chunk64;
  }
  static_assert(kDqInScores || 256 + 3 * D <= 512, "TMEM columns");
};

__device__ __forceinline__ float bw_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool F16>
__device__ __forceinline__ uint32_t bw_pack(float a, float b) {
  if constexpr (F16) return pack_f16(a, b);
  else return pack_bf16(a, b);
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

struct TcBwdArgs {
  const float* lse;    // [B, H, Sq], natural log
  const float* delta;  // [B, H, Sq]
  float* dq_acc;       // [B, Sq, H, D] fp32
  uint16_t* dk;
  uint16_t* dv;
  int B, H, Sq, Sk;
  long long dk_ld, dk_bs, dv_ld, dv_bs;
  float scale, scale_log2;
  int* status;
  int debug;         // diagnostics: bit 0 skips the dQ reductions, bit 1 the elementwise math
  long long* trace;  // diagnostics: clock64 stamps of CTA (0, 0) when non-null
};

// Trace slots: [0] entry, [1] after setup, then per step s (< 10, counted over
// the CTA's work items) 16 slots at 8 + 16 s:
// +0 MMA q_full ok, +1 S/dP issued, +2 p_ready seen, +3 dV/dK issued, +4 dQ issued,
// +5 elementwise sdp_full seen, +6 elementwise arrived, +7 dQ warp dq_full seen, +8 dQ warp done,
// +9 producer staged LSE / delta (TMA already issued), +10..+14 elementwise
// chunk 0 loaded, chunk 0 stored, chunk 1 loaded, chunk 1 stored, fences done.
constexpr int kBwTraceSlots = 168;
__device__ __forceinline__ void bw_stamp(const TcBwdArgs& a, int slot) {
  if (a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && slot < kBwTraceSlots) a.trace[slot] = clock64();
}

// Work item `idx` of a persistent CTA: one 128-key block of one (batch,
// head). Items are ordered key block first, so under causal masking the
// blocks with the most query blocks come first and the static round-robin
// assignment over CTAs stays balanced.
struct BwItem {
  int b, h, bh, k0, i_start, n_steps;
};

template <bool CAUSAL>
__device__ __forceinline__ BwItem bw_item(int idx, int H, int BH, int Sq) {
  BwItem it;
  const int j = idx / BH;
  it.bh = idx - j * BH;
  it.b = it.bh / H;
  it.h = it.bh - it.b * H;
  it.k0 = j * kBwBK;
  const int nq = (Sq + kBwBQ - 1) / kBwBQ;
  it.i_start = CAUSAL ? min(nq, it.k0 / kBwBQ) : 0;
  it.n_steps = nq - it.i_start;
  return it;
}

template <int D, bool CAUSAL, bool F16>
__global__ void __launch_bounds__(kBwThreads, 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                        const __grid_constant__ CUtensorMap tdq, const TcBwdArgs a) {
  using Cfg = TcBwdCfg<D>;
  constexpr int ST = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  {
    uint32_t dsz;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dsz));
    if ((uint32_t)(smem - smem_raw) + Cfg::kNeeded > dsz) {
      if (threadIdx.x == 0) record_status(a.status, kStatusBadArgs);
      return;
    }
  }
  uint8_t* sK = smem;
  uint8_t* sV = sK + Cfg::kTile;
  uint8_t* sQ = sV + Cfg::kTile;              // [ST]
  uint8_t* sDO = sQ + ST * Cfg::kTile;        // [ST]
  uint8_t* sDS = sDO + ST * Cfg::kTile;       // dS, MN-major (queries contiguous), two 64-query chunks
  uint8_t* sDQ = sDS + Cfg::kDsBuffers * Cfg::kDsBytes;  // fp32 dQ staging tile (D = 64)
  float* sLse = reinterpret_cast<float*>(sDQ + Cfg::kDqStageBytes);  // [ST][128] LSE (natural log)
  float* sDelta = sLse + ST * kBwBQ;                                   // [ST][128] delta
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDelta + ST * kBwBQ);
  uint64_t* kv_full = bars;           // K_j, V_j loaded
  uint64_t* kv_empty = kv_full + 1;   // every MMA of the item is done (K / V smem free)
  uint64_t* q_full = kv_empty + 1;    // [ST]: TMA arming + 32 lanes' LSE / delta copies
  uint64_t* q_empty = q_full + ST;    // [ST]
  uint64_t* sdp_full = q_empty + ST;  // S^T and dP^T are in TMEM
  uint64_t* p_ready = sdp_full + 1;   // P^T, dS^T written (8 warps)
  uint64_t* dq_full = p_ready + 1;    // dQ_i is in TMEM
  uint64_t* dq_empty = dq_full + 1;   // dQ_i read out (4 warps)
  uint64_t* kv_done = dq_empty + 1;   // dK, dV of the item final
  uint64_t* kvo_empty = kv_done + 1;  // dK, dV read out of TMEM (8 warps)
  uint64_t* drain = kvo_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) bw_stamp(a, 0);
  const int BH = a.B * a.H;
  const int n_items = ((a.Sk + kBwBK - 1) / kBwBK) * BH;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&q_full[s], 33);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(sdp_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    mbar_init(kv_done, 1);
    mbar_init(kvo_empty, 8);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    tma_prefetch_desc(&tdo);
    if (Cfg::kDqTma) tma_prefetch_desc(&tdq);
  }
  if (warp == 1) tmem_alloc(tmem_holder, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  if (threadIdx.x == 0) bw_stamp(a, 1);

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(BwRegs<D>::kCtl));
    if (warp == 0) {
      // ---------------------------------------------------------------- producer (whole warp)
      uint32_t armed = 0, armed_par = 0, kv_armed = 0, kv_par = 0;
      bool ok = true;
      int step = 0, n_it = 0;
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ++n_it) {
        const BwItem it = bw_item<CAUSAL>(idx, a.H, BH, a.Sq);
        if (!mbar_wait(kv_empty, (n_it & 1) ^ 1, abort_flag, a.status, kStatusTimeoutProducer)) ok = false;
        if (!__all_sync(0xffffffffu, ok)) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(kv_full, 2 * Cfg::kTile);
          kv_armed = 1;
          kv_par = n_it & 1;
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            tma_load_4d(&tk, kv_full, sK + c * (kBwBK * 128), 64 * c, it.k0, it.h, it.b);
            tma_load_4d(&tv, kv_full, sV + c * (kBwBK * 128), 64 * c, it.k0, it.h, it.b);
          }
        }
        for (int st_i = 0; st_i < it.n_steps; ++st_i, ++step) {
          const int st = step % ST;
          const uint32_t ph = (step / ST) & 1;
          if (!mbar_wait(&q_empty[st], ph ^ 1, abort_flag, a.status, kStatusTimeoutProducer)) ok = false;
          if (!__all_sync(0xffffffffu, ok)) break;
          const int q0 = (it.i_start + st_i) * kBwBQ;
          // q_full takes 33 arrivals: the TMA arming by lane 0 and one
          // asynchronous arrival per lane when its LSE / delta copies land.
          if (lane == 0) {
            mbar_arrive_expect_tx(&q_full[st], 2 * Cfg::kTile);
            armed |= 1u << st;
            armed_par = (armed_par & ~(1u << st)) | (ph << st);
#pragma unroll
            for (int c = 0; c < D / 64; ++c) {
              tma_load_4d(&tq, &q_full[st], sQ + st * Cfg::kTile + c * (kBwBQ * 128), 64 * c, q0, it.h, it.b);
              tma_load_4d(&tdo, &q_full[st], sDO + st * Cfg::kTile + c * (kBwBQ * 128), 64 * c, q0, it.h, it.b);
            }
          }
          // LSE and delta of the block by asynchronous 4-byte copies (zero past
          // Sq; those queries are masked), each lane's copies tracked by q_full.
          const long long vbase = (long long)it.bh * a.Sq;
#pragma unroll
          for (int t = lane; t < kBwBQ; t += 32) {
            const int q = q0 + t;
            const bool in = q < a.Sq;
            const long long gi = vbase + (in ? q : 0);
            cp_async_4_zfill(&sLse[st * kBwBQ + t], a.lse + gi, in);
            cp_async_4_zfill(&sDelta[st * kBwBQ + t], a.delta + gi, in);
          }
          cp_async_mbar_arrive_noinc(&q_full[st]);
          if (lane == 0) bw_stamp(a, 8 + 16 * step + 9);
        }
      }
      if (lane == 0) {
        // Every issued copy must land before the CTA may exit (the last arming
        // of each barrier is its newest phase).
        volatile int never = 0;
        if (kv_armed) mbar_wait(kv_full, kv_par, &never, a.status, kStatusTimeoutDrain);
        for (int s = 0; s < ST; ++s)
          if (armed & (1u << s))
            if (!mbar_wait(&q_full[s], (armed_par >> s) & 1u, &never, a.status, kStatusTimeoutDrain)) break;
      }
    } else if (warp == 1 && lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc_t = idesc_f16(kBwBK, kBwBQ, F16, false, false);  // S^T, dP^T
      constexpr uint32_t idesc_kv = idesc_f16(kBwBK, D, F16, false, true);      // dV, dK (B MN-major)
      constexpr uint32_t idesc_q = idesc_f16(kBwBQ, 64, F16, true, true);       // dQ, per 64 columns (A, B MN-major)
      bool ok = true, issued = false;
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      int step = 0, n_it = 0;
      // S^T and dP^T of `stp` (a step of the current item) into TMEM.
      auto issue_sdp = [&](int stp) -> bool {
        const int st = stp % ST;
        if (!mbar_wait(&q_full[st], (stp / ST) & 1, abort_flag, a.status, kStatusTimeoutMma)) return false;
        // dQ of the previous step lives in the score columns at D = 128: it
        // must be read out before S^T / dP^T overwrite them.
        if (Cfg::kDqInScores && !mbar_wait(dq_empty, (stp & 1) ^ 1, abort_flag, a.status, kStatusTimeoutMma))
          return false;
        tc_fence_after();
        bw_stamp(a, 8 + 16 * stp);
        const uint32_t q_addr = smem_u32(sQ + st * Cfg::kTile), do_addr = smem_u32(sDO + st * Cfg::kTile);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem, sw128_desc(k_addr + off, 16, 1024), sw128_desc(q_addr + off, 16, 1024), idesc_t,
                      kk != 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (128 * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + Cfg::kColDP, sw128_desc(v_addr + off, 16, 1024), sw128_desc(do_addr + off, 16, 1024),
                      idesc_t, kk != 0 ? 1u : 0u);
        }
        umma_commit(sdp_full);
        bw_stamp(a, 8 + 16 * stp + 1);
        issued = true;
        return true;
      };
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ++n_it) {
        const BwItem it = bw_item<CAUSAL>(idx, a.H, BH, a.Sq);
        if (!mbar_wait(kv_full, n_it & 1, abort_flag, a.status, kStatusTimeoutMma) || !issue_sdp(step)) {
          ok = false;
          break;
        }
        for (int st_i = 0; st_i < it.n_steps && ok; ++st_i, ++step) {
          const int st = step % ST;
          const bool more = st_i + 1 < it.n_steps;
          if (!mbar_wait(p_ready, step & 1, abort_flag, a.status, kStatusTimeoutMma) ||
              (st_i == 0 && !mbar_wait(kvo_empty, (n_it & 1) ^ 1, abort_flag, a.status, kStatusTimeoutMma))) {
            ok = false;
            break;
          }
          bw_stamp(a, 8 + 16 * step + 2);
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sQ + st * Cfg::kTile), do_addr = smem_u32(sDO + st * Cfg::kTile);
          const uint32_t ds_addr = smem_u32(sDS + (Cfg::kDsBuffers == 2 ? (step & 1) * Cfg::kDsBytes : 0));
          auto issue_dq = [&]() {
#pragma unroll
            for (int h2 = 0; h2 < D / 64; ++h2)
#pragma unroll
              for (int kk = 0; kk < kBwBK / 16; ++kk)
                umma_f16_ss(tmem + Cfg::dq_col(h2), sw128_desc(ds_addr + kk * 2048, 128 * 128, 1024),
                            sw128_desc(k_addr + h2 * (128 * 128) + kk * 2048, 128 * 128, 1024), idesc_q,
                            kk != 0 ? 1u : 0u);
            umma_commit(dq_full);
            bw_stamp(a, 8 + 16 * step + 4);
          };
          // D = 128: dQ goes first; its commit covers only the dQ MMAs, so the
          // dQ warps read it out while the tensor cores run dV / dK, and the
          // next step's scores (which reuse dQ's columns) are not held up by
          // the readout.
          if (Cfg::kDqInScores) issue_dq();
#pragma unroll
          for (int kk = 0; kk < kBwBQ / 16; ++kk) {
            const uint32_t acc = (st_i | kk) != 0 ? 1u : 0u;
            umma_f16_ts(tmem + Cfg::kColDV, tmem + Cfg::a_col(kk), sw128_desc(do_addr + kk * 2048, 128 * 128, 1024),
                        idesc_kv, acc);
            umma_f16_ts(tmem + Cfg::kColDK, tmem + Cfg::kColDP + Cfg::a_col(kk),
                        sw128_desc(q_addr + kk * 2048, 128 * 128, 1024), idesc_kv, acc);
          }
          bw_stamp(a, 8 + 16 * step + 3);
          // D = 64: the next step's scores go ahead of this step's dQ (which
          // reads only shared memory), so its elementwise work overlaps dQ.
          if (!Cfg::kDqInScores && more && !issue_sdp(step + 1)) {
            ok = false;
            break;
          }
          if (!Cfg::kDqInScores) {
            if (!mbar_wait(dq_empty, (step & 1) ^ 1, abort_flag, a.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_dq();
          }
          umma_commit(&q_empty[st]);
          if (Cfg::kDqInScores && more && !issue_sdp(step + 1)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
        umma_commit(kv_done);
        umma_commit(kv_empty);
      }
      if (issued) {
        umma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, a.status, kStatusTimeoutDrain);
      }
      if (!ok) *abort_flag = 1;
    }
    tc_fence_before();
    named_bar_sync(1, kBwThreads);
    if (warp == 1) tmem_dealloc(tmem, 512);
  } else if (warp < 12) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(BwRegs<D>::kMath));
    // ---------------------------------------------------------------- elementwise + dK / dV epilogue
    // Thread = one key row (TMEM lane); warps 4..7 take queries 0..63 of the
    // block, warps 8..11 queries 64..127.
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;
    const int kr = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off, t_dp = tmem + lane_off + Cfg::kColDP;
    bool ok = true;
    int step = 0, n_it = 0;
    for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ++n_it) {
      const BwItem it = bw_item<CAUSAL>(idx, a.H, BH, a.Sq);
      const int kg = it.k0 + kr;
      for (int st_i = 0; st_i < it.n_steps; ++st_i, ++step) {
        const int st = step % ST;
        const bool got = mbar_wait(&q_full[st], (step / ST) & 1, abort_flag, a.status, kStatusTimeoutEpilogue) &&
                         mbar_wait(sdp_full, step & 1, abort_flag, a.status, kStatusTimeoutEpilogue);
        if (Cfg::kOwnRegion && !got) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (threadIdx.x == 128) bw_stamp(a, 8 + 16 * step + 5);
        const int q0 = (it.i_start + st_i) * kBwBQ + 64 * half;  // first query of this warp's columns
        // Masked: queries before the key (causal) and queries past Sq.
        const bool need_mask = (CAUSAL && q0 < it.k0 + kBwBK - 1) || q0 + 64 > a.Sq;
        const float* ls = sLse + st * kBwBQ + 64 * half;
        const float* dl_s = sDelta + st * kBwBQ + 64 * half;
        if (!Cfg::kOwnRegion && (a.debug & 2) && !got) {
          ok = false;
          break;
        }
        if (!(a.debug & 2)) {
          // Scores of this warp's 64 queries: at D = 64 in two 32-column
          // chunks, each thread writing P / dS over its own region (see
          // Cfg::p_col); at D = 128 all 64 at once, then the two warps of the
          // row quarter meet before either writes, since P / dS of queries
          // 64..127 land over scores of queries 32..63.
          uint32_t sv[64], dv[64];
          if constexpr (!Cfg::kOwnRegion) {
            if (got) {
              tmem_ld_32x32b_x64(t_s + 64 * half, sv);
              tmem_ld_32x32b_x64(t_dp + 64 * half, dv);
              tmem_wait_ld_dep64(sv);
              tmem_wait_ld_dep64(dv);
            }
            // Both warps of the quarter reach this barrier whether or not
            // their waits succeeded; a failed wait has raised the abort flag
            // before it, so both leave together.
            named_bar_sync(3 + quarter, 64);
            if (!got || *abort_flag) {
              ok = false;
              break;
            }
          }
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            if constexpr (Cfg::kOwnRegion) {
              tmem_ld_32x32b_x32(t_s + 64 * half + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sv[32 * c]));
              tmem_ld_32x32b_x32(t_dp + 64 * half + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&dv[32 * c]));
              tmem_wait_ld_dep(*reinterpret_cast<uint32_t(*)[32]>(&sv[32 * c]));
              tmem_wait_ld_dep(*reinterpret_cast<uint32_t(*)[32]>(&dv[32 * c]));
              if (threadIdx.x == 128) bw_stamp(a, 8 + 16 * step + 10 + 2 * c);
            }
            uint32_t pk[16], dk[16];
#pragma unroll
            for (int t = 0; t < 32; t += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(ls + 32 * c + t);
              const float4 d4 = *reinterpret_cast<const float4*>(dl_s + 32 * c + t);
              const float2 nlog2 = make_float2(-1.4426950408889634f, -1.4426950408889634f);
              const float2 sc2 = make_float2(a.scale_log2, a.scale_log2);
              float2 p[2], ds[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float2 l2 = mul2(e == 0 ? make_float2(l4.x, l4.y) : make_float2(l4.z, l4.w), nlog2);
                const float2 x = fma2(make_float2(__uint_as_float(sv[32 * c + t + 2 * e]),
                                                  __uint_as_float(sv[32 * c + t + 2 * e + 1])),
                                      sc2, l2);
                p[e] = make_float2(bw_ex2(x.x), bw_ex2(x.y));
                if (need_mask) {
                  const int q = q0 + 32 * c + t + 2 * e;
                  if (q >= a.Sq || (CAUSAL && q < kg)) p[e].x = 0.f;
                  if (q + 1 >= a.Sq || (CAUSAL && q + 1 < kg)) p[e].y = 0.f;
                }
                const float2 nd2 = e == 0 ? make_float2(-d4.x, -d4.y) : make_float2(-d4.z, -d4.w);
                ds[e] = mul2(p[e], add2(make_float2(__uint_as_float(dv[32 * c + t + 2 * e]),
                                                    __uint_as_float(dv[32 * c + t + 2 * e + 1])),
                                        nd2));
              }
              pk[t / 2] = bw_pack<F16>(p[0].x, p[0].y);
              pk[t / 2 + 1] = bw_pack<F16>(p[1].x, p[1].y);
              dk[t / 2] = bw_pack<F16>(ds[0].x, ds[0].y);
              dk[t / 2 + 1] = bw_pack<F16>(ds[1].x, ds[1].y);
            }
            tmem_st_32x32b_x16(t_s + Cfg::p_col(half) + 16 * c, pk);
            tmem_st_32x32b_x16(t_dp + Cfg::p_col(half) + 16 * c, dk);
            // dS row kr, queries 64*half + 32c .. +31: MN-major 128-byte swizzled
            // rows of 64 queries, 16-byte units XOR-ed with the row's low bits.
            uint8_t* row = sDS + (Cfg::kDsBuffers == 2 ? (step & 1) * Cfg::kDsBytes : 0) + half * (kBwBK * 128) +
                           kr * 128;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int unit = (c * 4 + u) ^ (kr & 7);
              *reinterpret_cast<uint4*>(row + unit * 16) =
                  make_uint4(dk[4 * u], dk[4 * u + 1], dk[4 * u + 2], dk[4 * u + 3]);
            }
            if (threadIdx.x == 128) bw_stamp(a, 8 + 16 * step + 11 + 2 * c);
          }
        }
        fence_proxy_async_smem();
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (threadIdx.x == 128) bw_stamp(a, 8 + 16 * step + 14);
        if (lane == 0) mbar_arrive(p_ready);
        if (threadIdx.x == 128) bw_stamp(a, 8 + 16 * step + 6);
      }
      // dK, dV rows of this key: this warp writes columns [D/2 * half, D/2 * (half + 1)).
      if (!ok || !mbar_wait(kv_done, n_it & 1, abort_flag, a.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint16_t* dkr = a.dk + (long long)it.b * a.dk_bs + (long long)kg * a.dk_ld + (long long)it.h * D;
      uint16_t* dvr = a.dv + (long long)it.b * a.dv_bs + (long long)kg * a.dv_ld + (long long)it.h * D;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        uint16_t* outr = which == 0 ? dkr : dvr;
        const float mul = which == 0 ? a.scale : 1.f;
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          const int col = (D / 2) * half + 32 * c;
          uint32_t ov[32];
          tmem_ld_32x32b_x32(tmem + lane_off + (which == 0 ? Cfg::kColDK : Cfg::kColDV) + col, ov);
          tmem_wait_ld_dep(ov);
          if (kg < a.Sk) {
#pragma unroll
            for (int d = 0; d < 32; d += 8) {
              uint4 w;
              w.x = bw_pack<F16>(__uint_as_float(ov[d]) * mul, __uint_as_float(ov[d + 1]) * mul);
              w.y = bw_pack<F16>(__uint_as_float(ov[d + 2]) * mul, __uint_as_float(ov[d + 3]) * mul);
              w.z = bw_pack<F16>(__uint_as_float(ov[d + 4]) * mul, __uint_as_float(ov[d + 5]) * mul);
              w.w = bw_pack<F16>(__uint_as_float(ov[d + 6]) * mul, __uint_as_float(ov[d + 7]) * mul);
              *reinterpret_cast<uint4*>(outr + col + d) = w;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(kvo_empty);
    }
    if (!ok) *abort_flag = 1;
    tc_fence_before();
    named_bar_sync(1, kBwThreads);
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(BwRegs<D>::kDq));
    // ---------------------------------------------------------------- dQ readout (one query row per thread)
    const int quarter = warp & 3;
    const int qr = quarter * 32 + lane;
    const bool leader = warp == 12 && lane == 0;
    const uint32_t t_dq = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    bool ok = true;
    int step = 0, n_it = 0;
    for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ++n_it) {
      const BwItem it = bw_item<CAUSAL>(idx, a.H, BH, a.Sq);
      for (int st_i = 0; st_i < it.n_steps; ++st_i, ++step) {
        const bool got = mbar_wait(dq_full, step & 1, abort_flag, a.status, kStatusTimeoutEpilogue);
        if (!Cfg::kDqTma && !got) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (threadIdx.x == 384) bw_stamp(a, 8 + 16 * step + 7);
        const int qb0 = (it.i_start + st_i) * kBwBQ;
        const int qg = qb0 + qr;
        if constexpr (Cfg::kDqTma) {
          // The staging tile was last read by the reduction of the previous
          // step. All four warps reach the barrier whether or not their wait
          // succeeded; a failed wait raised the abort flag before it.
          if (leader) bulk_wait_read<0>();
          named_bar_sync(2, 128);
          if (!got || *abort_flag) {
            ok = false;
            break;
          }
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_dq + Cfg::dq_col(c >> 1) + 32 * (c & 1), v);
            tmem_wait_ld_dep(v);
            uint8_t* row = sDQ + c * (kBwBQ * 128) + qr * 128;
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              *reinterpret_cast<float4*>(row + ((u ^ (qr & 7)) * 16)) =
                  make_float4(__uint_as_float(v[4 * u]) * a.scale, __uint_as_float(v[4 * u + 1]) * a.scale,
                              __uint_as_float(v[4 * u + 2]) * a.scale, __uint_as_float(v[4 * u + 3]) * a.scale);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dq_empty);
          fence_proxy_async_smem();
          named_bar_sync(2, 128);
          if (leader && !(a.debug & 1)) {
#pragma unroll
            for (int c = 0; c < D / 32; ++c)
              tma_reduce_add_4d(&tdq, sDQ + c * (kBwBQ * 128), 32 * c, qb0, it.h, it.b);
            bulk_commit();
          }
        } else {
          float* dst = a.dq_acc + (((long long)it.b * a.Sq + qg) * a.H + it.h) * D;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_dq + Cfg::dq_col(c >> 1) + 32 * (c & 1), v);
            tmem_wait_ld_dep(v);
            if (qg < a.Sq && !(a.debug & 1)) {
#pragma unroll
              for (int d = 0; d < 32; d += 4)
                red_add_v4(dst + 32 * c + d, __uint_as_float(v[d]) * a.scale, __uint_as_float(v[d + 1]) * a.scale,
                           __uint_as_float(v[d + 2]) * a.scale, __uint_as_float(v[d + 3]) * a.scale);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dq_empty);
        }
        if (threadIdx.x == 384) bw_stamp(a, 8 + 16 * step + 8);
      }
    }
    if (Cfg::kDqTma && leader) bulk_wait_all();
    if (!ok) *abort_flag = 1;
    tc_fence_before();
    named_bar_sync(1, kBwThreads);
  }
}

// 4-D view {D, S, H, B} of a [B, S, H, D] tensor, 128-row x 64-column boxes.
CUtensorMap bw_bshd_map(const at::Tensor& t) {
  const int64_t es = 2;
  uint64_t dims[4] = {(uint64_t)t.size(3), (uint64_t)t.size(1), (uint64_t)t.size(2), (uint64_t)t.size(0)};
  uint64_t strides[3] = {(uint64_t)(t.stride(1) * es), (uint64_t)(t.stride(2) * es), (uint64_t)(t.stride(0) * es)};
  uint32_t box[4] = {64, 128, 1, 1};
  return make_tma(t.data_ptr(), t.scalar_type(), 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D, bool CAUSAL, bool F16>
void launch_bwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& dout,
                   const at::Tensor& lse, const float* delta, float* dq_acc, at::Tensor& dk, at::Tensor& dv,
                   float scale, cudaStream_t s) {
  using Cfg = TcBwdCfg<D>;
  const int B = (int)q.size(0), Sq = (int)q.size(1), H = (int)q.size(2), Sk = (int)k.size(1);
  const CUtensorMap tq = bw_bshd_map(q), tk = bw_bshd_map(k), tv = bw_bshd_map(v), tdo = bw_bshd_map(dout);
  // fp32 dQ accumulator [B, Sq, H, D] as {D, Sq, H, B}, 32 x 128 boxes, 128-byte swizzle.
  CUtensorMap tdq;
  std::memset(&tdq, 0, sizeof(tdq));
  if (Cfg::kDqTma) {
    uint64_t dims[4] = {(uint64_t)D, (uint64_t)Sq, (uint64_t)H, (uint64_t)B};
    uint64_t strides[3] = {(uint64_t)H * D * 4, (uint64_t)D * 4, (uint64_t)Sq * H * D * 4};
    uint32_t box[4] = {32, 128, 1, 1};
    tdq = make_tma(dq_acc, at::kFloat, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  TcBwdArgs args;
  args.lse = lse.data_ptr<float>();
  args.delta = delta;
  args.dq_acc = dq_acc;
  args.dk = (uint16_t*)dk.data_ptr();
  args.dv = (uint16_t*)dv.data_ptr();
  args.B = B;
  args.H = H;
  args.Sq = Sq;
  args.Sk = Sk;
  args.dk_ld = dk.stride(1);
  args.dk_bs = dk.stride(0);
  args.dv_ld = dv.stride(1);
  args.dv_bs = dv.stride(0);
  args.scale = scale;
  args.scale_log2 = scale * 1.4426950408889634f;
  args.status = device_status_ptr(q.get_device());
  args.debug = g_attn_bwd_debug;
  args.trace = g_attn_bwd_trace;
  auto kern = flash_bwd_tc_kernel<D, CAUSAL, F16>;
  static bool set = false;
  if (!set) {
    KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    set = true;
  }
  const long long items = (long long)((Sk + kBwBK - 1) / kBwBK) * B * H;
  const int grid = (int)std::min<long long>(items, compute_sms(q.get_device()));
  kern<<<grid, kBwThreads, Cfg::kSmemBytes, s>>>(tq, tk, tv, tdo, tdq, args);
  KB_LAUNCHED();
}

}  // namespace

// Runs the tcgen05 backward (dQ accumulated into `dq_acc`, dK and dV written)
// when the shape allows it; returns false otherwise.
bool flash_attention_backward_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                 const at::Tensor& dout, const at::Tensor& lse, const float* delta, float* dq_acc,
                                 at::Tensor& dk, at::Tensor& dv, double scale, bool causal, cudaStream_t s) {
  const int64_t D = q.size(3);
  if (D != 64 && D != 128) return false;
  if (k.size(1) > INT32_MAX / 2 || q.size(1) > INT32_MAX / 2) return false;
  if (q.size(1) == 0 || k.size(1) == 0 || q.size(0) * q.size(2) == 0) return false;
  const bool f16 = q.scalar_type() == at::kHalf;
  const float sc = (float)scale;
#define KB_BTC(DD, CC, FF) launch_bwd_tc<DD, CC, FF>(q, k, v, dout, lse, delta, dq_acc, dk, dv, sc, s)
  if (D == 64) {
    if (causal) { if (f16) KB_BTC(64, true, true); else KB_BTC(64, true, false); }
    else { if (f16) KB_BTC(64, false, true); else KB_BTC(64, false, false); }
  } else {
    if (causal) { if (f16) KB_BTC(128, true, true); else KB_BTC(128, true, false); }
    else { if (f16) KB_BTC(128, false, true); else KB_BTC(128, false, false); }
  }
#undef KB_BTC
  return true;
}

}  // namespace kb
