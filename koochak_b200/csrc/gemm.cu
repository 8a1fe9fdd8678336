// Persistent, warp-specialised tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[b] = epilogue( alpha * A[b] . B[b]^T )        (A: M x K, B: N x K logically)
//
// Each operand is given either K-major (K contiguous) or MN-major (M or N
// contiguous), so forward (x W^T), data-gradient (dy W) and weight-gradient
// (dy^T x) products, and the Newton-Schulz products of the Muon optimizer,
// all run without a transpose copy.
//
// Roles inside one CTA (320 threads, one CTA per SM, grid = #SMs):
//   warp 0      TMA producer: 128-byte-swizzled tiles into a STAGES-deep ring
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue: two warps per TMEM lane quarter, each taking half the
//               columns; tcgen05.ld double-buffered against the math and stores
// The fp32 accumulator is double-buffered in TMEM (2 x BN columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// Epilogue, in order:  v = alpha*acc (+ bias[n])
//   ACT_GELU      : aux = bf16(v); v = gelu_tanh(v)
//   ACT_GELU_BWD  : v = v * gelu_tanh'(D[m,n])           (D = saved pre-activation)
//   otherwise     : v = v + beta * D[m,n]                 (residual add / accumulate)
//   C[m,n] = v  (bf16, fp16 or fp32)
//
// There is no TMA multicast here: every CTA loads its own tiles.
#include "host_utils.h"
#include "sm100.cuh"

#include <torch/extension.h>

#include <cstring>
#include <type_traits>

namespace kb {

enum GemmAct : int { ACT_NONE = 0, ACT_GELU = 1, ACT_GELU_BWD = 2 };

struct GemmParams {
  int M, N, K, batch;
  int a_mn_major, b_mn_major;
  int fp16_inputs;
  void* C;
  long long ldc, strideC;
  const void* D;
  long long ldd, strideD;
  float alpha, beta;
  const float* bias;
  void* aux;
  long long ldaux, strideAux;
  int vec_ok;  // C/D/aux rows 16-byte aligned for vector access
  int splits;  // split-K factor; > 1 means fp32 C is accumulated with atomics
  int kb_per_split;  // 64-wide K blocks per split (every split non-empty)
  int tma_store;     // epilogue writes C (and aux) through staged TMA stores
  int stream_k;      // K-iterations of all tiles split evenly over the workers (fp32 atomics)
  int group_n;       // tile order: > 1 takes the tile columns group_n at a time (see tile_mn)
  int sym;           // symmetric output (M == N): only tiles touching the upper triangle, mirrored
  int* status;
  // Optional pipeline profile (null: off). Per CTA, 8 counters of clock64
  // cycles: [0] producer waiting for a free stage, [1] MMA waiting for
  // operands, [2] MMA waiting for a free accumulator, [3] epilogue warps
  // waiting for a full accumulator (summed over warps), [4] producer role
  // total, [5] tiles issued by the MMA thread.
  unsigned long long* prof;
  // Extents (elements from the base pointer) of C, D and aux that a
  // KB_DEBUG_BOUNDS build checks every epilogue tile against.
  long long dbg_c_extent, dbg_d_extent, dbg_aux_extent;
  // Diagnostic modes (0 in normal use): bit 0 skips the operand loads (MMAs
  // read whatever the ring holds), bit 1 skips the epilogue's math and
  // stores, bit 2 keeps only the epilogue's TMEM loads (32 columns each; with
  // bit 3: 16, with bit 4: 64). Results are meaningless; only the timing is
  // of interest.
  int debug;
};

// KB_DEBUG_BOUNDS: the last element of rows [row0, row0 + 32) x columns
// [col0, col1) of batch b, clipped to M x N, must lie inside C (and D, aux).
__device__ __forceinline__ bool debug_tile_ok(const GemmParams& p, int b, int row0, int col0, int col1) {
  if constexpr (!kDebugBounds) {
    return true;
  } else {
    const int r1 = min(row0 + 32, p.M), c1 = min(col1, p.N);
    if (row0 >= r1 || col0 >= c1) return true;  // nothing of this slice is written
    const long long r = r1 - 1, c = c1 - 1;
    bool ok = debug_bounds_ok(p.status, kSiteGemmC, (long long)b * p.strideC + r * p.ldc + c, p.dbg_c_extent);
    if (p.D != nullptr)
      ok = ok && debug_bounds_ok(p.status, kSiteGemmD, (long long)b * p.strideD + r * p.ldd + c, p.dbg_d_extent);
    if (p.aux != nullptr)
      ok = ok && debug_bounds_ok(p.status, kSiteGemmAux, (long long)b * p.strideAux + r * p.ldaux + c,
                                 p.dbg_aux_extent);
    return ok;
  }
}

// Bulk reduce-add of a staged 3-D tile into global memory (fp32 add, per element).
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ bool prof_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                          int code, bool on, long long& acc) {
  if (!on) return mbar_wait(bar, parity, abort_flag, status, code);
  const long long t0 = clock64();
  const bool ok = mbar_wait(bar, parity, abort_flag, status, code);
  acc += clock64() - t0;
  return ok;
}

__device__ __forceinline__ void prof_add(const GemmParams& p, int idx, long long v) {
  if (p.prof) atomicAdd(p.prof + blockIdx.x * 8 + idx, (unsigned long long)v);
}

// Work unit k of worker w (a CTA, or a CTA pair) out of nw: output tile t and
// the K-block range [kb0, kb1) it covers. Without stream-K a unit is one tile
// (or one split of it); with stream-K the K-iterations of all tiles are cut
// into nw equal contiguous ranges, so a worker may finish one tile and start
// the next, and every partial tile is added into C with fp32 atomics.
__device__ __forceinline__ bool work_unit(const GemmParams& p, int w, int nw, int k, int total_tiles,
                                          int tiles_per_split, int num_kb, int& t, int& kb0, int& kb1) {
  if (!p.stream_k) {
    t = w + k * nw;
    if (t >= total_tiles) return false;
    const int split = t / tiles_per_split;
    kb0 = split * p.kb_per_split;
    kb1 = min(num_kb, kb0 + p.kb_per_split);
    return true;
  }
  const long long iters = (long long)total_tiles * num_kb;
  const long long begin = iters * w / nw, end = iters * (w + 1) / nw;
  const long long first = begin / num_kb;
  const long long start = (k == 0) ? begin : (first + k) * num_kb;
  if (start >= end) return false;
  t = (int)(first + k);
  kb0 = (int)(start - (long long)t * num_kb);
  kb1 = (int)min((long long)num_kb, end - (long long)t * num_kb);
  return true;
}

// Symmetric products (X X^T, and A A or b A + c A A with A symmetric) compute
// only the tiles that hold an element on or above the diagonal: in tile
// column n_blk the first sym_rows(n_blk) row blocks. The epilogue writes each
// such tile and, for its elements with column > row, the mirrored element.
__device__ __forceinline__ int sym_rows(int n_blk, int num_m, int bm, int bn) {
  return min(num_m, (n_blk * bn + bn - 1) / bm + 1);
}

__device__ __forceinline__ int tiles_in_batch(const GemmParams& p, int num_m, int num_n, int bm, int bn) {
  if (!p.sym) return num_m * num_n;
  int t = 0;
  for (int n = 0; n < num_n; ++n) t += sym_rows(n, num_m, bm, bn);
  return t;
}

// Output tile r of one batch as (m_blk, n_blk). Plain order: row blocks run
// fastest down each tile column, so the tiles in flight together span few
// columns and many row blocks (every A panel, few B panels). With group_n = G
// the columns are taken G at a time and, inside a group, the G tiles of one
// row block are consecutive: the tiles in flight then cover a patch about
// (workers / G) x G, and read about that many A plus G B panels -- for long K
// (weight gradients) that is what decides whether the panels stay in L2.
__device__ __forceinline__ void tile_mn(const GemmParams& p, int r, int num_m, int num_n, int bm, int bn, int& m_blk,
                                        int& n_blk) {
  if (p.sym) {
    int n = 0;
    for (;; ++n) {
      const int c = sym_rows(n, num_m, bm, bn);
      if (r < c || n == num_n - 1) break;
      r -= c;
    }
    n_blk = n;
    m_blk = r;
    return;
  }
  const int G = p.group_n <= 1 ? 1 : min(p.group_n, num_n);
  if (G == 1) {
    n_blk = r / num_m;
    m_blk = r - n_blk * num_m;
    return;
  }
  const int per_group = G * num_m;
  const int g = r / per_group;
  const int i = r - g * per_group;
  const int w = min(G, num_n - g * G);  // the last group may be narrower
  m_blk = i / w;
  n_blk = g * G + (i - m_blk * w);
}

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 320;  // producer warp, MMA warp, 8 epilogue warps
// Dynamic shared memory a CTA may use on sm_100 (227 KB), less the 1 KB
// alignment slack and the barrier block.
constexpr int kSmemBudget = 232448 - 1024 - 256;

// Per-warp epilogue staging for TMA stores: two ping-pong 32 x 32 tiles of the
// output type, plus two bf16 tiles for the pre-activation when GELU is fused.
// The rest of shared memory goes to the operand ring.
template <typename OutT, int ACT>
struct EpiStage {
  static constexpr int kCTile = 32 * 32 * (int)sizeof(OutT);
  static constexpr int kWarpBytes = 2 * kCTile + (ACT == ACT_GELU ? 2 * 2048 : 0);
  static constexpr int kBytes = kEpiWarps * kWarpBytes;
};

template <int BN, typename OutT, int ACT>
struct GemmCfg {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBytes = EpiStage<OutT, ACT>::kBytes;
  static constexpr int kStagesFit = (kSmemBudget - kEpiBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kTmemCols = 2 * BN;  // 256 or 512: power of two
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 + 256;
};

template <typename OutT>
__device__ __forceinline__ void store_row32(OutT* dst, const float (&v)[32], int valid, bool vec);

template <>
__device__ __forceinline__ void store_row32<float>(float* dst, const float (&v)[32], int valid, bool vec) {
  if (vec && valid == 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) dst[j] = v[j];
  }
}

template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16* dst, const float (&v)[32], int valid,
                                                          bool vec) {
  if (vec && valid == 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 p;
      p.x = pack_bf16(v[j], v[j + 1]);
      p.y = pack_bf16(v[j + 2], v[j + 3]);
      p.z = pack_bf16(v[j + 4], v[j + 5]);
      p.w = pack_bf16(v[j + 6], v[j + 7]);
      *reinterpret_cast<uint4*>(dst + j) = p;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

template <>
__device__ __forceinline__ void store_row32<__half>(__half* dst, const float (&v)[32], int valid, bool vec) {
  if (vec && valid == 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 p;
      p.x = pack_f16(v[j], v[j + 1]);
      p.y = pack_f16(v[j + 2], v[j + 3]);
      p.z = pack_f16(v[j + 4], v[j + 5]);
      p.w = pack_f16(v[j + 6], v[j + 7]);
      *reinterpret_cast<uint4*>(dst + j) = p;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) dst[j] = __float2half_rn(v[j]);
  }
}

template <typename T>
__device__ __forceinline__ void load_row32(const T* src, float (&v)[32], int valid, bool vec) {
  if (vec && valid == 32) {
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 q = *reinterpret_cast<const float4*>(src + j);
        v[j] = q.x; v[j + 1] = q.y; v[j + 2] = q.z; v[j + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 q = *reinterpret_cast<const uint4*>(src + j);
        const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
        for (int t = 0; t < 8; ++t) v[j + t] = to_f32<T>(e[t]);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (j < valid) ? to_f32<T>(src[j]) : 0.f;
  }
}

// Epilogue math for 32 consecutive accumulator columns of one row (one thread):
// pre = alpha*acc (+ bias), v = the value to store (activation / D term applied).
template <typename OutT, int ACT>
__device__ __forceinline__ void epi_values(const GemmParams& p, const uint32_t (&raw)[32], const OutT* drow, int col0,
                                           int valid, int split, bool vec, float (&v)[32], float (&pre)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) pre[j] = __uint_as_float(raw[j]) * p.alpha;
  if (p.bias && split == 0) {
#pragma unroll
    for (int j = 0; j < 32; ++j) pre[j] += (j < valid) ? p.bias[col0 + j] : 0.f;
  }
  if constexpr (ACT == ACT_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(pre[j]);
  } else if constexpr (ACT == ACT_GELU_BWD) {
    float h[32];
    load_row32<OutT>(drow + col0, h, valid, vec);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = pre[j] * gelu_tanh_grad(h[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = pre[j];
    if (drow != nullptr && p.beta != 0.f) {
      float d[32];
      load_row32<OutT>(drow + col0, d, valid, vec);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += p.beta * d[j];
    }
  }
}

// Writes one thread's 32 values (its row) into a warp staging tile laid out as
// the TMA store expects: 32 rows x 32 elements, 128-byte rows (fp32, 128-byte
// swizzle) or 64-byte rows (16-bit types, 64-byte swizzle), so the 16-byte
// writes of a warp are bank-conflict free.
template <typename T>
__device__ __forceinline__ void stage_row32(uint8_t* tile, int r, const float (&v)[32]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int pc = c ^ (r & 7);
      *reinterpret_cast<float4*>(tile + r * 128 + pc * 16) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int pc = c ^ ((r >> 1) & 3);
      uint4 q;
      if constexpr (std::is_same<T, __half>::value) {
        q.x = pack_f16(v[8 * c], v[8 * c + 1]);
        q.y = pack_f16(v[8 * c + 2], v[8 * c + 3]);
        q.z = pack_f16(v[8 * c + 4], v[8 * c + 5]);
        q.w = pack_f16(v[8 * c + 6], v[8 * c + 7]);
      } else {
        q.x = pack_bf16(v[8 * c], v[8 * c + 1]);
        q.y = pack_bf16(v[8 * c + 2], v[8 * c + 3]);
        q.z = pack_bf16(v[8 * c + 4], v[8 * c + 5]);
        q.w = pack_bf16(v[8 * c + 6], v[8 * c + 7]);
      }
      *reinterpret_cast<uint4*>(tile + r * 64 + pc * 16) = q;
    }
  }
}

struct EpiMaps {
  CUtensorMap c;    // C: dims {N, M, batch}, box {32, 32, 1}
  CUtensorMap aux;  // pre-activation, bf16
};

// One warp's share of a tile's epilogue: its 32 accumulator rows (TMEM lane
// quarter) x columns [c_begin, c_end). TMEM loads are double-buffered so the
// load of chunk i+1 overlaps the math of chunk i. With `use_tma`, each 32 x 32
// chunk is staged in shared memory and written by one TMA store (full-line
// writes instead of 32 scattered row segments per warp instruction).
template <typename OutT, int ACT>
__device__ __forceinline__ void epilogue_rows(const GemmParams& p, const EpiMaps& maps, uint8_t* wstage,
                                              int& stage_pp, uint32_t tmem_row, int row0, int b, int n0, int split,
                                              int c_begin, int c_end, bool vec, bool use_tma) {
  const int lane = threadIdx.x & 31;
  const int row = row0 + lane;
  const bool row_ok = row < p.M;
  OutT* crow = reinterpret_cast<OutT*>(p.C) + (long long)b * p.strideC + (long long)row * p.ldc;
  const OutT* drow =
      p.D ? reinterpret_cast<const OutT*>(p.D) + (long long)b * p.strideD + (long long)row * p.ldd : nullptr;
  // The GELU pre-activation is stored in the output's 16-bit type (bf16 for fp32 outputs).
  using AuxT = typename std::conditional<sizeof(OutT) == 2, OutT, __nv_bfloat16>::type;
  AuxT* arow = p.aux ? reinterpret_cast<AuxT*>(p.aux) + (long long)b * p.strideAux + (long long)row * p.ldaux : nullptr;
  const bool atomic_out = std::is_same<OutT, float>::value && ACT == ACT_NONE && (p.splits > 1 || p.stream_k);
  uint32_t r0[32], r1[32];

  auto handle = [&](const uint32_t (&raw)[32], int c) {
    const int col0 = n0 + c;
    if (col0 >= p.N) return;
    const int valid = min(32, p.N - col0);
    float v[32], pre[32];
    if (row_ok) {
      epi_values<OutT, ACT>(p, raw, drow, col0, valid, split, vec, v, pre);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = pre[j] = 0.f;  // rows past M: clipped by the TMA store
    }
    if (p.sym && row_ok) {
      // Mirror of the elements right of the diagonal: for each column j the
      // warp's 32 rows are consecutive in the transposed row, one coalesced store.
      OutT* cb = reinterpret_cast<OutT*>(p.C) + (long long)b * p.strideC;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int col = col0 + j;
        if (j < valid && col > row) {
          if constexpr (std::is_same<OutT, float>::value) cb[(long long)col * p.ldc + row] = v[j];
          else if constexpr (std::is_same<OutT, __half>::value) cb[(long long)col * p.ldc + row] = __float2half_rn(v[j]);
          else cb[(long long)col * p.ldc + row] = __float2bfloat16_rn(v[j]);
        }
      }
    }
    if (atomic_out && !use_tma) {
      if (!row_ok) return;
      float* dst = reinterpret_cast<float*>(crow) + col0;
      if (vec && valid == 32) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          atomicAdd(reinterpret_cast<float4*>(dst + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < valid) atomicAdd(dst + j, v[j]);
      }
      return;
    }
    if (!use_tma) {
      if (!row_ok) return;
      if constexpr (ACT == ACT_GELU) {
        if (arow) store_row32<AuxT>(arow + col0, pre, valid, vec);
      }
      store_row32<OutT>(crow + col0, v, valid, vec);
      return;
    }
    // TMA path: make sure the store that used this buffer two chunks ago has
    // finished reading shared memory, stage, then issue one bulk store.
    constexpr int kCTile = EpiStage<OutT, ACT>::kCTile;
    uint8_t* ctile = wstage + stage_pp * kCTile;
    uint8_t* atile = wstage + 2 * kCTile + stage_pp * 2048;
    if (lane == 0) bulk_wait_read<1>();
    __syncwarp();
    stage_row32<OutT>(ctile, lane, v);
    if constexpr (ACT == ACT_GELU) {
      if (p.aux) stage_row32<AuxT>(atile, lane, pre);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      // Partial tiles of split-K / stream-K are added into C by one bulk
      // reduction per 32 x 32 tile (whole lines at the L2) instead of a
      // per-row vector atomic from every thread.
      if (atomic_out) tma_reduce_add_3d(&maps.c, ctile, col0, row0, b);
      else tma_store_3d(&maps.c, ctile, col0, row0, b);
      if constexpr (ACT == ACT_GELU) {
        if (p.aux) tma_store_3d(&maps.aux, atile, col0, row0, b);
      }
      bulk_commit();
    }
    stage_pp ^= 1;
  };

  if (p.debug & 4) {
    // Diagnostic: TMEM reads only (no math, no stores), with 16-, 32- or
    // 64-column loads, to measure what the loads alone cost the MMA pipe.
    uint32_t acc = 0;
    if (p.debug & 8) {
      for (int c = c_begin; c < c_end; c += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tmem_row + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc ^= r[j];
      }
    } else if (p.debug & 16) {
      for (int c = c_begin; c < c_end; c += 64) {
        uint32_t r[64];
        tmem_ld_32x32b_x64(tmem_row + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 64; ++j) acc ^= r[j];
      }
    } else {
      for (int c = c_begin; c < c_end; c += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_row + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc ^= r[j];
      }
    }
    if (acc == 0x12345678u) atomicCAS(p.status, 0, kStatusBadArgs);
    return;
  }
  tmem_ld_32x32b_x32(tmem_row + c_begin, r0);
  tmem_wait_ld_dep(r0);
#pragma unroll 1
  for (int c = c_begin; c < c_end; c += 64) {
    const bool second = c + 32 < c_end;
    if (second) tmem_ld_32x32b_x32(tmem_row + c + 32, r1);
    handle(r0, c);
    if (second) {
      tmem_wait_ld_dep(r1);
      const bool third = c + 64 < c_end;
      if (third) tmem_ld_32x32b_x32(tmem_row + c + 64, r0);
      handle(r1, c + 32);
      if (third) tmem_wait_ld_dep(r0);
    }
  }
}
template <int BN, typename OutT, int ACT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmParams p, const __grid_constant__ EpiMaps maps) {
  using Cfg = GemmCfg<BN, OutT, ACT>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint8_t* sEpi = sB + S * Cfg::kBBytes;  // 1024-aligned: stage sizes are multiples of 8 KB
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + Cfg::kEpiBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_holder, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = (p.N + BN - 1) / BN;
  const int tiles_per_batch = tiles_in_batch(p, num_m, num_n, kBM, BN);
  const int tiles_per_split = tiles_per_batch * p.batch;
  const int total_tiles = tiles_per_split * p.splits;
  const int num_kb_total = (p.K + kBK - 1) / kBK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;  // per-stage bits (registers, not a local array)
      long long w_prod = 0;
      const long long t_role = clock64();
      bool ok = true;
      int t, kb0, kb1;
      for (int unit = 0; ok && work_unit(p, blockIdx.x, gridDim.x, unit, total_tiles, tiles_per_split, num_kb_total,
                                         t, kb0, kb1); ++unit) {
        const int split = t / tiles_per_split;
        const int ts = t - split * tiles_per_split;
        const int b = ts / tiles_per_batch;
        const int r = ts - b * tiles_per_batch;
        int m_blk, n_blk;
        tile_mn(p, r, num_m, num_n, kBM, BN, m_blk, n_blk);
        const int m0 = m_blk * kBM;
        const int n0 = n_blk * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!prof_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kStatusTimeoutProducer, p.prof != nullptr, w_prod)) {
            ok = false;
            break;
          }
          if (p.debug & 1) {
            mbar_arrive(&full[stage]);
            if (++stage == S) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          uint8_t* a_dst = sA + stage * Cfg::kABytes;
          uint8_t* b_dst = sB + stage * Cfg::kBBytes;
          const int k0 = kb * kBK;
          if (!p.a_mn_major) {
            tma_load_3d(&tmA, &full[stage], a_dst, k0, m0, b);
          } else {
            tma_load_3d(&tmA, &full[stage], a_dst, m0, k0, b);
            tma_load_3d(&tmA, &full[stage], a_dst + 8192, m0 + 64, k0, b);
          }
          if (!p.b_mn_major) {
            tma_load_3d(&tmB, &full[stage], b_dst, k0, n0, b);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_3d(&tmB, &full[stage], b_dst + c * 8192, n0 + c * 64, k0, b);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every armed stage must have landed before this CTA may exit.
      for (int s = 0; s < S; ++s) {
        if (armed & (1u << s)) {
          volatile int never = 0;
          if (!mbar_wait(&full[s], (armed_parity >> s) & 1u, &never, p.status, kStatusTimeoutDrain)) break;
        }
      }
      prof_add(p, 0, w_prod);
      prof_add(p, 4, clock64() - t_role);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_f16(kBM, BN, p.fp16_inputs != 0, p.a_mn_major != 0, p.b_mn_major != 0);
      // K-major: rows are 128 B, 8-row groups 1024 B apart, K step of 16 = +32 B.
      // MN-major: 64-wide chunks 8192 B apart (LBO), 8-row K groups 1024 B apart,
      // K step of 16 rows = +2048 B.
      const uint32_t a_lbo = p.a_mn_major ? 8192u : 16u;
      const uint32_t b_lbo = p.b_mn_major ? 8192u : 16u;
      const uint32_t a_kstep = p.a_mn_major ? 2048u : 32u;
      const uint32_t b_kstep = p.b_mn_major ? 2048u : 32u;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      long long w_ops = 0, w_acc = 0;
      int t, kb0, kb1;
      for (; ok && work_unit(p, blockIdx.x, gridDim.x, local, total_tiles, tiles_per_split, num_kb_total, t, kb0,
                             kb1); ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!prof_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.status, kStatusTimeoutMma, p.prof != nullptr, w_acc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int nkb = kb1 - kb0;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!prof_wait(&full[stage], phase, abort_flag, p.status, kStatusTimeoutMma, p.prof != nullptr, w_ops)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = sw128_desc(a_addr + k * a_kstep, a_lbo, 1024);
            const uint64_t bd = sw128_desc(b_addr + k * b_kstep, b_lbo, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      // Drain: wait until every MMA this thread issued has completed.
      if (issued_any) {
        umma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, p.status, kStatusTimeoutDrain);
      }
      prof_add(p, 1, w_ops);
      prof_add(p, 2, w_acc);
      prof_add(p, 5, local);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;   // two warps per quarter split the columns
    const bool vec = p.vec_ok != 0;
    const bool use_tma = p.tma_store != 0 && !(std::is_same<OutT, float>::value && ACT == ACT_GELU);
    uint8_t* wstage = sEpi + (warp - 2) * EpiStage<OutT, ACT>::kWarpBytes;
    int stage_pp = 0;
    long long w_epi = 0;
    int local = 0;
    int t, kb0, kb1;
    for (; work_unit(p, blockIdx.x, gridDim.x, local, total_tiles, tiles_per_split, num_kb_total, t, kb0, kb1);
         ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!prof_wait(&tfull[acc], acc_phase, abort_flag, p.status, kStatusTimeoutEpilogue, p.prof != nullptr, w_epi)) break;
      tc_fence_after();
      const int split = t / tiles_per_split;
      const int ts = t - split * tiles_per_split;
      const int b = ts / tiles_per_batch;
      const int r = ts - b * tiles_per_batch;
      int m_blk, n_blk;
      tile_mn(p, r, num_m, num_n, kBM, BN, m_blk, n_blk);
      if (!(p.debug & 2) && debug_tile_ok(p, b, m_blk * kBM + q * 32, n_blk * BN + half * (BN / 2),
                                          n_blk * BN + (half + 1) * (BN / 2)))
      epilogue_rows<OutT, ACT>(p, maps, wstage, stage_pp, tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN,
                               m_blk * kBM + q * 32, b, n_blk * BN, kb0 == 0 ? 0 : 1, half * (BN / 2), (half + 1) * (BN / 2), vec,
                               use_tma);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (use_tma && lane == 0) bulk_wait_all();
    if (lane == 0) prof_add(p, 3, w_epi);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------- 2-SM variant
//
// A cluster of two CTAs computes a 256 x BN tile with tcgen05.mma.cta_group::2:
// each CTA stages its own 128 rows of A and its own BN/2 rows of B (halving the
// operand traffic per SM against the 1-SM kernel), the even CTA issues the
// MMAs, and each CTA's TMEM receives the 128 x BN fp32 accumulator of its rows.
// Both CTAs' TMA loads signal the even CTA's "full" barrier; the MMA commit
// signals the "empty"/"tmem full" barriers of both CTAs; both CTAs' epilogues
// signal the even CTA's "tmem empty" barrier. No load uses cluster multicast.

template <int BN, typename OutT, int ACT>
struct Gemm2Cfg {
  static constexpr int kABytes = 128 * kBK * 2;
  static constexpr int kBBytes = (BN / 2) * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBytes = EpiStage<OutT, ACT>::kBytes;
  static constexpr int kStagesFit = (kSmemBudget - kEpiBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 + 256;
};

template <int BN, typename OutT, int ACT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const GemmParams p, const __grid_constant__ EpiMaps maps) {
  using Cfg = Gemm2Cfg<BN, OutT, ACT>;
  constexpr int S = Cfg::kStages;
  constexpr int BHALF = BN / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kABytes;
  uint8_t* sEpi = sB + S * Cfg::kBBytes;  // 1024-aligned: stage sizes are multiples of 8 KB
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + Cfg::kEpiBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 16);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, Cfg::kTmemCols);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int num_m = (p.M + 255) / 256;
  const int num_n = (p.N + BN - 1) / BN;
  const int tiles_per_batch = tiles_in_batch(p, num_m, num_n, 256, BN);
  const int tiles_per_split = tiles_per_batch * p.batch;
  const int total_tiles = tiles_per_split * p.splits;
  const int num_kb_total = (p.K + kBK - 1) / kBK;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producers (both CTAs)
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // leader's full[0]
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;  // per-stage bits (registers, not a local array)
      long long w_prod = 0;
      const long long t_role = clock64();
      bool ok = true;
      int t, kb0, kb1;
      for (int unit = 0; ok && work_unit(p, pair, npairs, unit, total_tiles, tiles_per_split, num_kb_total, t, kb0,
                                         kb1); ++unit) {
        const int split = t / tiles_per_split;
        const int ts = t - split * tiles_per_split;
        const int b = ts / tiles_per_batch;
        const int r = ts - b * tiles_per_batch;
        int m_blk, n_blk;
        tile_mn(p, r, num_m, num_n, 256, BN, m_blk, n_blk);
        const int m0 = m_blk * 256 + (int)rank * 128;
        const int n0 = n_blk * BN + (int)rank * BHALF;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!prof_wait(&empty[stage], phase ^ 1, abort_flag, p.status, kStatusTimeoutProducer, p.prof != nullptr, w_prod)) {
            ok = false;
            break;
          }
          if (p.debug & 1) {
            if (leader) mbar_arrive(&full[stage]);
            if (++stage == S) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          if (leader) {
            mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t fb = full0 + stage * 8;
          uint8_t* a_dst = sA + stage * Cfg::kABytes;
          uint8_t* b_dst = sB + stage * Cfg::kBBytes;
          const int k0 = kb * kBK;
          if (!p.a_mn_major) {
            tma_load_3d_pair(&tmA, fb, a_dst, k0, m0, b);
          } else {
            tma_load_3d_pair(&tmA, fb, a_dst, m0, k0, b);
            tma_load_3d_pair(&tmA, fb, a_dst + 8192, m0 + 64, k0, b);
          }
          if (!p.b_mn_major) {
            tma_load_3d_pair(&tmB, fb, b_dst, k0, n0, b);
          } else {
#pragma unroll
            for (int c = 0; c < BHALF / 64; ++c) tma_load_3d_pair(&tmB, fb, b_dst + c * 8192, n0 + c * 64, k0, b);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (leader) {
        // The leader's full barriers account for both CTAs' copies.
        for (int s = 0; s < S; ++s) {
          if (armed & (1u << s)) {
            volatile int never = 0;
            if (!mbar_wait(&full[s], (armed_parity >> s) & 1u, &never, p.status, kStatusTimeoutDrain)) break;
          }
        }
      }
      prof_add(p, 0, w_prod);
      prof_add(p, 4, clock64() - t_role);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (even CTA)
      const uint32_t idesc = idesc_f16(256, BN, p.fp16_inputs != 0, p.a_mn_major != 0, p.b_mn_major != 0);
      const uint32_t a_lbo = p.a_mn_major ? 8192u : 16u;
      const uint32_t b_lbo = p.b_mn_major ? 8192u : 16u;
      const uint32_t a_kstep = p.a_mn_major ? 2048u : 32u;
      const uint32_t b_kstep = p.b_mn_major ? 2048u : 32u;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      long long w_ops = 0, w_acc = 0;
      int t, kb0, kb1;
      for (; ok && work_unit(p, pair, npairs, local, total_tiles, tiles_per_split, num_kb_total, t, kb0, kb1);
           ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!prof_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.status, kStatusTimeoutMma, p.prof != nullptr, w_acc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int nkb = kb1 - kb0;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!prof_wait(&full[stage], phase, abort_flag, p.status, kStatusTimeoutMma, p.prof != nullptr, w_ops)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = sw128_desc(a_addr + k * a_kstep, a_lbo, 1024);
            const uint64_t bd = sw128_desc(b_addr + k * b_kstep, b_lbo, 1024);
            umma_f16_ss_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(&tfull[acc], 0x3);
      }
      if (issued_any) {
        umma_commit_pair(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, p.status, kStatusTimeoutDrain);
      }
      prof_add(p, 1, w_ops);
      prof_add(p, 2, w_acc);
      prof_add(p, 5, local);
    }
  } else {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const bool vec = p.vec_ok != 0;
    const bool use_tma = p.tma_store != 0 && !(std::is_same<OutT, float>::value && ACT == ACT_GELU);
    uint8_t* wstage = sEpi + (warp - 2) * EpiStage<OutT, ACT>::kWarpBytes;
    int stage_pp = 0;
    long long w_epi = 0;
    const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
    int local = 0;
    int t, kb0, kb1;
    for (; work_unit(p, pair, npairs, local, total_tiles, tiles_per_split, num_kb_total, t, kb0, kb1); ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!prof_wait(&tfull[acc], acc_phase, abort_flag, p.status, kStatusTimeoutEpilogue, p.prof != nullptr, w_epi)) break;
      tc_fence_after();
      const int split = t / tiles_per_split;
      const int ts = t - split * tiles_per_split;
      const int b = ts / tiles_per_batch;
      const int r = ts - b * tiles_per_batch;
      int m_blk, n_blk;
      tile_mn(p, r, num_m, num_n, 256, BN, m_blk, n_blk);
      if (!(p.debug & 2) && debug_tile_ok(p, b, m_blk * 256 + (int)rank * 128 + q * 32, n_blk * BN + half * (BN / 2),
                                          n_blk * BN + (half + 1) * (BN / 2)))
      epilogue_rows<OutT, ACT>(p, maps, wstage, stage_pp, tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN,
                               m_blk * 256 + (int)rank * 128 + q * 32, b, n_blk * BN, kb0 == 0 ? 0 : 1, half * (BN / 2),
                               (half + 1) * (BN / 2), vec, use_tma);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + acc * 8);
    }
    if (use_tma && lane == 0) bulk_wait_all();
    if (lane == 0) prof_add(p, 3, w_epi);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------- host

static bool is_mn_major_2d(const at::Tensor& t) {
  // For a [rows, cols] view: K-major means cols (K) contiguous.
  return t.stride(-1) != 1;
}

template <int BN, typename OutT, int ACT>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, const EpiMaps& maps,
                        int grid, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, OutT, ACT>;
  auto kern = gemm_tcgen05_kernel<BN, OutT, ACT>;
  static bool attr_set = false;
  if (!attr_set) {
    KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    attr_set = true;
  }
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, p, maps);
  KB_LAUNCHED();
}

template <int BN, typename OutT>
static void dispatch_act(int act, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, const EpiMaps& maps, int grid,
                         cudaStream_t s) {
  switch (act) {
    case ACT_NONE: launch_gemm<BN, OutT, ACT_NONE>(ta, tb, p, maps, grid, s); break;
    case ACT_GELU: launch_gemm<BN, OutT, ACT_GELU>(ta, tb, p, maps, grid, s); break;
    case ACT_GELU_BWD: launch_gemm<BN, OutT, ACT_GELU_BWD>(ta, tb, p, maps, grid, s); break;
    default: KB_CHECK(false, "bad activation");
  }
}

template <int BN, typename OutT, int ACT>
static void launch_gemm2(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, const EpiMaps& maps,
                         int grid, cudaStream_t stream) {
  using Cfg = Gemm2Cfg<BN, OutT, ACT>;
  auto kern = gemm_2sm_kernel<BN, OutT, ACT>;
  static bool attr_set = false;
  if (!attr_set) {
    KB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    attr_set = true;
  }
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, p, maps);
  KB_LAUNCHED();
}

template <int BN, typename OutT>
static void dispatch_act2(int act, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, const EpiMaps& maps, int grid,
                          cudaStream_t s) {
  switch (act) {
    case ACT_NONE: launch_gemm2<BN, OutT, ACT_NONE>(ta, tb, p, maps, grid, s); break;
    case ACT_GELU: launch_gemm2<BN, OutT, ACT_GELU>(ta, tb, p, maps, grid, s); break;
    case ACT_GELU_BWD: launch_gemm2<BN, OutT, ACT_GELU_BWD>(ta, tb, p, maps, grid, s); break;
    default: KB_CHECK(false, "bad activation");
  }
}

// Pipeline profile buffer for the GEMM kernels (see GemmParams::prof); null
// when profiling is off. Set from Python for diagnostics only.
static unsigned long long* g_gemm_prof = nullptr;
static int g_gemm_debug = 0;
// Tile-column group width override for timing studies (-1: the host's rule).
static int g_gemm_group = -1;
// K-cut override for fp32 outputs, for timing studies: -1 the host's rule,
// 0 never cut, 1 stream-K, s >= 2 split-K into s parts.
static int g_gemm_split = -1;

void gemm_set_debug(int64_t mode) { g_gemm_debug = (int)mode; }
void gemm_set_group(int64_t g) { g_gemm_group = (int)g; }
void gemm_set_split(int64_t s) { g_gemm_split = (int)s; }

static int64_t sym_tile_count(int64_t num_m, int64_t num_n, int64_t bm, int64_t bn) {
  int64_t t = 0;
  for (int64_t n = 0; n < num_n; ++n) t += std::min<int64_t>(num_m, (n * bn + bn - 1) / bm + 1);
  return t;
}

void gemm_set_profile(const c10::optional<at::Tensor>& buf) {
  if (!buf.has_value() || !buf->defined()) {
    g_gemm_prof = nullptr;
    return;
  }
  check_cuda_tensor(*buf, "profile buffer");
  KB_CHECK(buf->scalar_type() == at::kLong && buf->is_contiguous() && buf->numel() >= 8 * 2 * 256,
           "gemm profile buffer must be int64 with at least 4096 entries");
  g_gemm_prof = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
}

// Operand description: `t` is a 2-D [rows, cols] or 3-D [batch, rows, cols] view.
// For A: logical (M x K). If K-major, t is [.., M, K] with stride(-1)==1. If
// M-major, t is [.., K, M] with stride(-1)==1 (flag mn_major=true).
static CUtensorMap operand_map(const at::Tensor& t, bool mn_major, int mn_extent, int k_extent, int box_rows) {
  const int64_t batch = t.dim() == 3 ? t.size(0) : 1;
  const int64_t bstride = t.dim() == 3 ? t.stride(0) : 0;
  const int64_t ld = t.stride(-2);
  const int64_t esz = t.element_size();
  uint64_t dims[3];
  uint64_t strides[2];
  uint32_t box[3];
  if (!mn_major) {
    dims[0] = (uint64_t)k_extent;
    dims[1] = (uint64_t)mn_extent;
    box[0] = 64;
    box[1] = (uint32_t)box_rows;
  } else {
    dims[0] = (uint64_t)mn_extent;
    dims[1] = (uint64_t)k_extent;
    box[0] = 64;
    box[1] = 64;
  }
  dims[2] = (uint64_t)batch;
  box[2] = 1;
  strides[0] = (uint64_t)(ld * esz);
  strides[1] = (uint64_t)((batch > 1 ? bstride : ld * (mn_major ? k_extent : mn_extent)) * esz);
  if (strides[1] % 16 != 0) strides[1] = ((strides[1] + 15) / 16) * 16;  // unused when batch == 1
  return make_tma(t.data_ptr(), t.scalar_type(), 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Public entry: see gemm() in bindings for argument meaning.
void gemm_launch(const at::Tensor& a, bool a_mn_major, const at::Tensor& b, bool b_mn_major, at::Tensor& c,
                 const c10::optional<at::Tensor>& d, double alpha, double beta, const c10::optional<at::Tensor>& bias,
                 const c10::optional<at::Tensor>& aux, int64_t act, int64_t block_n, int64_t flags) {
  check_cuda_tensor(a, "a");
  check_cuda_tensor(b, "b");
  check_cuda_tensor(c, "c");
  KB_CHECK(a.scalar_type() == b.scalar_type(), "A and B must have the same dtype");
  KB_CHECK(a.scalar_type() == at::kBFloat16 || a.scalar_type() == at::kHalf, "A/B must be bf16 or fp16");
  KB_CHECK(a.dim() == b.dim() && (a.dim() == 2 || a.dim() == 3), "A and B must both be 2-D or 3-D");
  KB_CHECK(a.stride(-1) == 1 && b.stride(-1) == 1, "A and B must have unit inner stride");
  const bool batched = a.dim() == 3;
  const int64_t batch = batched ? a.size(0) : 1;
  const int64_t M = a_mn_major ? a.size(-1) : a.size(-2);
  const int64_t K = a_mn_major ? a.size(-2) : a.size(-1);
  const int64_t N = b_mn_major ? b.size(-1) : b.size(-2);
  const int64_t Kb = b_mn_major ? b.size(-2) : b.size(-1);
  KB_CHECK(K == Kb, "inner dimensions differ");
  KB_CHECK(c.size(-2) == M && c.size(-1) == N && c.stride(-1) == 1, "C shape mismatch");
  KB_CHECK(!batched || (b.size(0) == batch && c.dim() == 3 && c.size(0) == batch), "batch mismatch");
  KB_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  const auto ct = c.scalar_type();
  KB_CHECK(ct == at::kFloat || ct == at::kBFloat16 || ct == at::kHalf, "C must be fp32, bf16 or fp16");
  KB_CHECK(ct == at::kFloat || ct == a.scalar_type(), "reduced-precision C must match the input dtype");

  // flags bit 0: the product is symmetric (X X^T, or A A / b A + c A A with A
  // and D symmetric); only tiles on or above the diagonal are computed.
  const bool sym = (flags & 1) != 0;
  KB_CHECK(!sym || (M == N && act == ACT_NONE && !(bias.has_value() && bias->defined()) &&
                    !(aux.has_value() && aux->defined()) && ct != at::kFloat &&
                    !(d.has_value() && d->defined() && d->data_ptr() == c.data_ptr())),
           "symmetric GEMM: square 16-bit output without bias, aux or activation, D not C itself "
           "(the mirrored stores would race with other tiles' reads of D)");
  const c10::cuda::CUDAGuard guard(a.device());
  const int dev = a.get_device();
  // Tile configuration: 1-SM 128 x {128, 256} or 2-SM 256 x {128, 256}.
  // block_n > 0 forces a 1-SM width, block_n < 0 forces a 2-SM width |block_n|;
  // 0 picks the configuration with the lowest estimated time (waves x tile work,
  // weighted by each configuration's measured relative efficiency).
  const int sms_all = compute_sms(dev);
  int bn = 0;
  bool pair_mode = false;
  if (block_n == 128 || block_n == 256) {
    bn = (int)block_n;
  } else if (block_n == -128 || block_n == -256) {
    bn = (int)-block_n;
    pair_mode = true;
  } else {
    // Relative time per unit of tile work, measured on the model shapes: an
    // N=128 MMA keeps the tensor pipe far less busy than an N=256 one, and the
    // 2-SM pair halves each SM's operand traffic.
    double best = 1e30;
    const int cand_bn[4] = {128, 256, 128, 256};
    const bool cand_pair[4] = {false, false, true, true};
    const double factor[4] = {1.6, 1.05, 1.6, 1.0};
    const bool sk_ok = c.scalar_type() == at::kFloat && act == ACT_NONE && (K + 63) / 64 >= 8;
    for (int i = 0; i < 4; ++i) {
      const int w = cand_bn[i];
      const bool pm = cand_pair[i];
      if (pm && M < 256) continue;
      const int rows = pm ? 256 : 128;
      const int64_t t = batch * (sym ? sym_tile_count((M + rows - 1) / rows, (N + w - 1) / w, rows, w)
                                     : ((M + rows - 1) / rows) * ((N + w - 1) / w));
      const int64_t slots = pm ? sms_all / 2 : sms_all;
      // With stream-K available the work spreads evenly (plus a partial-tile
      // overhead); otherwise whole waves count.
      const double waves = sk_ok ? double(t) / double(slots) + 0.15 : double((t + slots - 1) / slots);
      const double cost = waves * (double(w) / 256.0) * factor[i];
      if (cost < best - 1e-9) {
        best = cost;
        bn = w;
        pair_mode = pm;
      }
    }
  }
  const CUtensorMap ta = operand_map(a, a_mn_major, (int)M, (int)K, 128);
  const CUtensorMap tb = operand_map(b, b_mn_major, (int)N, (int)K, pair_mode ? bn / 2 : bn);

  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = (int)batch;
  p.a_mn_major = a_mn_major;
  p.b_mn_major = b_mn_major;
  p.fp16_inputs = a.scalar_type() == at::kHalf;
  p.C = c.data_ptr();
  p.dbg_c_extent = declared_extent(c);
  p.ldc = c.stride(-2);
  p.strideC = batched ? c.stride(0) : 0;
  p.alpha = (float)alpha;
  p.beta = (float)beta;
  bool vec = (p.ldc % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) && (!batched || p.strideC % 8 == 0);
  if (d.has_value() && d->defined()) {
    KB_CHECK(d->scalar_type() == ct && d->size(-2) == M && d->size(-1) == N && d->stride(-1) == 1, "D mismatch");
    p.D = d->data_ptr();
    p.dbg_d_extent = declared_extent(*d);
    p.ldd = d->stride(-2);
    p.strideD = batched ? d->stride(0) : 0;
    vec = vec && (p.ldd % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.D) & 15) == 0) && (!batched || p.strideD % 8 == 0);
  }
  if (bias.has_value() && bias->defined()) {
    KB_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == N && bias->is_contiguous(), "bias must be fp32 [N]");
    p.bias = bias->data_ptr<float>();
  }
  if (aux.has_value() && aux->defined()) {
    const at::ScalarType aux_t = (ct == at::kFloat) ? at::kBFloat16 : ct;
    KB_CHECK(aux->scalar_type() == aux_t && aux->size(-2) == M && aux->size(-1) == N,
             "aux must be [.., M, N] in the output's 16-bit type (bf16 for fp32 outputs)");
    p.aux = aux->data_ptr();
    p.dbg_aux_extent = declared_extent(*aux);
    p.ldaux = aux->stride(-2);
    p.strideAux = batched ? aux->stride(0) : 0;
    vec = vec && (p.ldaux % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.aux) & 15) == 0);
  }
  KB_CHECK(act != ACT_GELU_BWD || p.D != nullptr, "GELU backward needs the pre-activation as D");
  p.vec_ok = vec;
  p.status = device_status_ptr(dev);
  p.prof = g_gemm_prof;
  p.debug = g_gemm_debug;

  const int rows_per_tile = pair_mode ? 256 : 128;
  const int64_t num_m_tiles = (M + rows_per_tile - 1) / rows_per_tile, num_n_tiles = (N + bn - 1) / bn;
  const int64_t tiles = batch * (sym ? sym_tile_count(num_m_tiles, num_n_tiles, rows_per_tile, bn)
                                     : num_m_tiles * num_n_tiles);
  p.sym = sym ? 1 : 0;
  const int sms = pair_mode ? (sms_all / 2) : sms_all;  // concurrent tile slots
  const int64_t num_kb = (K + 63) / 64;
  // fp32 outputs without an activation (weight gradients, long K) whose whole
  // tiles would leave part of the last wave idle are cut along K, and the
  // partial tiles are summed into C with fp32 atomics (C first set to
  // beta * D, or zero):
  //  * split-K first: every tile cut at the same K boundaries, units of one
  //    split handed to neighbouring workers, so the workers running at the
  //    same time read the same K range of the operand panels and those stay
  //    in L2 (cutting the K-iterations of all tiles evenly over the workers,
  //    stream-K, puts every worker at a different K offset and, once the
  //    operands outgrow L2, re-reads them from DRAM). The smallest split
  //    count that fills the machine is taken, as long as its atomic traffic
  //    (splits x the size of C) stays moderate;
  //  * stream-K otherwise.
  // With a D operand (a residual to add) the copy of D into C and the
  // atomics cost more than a partly idle last wave, so those cut only when
  // whole tiles would leave a quarter of the machine idle -- unless D is C
  // itself with beta 1 (accumulation into an existing gradient), where the
  // partial tiles are simply added into C.
  int splits = 1;
  int stream_k = 0;
  if (ct == at::kFloat && act == ACT_NONE && num_kb >= 8) {
    auto fill = [&](int64_t units) {
      const int64_t waves = (units + sms - 1) / sms;
      return double(units) / double(waves * sms);
    };
    // C += A B^T in place (D is C, beta 1) needs no copy of D: the cut costs what it costs without D.
    const bool has_d = p.D != nullptr && p.beta != 0.f && !(p.D == p.C && p.beta == 1.f);
    // (At a fill of 0.865 -- the Llama-style q/k/v and output-projection
    // weight gradients -- whole tiles in the grouped order measured 7-9 %
    // faster than stream-K, so the bar for cutting is 0.85.)
    if (fill(tiles) < (has_d ? 0.75 : 0.85)) {
      const double c_bytes = double(batch) * double(M) * double(N) * 4.0;
      for (int sp = 2; sp <= 8 && sp * 4 <= num_kb; ++sp) {
        if (fill(tiles * sp) >= 0.9 && sp * c_bytes <= 96.0 * (1 << 20)) {
          splits = sp;
          break;
        }
      }
      if (splits == 1) stream_k = 1;
    }
    if (g_gemm_split >= 0) {
      splits = g_gemm_split >= 2 ? (int)std::min<int64_t>(g_gemm_split, std::max<int64_t>(1, num_kb / 4)) : 1;
      stream_k = g_gemm_split == 1 ? 1 : 0;
    }
  }
  p.splits = splits;
  p.kb_per_split = (int)((num_kb + splits - 1) / splits);
  p.stream_k = stream_k;
  // Tile order (measured on the GPT-2 and Llama-style shapes): columns taken
  // 8 at a time where the operand panels of the tiles in flight would not
  // stay in L2 in plain order -- long K (data and weight gradients, the LM
  // head's gradients) and batched products (Newton-Schulz) -- 4-14 % faster
  // there; plain order for short-K forward products, where grouping cost up
  // to 4 %, and under stream-K, whose workers are spread over K anyway.
  p.group_n = g_gemm_group >= 0 ? g_gemm_group : ((!stream_k && (batch > 1 || K >= 3072)) ? 8 : 0);
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev).stream();
  if (stream_k || splits > 1) {
    // C = beta * D (or 0); every split then adds its partial product.
    if (p.D != nullptr && p.beta != 0.f) {
      if (p.D != p.C || p.beta != 1.f) {
        at::Tensor cv = c;
        cv.copy_(*d);
        if (p.beta != 1.f) cv.mul_(p.beta);
      }
    } else {
      c.zero_();
    }
    p.D = nullptr;
    p.beta = 0.f;
  }
  // Staged TMA stores need 16-byte aligned rows (and batch strides) for C and aux.
  EpiMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  {
    const int64_t esz = c.element_size();
    bool ok = (p.ldc * esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.C) & 15) == 0 &&
              (!batched || (p.strideC * esz) % 16 == 0);
    if (ok && p.aux != nullptr)
      ok = (p.ldaux * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.aux) & 15) == 0 && (!batched || (p.strideAux * 2) % 16 == 0);
    if (ok) {
      auto make = [&](void* base, at::ScalarType t, int64_t ld, int64_t bstride, int64_t es) {
        uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)batch};
        uint64_t strides[2] = {(uint64_t)(ld * es), (uint64_t)((batched ? bstride : ld * M) * es)};
        if (strides[1] % 16) strides[1] = (strides[1] + 15) / 16 * 16;
        uint32_t box[3] = {32, 32, 1};
        return make_tma(base, t, 3, dims, strides, box, es == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
      };
      maps.c = make(p.C, ct, p.ldc, p.strideC, esz);
      if (p.aux != nullptr) maps.aux = make(p.aux, ct == at::kFloat ? at::kBFloat16 : ct, p.ldaux, p.strideAux, 2);
      p.tma_store = 1;
    }
  }
  if (pair_mode) {
    const int grid2 = 2 * (int)(stream_k ? std::min<int64_t>(tiles * num_kb, sms) : std::min<int64_t>(tiles * splits, sms));
    if (bn == 256) {
      if (ct == at::kFloat) dispatch_act2<256, float>((int)act, ta, tb, p, maps, grid2, stream);
      else if (ct == at::kBFloat16) dispatch_act2<256, __nv_bfloat16>((int)act, ta, tb, p, maps, grid2, stream);
      else dispatch_act2<256, __half>((int)act, ta, tb, p, maps, grid2, stream);
    } else {
      if (ct == at::kFloat) dispatch_act2<128, float>((int)act, ta, tb, p, maps, grid2, stream);
      else if (ct == at::kBFloat16) dispatch_act2<128, __nv_bfloat16>((int)act, ta, tb, p, maps, grid2, stream);
      else dispatch_act2<128, __half>((int)act, ta, tb, p, maps, grid2, stream);
    }
    return;
  }
  const int grid = (int)(stream_k ? std::min<int64_t>(tiles * num_kb, sms) : std::min<int64_t>(tiles * splits, sms));
  if (bn == 256) {
    if (ct == at::kFloat) dispatch_act<256, float>((int)act, ta, tb, p, maps, grid, stream);
    else if (ct == at::kBFloat16) dispatch_act<256, __nv_bfloat16>((int)act, ta, tb, p, maps, grid, stream);
    else dispatch_act<256, __half>((int)act, ta, tb, p, maps, grid, stream);
  } else {
    if (ct == at::kFloat) dispatch_act<128, float>((int)act, ta, tb, p, maps, grid, stream);
    else if (ct == at::kBFloat16) dispatch_act<128, __nv_bfloat16>((int)act, ta, tb, p, maps, grid, stream);
    else dispatch_act<128, __half>((int)act, ta, tb, p, maps, grid, stream);
  }
}

}  // namespace kb
