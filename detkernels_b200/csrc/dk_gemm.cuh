// Batch-invariant GEMM on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces kernels/matmul.py:64-100 (_matmul_kernel, the invariant direct tile
// GEMM) and, through the ATOMIC mode, kernels/matmul.py:102-145 (the split-K
// atomic twin used by matmul_batch_variant).
//
// C[M,N] = A[M,K] @ B[K,N], A and B row-major bf16/f16, f32 accumulation.
//
// When all M rows fit one 128-token tile, the activation TMA box covers only
// ceil8(M) rows; the instruction still spans 128 token columns, and columns
// beyond the box read stale shared memory.  Each output column depends only on
// its own token row, and stale columns are never stored.
//
// Formulation ("swap-AB"): the tensor-core instruction computes
//   D[n, m] = sum_k B[k, n] * A[m, k]
// with the 128 weight columns of a tile on the UMMA M axis (B read MN-major,
// straight from its row-major [K, N] layout) and 128 tokens on the UMMA N axis
// (A read K-major).  The tile shape (128 x 128 x 16 per instruction) is the
// same for every M.
//
// Fixed reduction structure (the definition of the output bits):
//   * K is cut into DK_MATMUL_K_SLICES = 8 slices of L = ceil16(ceil(K/8))
//     elements; slice s covers [s*L, min((s+1)*L, K)).
//   * Slice s is accumulated from zero in its own TMEM accumulator by
//     tcgen05.mma steps of 16 K-elements in ascending K order.
//   * The 8 f32 partials are folded in slice order ((p0 + p1) + p2) + ... + p7,
//     then rounded to the output dtype (round to nearest even).
// Nothing in that structure depends on M, N or the schedule, so a row's output
// bits do not depend on the batch.  Only the schedule does:
//   * FOLD:    a work unit = one output tile x all 8 slices; the epilogue warps
//              fold each partial into a third TMEM buffer (tcgen05.ld / add /
//              tcgen05.st), with the two accumulators double-buffered so slice
//              s+1 is multiplied while slice s is drained.  Used when there are
//              at least as many output tiles as SMs.
//   * SPLIT:   a work unit = one output tile x a group of 1/2/4 slices; every
//              partial goes to the workspace and the CTA that finishes a tile
//              last (atomic arrival counter, no spinning) folds all 8 in slice
//              order.  Used for small M to fill the GPU with K-parallel work.
//   * PARTIAL: slices [slice_begin, slice_end) only, partials written out
//              (row-parallel tensor parallelism).
//   * ATOMIC:  the deliberately batch-variant twin: split_k chunks added with
//              f32 atomics (scheduler-dependent order).
#pragma once

#include "dk_common.cuh"

namespace dk {
namespace gemm {

constexpr int kTileN = 128;  // weight columns per tile (UMMA M)
constexpr int kTileM = 128;  // tokens per tile (UMMA N)
constexpr int kBK = 64;      // K per pipeline stage: one 128-byte swizzle row of bf16
constexpr int kUK = 16;      // K per tcgen05.mma, kind::f16
constexpr int kStages = 6;
constexpr int kSlices = DK_MATMUL_K_SLICES;
constexpr int kWBoxBytes = 64 * kBK * 2;          // 64 columns x 64 k
constexpr int kWTileBytes = 2 * kWBoxBytes;       // 128 columns x 64 k
constexpr int kATileBytes = kTileM * kBK * 2;     // 128 tokens x 64 k
constexpr int kStageBytes = kWTileBytes + kATileBytes;
constexpr int kEpiWarps = 8;                      // two warps per TMEM lane quarter
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kEpiCols = kTileM / 2;              // token columns folded per epilogue thread
constexpr int kThreads = 64 + kEpiThreads;        // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kTmemCols = 512;                    // two 128-column f32 accumulators + fold buffer
constexpr int kSumCol = 2 * kTileM;               // TMEM column of the running slice fold
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;

enum Mode : int { FOLD = 0, SPLIT = 1, PARTIAL = 2, ATOMIC = 3 };

struct Params {
  int M, N, K;
  int slice_len;                 // elements per slice (multiple of 16)
  int slice_begin, slice_end;    // slices computed by this launch
  int group;                     // slices per work unit
  int n_tiles, m_tiles;
  int mode;
  int a_rows;      // rows of the activation TMA box (128, or fewer when M fits one tile)
  void* c;
  int64_t ldc;
  float* ws;       // SPLIT/PARTIAL: partials [slice][M][N]; ATOMIC: [M][N]
  int* counters;   // SPLIT: one arrival counter per output tile
};

// Detail codes recorded with a timeout (which wait expired).
enum : int {
  kDetProdEmpty = 0x100,
  kDetMmaAccEmpty = 0x101,
  kDetMmaFull = 0x102,
  kDetEpiAccFull = 0x103,
  kDetEpiSync = 0x104,
  kDetDrain = 0x105,
};

__device__ __forceinline__ void slice_bounds(const Params& p, int s, int& k0, int& k1) {
  k0 = s * p.slice_len;
  k1 = min(k0 + p.slice_len, p.K);
  if (k1 < k0) k1 = k0;
}

// Bounded barrier among the epilogue threads (an mbarrier, so a thread
// that gave up cannot leave the others blocked forever).
__device__ __forceinline__ bool epi_sync(uint64_t* bar, uint32_t& phase, bool& abort_flag) {
  if (abort_flag) return false;
  mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase, kDetEpiSync, abort_flag);
  phase ^= 1u;
  return ok;
}

template <typename T, int FMT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* ep_bar = acc_empty + 2;
  uint64_t* drain_bar = ep_bar + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
    mbar_init(&acc_empty[0], kEpiThreads);
    mbar_init(&acc_empty[1], kEpiThreads);
    mbar_init(ep_bar, kEpiThreads);
    mbar_init(drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmA);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int n_groups = (p.slice_end - p.slice_begin) / p.group;
  const int units = p.n_tiles * p.m_tiles * n_groups;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      int fills = 0;                     // stage fills issued so far (round robin)
      for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x) {
        const int g = u % n_groups;
        const int t = u / n_groups;
        const int mt = t % p.m_tiles;
        const int nt = t / p.m_tiles;
        for (int si = 0; si < p.group && !abort_flag; ++si) {
          const int s = p.slice_begin + g * p.group + si;
          int k0, k1;
          slice_bounds(p, s, k0, k1);
          const int nkb = (k1 - k0 + kBK - 1) / kBK;
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, kDetProdEmpty, abort_flag)) break;
            uint8_t* st = smem + stage * kStageBytes;
            mbar_arrive_expect_tx(&full[stage], kWTileBytes + p.a_rows * kBK * 2);
            const int kk = k0 + kb * kBK;
            tma_load_2d(st, &tmB, &full[stage], nt * kTileN, kk);
            tma_load_2d(st + kWBoxBytes, &tmB, &full[stage], nt * kTileN + 64, kk);
            tma_load_2d(st + kWTileBytes, &tmA, &full[stage], kk, mt * kTileM);
            ++fills;
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      // Drain: every copy this thread issued must have landed before the CTA exits.
      bool drain_abort = false;
#pragma unroll 1
      for (int f = (fills > kStages ? fills - kStages : 0); f < fills; ++f) {
        mbar_wait(&full[f % kStages], static_cast<uint32_t>((f / kStages) & 1), kDetDrain, drain_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer (one thread) ----------------
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      constexpr uint32_t idesc = umma_idesc_f16(FMT, /*a_mn=*/1, /*b_mn=*/0, kTileN, kTileM);
      for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x) {
        const int g = u % n_groups;
        for (int si = 0; si < p.group && !abort_flag; ++si) {
          const int s = p.slice_begin + g * p.group + si;
          int k0, k1;
          slice_bounds(p, s, k0, k1);
          const int nkb = (k1 - k0 + kBK - 1) / kBK;
          if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, kDetMmaAccEmpty, abort_flag)) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTileM);
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&full[stage], phase, kDetMmaFull, abort_flag)) break;
            tc_fence_after();
            const int kk = k0 + kb * kBK;
            const int nsteps = min(kBK / kUK, (k1 - kk + kUK - 1) / kUK);
            const uint32_t b_base = smem_u32(smem + stage * kStageBytes);
            const uint32_t a_base = b_base + kWTileBytes;
            for (int j = 0; j < nsteps; ++j) {
              // B (weights) MN-major, 128B swizzle: 64-column groups 8 KB apart (LBO),
              // 8-row K groups 1 KB apart (SBO); one 16-deep K step = 2 KB.
              const uint64_t bdesc = umma_sdesc(b_base + j * 2048, kWBoxBytes, 1024, 2);
              // A (tokens) K-major, 128B swizzle: 8-row groups 1 KB apart; 16 K = 32 bytes.
              const uint64_t adesc = umma_sdesc(a_base + j * 32, 16, 1024, 2);
              tc_mma_f16(d_tmem, bdesc, adesc, idesc, (kb > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit(&empty[stage]);
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (abort_flag) break;
          tc_commit(&acc_full[acc]);
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1u;
        }
      }
      // Drain: all MMAs issued by this thread complete before TMEM is released.
      bool drain_abort = false;
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, kDetDrain, drain_abort);
    }
  } else {
    // ---------------- epilogue: 8 warps ----------------
    // Warp w may only read TMEM lanes 32*(w%4)..+31 (its quarter); the two warps
    // of a quarter split the 128 token columns into halves.  Thread <-> TMEM
    // lane <-> output column n; each thread folds 64 token columns.
    bool abort_flag = false;
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int n_local = quarter * 32 + lane;      // D row = weight column inside the tile
    const int col0 = half * kEpiCols;             // first token column of this thread
    const int ep_tid = threadIdx.x - 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t ep_phase = 0;
    T* C = reinterpret_cast<T*>(p.c);
    const int64_t MN = static_cast<int64_t>(p.M) * p.N;
    for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x) {
      const int g = u % n_groups;
      const int t = u / n_groups;
      const int mt = t % p.m_tiles;
      const int nt = t / p.m_tiles;
      const int n = nt * kTileN + n_local;
      const int m0 = mt * kTileM + col0;
      const bool n_ok = n < p.N;
      const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      for (int si = 0; si < p.group; ++si) {
        const int s = p.slice_begin + g * p.group + si;
        int k0, k1;
        slice_bounds(p, s, k0, k1);
        const bool empty_slice = (k1 <= k0);
        if (!mbar_wait(&acc_full[acc], acc_phase, kDetEpiAccFull, abort_flag)) break;
        tc_fence_after();
        const uint32_t taddr = lane_base + static_cast<uint32_t>(acc * kTileM + col0);
        const uint32_t saddr = lane_base + static_cast<uint32_t>(kSumCol + col0);
#pragma unroll 1
        for (int c = 0; c < kEpiCols / 32; ++c) {
          float v[32];
          tmem_ld_32x32b_x32(taddr + c * 32, v);
          tmem_ld_wait();
          if (empty_slice) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
          }
          if (p.mode == FOLD) {
            // running fold ((p0 + p1) + p2) + ... kept in TMEM columns [kSumCol, kSumCol + 128)
            if (si > 0) {
              float w[32];
              tmem_ld_32x32b_x32(saddr + c * 32, w);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(w[j], v[j]);
            }
            if (si + 1 < p.group) {
              tmem_st_32x32b_x32(saddr + c * 32, v);
              tmem_st_wait();
            } else if (n_ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int m = m0 + c * 32 + j;
                if (m < p.M) C[static_cast<int64_t>(m) * p.ldc + n] = from_f32<T>(v[j]);
              }
            }
          } else if (p.mode == ATOMIC) {
            if (n_ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int m = m0 + c * 32 + j;
                if (m < p.M) atomicAdd(p.ws + static_cast<int64_t>(m) * p.N + n, v[j]);
              }
            }
          } else {  // SPLIT / PARTIAL: partial of slice s -> ws[s - slice_begin][m][n]
            if (n_ok) {
              float* dst = p.ws + static_cast<int64_t>(s - p.slice_begin) * MN;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int m = m0 + c * 32 + j;
                if (m < p.M) dst[static_cast<int64_t>(m) * p.N + n] = v[j];
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (abort_flag) break;

      if (p.mode == SPLIT) {
        // Last CTA to finish this tile folds all slices in slice order.
        __threadfence();
        if (!epi_sync(ep_bar, ep_phase, abort_flag)) break;
        if (ep_tid == 0) {
          const int tile = nt * p.m_tiles + mt;
          const int arrivals = (p.slice_end - p.slice_begin) / p.group;
          const int old = atomicAdd(p.counters + tile, 1);
          *last_flag = (old == arrivals - 1) ? 1 : 0;
          if (old == arrivals - 1) p.counters[tile] = 0;  // ready for the next launch
        }
        if (!epi_sync(ep_bar, ep_phase, abort_flag)) break;
        const bool is_last = *last_flag != 0;
        if (is_last && n_ok) {
          __threadfence();
          const int rows = min(kEpiCols, p.M - m0);
          // 4 rows x 8 slices of independent loads in flight per iteration
          for (int i0 = 0; i0 < rows; i0 += 4) {
            float part[4][kSlices];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const float* src = p.ws + static_cast<int64_t>(m0 + min(i0 + r, rows - 1)) * p.N + n;
#pragma unroll
              for (int s = 0; s < kSlices; ++s) part[r][s] = __ldcg(src + s * MN);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              if (i0 + r < rows) {
                float a = part[r][0];
#pragma unroll
                for (int s = 1; s < kSlices; ++s) a = __fadd_rn(a, part[r][s]);
                C[static_cast<int64_t>(m0 + i0 + r) * p.ldc + n] = from_f32<T>(a);
              }
            }
          }
        }
        // keep last_flag stable until every thread has read it
        if (!epi_sync(ep_bar, ep_phase, abort_flag)) break;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// out[m, n] = fold of 8 slice partials in slice order (row-parallel TP combine).
template <typename T>
__global__ void fold_slices_kernel(const float* __restrict__ partials, T* __restrict__ c, int64_t ldc, int M, int N) {
  const int64_t MN = static_cast<int64_t>(M) * N;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < MN;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = idx / N, n = idx - m * N;
    float a = partials[idx];
#pragma unroll
    for (int s = 1; s < kSlices; ++s) a = __fadd_rn(a, partials[idx + s * MN]);
    c[m * ldc + n] = from_f32<T>(a);
  }
}

// f32 [M][N] -> output dtype (batch-variant twin's final cast).
template <typename T>
__global__ void cast_out_kernel(const float* __restrict__ src, T* __restrict__ c, int64_t ldc, int M, int N) {
  const int64_t MN = static_cast<int64_t>(M) * N;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < MN;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = idx / N, n = idx - m * N;
    c[m * ldc + n] = from_f32<T>(src[idx]);
  }
}

}  // namespace gemm
}  // namespace dk
