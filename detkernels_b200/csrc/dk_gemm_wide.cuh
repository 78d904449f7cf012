// Batch-invariant GEMM on CTA pairs with 256 x 256 tiles (tcgen05.mma.cta_group::2, N = 256).
//
// Same output definition as gemm_kernel (dk_gemm.cuh): K in 8 fixed slices, each
// accumulated from zero in its own f32 TMEM accumulator in ascending 16-deep steps, the
// partials summed along the fixed tree ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)).  Only the tile
// one instruction covers changes (an output element's bits depend neither on the
// instruction's N nor on its CTA group).
//
// Why this shape: a pair tile of 256 weight columns x 256 tokens moves, per SM and per
// 16-deep step, 4 KB of weights (the CTA's 128 columns) and 4 KB of tokens (the CTA's 128
// rows) for 128 x 256 x 16 of work -- 64 bytes per tensor-core cycle instead of the 128 of
// the one-CTA 128 x 128 tile.  TMA delivery into shared memory (about 55-70 bytes per cycle
// per SM with every SM streaming) is what bounds the smaller tile.
//
// Operand roles: the 256 tokens of a pair tile are the instruction's M (each CTA's 128 token
// rows are its TMEM lanes) and the 256 weight columns its N, so an epilogue thread owns one
// token row of consecutive output columns and stores it without a transpose.  (The one-CTA
// kernel puts weights on M instead, so that a few decode tokens still fill the instruction;
// which operand is A does not change an output element's bits.)
//
// Accumulators: one slice partial of the CTA's 128 tokens x 256 columns takes 256 TMEM
// columns, so TMEM holds two (slots X and Y, used alternately).  The tree needs up to four
// live values, so the pending left operands live elsewhere:
//   * R: the epilogue threads' registers (thread = one TMEM lane x 128 weight columns,
//     128 f32 registers), holding p0 / p0+p1 (and p4 / p4+p5);
//   * p2 (p6) stays in its slot until p3 (p7) arrives;
//   * S: the 8-slice unit's left half (p0+p1)+(p2+p3), parked in a global stash (L2) while
//     the right half is computed: 128 KB per CTA per unit, written once and read once.
// Order of the sums (the tree exactly):
//   si 0: R = p0            si 1: R = R + p1          si 2: keep p2
//   si 3: R = R + (p2 + p3) [group 4: final; group 8: S = R]
//   si 4: R = p4            si 5: R = R + p5          si 6: keep p6
//   si 7: R = R + (p6 + p7); final = S + R
// Groups of 1 and 2 (SPLIT launches) end at si 0 / si 1.
//
// Registers: warpgroup 0 (TMA producer, MMA issuer, two idle warps) gives registers back
// with setmaxnreg.dec, the two epilogue warpgroups take them with setmaxnreg.inc.  The
// launch gives every thread kWideLaunchRegs; the host refuses to launch a build whose
// register count differs (the split below is exact only for that count).
//
// Synchronisation (no multicast data copy anywhere): full[s] (leader) counts both CTAs' stage
// bytes; empty[s] (each CTA) gets the leader's MMA commit, one commit signalled to both CTAs;
// slot_full[k] (each CTA) likewise when accumulator k is complete; slot_free[k] (leader) takes
// one arrival per epilogue warp of both CTAs.  Every wait is bounded.
#pragma once

#include "dk_gemm2.cuh"

namespace dk {
namespace gemm {

constexpr int kWideTileN = 256;                        // weight columns per pair tile (UMMA M)
constexpr int kWideTileM = 256;                        // tokens per pair tile (UMMA N)
constexpr int kWideRows = kWideTileM / 2;              // token rows each CTA loads per stage
constexpr int kWideSub = 2;                            // 64-deep K sub-blocks per stage
constexpr int kWideBK = kWideSub * kBK;                // K per stage (128)
constexpr int kWideSubBytes = kWTileBytes + kWideRows * kBK * 2;   // 32 KB: 128 columns + 128 rows x 64 k
constexpr int kWideStageBytes = kWideSub * kWideSubBytes;          // 64 KB
constexpr int kWideSlotCols = kWideTileM;              // TMEM columns per accumulator slot
constexpr int kWideSlots = 2;
constexpr int kWideEpiWarps = 8;                       // two warpgroups, two warps per lane quarter
constexpr int kWideThreads = 128 + 32 * kWideEpiWarps; // 384
constexpr int kWideEpiCols = kWideTileM / 2;           // token columns per epilogue thread (128)
constexpr int kWideChunks = kWideEpiCols / 32;         // 4 chunks of 32 columns
constexpr int kWideEpiArrivals = 2 * kWideEpiWarps;    // slot_free arrivals: epilogue warps of both CTAs
constexpr int kWideRingBytes = kSmemBytes - 1024 - kBarrierBytes;
constexpr int kWideStages = kWideRingBytes / kWideStageBytes;   // 3 (6 of one sub-block)
constexpr int kWideLaunchRegs = 168;                   // 65536 / 384, rounded down to 8
constexpr int kWideProducerRegs = 56;
constexpr int kWideEpiRegs = 224;                      // 128 x 56 + 256 x 224 = 384 x 168
constexpr int kWideStashFloats = 128 * kWideTileM;     // per CTA: 128 columns x 256 tokens
static_assert(kWideStages * kWideSub >= 6, "wide GEMM ring too shallow");
static_assert(128 * kWideProducerRegs + 32 * kWideEpiWarps * kWideEpiRegs == kWideThreads * kWideLaunchRegs,
              "register split must add up to the launch allocation");

// One commit that arrives on the barrier at this CTA-relative shared-memory address in BOTH CTAs
// of the pair once the leader's earlier MMAs complete (a completion signal, not a data copy;
// measured 18 % faster for the whole GEMM than two commits addressed to one CTA each).
__device__ __forceinline__ void tc_commit_both(const uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// Arrive (relaxed) on the mbarrier at cluster shared-memory address `addr`.
__device__ __forceinline__ void mbar_arrive_relaxed_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}

template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Unit u of the pair's work list -> (slice group g, pair tile t); tile -> (m-tile, n-tile)
// with p.n_tiles / p.m_tiles counting 256-wide tiles.
__device__ __forceinline__ void wide_unit(const Params& p, int u, int n_groups, int& g, int& mt, int& nt) {
  g = u % n_groups;
  tile_coords(p, u / n_groups, mt, nt);
}

// 32 columns (chunk c) of slot `slot` for this thread's lane, or zeros for an empty slice.
__device__ __forceinline__ void wide_ld(uint32_t lane_base, int slot, int c, bool empty, float (&v)[32]) {
  if (empty) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = 0.0f;
  } else {
    tmem_ld_32x32b_x32(lane_base + static_cast<uint32_t>(slot * kWideSlotCols + c * 32), v);
  }
}

// Final values (or, for SPLIT / PARTIAL, this unit's subtree sum) of one token row m, columns
// n_base .. n_base + 31 -> memory.  The thread owns the row, so no transpose is needed.  ARGMAX
// only folds the chunk into the thread's running key (one atomic per row per unit, after the
// last chunk).
template <typename T, bool FOLDK>
__device__ __forceinline__ void wide_emit(const Params& q, float* ws, T* C, int m, int n_base, const float (&v)[32],
                                          unsigned long long& best) {
  const int ncols = min(32, q.N - n_base);
  if (m >= q.M || ncols <= 0) return;
  if constexpr (FOLDK) {
    if (q.epi.mode == DK_EPI_ARGMAX) {
      const unsigned long long key = argmax_chunk_key<T>(v, ncols, n_base);
      best = key > best ? key : best;
      if (C) {
        float w[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) w[k] = v[k];
        T* dst = C + static_cast<int64_t>(m) * q.ldc + n_base;
        if (ncols == 32 && aligned_row<T>(C, q.ldc, n_base)) {
          store_row_vec<T>(dst, w, 32);
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (k < ncols) dst[k] = from_f32<T>(w[k]);
        }
      }
      return;
    }
    float w[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) w[k] = v[k];
    store_final_row<T>(q, C, m, n_base, ncols, w);
  } else {
    // SPLIT (ws already offset to this unit's group) or PARTIAL: the f32 subtree sum
    (void)C;
    (void)best;
    float* dst = ws + static_cast<int64_t>(m) * q.N + n_base;
    if (ncols == 32 && (q.N % 4) == 0) {
#pragma unroll
      for (int k = 0; k < 32; k += 4) *reinterpret_cast<float4*>(dst + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k)
        if (k < ncols) dst[k] = v[k];
    }
  }
}

// The epilogue warpgroups (warps 4..11).  Warp w reads TMEM lane quarter w % 4; the two warps
// of a quarter split the 256 weight columns into halves.  Thread <-> TMEM lane <-> token row.
template <typename T, bool FOLDK>
__device__ __forceinline__ void wide_epilogue(const Params& p, uint64_t* slot_full, uint64_t* slot_free,
                                              uint32_t tmem_base, int units, int n_groups, int pair, int n_pairs,
                                              uint32_t rank) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ew = warp - 4;
  const int quarter = warp & 3;
  const int half = ew >> 2;
  const int m_local = static_cast<int>(rank) * kWideRows + quarter * 32 + lane;   // token row in the pair tile
  const int col0 = half * kWideEpiCols;
  T* C = reinterpret_cast<T*>(p.c);
  const int64_t MN = static_cast<int64_t>(p.M) * p.N;
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(col0);
  // this thread's 128 stash floats as 32 float4: [half][chunk][quad][lane of the CTA's 128 rows],
  // so a warp's 16-byte accesses cover 512 contiguous bytes
  float4* stash = reinterpret_cast<float4*>(p.stash + static_cast<int64_t>(blockIdx.x) * kWideStashFloats) +
                  half * (kWideChunks * 8 * 128) + quarter * 32 + lane;
  auto release = [&](int s) {
    __syncwarp();
    // relaxed: the TMEM reads are complete (tcgen05.wait::ld); release semantics would also wait
    // for this thread's global stores, which the MMA issuer does not depend on
    if (lane == 0) mbar_arrive_relaxed_cluster(cluster_addr(&slot_free[s], 0));
  };
  bool abort_flag = false;
  uint32_t cnt = 0;
  float R[kWideChunks][32];
#pragma unroll 1
  for (int u = pair; u < units && !abort_flag; u += n_pairs) {
    int g, mt, nt;
    wide_unit(p, u, n_groups, g, mt, nt);
    const int m = mt * kWideTileM + m_local;
    const int n0 = nt * kWideTileN + col0;
    float* ws = (p.mode == SPLIT) ? p.ws + static_cast<int64_t>(g) * MN : p.ws;
    int prev_slot = 0;
    bool prev_empty = false;
#pragma unroll 1
    for (int si = 0; si < p.group; ++si) {
      const int s = p.slice_begin + g * p.group + si;
      int k0, k1;
      slice_bounds(p, s, k0, k1);
      const bool empty = (k1 <= k0);
      const int slot = static_cast<int>(cnt & 1u);
      const uint32_t par = (cnt >> 1) & 1u;
      ++cnt;
      if (!mbar_wait(&slot_full[slot], par, kDetEpiSlotFull, abort_flag)) break;
      tc_fence_after();
      const int kind = si & 3;
      if (kind == 0) {
        // R = p0 (p4)
#pragma unroll
        for (int c = 0; c < kWideChunks; ++c) wide_ld(lane_base, slot, c, empty, R[c]);
        tmem_ld_wait();
        tc_fence_before();
        release(slot);
      } else if (kind == 1) {
        // R = R + p1 (p5)
#pragma unroll
        for (int c = 0; c < kWideChunks; ++c) {
          float x[32];
          wide_ld(lane_base, slot, c, empty, x);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) R[c][j] = __fadd_rn(R[c][j], x[j]);
        }
        tc_fence_before();
        release(slot);
      } else if (kind == 2) {
        // p2 (p6) waits in its slot for p3 (p7)
        prev_slot = slot;
        prev_empty = empty;
        continue;
      } else {
        // R = R + (p2 + p3)   (R + (p6 + p7))
#pragma unroll
        for (int c = 0; c < kWideChunks; ++c) {
          float x[32], y[32];
          wide_ld(lane_base, prev_slot, c, prev_empty, x);
          wide_ld(lane_base, slot, c, empty, y);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) R[c][j] = __fadd_rn(R[c][j], __fadd_rn(x[j], y[j]));
        }
        tc_fence_before();
        release(prev_slot);
        release(slot);
        if (si == 3 && p.group == 8) {
          // the left half of the tree waits in the stash while the right half is computed
#pragma unroll
          for (int c = 0; c < kWideChunks; ++c)
#pragma unroll
            for (int j = 0; j < 8; ++j)
              __stcg(stash + (c * 8 + j) * 128, make_float4(R[c][4 * j], R[c][4 * j + 1], R[c][4 * j + 2], R[c][4 * j + 3]));
        }
      }
      if (si + 1 == p.group) {
        unsigned long long best = 0ull;
        if (p.group == 8) {
          // final = S + R: the stash is read two chunks at a time, all of it before any store,
          // so its L2 round trips overlap instead of one per chunk between the stores
#pragma unroll
          for (int c = 0; c < kWideChunks; c += 2) {
            float4 s0[8], s1[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              s0[j] = __ldcg(stash + (c * 8 + j) * 128);
              s1[j] = __ldcg(stash + ((c + 1) * 8 + j) * 128);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              R[c][4 * j] = __fadd_rn(s0[j].x, R[c][4 * j]);
              R[c][4 * j + 1] = __fadd_rn(s0[j].y, R[c][4 * j + 1]);
              R[c][4 * j + 2] = __fadd_rn(s0[j].z, R[c][4 * j + 2]);
              R[c][4 * j + 3] = __fadd_rn(s0[j].w, R[c][4 * j + 3]);
              R[c + 1][4 * j] = __fadd_rn(s1[j].x, R[c + 1][4 * j]);
              R[c + 1][4 * j + 1] = __fadd_rn(s1[j].y, R[c + 1][4 * j + 1]);
              R[c + 1][4 * j + 2] = __fadd_rn(s1[j].z, R[c + 1][4 * j + 2]);
              R[c + 1][4 * j + 3] = __fadd_rn(s1[j].w, R[c + 1][4 * j + 3]);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < kWideChunks; ++c) wide_emit<T, FOLDK>(p, ws, C, m, n0 + c * 32, R[c], best);
        if constexpr (FOLDK) {
          if (p.epi.mode == DK_EPI_ARGMAX && best != 0ull) atomicMax(p.epi.argmax_keys + m, best);
        }
      }
    }
  }
}

// p.n_tiles / p.m_tiles count 256-wide pair tiles; the grid is 2 x pairs, clusters of 2.
// p.stash: kWideStashFloats floats per CTA of the grid (used by 8-slice units only).
template <typename T, int FMT, bool FOLDK>
__global__ void __launch_bounds__(kWideThreads, 1)
    gemm_wide_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWideRingBytes);
  uint64_t* empty = full + kWideStages;
  uint64_t* slot_full = empty + kWideStages;
  uint64_t* slot_free = slot_full + kWideSlots;
  uint64_t* drain_bar = slot_free + kWideSlots;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = (rank == 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWideStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
#pragma unroll
    for (int k = 0; k < kWideSlots; ++k) {
      mbar_init(&slot_full[k], 1);
      mbar_init(&slot_free[k], kWideEpiArrivals);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmA);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync_all();   // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
  const uint32_t tmem_base = *tmem_holder;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();

  const int n_groups = (p.slice_end - p.slice_begin) / p.group;
  const int units = p.n_tiles * p.m_tiles * n_groups;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int n_pairs = static_cast<int>(gridDim.x >> 1);

  if (warp < 4) {
    // The register split comes first in each role's branch, before any wait: warpgroup 0
    // gives back what the epilogue warpgroups take, so the increase can always be granted.
    regs_dec<kWideProducerRegs>();
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      int fills = 0;
      for (int u = pair; u < units && !abort_flag; u += n_pairs) {
        int g, mt, nt;
        wide_unit(p, u, n_groups, g, mt, nt);
        const int wcol = nt * kWideTileN + static_cast<int>(rank) * kTileN;
        const int trow = mt * kWideTileM + static_cast<int>(rank) * kWideRows;
        for (int si = 0; si < p.group && !abort_flag; ++si) {
          const int s = p.slice_begin + g * p.group + si;
          int k0, k1;
          slice_bounds(p, s, k0, k1);
          const int nkb = (k1 - k0 + kWideBK - 1) / kWideBK;
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, kDetProdEmpty, abort_flag)) break;
            uint8_t* st = smem + stage * kWideStageBytes;
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kWideStageBytes);
            const uint32_t bar = cluster_addr(&full[stage], 0);
            // every sub-block is loaded, also one past the slice's end (its MMAs are not issued;
            // past K the copy reads zeros), so the byte count never varies
#pragma unroll
            for (int sb = 0; sb < kWideSub; ++sb) {
              const int kl = k0 + kb * kWideBK + sb * kBK - p.k_base;
              uint8_t* sst = st + sb * kWTileBytes;
              tma_load_2d_pair(sst, &tmB, bar, wcol, kl);
              tma_load_2d_pair(sst + kWBoxBytes, &tmB, bar, wcol + 64, kl);
              tma_load_2d_pair(st + kWideSub * kWTileBytes + sb * kWideRows * kBK * 2, &tmA, bar, kl, trow);
            }
            ++fills;
            if (++stage == kWideStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      // Drain (leader): the full barriers count both CTAs' bytes.  The peer waits for this at
      // the final cluster barrier.
      if (leader) {
        bool drain_abort = false;
        for (int f = (fills > kWideStages ? fills - kWideStages : 0); f < fills; ++f)
          mbar_wait(&full[f % kWideStages], static_cast<uint32_t>((f / kWideStages) & 1), kDetDrain, drain_abort);
      }
    }
    if (warp == 1 && lane == 0 && leader) {
      // ---------------- MMA issuer (leader, one thread) ----------------
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t cnt = 0;   // slice partials issued; slot = cnt & 1
      // A = tokens (K-major, 128 rows in each CTA: UMMA M = 256 tokens, TMEM lanes), B = weights
      // (MN-major, 128 columns in each CTA: UMMA N = 256 columns)
      constexpr uint32_t idesc = umma_idesc_f16(FMT, /*a_mn=*/0, /*b_mn=*/1, kWideTileM, kWideTileN);
      for (int u = pair; u < units && !abort_flag; u += n_pairs) {
        const int g = u % n_groups;
        for (int si = 0; si < p.group && !abort_flag; ++si) {
          const int s = p.slice_begin + g * p.group + si;
          int k0, k1;
          slice_bounds(p, s, k0, k1);
          const int nkb = (k1 - k0 + kWideBK - 1) / kWideBK;
          const int slot = static_cast<int>(cnt & 1u);
          const uint32_t use = (cnt >> 1) & 1u;
          ++cnt;
          if (!mbar_wait(&slot_free[slot], use ^ 1u, kDetMmaSlotFree, abort_flag)) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * kWideSlotCols);
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&full[stage], phase, kDetMmaFull, abort_flag)) break;
            tc_fence_after();
            const int kk = k0 + kb * kWideBK;
            const int nsteps = min(kWideBK / kUK, (k1 - kk + kUK - 1) / kUK);
            const uint32_t b_base = smem_u32(smem + stage * kWideStageBytes);
            const uint32_t a_base = b_base + kWideSub * kWTileBytes;
            for (int j = 0; j < nsteps; ++j) {
              // weights MN-major (128 columns here, 128 at the same address in the peer); tokens
              // K-major (128 rows here, 128 in the peer); sub-block j / 4, K step j % 4 inside it
              const int sb = j >> 2, jj = j & 3;
              const uint64_t bdesc = umma_sdesc(b_base + sb * kWTileBytes + jj * 2048, kWBoxBytes, 1024, 2);
              const uint64_t adesc = umma_sdesc(a_base + sb * (kWideRows * kBK * 2) + jj * 32, 16, 1024, 2);
              tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit_both(&empty[stage]);
            if (++stage == kWideStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (abort_flag) break;
          tc_commit_both(&slot_full[slot]);
        }
      }
      bool drain_abort = false;
      tc_commit_pair(cluster_addr(drain_bar, 0));
      mbar_wait(drain_bar, 0, kDetDrain, drain_abort);
    }
  } else {
    regs_inc<kWideEpiRegs>();
    wide_epilogue<T, FOLDK>(p, slot_full, slot_free, tmem_base, units, n_groups, pair, n_pairs, rank);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();   // the leader's MMAs and copies drained, both epilogues done with TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace gemm
}  // namespace dk
