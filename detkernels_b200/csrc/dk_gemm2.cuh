// Batch-invariant GEMM on CTA pairs: tcgen05.mma.cta_group::2.
//
// Same output definition as gemm_kernel (dk_gemm.cuh): K in 8 fixed slices,
// each accumulated from zero in its own f32 TMEM accumulator in ascending
// 16-deep steps, the partials summed along the fixed tree.  Only the tile a
// tensor-core instruction covers changes: a pair of CTAs (a cluster of 2)
// computes a 256-weight-column x 128-token tile.  CTA r of the pair owns weight
// columns [256 nt + 128 r, +128) -- its TMEM accumulators hold those 128 columns
// x the tile's 128 tokens, exactly the per-CTA tile of gemm_kernel -- and
// loads its 128 weight columns and token rows [128 mt + 64 r, +64) of every K
// stage.  One instruction (M = 256 weight columns, N = 128 tokens, K = 16),
// issued by the leader CTA, reads both CTAs' shared memory, so each SM moves
// 24 KB per 128 x 128 x 64 of work instead of 32 KB.
//
// Synchronisation (no cluster multicast anywhere):
//   * full[s]  (leader): the leader's producer expects the stage bytes of BOTH
//     CTAs; both CTAs' TMA loads complete on it (cta_group::2 copies addressed
//     to the leader's barrier).
//   * empty[s] (each CTA): the leader's MMA commit arrives on both CTAs' copy.
//   * slot_full[k] (each CTA): accumulator k complete, committed to both CTAs.
//   * slot_free[k] (leader): one arrival per epilogue warp of both CTAs.
// Every wait is bounded (mbar_wait); the pair meets at cluster barriers only
// after every role has finished or given up, so no path can leave a CTA
// waiting for its peer.
#pragma once

#include "dk_gemm.cuh"

namespace dk {
namespace gemm {

constexpr int kPairTileN = 2 * kTileN;                     // weight columns per pair tile
constexpr int kPairRows = kTileM / 2;                      // token rows each CTA loads per stage
constexpr int kPairStageBytes = kWTileBytes + kPairRows * kBK * 2;   // 24 KB, a multiple of 1 KB
constexpr int kPairEpiArrivals = 2 * kEpiWarps;            // slot_free arrivals: every epilogue warp of both CTAs

__host__ __device__ __forceinline__ int pair_stages_for(int mode) {
  const int n = ring_bytes_for(mode) / kPairStageBytes;
  return n < kMaxStages ? n : kMaxStages;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory address of the same variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at cluster address `bar` once this thread's earlier pair MMAs complete.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 2-D tile copy into this CTA's shared memory whose completion is counted on the barrier at
// cluster address `bar` (the leader's).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* m, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// p.n_tiles counts PAIR tiles (256 weight columns); the grid is 2 x pairs, clusters of 2.
template <typename T, int FMT, bool FOLDK>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int n_stages = pair_stages_for(p.mode);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingBytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* slot_full = empty + kMaxStages;
  uint64_t* slot_free = slot_full + kSlots;
  uint64_t* drain_bar = slot_free + kSlots;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = (rank == 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
#pragma unroll
    for (int k = 0; k < kSlots; ++k) {
      mbar_init(&slot_full[k], 1);
      mbar_init(&slot_free[k], kPairEpiArrivals);
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

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      int fills = 0;
      for (int u = pair; u < units && !abort_flag; u += n_pairs) {
        const int g = u % n_groups;
        const int t = u / n_groups;
        int mt, nt;
        tile_coords(p, t, mt, nt);
        const int wcol = nt * kPairTileN + static_cast<int>(rank) * kTileN;
        const int trow = mt * kTileM + static_cast<int>(rank) * kPairRows;
        for (int si = 0; si < p.group && !abort_flag; ++si) {
          const int s = p.slice_begin + g * p.group + si;
          int k0, k1;
          slice_bounds(p, s, k0, k1);
          const int nkb = (k1 - k0 + kBK - 1) / kBK;
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, kDetProdEmpty, abort_flag)) break;
            uint8_t* st = smem + stage * kPairStageBytes;
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * kPairStageBytes);
            const uint32_t bar = cluster_addr(&full[stage], 0);
            const int kl = k0 + kb * kBK - p.k_base;
            tma_load_2d_pair(st, &tmB, bar, wcol, kl);
            tma_load_2d_pair(st + kWBoxBytes, &tmB, bar, wcol + 64, kl);
            tma_load_2d_pair(st + kWTileBytes, &tmA, bar, kl, trow);
            ++fills;
            if (++stage == n_stages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      // Drain (leader): the full barriers count both CTAs' bytes, so their completion means
      // every copy of the pair has landed.  The peer waits for this at the final cluster barrier.
      if (leader) {
        bool drain_abort = false;
        for (int f = (fills > n_stages ? fills - n_stages : 0); f < fills; ++f)
          mbar_wait(&full[f % n_stages], static_cast<uint32_t>((f / n_stages) & 1), kDetDrain, drain_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader, one thread) ----------------
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t use_par = 0;
      int ordinal = 0;
      constexpr uint32_t idesc = umma_idesc_f16(FMT, /*a_mn=*/1, /*b_mn=*/0, kPairTileN, kTileM);
      for (int u = pair; u < units && !abort_flag; u += n_pairs, ++ordinal) {
        const int g = u % n_groups;
        for (int si = 0; si < p.group && !abort_flag; ++si) {
          const int s = p.slice_begin + g * p.group + si;
          int k0, k1;
          slice_bounds(p, s, k0, k1);
          const int nkb = (k1 - k0 + kBK - 1) / kBK;
          const int slot = slot_of(si, ordinal, p.group);
          if (!mbar_wait(&slot_free[slot], ((use_par >> slot) & 1u) ^ 1u, kDetMmaSlotFree, abort_flag)) break;
          use_par ^= 1u << slot;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * kTileM);
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&full[stage], phase, kDetMmaFull, abort_flag)) break;
            tc_fence_after();
            const int kk = k0 + kb * kBK;
            const int nsteps = min(kBK / kUK, (k1 - kk + kUK - 1) / kUK);
            const uint32_t b_base = smem_u32(smem + stage * kPairStageBytes);
            const uint32_t a_base = b_base + kWTileBytes;
            for (int j = 0; j < nsteps; ++j) {
              // weights MN-major (the pair's 256 columns: 128 here, 128 at the same address in the
              // peer); tokens K-major (64 rows here, 64 in the peer)
              const uint64_t bdesc = umma_sdesc(b_base + j * 2048, kWBoxBytes, 1024, 2);
              const uint64_t adesc = umma_sdesc(a_base + j * 32, 16, 1024, 2);
              tc_mma_f16_pair(d_tmem, bdesc, adesc, idesc, (kb > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit_pair(cluster_addr(&empty[stage], 0));
            tc_commit_pair(cluster_addr(&empty[stage], 1));
            if (++stage == n_stages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (abort_flag) break;
          tc_commit_pair(cluster_addr(&slot_full[slot], 0));
          tc_commit_pair(cluster_addr(&slot_full[slot], 1));
        }
      }
      bool drain_abort = false;
      tc_commit_pair(cluster_addr(drain_bar, 0));
      mbar_wait(drain_bar, 0, kDetDrain, drain_abort);
    }
  } else {
    // ---------------- epilogue: 8 warps per CTA, this CTA's 128 weight columns ----------------
    bool abort_flag = false;
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int n_local = quarter * 32 + lane;
    const int col0 = half * kEpiCols;
    uint32_t use_par = 0;
    int ordinal = 0;
    T* C = reinterpret_cast<T*>(p.c);
    float* stage = reinterpret_cast<float*>(smem + kRingBytes - kEpiStageBytes) + (warp - 2) * (32 * kStagePitch);
    const int64_t MN = static_cast<int64_t>(p.M) * p.N;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(col0);
    // one arrival per warp on the leader's slot_free, after every lane's TMEM reads
    auto release = [&](int s) {
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&slot_free[s], 0));
    };
    for (int u = pair; u < units && !abort_flag; u += n_pairs, ++ordinal) {
      const int g = u % n_groups;
      const int t = u / n_groups;
      int mt, nt;
      tile_coords(p, t, mt, nt);
      const int n_first = nt * kPairTileN + static_cast<int>(rank) * kTileN;
      const int n = n_first + n_local;
      const int m0 = mt * kTileM + col0;
      const bool n_ok = n < p.N;
      Params q = p;
      if (p.mode == SPLIT) q.ws = p.ws + static_cast<int64_t>(g) * MN;
      uint32_t stack = 0;
      for (int si = 0; si < p.group; ++si) {
        const int s = p.slice_begin + g * p.group + si;
        int k0, k1;
        slice_bounds(p, s, k0, k1);
        const bool empty_slice = (k1 <= k0);
        const int slot = slot_of(si, ordinal, p.group);
        if (!mbar_wait(&slot_full[slot], (use_par >> slot) & 1u, kDetEpiSlotFull, abort_flag)) break;
        use_par ^= 1u << slot;
        tc_fence_after();
        const int nlev = __ffs(~si) - 1;
        const bool last = (si + 1 == p.group);
        const uint32_t x_addr = lane_base + static_cast<uint32_t>(slot * kTileM);
        if (nlev == 0 && !last) {
          if (empty_slice) {
            float z[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) z[j] = 0.0f;
#pragma unroll
            for (int c = 0; c < kEpiCols / 32; ++c) tmem_st_32x32b_x32(x_addr + c * 32, z);
            tmem_st_wait();
          }
          stack = (stack & ~3u) | static_cast<uint32_t>(slot);
          continue;
        }
        const int res_slot = (nlev > 0) ? static_cast<int>((stack >> (2 * (nlev - 1))) & 3u) : slot;
#pragma unroll 1
        for (int c = 0; c < kEpiCols / 32; ++c) {
          float acc[32];
          if (empty_slice) {
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
          } else {
            tmem_ld_32x32b_x32(x_addr + c * 32, acc);
            tmem_ld_wait();
          }
#pragma unroll 1
          for (int l = 0; l < nlev; ++l) {
            float left[32];
            const uint32_t ls = (stack >> (2 * l)) & 3u;
            tmem_ld_32x32b_x32(lane_base + ls * kTileM + c * 32, left);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(left[j], acc[j]);
          }
          if (last) {
            if constexpr (FOLDK) {
              emit_rows<T>(q, C, stage, p.mode, n_first + quarter * 32, m0 + c * 32, acc);
            } else {
              emit_chunk<T>(q, C, p.mode, n, n_ok, m0 + c * 32, acc);
            }
          } else {
            tmem_st_32x32b_x32(lane_base + static_cast<uint32_t>(res_slot * kTileM) + c * 32, acc);
          }
        }
        if (!last) tmem_st_wait();
        tc_fence_before();
        if (nlev > 0) release(slot);
        for (int l = 0; l + 1 < nlev; ++l) release(static_cast<int>((stack >> (2 * l)) & 3u));
        if (last) release(res_slot);
        if (!last) stack = (stack & ~(3u << (2 * nlev))) | (static_cast<uint32_t>(res_slot) << (2 * nlev));
      }
      if (abort_flag) break;
    }
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
