// Batch-invariant split-KV decode attention.
//
// Replaces kernels/attention.py:86-143 (_attn_direct_kernel) behind
// attention_batch_invariant (attention.py:289-298), extended with grouped
// query heads (GQA), per-row KV lengths and multi-row tiles (prefill rows of
// one sequence processed together with exactly the per-row arithmetic of a
// decode step).
//
// Fixed reduction structure (the definition of the output bits of a row):
//   * The row's KV tokens [0, kv_len) are cut into splits of DK_ATTN_KV_SPLIT
//     = 256 tokens (a fixed SIZE, so the split count follows the row's own
//     length and nothing else).
//   * Inside a split, tokens are visited in blocks of 64; warp w of the CTA
//     always owns tokens [16w, 16w+16) of every block and keeps its own
//     online-softmax state (running max m, running sum l, f32 accumulator O).
//     Scores come from mma.m16n8k16 (bf16/f16 in, f32 accumulate) with the q
//     vector as one of the 16 MMA rows; probabilities are rounded to the input
//     type for the P.V product and the same rounded values are summed into l.
//   * The four warp states of a split are merged in warp order 0..3 with
//     weights exp2(m_w - max_w m_w) into the split's (m, l, O).
//   * The split states are merged in split order by a running (online) merge:
//     m' = max(m, m_s); (l, O) <- (l, O) * exp2(m - m') + (l_s, O_s) * exp2(m_s - m');
//     out = O / l.
// A row's arithmetic therefore depends on its q, its KV sequence and its
// kv_len only -- not on the batch, the other rows of its tile, or the grid.
//
// Work decomposition: a work item is (row tile, kv head, run of up to `spu`
// consecutive splits).  The grid is persistent (as many CTAs as fit on the GPU
// at once) and CTA b takes items b, b + grid, ...  A producer warp streams
// 64-token K/V blocks with TMA (4-D tensor map over the cache, 128- or 64-byte
// swizzle) into a ring of shared-memory stages that keeps flowing across split
// AND item boundaries, so the next item's first blocks are in flight while the
// current one finishes; four consumer warps compute.  When an item covers all of
// a tile's splits it merges them as it goes and writes the output; otherwise each
// item writes its splits' (m, l, O) to the workspace and the last to arrive
// (atomic counter, no spinning) replays the same split-order merge over them.
// Which CTA computes an item never changes the arithmetic.
#pragma once

#include "dk_common.cuh"

namespace dk {
namespace attn {

constexpr int kSplit = DK_ATTN_KV_SPLIT;
constexpr int kBlock = 64;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr int kRows = 16;
constexpr int kItemSlots = 2;   // work items staged ahead of the consumers
constexpr int kItemInts = 32;   // ints per staged item: description [0, 11), kv lengths [16, 32)

// ONE: the single-row (transposed) instances, which run 4 CTAs per SM for d <= 64 on a
// 3-stage ring (measured 3 % faster than 3 CTAs on 4 stages).
template <int D, bool ONE = false>
struct Cfg {
  static_assert(D == 32 || D == 64 || D == 128, "head_dim");
  static constexpr int BOXD = D < 64 ? D : 64;          // elements per TMA box row
  static constexpr int NBOX = D / BOXD;                 // boxes per tensor per block
  static constexpr int ROWB = BOXD * 2;                 // bytes per token row in a box
  static constexpr int CPB = ROWB / 16;                 // 16-byte chunks per box row
  static constexpr int BOX_BYTES = kBlock * ROWB;
  static constexpr int TENSOR_BYTES = NBOX * BOX_BYTES;  // 64 tokens x D
  static constexpr int STAGE_BYTES = 2 * TENSOR_BYTES;   // K block + V block
  static constexpr int STAGES = (D == 128 || ONE) ? 3 : 4;
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  static constexpr int CSTRIDE = D + 8;                  // padded row of the warp-merge buffer (floats)
  static constexpr int KMAX = (kRows * D + kConsumerWarps * 32 - 1) / (kConsumerWarps * 32);
  // dynamic shared memory for a launch whose tiles hold up to `rows` mma rows
  static __host__ __device__ int smem_bytes(int rows) {
    return 1024 + RING_BYTES + kConsumerWarps * rows * (CSTRIDE + 2) * 4 + 512 +
           kItemSlots * (kItemInts * 4 + rows * D * 2 + 16) + 128;
  }
};

struct Params {
  const void* q;
  int64_t q_sr, q_sh;
  void* out;
  int64_t o_sr, o_sh;
  const int32_t* kv_lens;
  int32_t uniform_len;
  const int32_t* tiles;
  int32_t n_tiles;
  int32_t rows_cap;   // mma rows per tile (workspace rows and merge-buffer rows) = rows_per_tile * G
  int32_t n_rows, hq, hkv, G;
  int32_t max_splits;
  int32_t spu;        // splits per CTA
  int32_t upt;        // CTAs per (tile, kv head) = ceil(max_splits / spu)
  int32_t kv_capacity;
  int32_t kv_n_seq;
  // paged KV (block_table != null): the tensor maps cover a block pool [n_blocks, hkv, page, d];
  // token t of sequence s lives in block block_table[s * bt_stride + t / page] at t % page
  const int32_t* block_table;
  int64_t bt_stride;
  int32_t page;       // tokens per block, a multiple of kBlock
  int32_t n_blocks;
  float scale_log2;   // softmax scale * log2(e)
  float* ws_o;        // [n_tiles][hkv][max_splits][rows_cap][D]
  float* ws_ml;       // [n_tiles][hkv][max_splits][rows_cap][2]
  int32_t* counters;  // [n_tiles][hkv]
};

// K and V tensor maps: 64-token boxes for whole blocks and 16-token boxes for the tail of a
// split whose end falls inside a block, so a row's last block moves only the 16-token groups it
// needs (a row of ~330 tokens otherwise fetches ~10 % beyond its end).
struct KvMaps {
  CUtensorMap k, v, k16, v16;
};
constexpr int kTailRows = 16;

enum : int {
  kDetProdEmpty = 0x200,
  kDetFull = 0x201,
  kDetSync = 0x202,
  kDetDrain = 0x203,
  kDetItem = 0x204,
  kDetLen = 0x210,   // a kv_len exceeds the cache capacity or max_kv_len
  kDetTile = 0x211,  // a row tile is malformed
  kDetPage = 0x212,  // a block table entry outside the block pool
};

// TMA coordinates (token, slab) of the 64-token block starting at token t0 of sequence seq:
// (t0, seq) for a contiguous cache; (t0 mod page, block) through the block table for a paged
// one.  A table entry outside the pool is recorded (DK_ERR_DEVICE_CHECK) and replaced by block 0,
// so the copy always stays inside the pool.
__device__ __forceinline__ void kv_block_coords(const Params& p, int seq, int t0, int& tok, int& slab) {
  if (p.block_table == nullptr) {
    tok = t0;
    slab = seq;
    return;
  }
  const int pg = t0 / p.page;
  tok = t0 - pg * p.page;
  slab = p.block_table[static_cast<int64_t>(seq) * p.bt_stride + pg];
  if (slab < 0 || slab >= p.n_blocks) {
    report_error(DK_ERR_DEVICE_CHECK, kDetPage);
    slab = 0;
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The low / high 16-bit element of a packed pair as f32.
template <typename T>
__device__ __forceinline__ float lo_f32(uint32_t v);
template <typename T>
__device__ __forceinline__ float hi_f32(uint32_t v);
template <>
__device__ __forceinline__ float lo_f32<__nv_bfloat16>(uint32_t v) { return __uint_as_float(v << 16); }
template <>
__device__ __forceinline__ float hi_f32<__nv_bfloat16>(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
template <>
__device__ __forceinline__ float lo_f32<__half>(uint32_t v) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xffffu)));
}
template <>
__device__ __forceinline__ float hi_f32<__half>(uint32_t v) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
}

// Round two probabilities to the input type, pack them, and return the rounded values.
template <typename T>
__device__ __forceinline__ uint32_t pack_round(float lo, float hi, float& rlo, float& rhi);
template <>
__device__ __forceinline__ uint32_t pack_round<__nv_bfloat16>(float lo, float hi, float& rlo, float& rhi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  rlo = __low2float(v);
  rhi = __high2float(v);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack_round<__half>(float lo, float hi, float& rlo, float& rhi) {
  __half2 v = __floats2half2_rn(lo, hi);
  rlo = __low2float(v);
  rhi = __high2float(v);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Shared-memory address of 16-byte chunk `c` (along d) of token row `r` inside
// one tensor block of a stage, following the TMA swizzle of the box.
template <int D>
__device__ __forceinline__ uint32_t chunk_addr(uint32_t tensor_base, int r, int c) {
  using C = Cfg<D>;
  const int box = c / C::CPB;
  const int cc = c % C::CPB;
  const int swz = (C::ROWB == 128) ? (r & 7) : ((r >> 1) & 3);
  return tensor_base + box * C::BOX_BYTES + r * C::ROWB + ((cc ^ swz) << 4);
}

// Bounded barrier among the 128 consumer threads.
__device__ __forceinline__ bool csync(uint64_t* bar, uint32_t& phase, bool& abort_flag) {
  if (abort_flag) return false;
  mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase, kDetSync, abort_flag);
  phase ^= 1u;
  return ok;
}

// 2^x with the single-instruction hardware approximation (relative error < 2^-22);
// 2^-inf = +0 and 2^0 = 1 exactly.  Every weight of the softmax and of both merges
// goes through this one function.
__device__ __forceinline__ float exp2_hw(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float weight_of(float m, float mref) {
  // exp2(m - mref); m == -inf gives 0.
  return exp2_hw(__fsub_rn(m, mref));
}

// One step of the split-order merge: (m, l, o) <- merge((m, l, o), (ms, ls, os)).
// `first` starts the merge with split 0's state.
__device__ __forceinline__ void merge_split(bool first, float& m, float& l, float& o, float ms, float ls, float os) {
  if (first) {
    m = ms;
    l = ls;
    o = os;
    return;
  }
  const float mn = fmaxf(m, ms);
  const float mref = (mn == -INFINITY) ? 0.0f : mn;
  const float a = weight_of(m, mref), b = weight_of(ms, mref);
  l = __fadd_rn(__fmul_rn(l, a), __fmul_rn(ls, b));
  o = __fadd_rn(__fmul_rn(o, a), __fmul_rn(os, b));
  m = mn;
}

// One work item: a row tile, a run of consecutive splits of it, and a kv head.
struct Item {
  int tile, unit, kvh;
  int r0, nr, seq;
  int max_len, nsplits, s_begin, s_end;
};

// Decode item w (tile-major, kv head fastest).  Returns 0 for work, 1 when the item's
// split run is past the tile's last split or the tile is empty (nsplits == 0), 2 for a
// malformed tile, 3 for a length outside the cache.  Every warp computes the same
// answer from the same memory.
__device__ __forceinline__ int describe_item(const Params& p, int64_t w, Item& it) {
  const int64_t tu = w / p.hkv;
  it.kvh = static_cast<int>(w - tu * p.hkv);
  it.tile = static_cast<int>(tu / p.upt);
  it.unit = static_cast<int>(tu - static_cast<int64_t>(it.tile) * p.upt);
  if (p.tiles != nullptr) {
    it.r0 = p.tiles[3 * it.tile + 0];
    it.nr = p.tiles[3 * it.tile + 1];
    it.seq = p.tiles[3 * it.tile + 2];
  } else {
    it.r0 = it.tile;
    it.nr = 1;
    it.seq = it.tile;
  }
  it.max_len = 0;
  it.nsplits = 0;
  it.s_begin = it.s_end = 0;
  const int rows_per_tile_max = kRows / p.G;
  if (it.nr < 1 || it.nr > rows_per_tile_max || it.r0 < 0 || it.r0 + it.nr > p.n_rows || it.seq < 0 ||
      it.seq >= p.kv_n_seq || it.nr * p.G > p.rows_cap)
    return 2;
  for (int i = 0; i < it.nr; ++i) {
    const int L = p.kv_lens ? p.kv_lens[it.r0 + i] : p.uniform_len;
    if (L < 0 || L > p.kv_capacity || L > p.max_splits * kSplit) return 3;
    it.max_len = max(it.max_len, L);
  }
  it.nsplits = (it.max_len + kSplit - 1) / kSplit;
  it.s_begin = it.unit * p.spu;
  it.s_end = min(it.s_begin + p.spu, it.nsplits);
  return (it.nsplits == 0 || it.s_begin >= it.nsplits) ? 1 : 0;
}

// KM: merge elements per consumer thread (ceil(rows x D / 128)); decode launches
// without row tiles have at most G rows and use a narrow instance.
// T1: launches whose tiles hold one mma row (rows_cap == 1: decode without grouped
// query heads).  The products are formed transposed -- S^T = K q^T and O^T = V^T P^T,
// the 16 tokens of a warp as the MMA's M dimension instead of 15 idle query rows --
// which halves the MMAs and the accumulator.  Every sum keeps the 16-row form's
// operands and order (per token the same 16-deep MMA dot products over the same
// k steps; l from the same four tokens per lane, (p0 + p1) + (p2 + p3), and the
// same butterfly), so a row's bits are those of the 16-row form.
// Occupancy: 3 CTAs per SM for d <= 64, except the wide multi-row (prefill) instances
// (KM >= 8), which run 2 per SM without register spills, and the single-row instances,
// 4 per SM (both measured faster).
template <typename T, int D, int KM, bool T1>
__global__ void __launch_bounds__(kThreads, (D == 128 || (!T1 && KM >= 8)) ? 2 : (T1 ? 4 : 3))
    attn_kernel(const __grid_constant__ KvMaps maps, const Params p) {
  using C = Cfg<D, T1>;
  static_assert(KM <= C::KMAX, "merge elements per thread");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* comb_o = reinterpret_cast<float*>(ring + C::RING_BYTES);               // [4][rows_cap][CSTRIDE]
  float* comb_ml = comb_o + kConsumerWarps * p.rows_cap * C::CSTRIDE;          // [4][rows_cap][2]
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(comb_ml + kConsumerWarps * p.rows_cap * 2) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + C::STAGES;
  uint64_t* cbar = empty + C::STAGES;
  int* s_misc = reinterpret_cast<int*>(cbar + 1);  // [0] last-arriver flag
  // item ring: per slot the item description and its rows' kv lengths, and the tile's q rows
  int* islot = s_misc + 16;                                                  // [kItemSlots][kItemInts]
  T* iq = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(islot + kItemSlots * kItemInts) + 15) &
                               ~uintptr_t(15));                              // [kItemSlots][rows_cap][D]
  uint64_t* ifull = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(iq + kItemSlots * p.rows_cap * D) + 7) & ~uintptr_t(7));
  uint64_t* iempty = ifull + kItemSlots;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init(cbar, kConsumerWarps * 32);
    for (int s = 0; s < kItemSlots; ++s) {
      mbar_init(&ifull[s], 31);
      mbar_init(&iempty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  if (warp == kConsumerWarps && lane == 0) {
    tma_prefetch_desc(&maps.k);
    tma_prefetch_desc(&maps.v);
    tma_prefetch_desc(&maps.k16);
    tma_prefetch_desc(&maps.v16);
  }
  pdl_wait();   // lengths, tiles and q may come from the previous kernel
  if (threadIdx.x == 0) pdl_launch_dependents();
  __syncthreads();   // barrier initialisation visible to every warp

  // Persistent loop over work items (tile, split run, kv head); the producer warp
  // and the consumer warps walk the same items in the same order, so the producer
  // streams the next item's blocks while the consumers finish the current one.
  const int64_t n_items = static_cast<int64_t>(p.n_tiles) * p.upt * p.hkv;

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      int fills = 0;
      for (int64_t w = blockIdx.x; w < n_items && !abort_flag; w += gridDim.x) {
        Item it;
        if (describe_item(p, w, it) != 0) continue;
        for (int sp = it.s_begin; sp < it.s_end && !abort_flag; ++sp) {
          const int tb = sp * kSplit;
          const int nblk = (min(tb + kSplit, it.max_len) - tb + kBlock - 1) / kBlock;
          for (int b = 0; b < nblk; ++b) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, kDetProdEmpty, abort_flag)) break;
            uint8_t* st = ring + stage * C::STAGE_BYTES;
            const int t0 = tb + b * kBlock;
            int tok, slab;
            kv_block_coords(p, it.seq, t0, tok, slab);
            const int need = min(kBlock, min(tb + kSplit, it.max_len) - t0);   // tokens of the block in use
            if (need == kBlock) {
              mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
#pragma unroll
              for (int bx = 0; bx < C::NBOX; ++bx) {
                tma_load_4d(st + bx * C::BOX_BYTES, &maps.k, &full[stage], bx * C::BOXD, tok, it.kvh, slab);
                tma_load_4d(st + C::TENSOR_BYTES + bx * C::BOX_BYTES, &maps.v, &full[stage], bx * C::BOXD, tok, it.kvh,
                            slab);
              }
            } else {
              // the block's used 16-token groups only; the consumers mask the rest (K by select,
              // V rows zeroed) as for tokens past the end of a whole block
              const int nq = (need + kTailRows - 1) / kTailRows;
              mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(nq * kTailRows * C::ROWB * C::NBOX * 2));
              for (int qi = 0; qi < nq; ++qi) {
#pragma unroll
                for (int bx = 0; bx < C::NBOX; ++bx) {
                  const int off = bx * C::BOX_BYTES + qi * kTailRows * C::ROWB;
                  tma_load_4d(st + off, &maps.k16, &full[stage], bx * C::BOXD, tok + qi * kTailRows, it.kvh, slab);
                  tma_load_4d(st + C::TENSOR_BYTES + off, &maps.v16, &full[stage], bx * C::BOXD, tok + qi * kTailRows,
                              it.kvh, slab);
                }
              }
            }
            ++fills;
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      bool drain_abort = false;
      for (int f = (fills > C::STAGES ? fills - C::STAGES : 0); f < fills; ++f)
        mbar_wait(&full[f % C::STAGES], static_cast<uint32_t>((f / C::STAGES) & 1), kDetDrain, drain_abort);
    } else {
      // lanes 1..31: stage each item's description, kv lengths and q rows in the item ring,
      // up to kItemSlots items ahead of the consumers
      bool abort_flag = false;
      const int ml = lane - 1;
      int slot = 0;
      uint32_t iphase = 0;
      const T* q = reinterpret_cast<const T*>(p.q);
      for (int64_t w = blockIdx.x; w < n_items && !abort_flag; w += gridDim.x) {
        if (!mbar_wait(&iempty[slot], iphase ^ 1u, kDetItem, abort_flag)) break;
        Item it;
        const int bad = describe_item(p, w, it);
        int* m = islot + slot * kItemInts;
        if (ml == 0) {
          m[0] = bad;
          m[1] = it.tile;
          m[2] = it.unit;
          m[3] = it.kvh;
          m[4] = it.r0;
          m[5] = it.nr;
          m[6] = it.seq;
          m[7] = it.max_len;
          m[8] = it.nsplits;
          m[9] = it.s_begin;
          m[10] = it.s_end;
        }
        if (ml < kRows) m[16 + ml] = (bad <= 1 && ml < it.nr) ? (p.kv_lens ? p.kv_lens[it.r0 + ml] : p.uniform_len) : 0;
        if (bad == 0) {
          T* qs = iq + slot * p.rows_cap * D;
          const int chunks = it.nr * p.G * (D / 8);
          for (int e = ml; e < chunks; e += 31) {
            const int rho = e / (D / 8), c = e - rho * (D / 8);
            const int i = rho / p.G, gh = rho - i * p.G;
            const T* src = q + (int64_t)(it.r0 + i) * p.q_sr + (int64_t)(it.kvh * p.G + gh) * p.q_sh + c * 8;
            uint4 v;
            if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
              v = *reinterpret_cast<const uint4*>(src);
            } else {
              uint16_t h[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) h[j] = reinterpret_cast<const uint16_t*>(src)[j];
              v = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16), h[4] | (uint32_t(h[5]) << 16),
                             h[6] | (uint32_t(h[7]) << 16));
            }
            *reinterpret_cast<uint4*>(qs + rho * D + c * 8) = v;
          }
        }
        mbar_arrive(&ifull[slot]);
        if (++slot == kItemSlots) {
          slot = 0;
          iphase ^= 1u;
        }
      }
    }
    return;  // the producer warp takes no part in the merges
  }

  // ---------------- consumers ----------------
  bool abort_flag = false;
  const int g = lane >> 2;
  const int t4 = lane & 3;
  const int rho0 = g, rho1 = g + 8;
  const int ctid = threadIdx.x;  // 0..127
  constexpr int KC = D / 16;
  constexpr int NT = D / 8;  // output n-tiles of 8 along d
  const int wr = warp * 16;  // this warp's first token row inside a block
  T* out = reinterpret_cast<T*>(p.out);
  int stage = 0;
  uint32_t phase = 0;
  uint32_t cphase = 0;

  // ldmatrix source offsets inside a stage's K and V tensors (fixed per thread)
  uint32_t k_off[KC], v_off[D / 16];
  {
    const int mi = lane >> 3, ri = lane & 7;
    // K as the B operand (two n-tiles of 8 tokens) or, for T1, as the A operand (16
    // tokens x 16 d); V the other way round (ldmatrix.trans either way)
    const int r_a = wr + (mi & 1) * 8 + ri, c_a = mi >> 1;
    const int r_b = wr + (mi >> 1) * 8 + ri, c_b = mi & 1;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc)
      k_off[kc] = T1 ? chunk_addr<D>(0u, r_a, 2 * kc + c_a) : chunk_addr<D>(0u, r_b, 2 * kc + c_b);
#pragma unroll
    for (int pc = 0; pc < D / 16; ++pc)
      v_off[pc] = T1 ? chunk_addr<D>(0u, r_b, 2 * pc + c_b) : chunk_addr<D>(0u, r_a, 2 * pc + c_a);
  }
  int islot_i = 0;
  uint32_t iph = 0;
  for (int64_t w = blockIdx.x; w < n_items && !abort_flag; w += gridDim.x) {
    if (!mbar_wait(&ifull[islot_i], iph, kDetItem, abort_flag)) break;
    const int* m = islot + islot_i * kItemInts;
    const int* s_len = m + 16;   // kv length of each tile row
    const T* qs = iq + islot_i * p.rows_cap * D;
    do {
    const int bad = m[0];
    const int tile = m[1], unit = m[2], kvh = m[3], r0 = m[4], nr = m[5];
    const int max_len = m[7], nsplits = m[8];
    if (bad > 1) {
      if (ctid == 0 && unit == 0 && kvh == 0) report_error(DK_ERR_DEVICE_CHECK, bad == 2 ? kDetTile : kDetLen);
      break;
    }
    const int valid_rows = nr * p.G;
    if (nsplits == 0) {
      // every row of the tile has an empty KV sequence: output zeros
      if (unit == 0) {
        for (int e = ctid; e < valid_rows * D; e += kConsumerWarps * 32) {
          const int rho = e / D, d = e % D;
          const int i = rho / p.G, gh = rho % p.G;
          out[(int64_t)(r0 + i) * p.o_sr + (int64_t)(kvh * p.G + gh) * p.o_sh + d] = from_f32<T>(0.0f);
        }
      }
      break;
    }
    if (bad == 1) break;  // no split of this tile falls in this item's run
    const int s_begin = m[9], s_end = m[10];
    const bool direct = (nsplits <= p.spu);        // this item owns every split of the tile

    const bool v0 = rho0 < valid_rows, v1 = rho1 < valid_rows;
    const int i0 = v0 ? rho0 / p.G : 0, i1 = v1 ? rho1 / p.G : 0;

    // Q fragments (A operand, rows rho0/rho1) from the staged q rows; for T1 the B
    // operand q^T (column g = query row g: only column 0 is a row)
    uint32_t qa[KC][4];
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      const int d0 = kc * 16 + 2 * t4;
      if constexpr (T1) {
        qa[kc][0] = v0 ? *reinterpret_cast<const uint32_t*>(qs + d0) : 0u;
        qa[kc][1] = v0 ? *reinterpret_cast<const uint32_t*>(qs + d0 + 8) : 0u;
        qa[kc][2] = qa[kc][3] = 0u;
      } else {
        qa[kc][0] = v0 ? *reinterpret_cast<const uint32_t*>(qs + rho0 * D + d0) : 0u;
        qa[kc][1] = v1 ? *reinterpret_cast<const uint32_t*>(qs + rho1 * D + d0) : 0u;
        qa[kc][2] = v0 ? *reinterpret_cast<const uint32_t*>(qs + rho0 * D + d0 + 8) : 0u;
        qa[kc][3] = v1 ? *reinterpret_cast<const uint32_t*>(qs + rho1 * D + d0 + 8) : 0u;
      }
    }

    // running split-order merge of the elements this thread owns (direct path)
    float run_m[KM], run_l[KM], run_o[KM];
#pragma unroll
    for (int k = 0; k < KM; ++k) {
      run_m[k] = -INFINITY;
      run_l[k] = 0.0f;
      run_o[k] = 0.0f;
    }
    const int64_t slot = ((int64_t)tile * p.hkv + kvh) * p.max_splits;

    for (int sp = s_begin; sp < s_end && !abort_flag; ++sp) {
      const int tok_begin = sp * kSplit;
      const int tok_end = min(tok_begin + kSplit, max_len);
      const int nblk = (tok_end - tok_begin + kBlock - 1) / kBlock;
      const int end0 = v0 ? min(s_len[i0], tok_begin + kSplit) : 0;  // row's own token end in this split
      const int end1 = v1 ? min(s_len[i1], tok_begin + kSplit) : 0;

      // O (NT n-tiles of 8 d) or, for T1, O^T (D / 16 m-tiles of 16 d; column 0 = the row)
      constexpr int NO = T1 ? D / 16 : NT;
      float o[NO][4];
#pragma unroll
      for (int j = 0; j < NO; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
      const int end_t1 = min(s_len[0], tok_begin + kSplit);   // T1: the row's token end in this split
      float m_r[2] = {-INFINITY, -INFINITY};
      float l_r[2] = {0.0f, 0.0f};

      for (int b = 0; b < nblk; ++b) {
        if (!mbar_wait(&full[stage], phase, kDetFull, abort_flag)) break;
        const uint32_t kbase = smem_u32(ring + stage * C::STAGE_BYTES);
        const uint32_t vbase = kbase + C::TENSOR_BYTES;
        const int t0 = tok_begin + b * kBlock + wr;  // token of this warp's row 0

        // Tokens no row of the tile may read: zero their V rows (K is masked by select).
        if (t0 + 16 > tok_end) {
          uint8_t* vgen = ring + stage * C::STAGE_BYTES + C::TENSOR_BYTES;
          for (int e = lane; e < 16 * (D / 8); e += 32) {
            const int rr = e / (D / 8), c = e % (D / 8);
            if (t0 + rr >= tok_end) {
              const uint32_t a = chunk_addr<D>(0u, wr + rr, c);
              *reinterpret_cast<uint4*>(vgen + a) = make_uint4(0u, 0u, 0u, 0u);
            }
          }
          // order these generic-proxy writes before the next TMA write of the stage
          fence_proxy_async_smem();
          __syncwarp();
        }

        if constexpr (T1) {
          // S^T = K q^T: c[0] = token t0 + g, c[2] = token t0 + g + 8 (column 2*t4: only t4 == 0 is the row)
          float st[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int kc = 0; kc < KC; ++kc) {
            uint32_t ka[4];
            ldsm_x4(kbase + k_off[kc], ka[0], ka[1], ka[2], ka[3]);
            mma16816<T>(st, ka, qa[kc][0], qa[kc][1]);
          }
          // V^T fragments into registers now, so the stage goes back to the producer before the
          // softmax and the P.V products (the same operands, read earlier)
          uint32_t vfr[D / 16][4];
#pragma unroll
          for (int pc = 0; pc < D / 16; ++pc) ldsm_x4_t(vbase + v_off[pc], vfr[pc][0], vfr[pc][1], vfr[pc][2], vfr[pc][3]);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[stage]);
          const int tk = t0 + g;
          float x0 = __fmul_rn(st[0], p.scale_log2);
          float x1 = __fmul_rn(st[2], p.scale_log2);
          if (t4 != 0 || tk >= end_t1) x0 = -INFINITY;
          if (t4 != 0 || tk + 8 >= end_t1) x1 = -INFINITY;
          float mx = fmaxf(x0, x1);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          mx = __shfl_sync(0xffffffffu, mx, 0);   // the row's max on every lane (lanes t4 != 0 hold -inf)
          const float m_new = fmaxf(m_r[0], mx);
          const float mref = (m_new == -INFINITY) ? 0.0f : m_new;
          const float alpha = weight_of(m_r[0], mref);
          float r0f, r1f;
          const uint32_t pk = pack_round<T>(weight_of(x0, mref), weight_of(x1, mref), r0f, r1f);   // tokens g | g+8
          // P^T as the B operand: lane t4 of column 0 takes tokens 2t4, 2t4+1 (b0) and
          // 2t4+8, 2t4+9 (b1) from lanes 8*t4 and 8*t4+4
          const uint32_t ua = __shfl_sync(0xffffffffu, pk, 8 * t4);
          const uint32_t ub = __shfl_sync(0xffffffffu, pk, 8 * t4 + 4);
          uint32_t pb0 = __byte_perm(ua, ub, 0x5410);
          uint32_t pb1 = __byte_perm(ua, ub, 0x7632);
          if (g != 0) pb0 = pb1 = 0u;
          // l from the same four tokens per lane and in the same order as the 16-row form
          const float psum =
              __fadd_rn(__fadd_rn(lo_f32<T>(pb0), hi_f32<T>(pb0)), __fadd_rn(lo_f32<T>(pb1), hi_f32<T>(pb1)));
          l_r[0] = __fadd_rn(__fmul_rn(l_r[0], alpha), psum);
          m_r[0] = m_new;
          if (alpha != 1.0f) {   // multiplying by exactly 1 changes nothing
#pragma unroll
            for (int j = 0; j < NO; ++j) {
              o[j][0] = __fmul_rn(o[j][0], alpha);
              o[j][2] = __fmul_rn(o[j][2], alpha);
            }
          }
          // O^T += V^T P^T
#pragma unroll
          for (int pc = 0; pc < D / 16; ++pc) mma16816<T>(o[pc], vfr[pc], pb0, pb1);
        } else {
          // S = Q K^T for this warp's 16 tokens (two n-tiles of 8 tokens).
          float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
  #pragma unroll
          for (int kc = 0; kc < KC; ++kc) {
            uint32_t b00, b01, b10, b11;
            ldsm_x4(kbase + k_off[kc], b00, b01, b10, b11);
            mma16816<T>(s0, qa[kc], b00, b01);
            mma16816<T>(s1, qa[kc], b10, b11);
          }

          // scale, mask, online softmax update (rows rho0 -> s*[0..1], rho1 -> s*[2..3])
          const int tk = t0 + 2 * t4;
          float sc[2][4];
          sc[0][0] = __fmul_rn(s0[0], p.scale_log2);
          sc[0][1] = __fmul_rn(s0[1], p.scale_log2);
          sc[0][2] = __fmul_rn(s1[0], p.scale_log2);
          sc[0][3] = __fmul_rn(s1[1], p.scale_log2);
          sc[1][0] = __fmul_rn(s0[2], p.scale_log2);
          sc[1][1] = __fmul_rn(s0[3], p.scale_log2);
          sc[1][2] = __fmul_rn(s1[2], p.scale_log2);
          sc[1][3] = __fmul_rn(s1[3], p.scale_log2);
          if (tk + 9 >= end0 || tk + 9 >= end1) {   // some of this thread's tokens are past a row's end
            if (tk + 0 >= end0) sc[0][0] = -INFINITY;
            if (tk + 1 >= end0) sc[0][1] = -INFINITY;
            if (tk + 8 >= end0) sc[0][2] = -INFINITY;
            if (tk + 9 >= end0) sc[0][3] = -INFINITY;
            if (tk + 0 >= end1) sc[1][0] = -INFINITY;
            if (tk + 1 >= end1) sc[1][1] = -INFINITY;
            if (tk + 8 >= end1) sc[1][2] = -INFINITY;
            if (tk + 9 >= end1) sc[1][3] = -INFINITY;
          }

          uint32_t pa[4];
          float alpha[2];
  #pragma unroll
          for (int h = 0; h < 2; ++h) {
            float mx = fmaxf(fmaxf(sc[h][0], sc[h][1]), fmaxf(sc[h][2], sc[h][3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float m_new = fmaxf(m_r[h], mx);
            const float mref = (m_new == -INFINITY) ? 0.0f : m_new;
            alpha[h] = weight_of(m_r[h], mref);
            float pr[4];
            const uint32_t lo = pack_round<T>(weight_of(sc[h][0], mref), weight_of(sc[h][1], mref), pr[0], pr[1]);
            const uint32_t hi = pack_round<T>(weight_of(sc[h][2], mref), weight_of(sc[h][3], mref), pr[2], pr[3]);
            pa[h] = lo;      // a0 (row g) / a1 (row g+8): tokens 2t, 2t+1
            pa[h + 2] = hi;  // a2 / a3: tokens 8+2t, 8+2t+1
            const float psum = __fadd_rn(__fadd_rn(pr[0], pr[1]), __fadd_rn(pr[2], pr[3]));
            l_r[h] = __fadd_rn(__fmul_rn(l_r[h], alpha[h]), psum);
            m_r[h] = m_new;
          }
          if (alpha[0] != 1.0f || alpha[1] != 1.0f) {   // multiplying by exactly 1 changes nothing
  #pragma unroll
            for (int j = 0; j < NT; ++j) {
              o[j][0] = __fmul_rn(o[j][0], alpha[0]);
              o[j][1] = __fmul_rn(o[j][1], alpha[0]);
              o[j][2] = __fmul_rn(o[j][2], alpha[1]);
              o[j][3] = __fmul_rn(o[j][3], alpha[1]);
            }
          }
          // O += P V
  #pragma unroll
          for (int pc = 0; pc < D / 16; ++pc) {
            uint32_t b0a, b1a, b0b, b1b;
            ldsm_x4_t(vbase + v_off[pc], b0a, b1a, b0b, b1b);
            mma16816<T>(o[2 * pc], pa, b0a, b1a);
            mma16816<T>(o[2 * pc + 1], pa, b0b, b1b);
          }
        }
        if constexpr (!T1) {   // (the single-row path released the stage above)
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[stage]);
        }
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }

      // quad-reduce l (fixed butterfly; m is already quad-uniform)
#pragma unroll
      for (int h = 0; h < (T1 ? 1 : 2); ++h) {
        l_r[h] = __fadd_rn(l_r[h], __shfl_xor_sync(0xffffffffu, l_r[h], 1));
        l_r[h] = __fadd_rn(l_r[h], __shfl_xor_sync(0xffffffffu, l_r[h], 2));
      }

      // ---- merge the four warps of this split in warp order ----
      if (!csync(cbar, cphase, abort_flag)) break;   // the previous split's merge reads are done
      if constexpr (T1) {
        if (t4 == 0) {
#pragma unroll
          for (int j = 0; j < NO; ++j) {
            comb_o[warp * C::CSTRIDE + j * 16 + g] = o[j][0];
            comb_o[warp * C::CSTRIDE + j * 16 + g + 8] = o[j][2];
          }
        }
        if (lane == 0) {
          comb_ml[warp * 2 + 0] = m_r[0];
          comb_ml[warp * 2 + 1] = l_r[0];
        }
      } else if (v0) {
#pragma unroll
        for (int j = 0; j < NT; ++j)
          *reinterpret_cast<float2*>(comb_o + (warp * p.rows_cap + rho0) * C::CSTRIDE + j * 8 + 2 * t4) =
              make_float2(o[j][0], o[j][1]);
        if (t4 == 0) {
          comb_ml[(warp * p.rows_cap + rho0) * 2 + 0] = m_r[0];
          comb_ml[(warp * p.rows_cap + rho0) * 2 + 1] = l_r[0];
        }
      }
      if (!T1 && v1) {
#pragma unroll
        for (int j = 0; j < NT; ++j)
          *reinterpret_cast<float2*>(comb_o + (warp * p.rows_cap + rho1) * C::CSTRIDE + j * 8 + 2 * t4) =
              make_float2(o[j][2], o[j][3]);
        if (t4 == 0) {
          comb_ml[(warp * p.rows_cap + rho1) * 2 + 0] = m_r[1];
          comb_ml[(warp * p.rows_cap + rho1) * 2 + 1] = l_r[1];
        }
      }
      if (!csync(cbar, cphase, abort_flag)) break;

#pragma unroll
      for (int k = 0; k < KM; ++k) {
        const int e = ctid + k * (kConsumerWarps * 32);
        if (e < valid_rows * D) {
          const int rho = e / D, d = e % D;
          float mw[kConsumerWarps];
          float M = -INFINITY;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) {
            mw[w] = comb_ml[(w * p.rows_cap + rho) * 2];
            M = fmaxf(M, mw[w]);
          }
          const float mref = (M == -INFINITY) ? 0.0f : M;
          float L = 0.0f, O = 0.0f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) {
            const float wt = weight_of(mw[w], mref);
            L = __fadd_rn(L, __fmul_rn(comb_ml[(w * p.rows_cap + rho) * 2 + 1], wt));
            O = __fadd_rn(O, __fmul_rn(comb_o[(w * p.rows_cap + rho) * C::CSTRIDE + d], wt));
          }
          if (direct) {
            const int own = (s_len[rho / p.G] + kSplit - 1) / kSplit;
            if (sp < own) merge_split(sp == 0, run_m[k], run_l[k], run_o[k], M, L, O);
          } else {
            const int64_t base = (slot + sp) * p.rows_cap + rho;
            p.ws_o[base * D + d] = O;
            if (d == 0) {
              p.ws_ml[base * 2 + 0] = M;
              p.ws_ml[base * 2 + 1] = L;
            }
          }
        }
      }
    }
    if (abort_flag) break;

    if (!direct) {
      // ---- the last CTA of this (tile, kv head) replays the split-order merge ----
      __threadfence();
      if (!csync(cbar, cphase, abort_flag)) break;
      if (ctid == 0) {
        const int arrivals = (nsplits + p.spu - 1) / p.spu;
        const int old = atomicAdd(p.counters + (int64_t)tile * p.hkv + kvh, 1);
        const bool last = (old == arrivals - 1);
        s_misc[0] = last ? 1 : 0;
        if (last) p.counters[(int64_t)tile * p.hkv + kvh] = 0;
      }
      if (!csync(cbar, cphase, abort_flag)) break;
      if (s_misc[0] == 0) break;
      __threadfence();
#pragma unroll
      for (int k = 0; k < KM; ++k) {
        const int e = ctid + k * (kConsumerWarps * 32);
        if (e < valid_rows * D) {
          const int rho = e / D, d = e % D;
          const int own = (s_len[rho / p.G] + kSplit - 1) / kSplit;
          for (int s = 0; s < own; ++s) {
            const int64_t base = (slot + s) * p.rows_cap + rho;
            merge_split(s == 0, run_m[k], run_l[k], run_o[k], __ldcg(p.ws_ml + base * 2), __ldcg(p.ws_ml + base * 2 + 1),
                        __ldcg(p.ws_o + base * D + d));
          }
        }
      }
    }

#pragma unroll
    for (int k = 0; k < KM; ++k) {
      const int e = ctid + k * (kConsumerWarps * 32);
      if (e < valid_rows * D) {
        const int rho = e / D, d = e % D;
        const int i = rho / p.G, gh = rho % p.G;
        const float r = (s_len[i] == 0) ? 0.0f : __fdiv_rn(run_o[k], run_l[k]);
        out[(int64_t)(r0 + i) * p.o_sr + (int64_t)(kvh * p.G + gh) * p.o_sh + d] = from_f32<T>(r);
      }
    }
    } while (0);
    // this warp is done with the staged item: release its slot
    __syncwarp();
    if (lane == 0) mbar_arrive(&iempty[islot_i]);
    if (++islot_i == kItemSlots) {
      islot_i = 0;
      iph ^= 1u;
    }
  }
}

}  // namespace attn
}  // namespace dk
