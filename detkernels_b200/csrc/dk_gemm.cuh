// Batch-invariant GEMM on 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces kernels/matmul.py:64-100 (_matmul_kernel, the invariant direct tile
// GEMM) and, through the ATOMIC mode, kernels/matmul.py:102-145 (the split-K
// atomic twin used by matmul_batch_variant).
//
// C[M,N] = A[M,K] @ B[K,N], A and B row-major bf16/f16, f32 accumulation.
//
// Formulation ("swap-AB"): the tensor-core instruction computes
//   D[n, m] = sum_k B[k, n] * A[m, k]
// with the 128 weight columns of a tile on the UMMA M axis (B read MN-major,
// straight from its row-major [K, N] layout) and 128 tokens on the UMMA N axis
// (A read K-major).  The tile is 128 weight columns x 128 tokens for every M.
// When all M rows fit one 128-token tile, the activation TMA box covers only
// ceil8(M) rows and the instruction spans ceil16(M) token columns (an element's
// bits do not depend on the instruction's N); a column beyond the box reads
// stale shared memory.  Each output column depends only on its own token row,
// stale columns are never stored, and the epilogue skips 32-token chunks that
// hold no token below M.
//
// Fixed reduction structure (the definition of the output bits):
//   * K is cut into DK_MATMUL_K_SLICES = 8 slices of L = ceil16(ceil(K/8))
//     elements; slice s covers [s*L, min((s+1)*L, K)).
//   * Slice s is accumulated from zero in its own TMEM accumulator by
//     tcgen05.mma steps of 16 K-elements in ascending K order: partial p_s.
//   * The partials are summed in f32 along a fixed binary tree,
//       ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)),
//     then rounded to the output dtype (round to nearest even).
// Nothing in that structure depends on M, N or the schedule, so a row's output
// bits do not depend on the batch.  The tree makes every aligned group of 1, 2,
// 4 or 8 slices a subtree, so a group can be summed on its own and contribute
// ONE partial; only the schedule decides where the groups are summed:
//   * FOLD:    a work unit = one output tile x all 8 slices, summed in TMEM.
//   * SPLIT:   a work unit = one output tile x an aligned group of 1, 2 or 4
//              slices; each unit writes its subtree sum to the workspace and a
//              second, fully parallel kernel (fold_groups_kernel, launched as a
//              programmatic dependent of this one) adds the 8/g subtree sums
//              along the upper tree levels.
//   * PARTIAL: one aligned slice group per launch, its subtree sum written out
//              (row-parallel tensor parallelism: a rank per group).
//   * ATOMIC:  the deliberately batch-variant twin: split_k chunks added with
//              f32 atomics (scheduler-dependent order).
//
// Accumulators: TMEM holds 4 slots of 128 columns.  Slice i of a unit is
// multiplied into slot (kSlotTable[i] + unit_ordinal * step(g)) mod 4; the
// epilogue keeps the tree's pending left operands in their slots, adds right
// operands into them (tcgen05.ld / add / tcgen05.st) and releases every slot it
// consumed.  The table guarantees that a slot's previous value is always
// released by the epilogue of an EARLIER slice, so the MMA issuer never waits on
// work that depends on itself, and with one exception per 8-slice unit it never
// waits on the epilogue of the slice just before.
#pragma once

#include "dk_common.cuh"
#include "dk_rmsnorm.cuh"

namespace dk {
namespace gemm {

constexpr int kTileN = 128;  // weight columns per tile (UMMA M)
constexpr int kTileM = 128;  // tokens per tile (UMMA N)
constexpr int kBK = 64;      // K per sub-block: one 128-byte swizzle row of bf16
constexpr int kSub = 2;      // sub-blocks per pipeline stage of the one-CTA kernel
constexpr int kStageK = kSub * kBK;   // K per pipeline stage (128): fewer barrier round trips per MMA
constexpr int kUK = 16;      // K per tcgen05.mma, kind::f16
constexpr int kMaxStages = 16;   // ring depth is chosen per launch from the stage size
constexpr int kSlices = DK_MATMUL_K_SLICES;
constexpr int kWBoxBytes = 64 * kBK * 2;          // 64 columns x 64 k
constexpr int kWTileBytes = 2 * kWBoxBytes;       // 128 columns x 64 k
constexpr int kATileBytes = kTileM * kBK * 2;     // 128 tokens x 64 k
constexpr int kEpiWarps = 8;                      // two warps per TMEM lane quarter
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kEpiCols = kTileM / 2;              // token columns handled per epilogue thread
constexpr int kThreads = 64 + kEpiThreads;        // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kSlots = 4;
constexpr int kTmemCols = kSlots * kTileM;        // 512: the whole tensor memory of the SM
constexpr int kBarrierBytes = 512;
constexpr int kStagePitch = 33;                   // floats per row of an epilogue transpose tile (32 + 1 pad)
constexpr int kEpiStageBytes = kEpiWarps * 32 * kStagePitch * 4;   // one 32 x 32 f32 tile per epilogue warp
constexpr int kSmemBytes = 232448;               // the sm_100 per-CTA maximum
// [ring (kRingBytes) | barriers].  The FOLD epilogue's transpose tiles take the last
// kEpiStageBytes of the ring region, so FOLD launches run a shorter ring.
constexpr int kRingBytes = kSmemBytes - 1024 /*align*/ - kBarrierBytes;

// Stage layout for an activation box of a_rows rows (a multiple of 8):
//   [weights sub-block 0 | weights sub-block 1 | tokens sub-block 0 | tokens sub-block 1]
// with 16 KB per weight sub-block (128 columns x 64 k) and a_rows x 128 B per token
// sub-block (each a multiple of the 1 KB swizzle period), the whole rounded up to 1 KB.
// The MMA always reads 128 token rows (16 KB) from a token sub-block, i.e. up to
// (128 - a_rows) x 128 B past its loaded rows: into the next sub-block or stage (stale
// data, feeding columns that are never stored) and, after the last stage, into a guard
// area kept free at the end of the ring so that every read stays inside the CTA's
// shared memory.
__host__ __device__ __forceinline__ int stage_bytes_for(int a_rows) {
  return ((kSub * (kWTileBytes + a_rows * kBK * 2) + 1023) / 1024) * 1024;
}
__host__ __device__ __forceinline__ int overhang_bytes_for(int a_rows) { return (kTileM - a_rows) * kBK * 2; }
__host__ __device__ __forceinline__ int ring_bytes_for(int mode) {
  return kRingBytes - (mode == 0 /*FOLD*/ ? kEpiStageBytes : 0);
}
__host__ __device__ __forceinline__ int stages_for(int a_rows, int mode) {
  const int n = (ring_bytes_for(mode) - overhang_bytes_for(a_rows)) / stage_bytes_for(a_rows);
  return n < kMaxStages ? n : kMaxStages;
}

// kSlotTable[i] for i = 0..7 packed 2 bits each: {0, 1, 2, 1, 3, 1, 2, 1}.
constexpr uint32_t kSlotTable = 0u | (1u << 2) | (2u << 4) | (1u << 6) | (3u << 8) | (1u << 10) | (2u << 12) |
                                (1u << 14);

__host__ __device__ __forceinline__ int slot_of(int i, int unit_ordinal, int group) {
  const int step = (group == 2) ? 2 : (group == 4 ? 3 : 1);
  return (static_cast<int>((kSlotTable >> (2 * i)) & 3u) + unit_ordinal * step) & 3;
}

enum Mode : int { FOLD = 0, SPLIT = 1, PARTIAL = 2, ATOMIC = 3 };

struct Params {
  dk_matmul_epilogue epi;        // what is done with each final value (DK_EPI_*)
  int M, N, K;
  int k_base;      // global K index of the first column of A / row of B held in memory (K shards)
  int k_extent;    // K columns of A / rows of B held in memory (0: K)
  int slice_len;                 // elements per slice (multiple of 16)
  int slice_begin, slice_end;    // slices computed by this launch
  int group;                     // slices per work unit (aligned group, power of two)
  int n_tiles, m_tiles;
  int mode;
  int pair;        // 1: CTA-pair kernel (n_tiles counts 256-column pair tiles)
  int a_rows;      // rows of the activation TMA box (128, or fewer when M fits one tile)
  void* c;
  int64_t ldc;
  float* ws;       // SPLIT: subtree sums [8/g][M][N]; PARTIAL: [M][N]; ATOMIC: [M][N]
  float* stash;    // wide kernel, 8-slice units: a parking place per CTA for the tree's left half
};

// Detail codes recorded with a timeout (which wait expired).
enum : int {
  kDetProdEmpty = 0x100,
  kDetMmaSlotFree = 0x101,
  kDetMmaFull = 0x102,
  kDetEpiSlotFull = 0x103,
  kDetDrain = 0x105,
};

// Output tile t -> (m-tile, n-tile).  Tiles go in bands of kBandM m-tiles; inside a
// band the m-tile varies fastest, then the n-tile.  The ~SM-count tiles in flight at
// once then share a few activation and weight tiles in L2, and a tall activation
// matrix streams from DRAM about once per GEMM instead of once per n-tile.  This is
// order only: a tile's arithmetic does not depend on when or where it runs.
constexpr int kBandM = 16;
__device__ __forceinline__ void tile_coords(const Params& p, int t, int& mt, int& nt) {
  const int per_band = kBandM * p.n_tiles;
  const int band = t / per_band;
  const int r = t - band * per_band;
  const int bm = min(kBandM, p.m_tiles - band * kBandM);
  nt = r / bm;
  mt = band * kBandM + (r - nt * bm);
}

__device__ __forceinline__ void slice_bounds(const Params& p, int s, int& k0, int& k1) {
  k0 = s * p.slice_len;
  k1 = min(k0 + p.slice_len, p.K);
  if (k1 < k0) k1 = k0;
}

// Upper levels of the slice tree: sum of n (1, 2, 4 or 8) aligned subtree sums.
__device__ __forceinline__ float tree_sum(const float* v, int n) {
  if (n == 1) return v[0];
  if (n == 2) return __fadd_rn(v[0], v[1]);
  if (n == 4) return __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
  return __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])),
                   __fadd_rn(__fadd_rn(v[4], v[5]), __fadd_rn(v[6], v[7])));
}

__device__ __forceinline__ float silu_f32(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

template <typename T>
__device__ __forceinline__ float rnd(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// Element offset of (row m's sequence, head, row m's position, d) in a K/V cache: contiguous
// [n_seq, heads, capacity, d], or paged through the block table (block = table[seq][pos / page],
// token pos % page of a [n_blocks, heads, page, d] pool).  A position beyond the table row or a
// table entry outside the pool is recorded (DK_ERR_DEVICE_CHECK) and the store skipped (ok = false).
__device__ __forceinline__ int64_t kv_cache_offset(const dk_matmul_epilogue& e, int m, int head, int d, bool& ok) {
  const int64_t seq = e.row_seq ? e.row_seq[m] : m;
  int64_t pos = e.row_pos[m];
  int64_t slab = seq;
  ok = true;
  if (e.block_table) {
    const int64_t pg = pos / e.page_size;
    if (pos < 0 || pg >= e.blocks_per_seq) {
      report_error(DK_ERR_DEVICE_CHECK, 0x600);
      ok = false;
      return 0;
    }
    slab = e.block_table[seq * e.block_table_stride + pg];
    if (slab < 0 || slab >= e.n_blocks) {
      report_error(DK_ERR_DEVICE_CHECK, 0x601);
      ok = false;
      return 0;
    }
    pos -= pg * e.page_size;
  }
  return slab * e.cache_stride_seq + head * e.cache_stride_head + pos * e.cache_stride_tok + d;
}

// Final value v of output element (m, n) -> memory, per the epilogue mode (all but SILU_MUL).
template <typename T>
__device__ __forceinline__ void store_final(const Params& p, T* C, int m, int n, float v) {
  const dk_matmul_epilogue& e = p.epi;
  switch (e.mode) {
    case DK_EPI_RESIDUAL: {
      const float r = to_f32<T>(static_cast<const T*>(e.resid)[static_cast<int64_t>(m) * e.ld_resid + n]);
      C[static_cast<int64_t>(m) * p.ldc + n] = from_f32<T>(__fadd_rn(r, rnd<T>(v)));
      break;
    }
    case DK_EPI_SILU:
      C[static_cast<int64_t>(m) * p.ldc + n] = from_f32<T>(silu_f32(rnd<T>(v)));
      break;
    case DK_EPI_QKV_CACHE: {
      if (n < e.q_cols) {
        C[static_cast<int64_t>(m) * p.ldc + n] = from_f32<T>(v);
      } else {
        const int j = n - e.q_cols;
        const int which = j / e.kv_cols;
        const int jj = j - which * e.kv_cols;
        const int head = jj / e.head_dim, d = jj - head * e.head_dim;
        T* cache = static_cast<T*>(which == 0 ? e.k_cache : e.v_cache);
        bool ok;
        const int64_t off = kv_cache_offset(e, m, head, d, ok);
        if (ok) cache[off] = from_f32<T>(v);
      }
      break;
    }
    default:
      C[static_cast<int64_t>(m) * p.ldc + n] = from_f32<T>(v);
  }
}

// Argmax key of the rounded value v at column n: larger key = larger value, and among equal values
// the smaller column.  NaN sorts above everything; -0 and +0 are equal.  Every real key is > 0.
template <typename T>
__device__ __forceinline__ uint32_t argmax_hi(float v) {
  const float r = rnd<T>(v);
  if (r != r) return 0xffffffffu;
  const uint32_t b = __float_as_uint(r == 0.0f ? 0.0f : r);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
template <typename T>
__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
  return (static_cast<unsigned long long>(argmax_hi<T>(v)) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(n));
}

// The largest argmax_key of columns n_base .. n_base + ncols - 1 with values v[0..ncols) (0 when
// ncols <= 0).  Four independent running maxima (column k goes to k % 4, a strictly larger value
// replaces, so each keeps its first maximal column) merged at the end: the same key as a serial
// max over the 32 keys, without its 32-long dependent chain of 64-bit compares.
template <typename T>
__device__ __forceinline__ unsigned long long argmax_chunk_key(const float (&v)[32], int ncols, int n_base) {
  uint32_t bh[4] = {0u, 0u, 0u, 0u};
  int bk[4] = {0, 1, 2, 3};
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const uint32_t h = (k < ncols) ? argmax_hi<T>(v[k]) : 0u;   // every real hi is > 0
    if (h > bh[k & 3]) {
      bh[k & 3] = h;
      bk[k & 3] = k;
    }
  }
  uint32_t h = bh[0];
  int kk = bk[0];
#pragma unroll
  for (int i = 1; i < 4; ++i) {
    if (bh[i] > h || (bh[i] == h && bk[i] < kk)) {
      h = bh[i];
      kk = bk[i];
    }
  }
  return h ? ((static_cast<unsigned long long>(h) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(n_base + kk)))
           : 0ull;
}

// Max over the 32 lanes (columns) of each of 32 token values k[0..31]; lane L ends with token L's
// maximum in k[0].  Reduce-scatter butterfly: 31 exchanges instead of 32 x 5.
__device__ __forceinline__ unsigned long long warp_max_scatter(unsigned long long (&k)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool upper = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const unsigned long long send = upper ? k[i] : k[i + w];
      const unsigned long long keep = upper ? k[i + w] : k[i];
      const unsigned long long recv = __shfl_xor_sync(0xffffffffu, send, w);
      k[i] = keep > recv ? keep : recv;
    }
  }
  return k[0];
}

// gate value g (column 2j) and up value u (column 2j+1) -> C[m, j]
template <typename T>
__device__ __forceinline__ void store_silu_mul(const Params& p, T* C, int m, int j, float g, float u) {
  const float s = rnd<T>(silu_f32(rnd<T>(g)));
  C[static_cast<int64_t>(m) * p.ldc + j] = from_f32<T>(__fmul_rn(s, rnd<T>(u)));
}

// ---- row-wise epilogue: a warp's 32 columns x 32 tokens, transposed through shared memory so
// that each lane owns one token row of 32 consecutive columns and writes it with 16-byte stores.

template <typename T>
__device__ __forceinline__ bool aligned_row(const void* base, int64_t ld, int64_t col) {
  // 16-byte stores of 8 elements need a 16-byte aligned row start at every row
  return (reinterpret_cast<uintptr_t>(base) % 16 == 0) && (ld % 8 == 0) && (col % 8 == 0);
}

template <typename T>
__device__ __forceinline__ void store_row_vec(T* dst, const float (&v)[32], int count) {
  // count is 16 or 32 (multiple of 8); dst 16-byte aligned
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q * 8 < count) {
      uint4 w;
      uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const T lo = from_f32<T>(v[q * 8 + 2 * e]), hi = from_f32<T>(v[q * 8 + 2 * e + 1]);
        wp[e] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&lo)) |
                (static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
      }
      reinterpret_cast<uint4*>(dst)[q] = w;
    }
  }
}

template <typename T>
__device__ __forceinline__ void load_row_vec(const T* src, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 w = reinterpret_cast<const uint4*>(src)[q];
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint16_t lo = static_cast<uint16_t>(wp[e] & 0xffffu), hi = static_cast<uint16_t>(wp[e] >> 16);
      v[q * 8 + 2 * e] = to_f32<T>(*reinterpret_cast<const T*>(&lo));
      v[q * 8 + 2 * e + 1] = to_f32<T>(*reinterpret_cast<const T*>(&hi));
    }
  }
}

// Final values of token row m, columns n_base .. n_base + ncols - 1 (ncols <= 32) -> memory.
template <typename T>
__device__ __forceinline__ void store_final_row(const Params& p, T* C, int m, int n_base, int ncols, float (&v)[32]) {
  const dk_matmul_epilogue& e = p.epi;
  const bool full = (ncols == 32);
  switch (e.mode) {
    case DK_EPI_ARGMAX: {
      const unsigned long long best = argmax_chunk_key<T>(v, ncols, n_base);
      if (best != 0ull) atomicMax(e.argmax_keys + m, best);
      if (!C) return;
      break;   // logits stored as plain values below
    }
    case DK_EPI_RESIDUAL: {
      const T* R = static_cast<const T*>(e.resid) + static_cast<int64_t>(m) * e.ld_resid + n_base;
      float r[32];
      if (full && aligned_row<T>(e.resid, e.ld_resid, n_base)) {
        load_row_vec<T>(R, r);
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) r[k] = (k < ncols) ? to_f32<T>(R[k]) : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = __fadd_rn(r[k], rnd<T>(v[k]));
      break;
    }
    case DK_EPI_SILU:
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = silu_f32(rnd<T>(v[k]));
      break;
    case DK_EPI_SILU_MUL: {
      // columns (2j, 2j+1) are (gate, up); outputs n_base / 2 + j
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float s_ = rnd<T>(silu_f32(rnd<T>(v[2 * j])));
        v[j] = __fmul_rn(s_, rnd<T>(v[2 * j + 1]));
      }
      T* dst = C + static_cast<int64_t>(m) * p.ldc + n_base / 2;
      const int nout = ncols / 2;
      if (full && aligned_row<T>(C, p.ldc, n_base / 2)) {
        store_row_vec<T>(dst, v, 16);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < nout) dst[j] = from_f32<T>(v[j]);
      }
      return;
    }
    case DK_EPI_QKV_CACHE: {
      if (n_base >= e.q_cols && (e.q_cols % 32) == 0 && (e.head_dim % 32) == 0 && full) {
        const int j = n_base - e.q_cols;
        const int which = j / e.kv_cols;
        const int jj = j - which * e.kv_cols;
        const int head = jj / e.head_dim, d0 = jj - head * e.head_dim;
        T* cache = static_cast<T*>(which == 0 ? e.k_cache : e.v_cache);
        bool ok;
        const int64_t off = kv_cache_offset(e, m, head, d0, ok);
        if (!ok) return;
        if (reinterpret_cast<uintptr_t>(cache + off) % 16 == 0) {
          store_row_vec<T>(cache + off, v, 32);
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) cache[off + k] = from_f32<T>(v[k]);
        }
        return;
      }
      if (n_base + ncols <= e.q_cols) break;   // all in the q part: plain store below
#pragma unroll
      for (int k = 0; k < 32; ++k)
        if (k < ncols) store_final<T>(p, C, m, n_base + k, v[k]);
      return;
    }
    default:
      break;
  }
  T* dst = C + static_cast<int64_t>(m) * p.ldc + n_base;
  if (full && aligned_row<T>(C, p.ldc, n_base)) {
    store_row_vec<T>(dst, v, 32);
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k)
      if (k < ncols) dst[k] = from_f32<T>(v[k]);
  }
}

// FOLD: a warp's tile t[j] = final value of (token m_first + j, column n_base + lane), transposed
// through the warp's stage tile; then lane L handles token m_first + L.  All 32 lanes call this.
template <typename T>
__device__ __forceinline__ void emit_rows(const Params& p, T* C, float* stage, int mode, int n_base, int m_first,
                                          const float (&t)[32]) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 32; ++j) stage[j * kStagePitch + lane] = t[j];
  __syncwarp();
  float v[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = stage[lane * kStagePitch + k];
  const int m = m_first + lane;
  const int ncols = min(32, p.N - n_base);
  if (m >= p.M || ncols <= 0) return;
  (void)mode;
  store_final_row<T>(p, C, m, n_base, ncols, v);
}

// Thread <-> column n (consecutive columns in consecutive lanes), 32 tokens from m_first.
// Every lane of the warp calls this (the gate/up exchange is a shuffle).
template <typename T>
__device__ __forceinline__ void emit_chunk(const Params& p, T* C, int mode, int n, bool n_ok, int m_first,
                                           const float (&t)[32]) {
  if (mode == FOLD && p.epi.mode == DK_EPI_ARGMAX) {
    unsigned long long k[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int m = m_first + j;
      k[j] = (n_ok && m < p.M) ? argmax_key<T>(t[j], n) : 0ull;
      if (n_ok && m < p.M && C) C[static_cast<int64_t>(m) * p.ldc + n] = from_f32<T>(t[j]);
    }
    const unsigned long long best = warp_max_scatter(k);
    const int m = m_first + (threadIdx.x & 31);
    if (best != 0ull && m < p.M) atomicMax(p.epi.argmax_keys + m, best);
    return;
  }
  if (mode == FOLD && p.epi.mode == DK_EPI_SILU_MUL) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float partner = __shfl_xor_sync(0xffffffffu, t[j], 1);
      const int m = m_first + j;
      if (n_ok && (n & 1) == 0 && m < p.M) store_silu_mul<T>(p, C, m, n >> 1, t[j], partner);
    }
    return;
  }
  if (!n_ok) return;
  if (mode == FOLD) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int m = m_first + j;
      if (m < p.M) store_final<T>(p, C, m, n, t[j]);
    }
  } else if (mode == ATOMIC) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int m = m_first + j;
      if (m < p.M) atomicAdd(p.ws + static_cast<int64_t>(m) * p.N + n, t[j]);
    }
  } else {
    // SPLIT (ws already offset to this unit's group) or PARTIAL
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int m = m_first + j;
      if (m < p.M) p.ws[static_cast<int64_t>(m) * p.N + n] = t[j];
    }
  }
}

// FOLDK: compiled for FOLD launches (final values through the row epilogue); the other
// schedules use the instantiation without it, which keeps their kernel small.
template <typename T, int FMT, bool FOLDK>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int n_stages = stages_for(p.a_rows, p.mode);
  const int stage_bytes = stage_bytes_for(p.a_rows);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingBytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* slot_full = empty + kMaxStages;
  uint64_t* slot_free = slot_full + kSlots;
  uint64_t* drain_bar = slot_free + kSlots;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
#pragma unroll
    for (int k = 0; k < kSlots; ++k) {
      mbar_init(&slot_full[k], 1);
      mbar_init(&slot_free[k], kEpiThreads);
    }
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
  pdl_wait();                 // inputs of this call may come from the previous kernel
  if (threadIdx.x == 0) pdl_launch_dependents();

  const int n_groups = (p.slice_end - p.slice_begin) / p.group;
  const int units = p.n_tiles * p.m_tiles * n_groups;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      int fills = 0;                     // stage fills issued so far (round robin)
      const uint32_t tx_bytes = kSub * (kWTileBytes + p.a_rows * kBK * 2);
      for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x) {
        const int g = u % n_groups;
        const int t = u / n_groups;
        int mt, nt;
        tile_coords(p, t, mt, nt);
        for (int si = 0; si < p.group && !abort_flag; ++si) {
          const int s = p.slice_begin + g * p.group + si;
          int k0, k1;
          slice_bounds(p, s, k0, k1);
          const int nkb = (k1 - k0 + kStageK - 1) / kStageK;
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, kDetProdEmpty, abort_flag)) break;
            uint8_t* st = smem + stage * stage_bytes;
            mbar_arrive_expect_tx(&full[stage], tx_bytes);
            // both sub-blocks are always loaded (past the slice's end their MMAs are not issued;
            // past the K range held in memory the copy reads zeros), so the byte count is fixed
#pragma unroll
            for (int sb = 0; sb < kSub; ++sb) {
              const int kl = k0 + kb * kStageK + sb * kBK - p.k_base;   // inside the K range in memory
              uint8_t* wst = st + sb * kWTileBytes;
              tma_load_2d(wst, &tmB, &full[stage], nt * kTileN, kl);
              tma_load_2d(wst + kWBoxBytes, &tmB, &full[stage], nt * kTileN + 64, kl);
              tma_load_2d(st + kSub * kWTileBytes + sb * p.a_rows * kBK * 2, &tmA, &full[stage], kl, mt * kTileM);
            }
            ++fills;
            if (++stage == n_stages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      // Drain: every copy this thread issued must have landed before the CTA exits.
      bool drain_abort = false;
      for (int f = (fills > n_stages ? fills - n_stages : 0); f < fills; ++f) {
        mbar_wait(&full[f % n_stages], static_cast<uint32_t>((f / n_stages) & 1), kDetDrain, drain_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer (one thread) ----------------
      bool abort_flag = false;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t use_par = 0;   // bit k: parity of the number of times slot k has been written
      int ordinal = 0;
      // token columns per instruction: the loaded rows rounded up to 16 (an element's bits do not
      // depend on the instruction's N), so a few decode tokens do not read 128 rows of operand
      const uint32_t n_mma = static_cast<uint32_t>((p.a_rows + 15) / 16 * 16);
      const uint32_t idesc = umma_idesc_f16(FMT, /*a_mn=*/1, /*b_mn=*/0, kTileN, n_mma);
      for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x, ++ordinal) {
        const int g = u % n_groups;
        for (int si = 0; si < p.group && !abort_flag; ++si) {
          const int s = p.slice_begin + g * p.group + si;
          int k0, k1;
          slice_bounds(p, s, k0, k1);
          const int nkb = (k1 - k0 + kStageK - 1) / kStageK;
          const int slot = slot_of(si, ordinal, p.group);
          // the slot's previous value must have been released by the epilogue
          if (!mbar_wait(&slot_free[slot], ((use_par >> slot) & 1u) ^ 1u, kDetMmaSlotFree, abort_flag)) break;
          use_par ^= 1u << slot;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * kTileM);
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&full[stage], phase, kDetMmaFull, abort_flag)) break;
            tc_fence_after();
            const int kk = k0 + kb * kStageK;
            const int nsteps = min(kStageK / kUK, (k1 - kk + kUK - 1) / kUK);
            const uint32_t b_base = smem_u32(smem + stage * stage_bytes);
            const uint32_t a_base = b_base + kSub * kWTileBytes;
            for (int j = 0; j < nsteps; ++j) {
              const int sb = j >> 2, jj = j & 3;   // sub-block, 16-deep step inside it
              // B (weights) MN-major, 128B swizzle: 64-column groups 8 KB apart (LBO),
              // 8-row K groups 1 KB apart (SBO); one 16-deep K step = 2 KB.
              const uint64_t bdesc = umma_sdesc(b_base + sb * kWTileBytes + jj * 2048, kWBoxBytes, 1024, 2);
              // A (tokens) K-major, 128B swizzle: 8-row groups 1 KB apart; 16 K = 32 bytes.
              const uint64_t adesc = umma_sdesc(a_base + sb * (p.a_rows * kBK * 2) + jj * 32, 16, 1024, 2);
              tc_mma_f16(d_tmem, bdesc, adesc, idesc, (kb > 0 || j > 0) ? 1u : 0u);
            }
            tc_commit(&empty[stage]);
            if (++stage == n_stages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (abort_flag) break;
          tc_commit(&slot_full[slot]);
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
    // lane <-> output column n; each thread handles 64 token columns.
    bool abort_flag = false;
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int n_local = quarter * 32 + lane;      // D row = weight column inside the tile
    const int col0 = half * kEpiCols;             // first token column of this thread
    uint32_t use_par = 0;                         // bit k: parity of slot k's fills consumed
    int ordinal = 0;
    T* C = reinterpret_cast<T*>(p.c);
    float* stage = reinterpret_cast<float*>(smem + kRingBytes - kEpiStageBytes) + (warp - 2) * (32 * kStagePitch);
    const int64_t MN = static_cast<int64_t>(p.M) * p.N;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(col0);
    for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x, ++ordinal) {
      const int g = u % n_groups;
      const int t = u / n_groups;
      int mt, nt;
      tile_coords(p, t, mt, nt);
      const int n = nt * kTileN + n_local;
      const int m0 = mt * kTileM + col0;
      // 32-token chunks of this thread's columns that hold tokens below M (warp-uniform): the
      // others are never stored, so their partial sums are neither read nor folded
      const int c_end = (p.M > m0) ? min(kEpiCols / 32, (p.M - m0 + 31) / 32) : 0;
      const bool n_ok = n < p.N;
      Params q = p;
      if (p.mode == SPLIT) q.ws = p.ws + static_cast<int64_t>(g) * MN;
      uint32_t stack = 0;                        // slot of the pending left operand of level l: bits 2l..2l+1

      for (int si = 0; si < p.group; ++si) {
        const int s = p.slice_begin + g * p.group + si;
        int k0, k1;
        slice_bounds(p, s, k0, k1);
        const bool empty_slice = (k1 <= k0);
        const int slot = slot_of(si, ordinal, p.group);
        if (!mbar_wait(&slot_full[slot], (use_par >> slot) & 1u, kDetEpiSlotFull, abort_flag)) break;
        use_par ^= 1u << slot;
        tc_fence_after();
        const int nlev = __ffs(~si) - 1;          // trailing ones of si: tree levels closed here
        const bool last = (si + 1 == p.group);
        const uint32_t x_addr = lane_base + static_cast<uint32_t>(slot * kTileM);
        if (nlev == 0 && !last) {
          // a left operand: it waits in its slot (an empty slice is stored as zeros)
          if (empty_slice) {
            float z[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) z[j] = 0.0f;
            for (int c = 0; c < c_end; ++c) tmem_st_32x32b_x32(x_addr + c * 32, z);
            tmem_st_wait();
          }
          stack = (stack & ~3u) | static_cast<uint32_t>(slot);
          continue;
        }
        const int res_slot = (nlev > 0) ? static_cast<int>((stack >> (2 * (nlev - 1))) & 3u) : slot;
#pragma unroll 1
        for (int c = 0; c < c_end; ++c) {
          // this slice's chunk and the pending left operand of the first level it closes, read
          // before one wait; further levels (groups of 4 and 8) are read one at a time
          float acc[32];
          float left[32];
          if (!empty_slice) tmem_ld_32x32b_x32(x_addr + c * 32, acc);
          if (nlev > 0) tmem_ld_32x32b_x32(lane_base + (stack & 3u) * kTileM + c * 32, left);
          tmem_ld_wait();
          if (empty_slice) {
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
          }
          // close the tree levels: acc = stack[l] + acc for l = 0 .. nlev-1
          if (nlev > 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(left[j], acc[j]);
          }
#pragma unroll 1
          for (int l = 1; l < nlev; ++l) {
            tmem_ld_32x32b_x32(lane_base + ((stack >> (2 * l)) & 3u) * kTileM + c * 32, left);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(left[j], acc[j]);
          }
          if (last) {
            if constexpr (FOLDK) {
              emit_rows<T>(q, C, stage, p.mode, nt * kTileN + quarter * 32, m0 + c * 32, acc);
            } else {
              // f32 partials: consecutive lanes write consecutive columns (128-byte warp stores)
              emit_chunk<T>(q, C, p.mode, n, n_ok, m0 + c * 32, acc);
            }
          } else {
            tmem_st_32x32b_x32(lane_base + static_cast<uint32_t>(res_slot * kTileM) + c * 32, acc);
          }
        }
        if (!last) tmem_st_wait();
        tc_fence_before();
        // release every slot consumed here; the result slot stays unless this was the unit's end
        if (nlev > 0) mbar_arrive_relaxed(&slot_free[slot]);
        for (int l = 0; l + 1 < nlev; ++l) mbar_arrive_relaxed(&slot_free[(stack >> (2 * l)) & 3u]);
        if (last) mbar_arrive_relaxed(&slot_free[res_slot]);
        if (!last) stack = (stack & ~(3u << (2 * nlev))) | (static_cast<uint32_t>(res_slot) << (2 * nlev));
      }
      if (abort_flag) break;

    }
  }

  // Each warp converges before the CTA barrier: in warps 0 and 1 only lane 0
  // ran the producer / MMA loop, and an aligned barrier must be reached by the
  // whole warp together, or it can release before the epilogue is done.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// out[m, n] = upper tree levels over n_parts aligned subtree sums, partials
// [n_parts][M][N] f32.  Used by SPLIT launches (as a programmatic dependent of
// the GEMM) and for the row-parallel TP combine.  Each thread sums 4
// consecutive columns with 16-byte loads when N allows.
template <typename T>
__global__ void __launch_bounds__(256) fold_groups_kernel(const float* __restrict__ partials, int n_parts, const Params p) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int M = p.M, N = p.N;
  T* c = static_cast<T*>(p.c);
  const int64_t MN = static_cast<int64_t>(M) * N;
  const int64_t quads = (static_cast<int64_t>(N) + 3) / 4;
  const int64_t total = static_cast<int64_t>(M) * quads;
  const bool vec = (N % 4) == 0;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = idx / quads;
    const int n0 = static_cast<int>(idx - m * quads) * 4;
    const int64_t base = m * N + n0;
    float v[kSlices][4];
#pragma unroll
    for (int j = 0; j < kSlices; ++j) {
      if (j < n_parts) {
        if (vec) {
          const float4 q = __ldcg(reinterpret_cast<const float4*>(partials + j * MN + base));
          v[j][0] = q.x;
          v[j][1] = q.y;
          v[j][2] = q.z;
          v[j][3] = q.w;
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) v[j][e] = (n0 + e < N) ? __ldcg(partials + j * MN + base + e) : 0.0f;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[j][e] = 0.0f;
      }
    }
    float fin[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float col[kSlices];
#pragma unroll
      for (int j = 0; j < kSlices; ++j) col[j] = v[j][e];
      fin[e] = tree_sum(col, n_parts);
    }
    if (p.epi.mode == DK_EPI_ARGMAX) {
      unsigned long long best = 0ull;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (n0 + e < N) {
          const unsigned long long key = argmax_key<T>(fin[e], n0 + e);
          best = key > best ? key : best;
          if (c) c[m * p.ldc + n0 + e] = from_f32<T>(fin[e]);
        }
      }
      atomicMax(p.epi.argmax_keys + m, best);
    } else if (p.epi.mode == DK_EPI_SILU_MUL) {
      // n0 is a multiple of 4: pairs (n0, n0+1) and (n0+2, n0+3); N is even
      if (n0 + 1 < N) store_silu_mul<T>(p, c, static_cast<int>(m), n0 >> 1, fin[0], fin[1]);
      if (n0 + 3 < N) store_silu_mul<T>(p, c, static_cast<int>(m), (n0 >> 1) + 1, fin[2], fin[3]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (n0 + e < N) store_final<T>(p, c, static_cast<int>(m), n0 + e, fin[e]);
    }
  }
}

// Four consecutive columns n0 .. n0+3 (n0 a multiple of 4) of row m of partial j of
// [n_parts][M][N] f32; vec: N % 4 == 0 (one 16-byte load).
__device__ __forceinline__ float4 load_quad(const float* __restrict__ partials, int j, int64_t MN, int N, int64_t m,
                                            int n0, bool vec) {
  const float* src = partials + j * MN + m * N + n0;
  if (vec) return __ldcg(reinterpret_cast<const float4*>(src));
  float4 q;
  q.x = __ldcg(src);
  q.y = (n0 + 1 < N) ? __ldcg(src + 1) : 0.0f;
  q.z = (n0 + 2 < N) ? __ldcg(src + 2) : 0.0f;
  q.w = (n0 + 3 < N) ? __ldcg(src + 3) : 0.0f;
  return q;
}

// DK_EPI_RESIDUAL_RMSNORM after a SPLIT launch: one CTA of kRmsThreads per row m.
// h[m, :] = round(R[m, :] + round(upper tree levels over the partials)) is stored to C,
// then y[m, :] = RMSNorm(h[m, :]) * w -- with the invariant RMSNorm kernel's chunk
// ownership (thread t: 16-byte chunks t, t + 256, ...), its x^2 accumulation order and
// its butterflies, so h and y carry the bits of the fold kernel followed by that kernel.
// Needs N % VEC == 0, N <= MAXC * 256 * VEC and 16-byte aligned rows of C and y.
template <typename T, typename W, int MAXC>
__global__ void __launch_bounds__(kRmsThreads) fold_residual_rmsnorm_kernel(const float* __restrict__ partials,
                                                                            int n_parts, const Params p,
                                                                            const W* __restrict__ w, T* y,
                                                                            int64_t ldy, float eps) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  constexpr int VEC = Vec16<T>::N;
  __shared__ float red[9];
  const int64_t m = blockIdx.x;
  const int N = p.N;
  const int64_t MN = static_cast<int64_t>(p.M) * N;
  const int nchunks = N / VEC;
  const T* R = static_cast<const T*>(p.epi.resid) + m * p.epi.ld_resid;
  T* hr = static_cast<T*>(p.c) + m * p.ldc;
  Vec16<T> keep[MAXC];
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * kRmsThreads;
    if (c < nchunks) {
#pragma unroll
      for (int q = 0; q < VEC / 4; ++q) {
        const int n0 = c * VEC + 4 * q;
        float4 v[kSlices];
#pragma unroll
        for (int j = 0; j < kSlices; ++j)
          v[j] = (j < n_parts) ? load_quad(partials, j, MN, N, m, n0, true) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float col[kSlices];
#pragma unroll
          for (int j = 0; j < kSlices; ++j) col[j] = e == 0 ? v[j].x : (e == 1 ? v[j].y : (e == 2 ? v[j].z : v[j].w));
          const float fin = tree_sum(col, n_parts);
          // the residual element is read before this thread overwrites it (R may be C)
          keep[i].v[4 * q + e] = from_f32<T>(__fadd_rn(to_f32<T>(R[n0 + e]), rnd<T>(fin)));
        }
      }
      *reinterpret_cast<Vec16<T>*>(hr + c * VEC) = keep[i];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = to_f32<T>(keep[i].v[j]);
        acc = __fmaf_rn(f, f, acc);
      }
    }
  }
  const float total = block_sum_256(acc, red);
  const float var = __fdiv_rn(total, static_cast<float>(N));
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  T* yr = y + m * ldy;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * kRmsThreads;
    if (c < nchunks) {
      Vec16<T> o;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float xn = __fmul_rn(to_f32<T>(keep[i].v[j]), rstd);
        o.v[j] = from_f32<T>(__fmul_rn(xn, to_f32<W>(w[c * VEC + j])));
      }
      *reinterpret_cast<Vec16<T>*>(yr + c * VEC) = o;
    }
  }
}

// keys[r] -> tokens[r] (column = ~low word), keys reset, lengths advanced.
__global__ void argmax_finish_kernel(unsigned long long* __restrict__ keys, int64_t n_rows, int64_t* tokens,
                                     int64_t* tokens_copy, int32_t* lens_a, int32_t* lens_b) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < n_rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long k = keys[r];
    const int64_t col = static_cast<int64_t>(~static_cast<uint32_t>(k & 0xffffffffull));
    tokens[r] = col;
    if (tokens_copy) tokens_copy[r] = col;
    keys[r] = 0ull;
    if (lens_a) lens_a[r] += 1;
    if (lens_b) lens_b[r] += 1;
  }
}

// Column offsets of the parts of a column-parallel argmax (at most 8 tensor-parallel ranks).
struct PartOffsets {
  int64_t v[8];
};

// Cross-part argmax: part p's keys (local column indices) become global by subtracting
// offsets.v[p] from the key (its low word is ~column), the largest key over the parts wins
// (largest value, then smallest global column), then as argmax_finish_kernel.
__global__ void argmax_finish_parts_kernel(const unsigned long long* __restrict__ keys, int n_parts,
                                           int64_t part_stride, PartOffsets offs, int64_t n_rows, int64_t* tokens,
                                           int64_t* tokens_copy, int32_t* lens_a, int32_t* lens_b,
                                           unsigned long long* reset_keys) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < n_rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    unsigned long long best = 0ull;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q < n_parts) {
        unsigned long long k = keys[q * part_stride + r];
        if (k != 0ull) k -= static_cast<unsigned long long>(offs.v[q]);
        best = k > best ? k : best;
      }
    }
    const int64_t col = static_cast<int64_t>(~static_cast<uint32_t>(best & 0xffffffffull));
    tokens[r] = col;
    if (tokens_copy) tokens_copy[r] = col;
    if (reset_keys) reset_keys[r] = 0ull;
    if (lens_a) lens_a[r] += 1;
    if (lens_b) lens_b[r] += 1;
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
