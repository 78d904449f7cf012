// Gated delta rule, chunked forward on 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// bf16 inputs, head dim 128.
//
// Chunk algebra (64-token chunks cut from each sequence's start; gamma = cumulative log decay):
//   A   = beta_t exp(gamma_t - gamma_j) (K K^T)_tj   for j < t           [64 x 64] f32
//   T   = (I + A)^-1                                   (forward substitution, f32)
//   R   = beta_t (V - exp(gamma_t) K S0)                                  [64 x 128]
//   V'  = T R
//   O   = scale exp(gamma_t) Q S0 + P V',   P_tj = scale exp(gamma_t - gamma_j) (Q K^T)_tj, j <= t
//   S1  = exp(gamma_last) S0 + K^T (w . V'),  w_t = exp(gamma_last - gamma_t)
//
// Every product with a 128-long dimension runs on tcgen05.mma with M = 128 (one TMEM lane per
// row, one thread per lane), arranged so that each operand is in a layout that is either loaded
// by TMA or written row by row by the thread that owns the row:
//   GQ   = [K; Q] K^T          M = 128 (K rows, then Q rows)   N = 64 tokens   K = 128 key dims
//   KS^T = S0^T K^T, QS^T = S0^T Q^T   M = 128 value dims      N = 64 tokens   K = 128 key dims
//   V'^T = R^T T^T             M = 128 value dims               N = 64 tokens   K = 64 tokens
//   O^T  = scale exp(gamma) QS^T + V'^T P^T                     N = 64 tokens   K = 64 tokens
//   S   += K^T (w . V')        M = 128 key dims                 N = 128 value dims, K = 64 tokens
// The state S (key dims x value dims) stays in TMEM in f32 for the whole sequence.  f32 operands
// (S0, R, T, V', P, w . V') enter as bf16 pairs x = hi + lo (hi = bf16(x), lo = bf16(x - hi)); a
// product of a split operand with an exact bf16 one is hi + lo, of two split operands
// hi.hi + hi.lo + lo.hi (the lo.lo term is below f32 rounding of the sum).
//
// One CTA (256 threads, two per TMEM lane) owns one (sequence, value head).  Every sum has a fixed order and a
// sequence's chunks never read another sequence's tokens (rows past the sequence's end are
// zeroed in shared memory), so results do not depend on the rest of the pack.  Thread 0 issues
// the tensor-core work and the TMA copies; every wait is bounded.
#pragma once

#include "dk_common.cuh"
#include "dk_gdn.cuh"

namespace dk {
namespace gdn {

constexpr int kUmThreads = 256;   // two threads per TMEM lane: warps w and w + 4 split the columns
constexpr int kUmD = 128;
// shared memory (bytes from the 1 KB aligned base)
constexpr int kUmKQ = 32768;                 // one [K; Q] chunk: 2 key-dim boxes x (K 8 KB, Q 8 KB)
constexpr int kUmOKQ0 = 0;
constexpr int kUmOKQ1 = kUmOKQ0 + kUmKQ;
constexpr int kUmOV = kUmOKQ1 + kUmKQ;       // V chunk: 2 value-dim boxes of [64 tokens x 64] (16 KB)
constexpr int kUmOS = kUmOV + 16384;         // S0^T hi, lo (2 x 32 KB); later A, T (f32), w.V' hi/lo
constexpr int kUmOR = kUmOS + 65536;         // R^T hi, lo (2 x 16 KB); later V'^T hi, lo
constexpr int kUmOP = kUmOR + 32768;         // P hi, lo (2 x 8 KB)
constexpr int kUmOT = kUmOP + 16384;         // T hi, lo (2 x 8 KB)
constexpr int kUmOVec = kUmOT + 16384;       // gamma, exp(gamma), beta, w (4 x 64 f32)
constexpr int kUmOBar = kUmOVec + 1024;      // mbarriers
constexpr int kUmSmem = kUmOBar + 128 + 1024;   // + alignment slack
constexpr int kUmFPitch = 65;                // f32 pitch of the A and T tiles
// TMEM columns
constexpr uint32_t kUmTmS = 0, kUmTmGQ = 128, kUmTmKS = 192, kUmTmO = 256, kUmTmVp = 320;
constexpr uint32_t kUmTmCols = 512;

// Byte offset of 16-byte chunk c of 128-byte row r in a 128B-swizzled tile (1 KB aligned).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

// 64 f32 values of one row -> bf16 hi and lo rows (128 B each) of two 128B-swizzled tiles.
__device__ __forceinline__ void store_split_row(uint8_t* hi_tile, uint8_t* lo_tile, int r, const float (&x)[64]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = x[8 * c + 2 * e], b = x[8 * c + 2 * e + 1];
      const __nv_bfloat16 ha = __float2bfloat16_rn(a), hb = __float2bfloat16_rn(b);
      const __nv_bfloat16 la = __float2bfloat16_rn(__fsub_rn(a, __bfloat162float(ha)));
      const __nv_bfloat16 lb = __float2bfloat16_rn(__fsub_rn(b, __bfloat162float(hb)));
      h[e] = static_cast<uint32_t>(__bfloat16_as_ushort(ha)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hb)) << 16);
      l[e] = static_cast<uint32_t>(__bfloat16_as_ushort(la)) | (static_cast<uint32_t>(__bfloat16_as_ushort(lb)) << 16);
    }
    *reinterpret_cast<uint4*>(hi_tile + sw128(r, c)) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_tile + sw128(r, c)) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// 32 f32 values -> the bf16 hi and lo of half h (16-byte chunks 4h .. 4h + 3) of row r.
__device__ __forceinline__ void store_split_half(uint8_t* hi_tile, uint8_t* lo_tile, int r, int h, const float (&x)[32]) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const int c = 4 * h + cc;
    uint32_t hv[4], lv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = x[8 * cc + 2 * e], b = x[8 * cc + 2 * e + 1];
      const __nv_bfloat16 ha = __float2bfloat16_rn(a), hb = __float2bfloat16_rn(b);
      const __nv_bfloat16 la = __float2bfloat16_rn(__fsub_rn(a, __bfloat162float(ha)));
      const __nv_bfloat16 lb = __float2bfloat16_rn(__fsub_rn(b, __bfloat162float(hb)));
      hv[e] = static_cast<uint32_t>(__bfloat16_as_ushort(ha)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hb)) << 16);
      lv[e] = static_cast<uint32_t>(__bfloat16_as_ushort(la)) | (static_cast<uint32_t>(__bfloat16_as_ushort(lb)) << 16);
    }
    *reinterpret_cast<uint4*>(hi_tile + sw128(r, c)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    *reinterpret_cast<uint4*>(lo_tile + sw128(r, c)) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
  }
}

// 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tm_ld32(uint32_t taddr, float (&x)[32]) {
  tmem_ld_32x32b_x32(taddr, x);
  tmem_ld_wait();
}

// 64 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tm_ld64(uint32_t taddr, float (&x)[64]) {
  float a[32], b[32];
  tmem_ld_32x32b_x32(taddr, a);
  tmem_ld_32x32b_x32(taddr + 32, b);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    x[j] = a[j];
    x[32 + j] = b[j];
  }
}

// K-major operand, 128B swizzle: 8-row groups 1 KB apart; a 16-deep K step advances 32 bytes.
__device__ __forceinline__ uint64_t kmaj(uint32_t saddr) { return umma_sdesc(saddr, 16, 1024, 2); }
// MN-major operand, 128B swizzle: 64-element M groups `group_bytes` apart; 8 K rows per 1 KB.
__device__ __forceinline__ uint64_t mnmaj(uint32_t saddr, uint32_t group_bytes) {
  return umma_sdesc(saddr, group_bytes, 1024, 2);
}

// exp(x) for x <= 0 as 2^(x log2 e) by the single hardware instruction (relative error ~2^-22);
// used for the decay factors exp(gamma_t - gamma_j) of the chunk's 64 x 64 matrices.
__device__ __forceinline__ float um_exp_nonpos(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmul_rn(x, 1.44269504088896341f)));
  return y;
}

enum : int {
  kDetUmLoad = 0x540,
  kDetUmMma = 0x541,
  kDetUmDrain = 0x542,
};

// Thread 0: the K, Q (both into buffer `kq`) and V copies of chunk rows [row0, row0 + 64).
__device__ __forceinline__ void um_issue_loads(const CUtensorMap* tmK, const CUtensorMap* tmQ, const CUtensorMap* tmV,
                                               uint8_t* kq, uint8_t* vt, uint64_t* bar, int kx, int vx, int row0) {
  mbar_arrive_expect_tx(bar, kUmKQ + 16384);   // K and Q 32 KB, V 16 KB
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    tma_load_2d(kq + b * 16384, tmK, bar, kx + 64 * b, row0);
    tma_load_2d(kq + b * 16384 + 8192, tmQ, bar, kx + 64 * b, row0);
    tma_load_2d(vt + b * 8192, tmV, bar, vx + 64 * b, row0);
  }
}

// Thread 0: the MMAs of one product, `steps` 16-deep K steps per operand pair, accumulate from
// the first step if `acc0`.
__device__ __forceinline__ void um_mma(uint32_t d, uint32_t idesc, uint64_t a, uint64_t b, int steps, uint32_t a_step,
                                       uint32_t b_step, bool acc0) {
  for (int s = 0; s < steps; ++s)
    tc_mma_f16(d, a + ((a_step * s) >> 4), b + ((b_step * s) >> 4), idesc, (acc0 || s > 0) ? 1u : 0u);
}

// One level of the blocked inverse: the blocks (b, c) with b - c = LVL from the levels below.
//   M_bc = sum_{d=c}^{b-1} A_bd T_dc,  then  T_bc = -T_bb M_bc   (thread: element e = tid + 256 i)
template <int LVL>
__device__ __forceinline__ void um_inverse_level(const float* Af, float* Tf, float* Mf, int tid) {
  constexpr int kBlocks = 4 - LVL;
#pragma unroll
  for (int i = 0; i < kBlocks; ++i) {
    const int e = tid + kUmThreads * i;
    const int cb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
    const int bb = cb + LVL;
    float acc = 0.0f;
#pragma unroll
    for (int dd = 0; dd < LVL; ++dd) {
      const int d = cb + dd;
      const float* arow = Af + (16 * bb + r) * kUmFPitch + 16 * d;
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) acc = __fmaf_rn(arow[kk], Tf[(16 * d + kk) * kUmFPitch + 16 * cb + cc], acc);
    }
    Mf[e] = acc;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kBlocks; ++i) {
    const int e = tid + kUmThreads * i;
    const int cb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
    const int bb = cb + LVL;
    const float* trow = Tf + (16 * bb + r) * kUmFPitch + 16 * bb;
    float acc = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 16; ++kk)
      if (kk <= r) acc = __fmaf_rn(trow[kk], Mf[(cb << 8) + (kk << 4) + cc], acc);
    Tf[(16 * bb + r) * kUmFPitch + 16 * cb + cc] = -acc;
  }
  __syncthreads();
}

// One CTA per (value head, sequence); D = 128, bf16 q / k / v / o.
__global__ void __launch_bounds__(kUmThreads, 1)
    gdn_chunk_umma_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t um_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(um_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kqb[2] = {sm + kUmOKQ0, sm + kUmOKQ1};
  uint8_t* Vt = sm + kUmOV;
  uint8_t* Sh = sm + kUmOS;                 // S0^T hi (MN-major, two 64-column groups of 16 KB)
  uint8_t* Sl = Sh + 32768;
  float* Af = reinterpret_cast<float*>(sm + kUmOS);   // after the S0 operands are consumed
  float* Tf = Af + kChunk * kUmFPitch;
  float* Mf = Tf + kChunk * kUmFPitch;      // [3][16][16] scratch of the blocked inverse
  uint8_t* Wh = sm + kUmOS + 32768;         // (w . V')^T hi, lo (after T is split)
  uint8_t* Wl = Wh + 16384;
  uint8_t* Rh = sm + kUmOR;                 // R^T hi, lo; then V'^T hi, lo
  uint8_t* Rl = Rh + 16384;
  uint8_t* Ph = sm + kUmOP;
  uint8_t* Pl = Ph + 8192;
  uint8_t* Th = sm + kUmOT;
  uint8_t* Tl = Th + 8192;
  float* gam = reinterpret_cast<float*>(sm + kUmOVec);
  float* egam = gam + kChunk;
  float* bet = egam + kChunk;
  float* wl = bet + kChunk;
  uint64_t* ld_bar = reinterpret_cast<uint64_t*>(sm + kUmOBar);   // [2], one per K/Q buffer
  uint64_t* mma_bar = ld_bar + 2;
  uint32_t* tm_holder = reinterpret_cast<uint32_t*>(mma_bar + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lrow = ((warp & 3) << 5) | (tid & 31);   // this thread's TMEM lane = the row it owns
  const int half = warp >> 2;                        // which half of the row's columns it handles
  const int hv = blockIdx.x;
  const int n = blockIdx.y;
  const int HV = p.HV;
  const int hq = hv / (HV / p.H);
  pdl_wait();
  int64_t bos, len;
  if (!seq_range(p, n, bos, len)) return;   // the same for every thread of the CTA
  const int nch = static_cast<int>((len + kChunk - 1) / kChunk);

  if (tid == 0) {
    mbar_init(&ld_bar[0], 1);
    mbar_init(&ld_bar[1], 1);
    mbar_init(mma_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 0) {
    tmem_alloc(tm_holder, kUmTmCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = *tm_holder;
  const uint32_t tl = tm + (static_cast<uint32_t>((warp & 3) * 32) << 16);   // this thread's TMEM lane
  const int kx = hq * kUmD, vx = hv * kUmD;
  int loads = 0;        // chunk loads issued (thread 0)
  int consumed = 0;     // chunk loads waited for
  uint32_t mma_phase = 0;
  if (tid == 0 && nch > 0) {
    um_issue_loads(&tmK, &tmQ, &tmV, kqb[0], Vt, &ld_bar[0], kx, vx, static_cast<int>(bos));
    loads = 1;
  }

  // ---- the initial state into TMEM: lane = key dim, column = value dim ----
  const int64_t sbase = (static_cast<int64_t>(n) * HV + hv) * kUmD * kUmD;
#pragma unroll 1
  for (int c = 2 * half; c < 2 * half + 2; ++c) {
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; ++j)
      x[j] = p.h0 ? load_any(p.h0, sbase + static_cast<int64_t>(lrow) * kUmD + 32 * c + j, p.h0_dtype) : 0.0f;
    tmem_st_32x32b_x32(tl + kUmTmS + 32 * c, x);
  }
  tmem_st_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  bool failed = false;
#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    const int buf = c & 1;
    uint8_t* kq = kqb[buf];
    const int64_t row0 = bos + static_cast<int64_t>(c) * kChunk;
    const int L = static_cast<int>((len - c * kChunk) < kChunk ? (len - c * kChunk) : kChunk);

    // ---- P1: chunk data in place; rows past the sequence zeroed; gamma, beta, w ----
    bool ok = mbar_wait(&ld_bar[buf], static_cast<uint32_t>((c >> 1) & 1), kDetUmLoad, failed);
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    consumed = c + 1;
    if (L < kChunk) {
      const int nr = kChunk - L;
      for (int e = tid; e < 6 * nr * 8; e += kUmThreads) {
        const int box = e / (nr * 8), r = L + (e / 8) % nr, ch = e % 8;
        uint8_t* base = (box < 4) ? kq + (box >> 1) * 16384 + (box & 1) * 8192 : Vt + (box - 4) * 8192;
        *reinterpret_cast<uint4*>(base + r * 128 + ch * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    if (tid < kChunk) {
      float gt = 0.0f, bt = 0.0f;
      if (tid < L) {
        gt = load_any(p.g, (row0 + tid) * HV + hv, p.gb_dtype);
        bt = load_any(p.beta, (row0 + tid) * HV + hv, p.gb_dtype);
      }
      const int ln = tid & 31;
      float acc = gt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float up = __shfl_up_sync(0xffffffffu, acc, off);
        if (ln >= off) acc = __fadd_rn(up, acc);
      }
      gam[tid] = acc;
      bet[tid] = bt;
    }
    __syncthreads();
    if (tid >= 32 && tid < kChunk) gam[tid] = __fadd_rn(gam[31], gam[tid]);
    __syncthreads();
    if (tid < kChunk) {
      egam[tid] = expf(gam[tid]);
      wl[tid] = (tid < L) ? expf(__fsub_rn(gam[L - 1], gam[tid])) : 0.0f;
    }
    __syncthreads();

    // ---- P2: S0 -> bf16 pair operand (row = key dim, MN-major); S <- exp(gamma_last) S0 ----
    {
      // thread (key dim lrow, half): value dims [64 half, +64) = one 128-byte row of group `half`
      const float el = egam[L - 1];
      float x[64];
      tm_ld64(tl + kUmTmS + 64 * half, x);
      store_split_row(Sh + half * 16384, Sl + half * 16384, lrow, x);
      float a[32], b[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        a[j] = __fmul_rn(el, x[j]);
        b[j] = __fmul_rn(el, x[32 + j]);
      }
      tmem_st_32x32b_x32(tl + kUmTmS + 64 * half, a);
      tmem_st_32x32b_x32(tl + kUmTmS + 64 * half + 32, b);
      tmem_st_wait();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- P3: GQ = [K; Q] K^T, KS^T = S0^T K^T, QS^T = S0^T Q^T ----
    if (tid == 0) {
      tc_fence_after();
      const uint32_t kqa = smem_u32(kq);
      constexpr uint32_t id_kk = umma_idesc_f16(1, 0, 0, 128, 64);
      constexpr uint32_t id_mk = umma_idesc_f16(1, 1, 0, 128, 64);
      // 16-deep steps over the 128 key dims: 32 bytes inside a 64-dim box, the next box 16 KB on
      for (int s = 0; s < 8; ++s) {
        const uint32_t off = (s >> 2) * 16384 + (s & 3) * 32;
        tc_mma_f16(tm + kUmTmGQ, kmaj(kqa + off), kmaj(kqa + off), id_kk, s > 0 ? 1u : 0u);
      }
      for (int part = 0; part < 2; ++part) {
        const uint32_t sa = smem_u32(part ? Sl : Sh);
        for (int s = 0; s < 8; ++s) {
          const uint32_t off = (s >> 2) * 16384 + (s & 3) * 32;
          const uint64_t a = mnmaj(sa + s * 2048, 16384);
          tc_mma_f16(tm + kUmTmKS, a, kmaj(kqa + off), id_mk, (part | s) ? 1u : 0u);
          tc_mma_f16(tm + kUmTmO, a, kmaj(kqa + 8192 + off), id_mk, (part | s) ? 1u : 0u);
        }
      }
      tc_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_phase, kDetUmMma, failed);
    mma_phase ^= 1u;
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    tc_fence_after();

    // ---- P4: A rows (lanes 0-63) and P rows (64-127); R^T rows; O^T <- scale exp(gamma) QS^T ----
    // (each thread: its lane's row, columns [32 half, +32))
    {
      float x[32];
      tm_ld32(tl + kUmTmGQ + 32 * half, x);
      if (lrow < kChunk) {
        const int t = lrow;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = 32 * half + jj;
          Af[t * kUmFPitch + j] =
              (t < L && j < t) ? __fmul_rn(__fmul_rn(bet[t], um_exp_nonpos(__fsub_rn(gam[t], gam[j]))), x[jj]) : 0.0f;
        }
      } else {
        const int t = lrow - kChunk;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = 32 * half + jj;
          x[jj] = (t < L && j <= t) ? __fmul_rn(__fmul_rn(p.scale, um_exp_nonpos(__fsub_rn(gam[t], gam[j]))), x[jj])
                                    : 0.0f;
        }
        store_split_half(Ph, Pl, t, half, x);
      }
    }
    {
      // lane = value dim dv: R^T[dv][t] = beta_t (V[t][dv] - exp(gamma_t) KS^T[dv][t])
      float x[32];
      tm_ld32(tl + kUmTmKS + 32 * half, x);
      const int b = lrow >> 6, e = lrow & 63;
      const uint8_t* vb = Vt + b * 8192;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int t = 32 * half + jj;
        const __nv_bfloat16 vv = *reinterpret_cast<const __nv_bfloat16*>(vb + sw128(t, e >> 3) + (e & 7) * 2);
        x[jj] = __fmul_rn(bet[t], __fsub_rn(__bfloat162float(vv), __fmul_rn(egam[t], x[jj])));
      }
      store_split_half(Rh, Rl, lrow, half, x);
    }
    {
      float x[32];
      tm_ld32(tl + kUmTmO + 32 * half, x);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) x[jj] = __fmul_rn(__fmul_rn(p.scale, egam[32 * half + jj]), x[jj]);
      tmem_st_32x32b_x32(tl + kUmTmO + 32 * half, x);
      tmem_st_wait();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // the next chunk's copies: its K/Q buffer was last read by the previous chunk's MMAs (done),
    // and V was last read just above
    if (tid == 0 && c + 1 < nch) {
      um_issue_loads(&tmK, &tmQ, &tmV, kqb[buf ^ 1], Vt, &ld_bar[buf ^ 1], kx, vx,
                     static_cast<int>(row0 + kChunk));
      ++loads;
    }

    // ---- P5: T = (I + A)^-1 by 16 x 16 blocks, then T rows -> bf16 pair ----
    // diagonal blocks by forward substitution (threads 0-63: block b, column j)
    if (tid < kChunk) {
      // column j of the block's inverse: x_i = -sum_{k<i} A_ik x_k (x_k = 0 for k < j, x_j = 1),
      // the sum split over even and odd k to halve the dependent chain
      const int b = tid >> 4, j = tid & 15;
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float* arow = Af + (16 * b + i) * kUmFPitch + 16 * b;
        float e0 = 0.0f, e1 = 0.0f;
#pragma unroll
        for (int kk = 0; kk < i; kk += 2) {
          e0 = __fmaf_rn(arow[kk], x[kk], e0);
          if (kk + 1 < i) e1 = __fmaf_rn(arow[kk + 1], x[kk + 1], e1);
        }
        x[i] = (i < j) ? 0.0f : ((i == j) ? 1.0f : -__fadd_rn(e0, e1));
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) Tf[(16 * b + i) * kUmFPitch + 16 * b + j] = x[i];
    }
    for (int e = tid; e < kChunk * kChunk; e += kUmThreads) {
      const int r = e >> 6, cc = e & 63;
      if ((cc >> 4) > (r >> 4)) Tf[r * kUmFPitch + cc] = 0.0f;   // strictly upper blocks
    }
    __syncthreads();
    um_inverse_level<1>(Af, Tf, Mf, tid);
    um_inverse_level<2>(Af, Tf, Mf, tid);
    um_inverse_level<3>(Af, Tf, Mf, tid);
    if (lrow < kChunk) {
      float x[32];
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) x[jj] = Tf[lrow * kUmFPitch + 32 * half + jj];
      store_split_half(Th, Tl, lrow, half, x);
    }
    fence_proxy_async_smem();
    __syncthreads();

    // ---- P6: V'^T = R^T T^T ----
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t id = umma_idesc_f16(1, 0, 0, 128, 64);
      const uint32_t rh = smem_u32(Rh), rl = smem_u32(Rl), th = smem_u32(Th), tlo = smem_u32(Tl);
      um_mma(tm + kUmTmVp, id, kmaj(rh), kmaj(th), 4, 32, 32, false);
      um_mma(tm + kUmTmVp, id, kmaj(rh), kmaj(tlo), 4, 32, 32, true);
      um_mma(tm + kUmTmVp, id, kmaj(rl), kmaj(th), 4, 32, 32, true);
      tc_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_phase, kDetUmMma, failed);
    mma_phase ^= 1u;
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    tc_fence_after();

    // ---- P7: V'^T rows -> bf16 pair (over R^T); (w . V')^T rows -> bf16 pair ----
    {
      float x[32];
      tm_ld32(tl + kUmTmVp + 32 * half, x);
      store_split_half(Rh, Rl, lrow, half, x);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) x[jj] = __fmul_rn(wl[32 * half + jj], x[jj]);
      store_split_half(Wh, Wl, lrow, half, x);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- P8: O^T += V'^T P^T;  S += K^T (w . V') ----
    if (tid == 0) {
      tc_fence_after();
      constexpr uint32_t id_o = umma_idesc_f16(1, 0, 0, 128, 64);
      constexpr uint32_t id_s = umma_idesc_f16(1, 1, 0, 128, 128);
      const uint32_t vh = smem_u32(Rh), vl = smem_u32(Rl), ph = smem_u32(Ph), pl = smem_u32(Pl);
      um_mma(tm + kUmTmO, id_o, kmaj(vh), kmaj(ph), 4, 32, 32, true);
      um_mma(tm + kUmTmO, id_o, kmaj(vh), kmaj(pl), 4, 32, 32, true);
      um_mma(tm + kUmTmO, id_o, kmaj(vl), kmaj(ph), 4, 32, 32, true);
      const uint32_t kqa = smem_u32(kq);
      um_mma(tm + kUmTmS, id_s, mnmaj(kqa, 16384), kmaj(smem_u32(Wh)), 4, 2048, 32, true);
      um_mma(tm + kUmTmS, id_s, mnmaj(kqa, 16384), kmaj(smem_u32(Wl)), 4, 2048, 32, true);
      tc_commit(mma_bar);
    }
    ok = mbar_wait(mma_bar, mma_phase, kDetUmMma, failed);
    mma_phase ^= 1u;
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    tc_fence_after();

    // ---- P9: O rows out (thread = value dim) ----
    {
      float x[32];
      tm_ld32(tl + kUmTmO + 32 * half, x);
      __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.o);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int t = 32 * half + jj;
        if (t < L) o[((row0 + t) * HV + hv) * kUmD + lrow] = __float2bfloat16_rn(x[jj]);
      }
    }
    tc_fence_before();
    __syncthreads();   // TMEM O and the operand tiles are free for the next chunk
    tc_fence_after();
  }

  if (failed) {
    // drain: copies and tensor-core work this CTA started must finish before it exits
    if (tid == 0) {
      bool da = false;
      for (int f = consumed; f < loads; ++f)
        mbar_wait(&ld_bar[f & 1], static_cast<uint32_t>((f >> 1) & 1), kDetUmDrain, da);
      tc_commit(mma_bar);
      da = false;
      mbar_wait(mma_bar, mma_phase, kDetUmDrain, da);
    }
  } else if (p.ht) {
#pragma unroll 1
    for (int c = 2 * half; c < 2 * half + 2; ++c) {
      float x[32];
      tmem_ld_32x32b_x32(tl + kUmTmS + 32 * c, x);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) p.ht[sbase + static_cast<int64_t>(lrow) * kUmD + 32 * c + j] = x[j];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tm, kUmTmCols);
  }
}

}  // namespace gdn
}  // namespace dk
