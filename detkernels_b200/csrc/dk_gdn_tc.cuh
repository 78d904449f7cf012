// Gated delta rule, chunked forward on tensor cores (bf16 inputs, head dims 64 and 128).
//
// The same chunk algebra as gdn_chunk_kernel (dk_gdn.cuh), with every product on
// mma.sync m16n8k16 (bf16 operands, f32 accumulation):
//
//   exact bf16 operands:  G = K K^T, QK = Q K^T, K S, Q S, K^T (w . V')
//   f32 operands (S, T, R, P, w . V') enter as a bf16 pair x = hi + lo with
//   hi = bf16(x), lo = bf16(x - hi); a product X Y of two split operands is
//   Xhi Yhi + Xhi Ylo + Xlo Yhi (the lo*lo term is below f32 rounding of the sum).
//
//   A   = beta_t exp(gamma_t - gamma_j) G_tj   (j < t)         [64 x 64], f32
//   T   = (I + A)^-1  by blocks of 16: diagonal blocks by forward substitution,
//         then T_bc = -T_bb (sum_{d=c}^{b-1} A_bd T_dc) level by level (b - c = 1, 2, 3)
//   R   = beta_t (V - exp(gamma_t) K S0)                       [64 x D]
//   V'  = T R
//   O   = scale exp(gamma_t) Q S0 + P V',  P_tj = scale exp(gamma_t - gamma_j) QK_tj (j <= t)
//   S1  = exp(gamma_last) S0 + K^T (w . V'),  w_t = exp(gamma_last - gamma_t)
//
// The state never leaves f32: it lives in registers as the accumulator fragments
// of the S1 product (each warp owns a fixed set of 16 x 8 state tiles) and is
// copied to shared memory as a bf16 pair only to serve as the B operand of K S0
// and Q S0.  One CTA owns one (sequence, value head); chunks are cut from the
// sequence's start; every sum has a fixed order, so results do not depend on the
// other sequences of the call.
#pragma once

#include "dk_common.cuh"
#include "dk_gdn.cuh"

namespace dk {
namespace gdn {

constexpr int kTcThreads = 256;   // 8 warps
constexpr int kTPitch = kChunk + 8;   // bf16 pitch of [64][64] tiles (T, P)
constexpr int kFPitch = kChunk + 4;   // f32 pitch of [64][64] tiles (A, T)

template <int D>
struct TcSmem {
  static constexpr int DP = D + 8;                          // bf16 pitch of [rows][D] tiles
  static constexpr int kTile = kChunk * DP * 2;             // one [64][D] bf16 tile, bytes
  static constexpr int kX = (2 * D * DP * 2 > 4 * kTile) ? 2 * D * DP * 2 : 4 * kTile;
  static constexpr int oK = 0;                              // K           [64][DP]
  static constexpr int oQ = oK + kTile;                     // Q, then R hi
  static constexpr int oV = oQ + kTile;                     // V, then R lo
  static constexpr int oX = oV + kTile;                     // S hi/lo [D][DP]; then V' hi/lo, wV' hi/lo
  static constexpr int oA = oX + kX;                        // A  f32 [64][kFPitch]
  static constexpr int oT = oA + kChunk * kFPitch * 4;      // T  f32 [64][kFPitch]
  static constexpr int oM = oT + kChunk * kFPitch * 4;      // level scratch f32 [3][16][16]
  static constexpr int oTh = oM + 3 * 256 * 4;              // T hi, T lo, P hi, P lo bf16 [64][kTPitch]
  static constexpr int oVec = oTh + 4 * kChunk * kTPitch * 2;   // gamma, exp(gamma), beta, w
  static constexpr int kBytes = oVec + 4 * kChunk * 4;
};

__device__ __forceinline__ void tc_ldsm(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void tc_ldsm_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void tc_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// x -> (bf16(x), bf16(x - bf16(x))) for two consecutive values, packed
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
  const __nv_bfloat16 l0 = __float2bfloat16_rn(__fsub_rn(x0, __bfloat162float(h0)));
  const __nv_bfloat16 l1 = __float2bfloat16_rn(__fsub_rn(x1, __bfloat162float(h1)));
  hi = static_cast<uint32_t>(__bfloat16_as_ushort(h0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
  lo = static_cast<uint32_t>(__bfloat16_as_ushort(l0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
}

// A fragment (16 rows x 16 k) of a row-major bf16 tile: rows r0.., k columns k0..
__device__ __forceinline__ void frag_a(const __nv_bfloat16* tile, int pitch, int r0, int k0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  const int r = r0 + (lane & 7) + 8 * ((lane >> 3) & 1);
  const int k = k0 + 8 * (lane >> 4);
  tc_ldsm(smem_u32(tile + r * pitch + k), a[0], a[1], a[2], a[3]);
}
// A fragment of the transpose of a row-major tile X[k][m]: A[m][k] = X[k][m]
__device__ __forceinline__ void frag_a_t(const __nv_bfloat16* tile, int pitch, int m0, int k0, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31;
  const int k = k0 + (lane & 7) + 8 * (lane >> 4);
  const int m = m0 + 8 * ((lane >> 3) & 1);
  tc_ldsm_t(smem_u32(tile + k * pitch + m), a[0], a[1], a[2], a[3]);
}
// B fragments of two adjacent n-tiles from a tile stored [n][k] (row-major by n)
__device__ __forceinline__ void frag_b_nk(const __nv_bfloat16* tile, int pitch, int n0, int k0, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31;
  const int n = n0 + (lane & 7) + 8 * (lane >> 4);
  const int k = k0 + 8 * ((lane >> 3) & 1);
  tc_ldsm(smem_u32(tile + n * pitch + k), b[0], b[1], b[2], b[3]);
}
// B fragments of two adjacent n-tiles from a tile stored [k][n] (row-major by k)
__device__ __forceinline__ void frag_b_kn(const __nv_bfloat16* tile, int pitch, int n0, int k0, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31;
  const int k = k0 + (lane & 7) + 8 * ((lane >> 3) & 1);
  const int n = n0 + 8 * (lane >> 4);
  tc_ldsm_t(smem_u32(tile + k * pitch + n), b[0], b[1], b[2], b[3]);
}

template <int D>
__global__ void __launch_bounds__(kTcThreads, 1) gdn_chunk_tc_kernel(const Params p) {
  using L_ = TcSmem<D>;
  constexpr int DP = L_::DP;
  constexpr int NTS = D / 8;              // n-tiles along d
  constexpr int MTS = D / 16;             // m-tiles along the state rows
  constexpr int SPW = MTS * NTS / 8;      // state tiles per warp
  constexpr int HN = NTS / 2;             // n-tiles per warp in the [64 x D] products
  extern __shared__ __align__(16) uint8_t sm_raw[];
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(sm_raw + L_::oK);
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(sm_raw + L_::oQ);   // later R hi
  __nv_bfloat16* Vs = reinterpret_cast<__nv_bfloat16*>(sm_raw + L_::oV);   // later R lo
  __nv_bfloat16* Shi = reinterpret_cast<__nv_bfloat16*>(sm_raw + L_::oX);
  __nv_bfloat16* Slo = Shi + D * DP;
  __nv_bfloat16* Vph = reinterpret_cast<__nv_bfloat16*>(sm_raw + L_::oX);  // after S hi/lo are consumed
  __nv_bfloat16* Vpl = Vph + kChunk * DP;
  __nv_bfloat16* Wvh = Vpl + kChunk * DP;
  __nv_bfloat16* Wvl = Wvh + kChunk * DP;
  float* Af = reinterpret_cast<float*>(sm_raw + L_::oA);
  float* Tf = reinterpret_cast<float*>(sm_raw + L_::oT);
  float* Mf = reinterpret_cast<float*>(sm_raw + L_::oM);
  __nv_bfloat16* Thi = reinterpret_cast<__nv_bfloat16*>(sm_raw + L_::oTh);
  __nv_bfloat16* Tlo = Thi + kChunk * kTPitch;
  __nv_bfloat16* Phi = Tlo + kChunk * kTPitch;
  __nv_bfloat16* Plo = Phi + kChunk * kTPitch;
  float* gam = reinterpret_cast<float*>(sm_raw + L_::oVec);
  float* egam = gam + kChunk;
  float* bet = egam + kChunk;
  float* wl = bet + kChunk;

  pdl_wait();
  const int hv = blockIdx.x;
  const int n = blockIdx.y;
  const int HV = p.HV;
  const int hq = hv / (HV / p.H);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  int64_t bos, len;
  if (!seq_range(p, n, bos, len)) return;
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(p.q);
  const __nv_bfloat16* k = static_cast<const __nv_bfloat16*>(p.k);
  const __nv_bfloat16* v = static_cast<const __nv_bfloat16*>(p.v);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.o);

  // ---- state tiles of this warp: flat tiles [warp * SPW, +SPW), (m-tile, n-tile) row-major ----
  const int64_t sbase = (static_cast<int64_t>(n) * HV + hv) * D * D;
  float S[SPW][4];
#pragma unroll
  for (int u = 0; u < SPW; ++u) {
    const int ft = warp * SPW + u;
    const int i0 = (ft / NTS) * 16 + g, c0 = (ft % NTS) * 8 + 2 * t4;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = i0 + (e >> 1) * 8, c = c0 + (e & 1);
      S[u][e] = p.h0 ? load_any(p.h0, sbase + static_cast<int64_t>(i) * D + c, p.h0_dtype) : 0.0f;
    }
  }

  // [64 x D] products: m-tile (warp % 4), n-tiles [HN * (warp / 4), +HN)
  const int pm = warp & 3;
  const int pn0 = (warp >> 2) * HN;

  for (int64_t c0 = 0; c0 < len; c0 += kChunk) {
    const int L = static_cast<int>((len - c0) < kChunk ? (len - c0) : kChunk);
    __syncthreads();   // the previous chunk is done with every tile

    // ---- A: chunk loads (bf16 rows, zero past L), gamma / beta ----
    {
      constexpr int CH = kChunk * D / 8;                    // 16-byte chunks per tensor
      constexpr int CPT = CH / kTcThreads;
      uint4 kr[CPT], qr[CPT], vr[CPT];
#pragma unroll
      for (int u = 0; u < CPT; ++u) {
        const int e = tid + u * kTcThreads;
        const int t = e / (D / 8), c = e - t * (D / 8);
        kr[u] = qr[u] = vr[u] = make_uint4(0u, 0u, 0u, 0u);
        if (t < L) {
          const int64_t kq = ((bos + c0 + t) * p.H + hq) * D + c * 8;
          kr[u] = *reinterpret_cast<const uint4*>(k + kq);
          qr[u] = *reinterpret_cast<const uint4*>(q + kq);
          vr[u] = *reinterpret_cast<const uint4*>(v + ((bos + c0 + t) * HV + hv) * D + c * 8);
        }
      }
      float gt = 0.0f, bt = 0.0f;
      if (tid < kChunk && tid < L) {
        gt = load_any(p.g, (bos + c0 + tid) * HV + hv, p.gb_dtype);
        bt = load_any(p.beta, (bos + c0 + tid) * HV + hv, p.gb_dtype);
      }
#pragma unroll
      for (int u = 0; u < CPT; ++u) {
        const int e = tid + u * kTcThreads;
        const int t = e / (D / 8), c = e - t * (D / 8);
        *reinterpret_cast<uint4*>(Ks + t * DP + c * 8) = kr[u];
        *reinterpret_cast<uint4*>(Qs + t * DP + c * 8) = qr[u];
        *reinterpret_cast<uint4*>(Vs + t * DP + c * 8) = vr[u];
      }
      if (tid < kChunk) {
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
    }
    // ---- B: state -> bf16 pair (the B operand of K S0 and Q S0) ----
#pragma unroll
    for (int u = 0; u < SPW; ++u) {
      const int ft = warp * SPW + u;
      const int i0 = (ft / NTS) * 16 + g, cc = (ft % NTS) * 8 + 2 * t4;
      uint32_t hi, lo;
      split2(S[u][0], S[u][1], hi, lo);
      *reinterpret_cast<uint32_t*>(Shi + i0 * DP + cc) = hi;
      *reinterpret_cast<uint32_t*>(Slo + i0 * DP + cc) = lo;
      split2(S[u][2], S[u][3], hi, lo);
      *reinterpret_cast<uint32_t*>(Shi + (i0 + 8) * DP + cc) = hi;
      *reinterpret_cast<uint32_t*>(Slo + (i0 + 8) * DP + cc) = lo;
    }
    __syncthreads();
    if (tid >= 32 && tid < kChunk) gam[tid] = __fadd_rn(gam[31], gam[tid]);
    __syncthreads();
    if (tid < kChunk) {
      egam[tid] = expf(gam[tid]);
      wl[tid] = (tid < L) ? expf(__fsub_rn(gam[L - 1], gam[tid])) : 0.0f;
    }
    __syncthreads();

    // ---- C1: G = K K^T (warps 0-3) and QK = Q K^T (warps 4-7) -> A (f32) and P (bf16 pair) ----
    {
      const __nv_bfloat16* Asrc = (warp < 4) ? Ks : Qs;
      float acc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t a[4];
        frag_a(Asrc, DP, pm * 16, ks * 16, a);
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
          uint32_t b[4];
          frag_b_nk(Ks, DP, jp * 16, ks * 16, b);
          tc_mma(acc[2 * jp], a, b[0], b[1]);
          tc_mma(acc[2 * jp + 1], a, b[2], b[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = pm * 16 + g + 8 * h;
          float val[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jj = j * 8 + 2 * t4 + e;
            const float x = acc[j][2 * h + e];
            if (warp < 4) {
              val[e] = (t < L && jj < t) ? __fmul_rn(__fmul_rn(bet[t], expf(__fsub_rn(gam[t], gam[jj]))), x) : 0.0f;
            } else {
              val[e] = (t < L && jj <= t)
                           ? __fmul_rn(__fmul_rn(p.scale, expf(__fsub_rn(gam[t], gam[jj]))), x)
                           : 0.0f;
            }
          }
          const int jj0 = j * 8 + 2 * t4;
          if (warp < 4) {
            Af[t * kFPitch + jj0] = val[0];
            Af[t * kFPitch + jj0 + 1] = val[1];
          } else {
            uint32_t hi, lo;
            split2(val[0], val[1], hi, lo);
            *reinterpret_cast<uint32_t*>(Phi + t * kTPitch + jj0) = hi;
            *reinterpret_cast<uint32_t*>(Plo + t * kTPitch + jj0) = lo;
          }
        }
      }
    }

    // ---- C2: K S0 and Q S0 for m-tile pm, n-tiles [pn0, pn0 + HN) ----
    float ks_acc[HN][4], qs_acc[HN][4];
#pragma unroll
    for (int j = 0; j < HN; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) ks_acc[j][e] = qs_acc[j][e] = 0.0f;
#pragma unroll 2
    for (int kst = 0; kst < D / 16; ++kst) {
      uint32_t ak[4], aq[4];
      frag_a(Ks, DP, pm * 16, kst * 16, ak);
      frag_a(Qs, DP, pm * 16, kst * 16, aq);
#pragma unroll
      for (int jp = 0; jp < HN / 2; ++jp) {
        uint32_t bh[4], bl[4];
        frag_b_kn(Shi, DP, (pn0 + 2 * jp) * 8, kst * 16, bh);
        frag_b_kn(Slo, DP, (pn0 + 2 * jp) * 8, kst * 16, bl);
        tc_mma(ks_acc[2 * jp], ak, bh[0], bh[1]);
        tc_mma(ks_acc[2 * jp], ak, bl[0], bl[1]);
        tc_mma(ks_acc[2 * jp + 1], ak, bh[2], bh[3]);
        tc_mma(ks_acc[2 * jp + 1], ak, bl[2], bl[3]);
        tc_mma(qs_acc[2 * jp], aq, bh[0], bh[1]);
        tc_mma(qs_acc[2 * jp], aq, bl[0], bl[1]);
        tc_mma(qs_acc[2 * jp + 1], aq, bh[2], bh[3]);
        tc_mma(qs_acc[2 * jp + 1], aq, bl[2], bl[3]);
      }
    }
    // R = beta (V - exp(gamma) K S0) in registers (V read before the barrier below);
    // O starts at scale exp(gamma) Q S0 and stays in qs_acc until P V' is added
#pragma unroll
    for (int j = 0; j < HN; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = pm * 16 + g + 8 * h;
        const int d0 = (pn0 + j) * 8 + 2 * t4;
        const __nv_bfloat162 vv = *reinterpret_cast<const __nv_bfloat162*>(Vs + t * DP + d0);
        const float vx[2] = {__low2float(vv), __high2float(vv)};
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          ks_acc[j][2 * h + e] = __fmul_rn(bet[t], __fsub_rn(vx[e], __fmul_rn(egam[t], ks_acc[j][2 * h + e])));
          qs_acc[j][2 * h + e] = __fmul_rn(__fmul_rn(p.scale, egam[t]), qs_acc[j][2 * h + e]);
        }
      }
    }
    __syncthreads();   // every warp is done reading Q, V and S hi/lo
    // R -> bf16 pair in the Q (hi) and V (lo) tiles
#pragma unroll
    for (int j = 0; j < HN; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = pm * 16 + g + 8 * h;
        const int d0 = (pn0 + j) * 8 + 2 * t4;
        uint32_t hi, lo;
        split2(ks_acc[j][2 * h], ks_acc[j][2 * h + 1], hi, lo);
        *reinterpret_cast<uint32_t*>(Qs + t * DP + d0) = hi;
        *reinterpret_cast<uint32_t*>(Vs + t * DP + d0) = lo;
      }
    }

    // ---- D: T = (I + A)^-1 by 16 x 16 blocks ----
    if (tid < kChunk) {
      // diagonal block b = tid / 16, column j = tid % 16: forward substitution
      const int b = tid >> 4, j = tid & 15;
      float x[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (i < j) {
          x[i] = 0.0f;
        } else if (i == j) {
          x[i] = 1.0f;
        } else {
          float acc = 0.0f;
          const float* arow = Af + (16 * b + i) * kFPitch + 16 * b;
#pragma unroll
          for (int kk = 0; kk < i; ++kk)
            if (kk >= j) acc = __fmaf_rn(arow[kk], x[kk], acc);
          x[i] = -acc;
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) Tf[(16 * b + i) * kFPitch + 16 * b + j] = x[i];
    }
    // zero the strictly upper blocks of T once per chunk (they stay zero)
    for (int e = tid; e < kChunk * kChunk; e += kTcThreads) {
      const int r = e / kChunk, c = e - r * kChunk;
      if ((c >> 4) > (r >> 4)) Tf[r * kFPitch + c] = 0.0f;
    }
    __syncthreads();
#pragma unroll 1
    for (int lvl = 1; lvl < 4; ++lvl) {
      const int nblk = 4 - lvl;   // blocks (b, c) with b - c = lvl, c = 0 .. nblk-1
      // M_bc = sum_{d=c}^{b-1} A_bd T_dc
      for (int e = tid; e < nblk * 256; e += kTcThreads) {
        const int cb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
        const int bb = cb + lvl;
        float acc = 0.0f;
        for (int d = cb; d < bb; ++d) {
          const float* arow = Af + (16 * bb + r) * kFPitch + 16 * d;
#pragma unroll
          for (int kk = 0; kk < 16; ++kk) acc = __fmaf_rn(arow[kk], Tf[(16 * d + kk) * kFPitch + 16 * cb + cc], acc);
        }
        Mf[e] = acc;
      }
      __syncthreads();
      // T_bc = -T_bb M_bc
      for (int e = tid; e < nblk * 256; e += kTcThreads) {
        const int cb = e >> 8, r = (e >> 4) & 15, cc = e & 15;
        const int bb = cb + lvl;
        const float* trow = Tf + (16 * bb + r) * kFPitch + 16 * bb;
        float acc = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
          if (kk <= r) acc = __fmaf_rn(trow[kk], Mf[(cb << 8) + (kk << 4) + cc], acc);
        Tf[(16 * bb + r) * kFPitch + 16 * cb + cc] = -acc;
      }
      __syncthreads();
    }
    // T -> bf16 pair
    for (int e = tid; e < kChunk * kChunk / 2; e += kTcThreads) {
      const int r = e / (kChunk / 2), c = 2 * (e - r * (kChunk / 2));
      uint32_t hi, lo;
      split2(Tf[r * kFPitch + c], Tf[r * kFPitch + c + 1], hi, lo);
      *reinterpret_cast<uint32_t*>(Thi + r * kTPitch + c) = hi;
      *reinterpret_cast<uint32_t*>(Tlo + r * kTPitch + c) = lo;
    }
    __syncthreads();

    // ---- E: V' = T R (same tiles as C2) -> V' and w.V' as bf16 pairs ----
    {
      float vp[HN][4];
#pragma unroll
      for (int j = 0; j < HN; ++j) vp[j][0] = vp[j][1] = vp[j][2] = vp[j][3] = 0.0f;
#pragma unroll
      for (int kst = 0; kst < kChunk / 16; ++kst) {
        uint32_t th[4], tl[4];
        frag_a(Thi, kTPitch, pm * 16, kst * 16, th);
        frag_a(Tlo, kTPitch, pm * 16, kst * 16, tl);
#pragma unroll
        for (int jp = 0; jp < HN / 2; ++jp) {
          uint32_t rh[4], rl[4];
          frag_b_kn(Qs, DP, (pn0 + 2 * jp) * 8, kst * 16, rh);
          frag_b_kn(Vs, DP, (pn0 + 2 * jp) * 8, kst * 16, rl);
          tc_mma(vp[2 * jp], th, rh[0], rh[1]);
          tc_mma(vp[2 * jp], th, rl[0], rl[1]);
          tc_mma(vp[2 * jp], tl, rh[0], rh[1]);
          tc_mma(vp[2 * jp + 1], th, rh[2], rh[3]);
          tc_mma(vp[2 * jp + 1], th, rl[2], rl[3]);
          tc_mma(vp[2 * jp + 1], tl, rh[2], rh[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < HN; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = pm * 16 + g + 8 * h;
          const int d0 = (pn0 + j) * 8 + 2 * t4;
          uint32_t hi, lo;
          split2(vp[j][2 * h], vp[j][2 * h + 1], hi, lo);
          *reinterpret_cast<uint32_t*>(Vph + t * DP + d0) = hi;
          *reinterpret_cast<uint32_t*>(Vpl + t * DP + d0) = lo;
          split2(__fmul_rn(wl[t], vp[j][2 * h]), __fmul_rn(wl[t], vp[j][2 * h + 1]), hi, lo);
          *reinterpret_cast<uint32_t*>(Wvh + t * DP + d0) = hi;
          *reinterpret_cast<uint32_t*>(Wvl + t * DP + d0) = lo;
        }
      }
    }
    __syncthreads();

    // ---- F: O = scale exp(gamma) Q S0 + P V' ----
#pragma unroll
    for (int kst = 0; kst < kChunk / 16; ++kst) {
      uint32_t ph[4], pl[4];
      frag_a(Phi, kTPitch, pm * 16, kst * 16, ph);
      frag_a(Plo, kTPitch, pm * 16, kst * 16, pl);
#pragma unroll
      for (int jp = 0; jp < HN / 2; ++jp) {
        uint32_t vh[4], vl[4];
        frag_b_kn(Vph, DP, (pn0 + 2 * jp) * 8, kst * 16, vh);
        frag_b_kn(Vpl, DP, (pn0 + 2 * jp) * 8, kst * 16, vl);
        tc_mma(qs_acc[2 * jp], ph, vh[0], vh[1]);
        tc_mma(qs_acc[2 * jp], ph, vl[0], vl[1]);
        tc_mma(qs_acc[2 * jp], pl, vh[0], vh[1]);
        tc_mma(qs_acc[2 * jp + 1], ph, vh[2], vh[3]);
        tc_mma(qs_acc[2 * jp + 1], ph, vl[2], vl[3]);
        tc_mma(qs_acc[2 * jp + 1], pl, vh[2], vh[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < HN; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = pm * 16 + g + 8 * h;
        if (t < L) {
          const int d0 = (pn0 + j) * 8 + 2 * t4;
          *reinterpret_cast<__nv_bfloat162*>(o + ((bos + c0 + t) * HV + hv) * D + d0) =
              __floats2bfloat162_rn(qs_acc[j][2 * h], qs_acc[j][2 * h + 1]);
        }
      }
    }

    // ---- G: S = exp(gamma_last) S + K^T (w . V') ----
    {
      const float el = egam[L - 1];
#pragma unroll
      for (int u = 0; u < SPW; ++u)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[u][e] = __fmul_rn(el, S[u][e]);
#pragma unroll
      for (int kst = 0; kst < kChunk / 16; ++kst) {
#pragma unroll
        for (int u = 0; u < SPW; u += 2) {
          // tiles u and u+1 share the m-tile (SPW and NTS are even)
          const int ft = warp * SPW + u;
          const int mt = ft / NTS, nt = ft % NTS;
          uint32_t a[4], wh[4], wlo[4];
          frag_a_t(Ks, DP, mt * 16, kst * 16, a);
          frag_b_kn(Wvh, DP, nt * 8, kst * 16, wh);
          frag_b_kn(Wvl, DP, nt * 8, kst * 16, wlo);
          tc_mma(S[u], a, wh[0], wh[1]);
          tc_mma(S[u], a, wlo[0], wlo[1]);
          tc_mma(S[u + 1], a, wh[2], wh[3]);
          tc_mma(S[u + 1], a, wlo[2], wlo[3]);
        }
      }
    }
  }
  __syncthreads();
  if (p.ht) {
#pragma unroll
    for (int u = 0; u < SPW; ++u) {
      const int ft = warp * SPW + u;
      const int i0 = (ft / NTS) * 16 + g, c0 = (ft % NTS) * 8 + 2 * t4;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        p.ht[sbase + static_cast<int64_t>(i0 + (e >> 1) * 8) * D + c0 + (e & 1)] = S[u][e];
    }
  }
}

}  // namespace gdn
}  // namespace dk
