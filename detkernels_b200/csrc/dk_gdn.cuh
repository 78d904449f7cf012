// Gated delta rule (Gated DeltaNet linear attention), forward, chunked.
//
// Replaces the third-party FLA `chunk_gated_delta_rule` that the reference's
// gdn/repro.py:76,161-162,293-294 calls.  The recurrence per value head, with
// state S in R^{DK x DV} (f32), decay g_t <= 0 (log space), beta_t in (0, 1):
//
//     S <- exp(g_t) S;   v'_t = beta_t (v_t - S^T k_t);   S <- S + k_t v'_t^T;
//     o_t = S^T (scale q_t)
//
// (the published gated delta rule; query/key head of value head j is
// j / (HV / H)).  Chunked form used here, for a chunk of L <= 64 tokens that
// starts with state S0, gamma_t = g_0 + ... + g_t (inclusive; a fixed-order scan):
//
//     A_tj = beta_t exp(gamma_t - gamma_j) k_t.k_j           (j < t)
//     R_t  = beta_t (v_t - exp(gamma_t) S0^T k_t)
//     (I + A) V' = R                                     (forward substitution)
//     o_t  = scale (exp(gamma_t) S0^T q_t + sum_{j<=t} exp(gamma_t - gamma_j) (q_t.k_j) v'_j)
//     S1   = exp(gamma_last) S0 + sum_t exp(gamma_last - gamma_t) k_t v'_t^T
//
// Determinism and invariance: one CTA owns one (sequence, value head) and
// walks its chunks in order; chunks are cut at multiples of 64 tokens from the
// SEQUENCE start, never from the packed-batch start; every reduction has a
// fixed order and all arithmetic is f32 with explicit _rn intrinsics.  A
// sequence's output therefore does not depend on the other sequences of the
// call, on its position in a packed batch, or on the call's total size.
#pragma once

#include "dk_common.cuh"

namespace dk {
namespace gdn {

constexpr int kChunk = 64;
constexpr int kThreads = 256;
constexpr int kPadC = kChunk + 4;  // row stride of transposed [D][chunk] tiles (keeps 16-byte rows)

struct Params {
  const void* q;      // [tokens, H, DK]
  const void* k;      // [tokens, H, DK]
  const void* v;      // [tokens, HV, DV]
  const void* g;      // [tokens, HV]
  const void* beta;   // [tokens, HV]
  void* o;            // [tokens, HV, DV], q's dtype
  const int64_t* cu_seqlens;  // device [n_seq + 1] or null (then sequence n = tokens [n*T, (n+1)*T))
  int64_t seq_len;            // T when cu_seqlens is null; else the packed length (bound of cu_seqlens)
  const void* h0;             // [n_seq, HV, DK, DV] or null (zeros)
  float* ht;                  // [n_seq, HV, DK, DV] f32 or null
  int H, HV;
  int gb_dtype;               // dtype code of g and beta
  int h0_dtype;               // dtype code of h0
  int chunk;                  // tokens per chunk: 64 (chunked) or 1 (token-by-token recurrence)
  float scale;
};

// Token range [bos, bos + len) of sequence n.  With cu_seqlens, p.seq_len holds the packed length
// and a pair outside [0, seq_len] or decreasing is recorded as DK_ERR_DEVICE_CHECK (detail 0x500)
// and the CTA skips the sequence (every thread of the CTA takes the same branch), so a bad
// cu_seqlens never makes a kernel read or write outside the caller's buffers.
__device__ __forceinline__ bool seq_range(const Params& p, int n, int64_t& bos, int64_t& len) {
  if (p.cu_seqlens) {
    const int64_t b = p.cu_seqlens[n], e = p.cu_seqlens[n + 1];
    if (b < 0 || e < b || e > p.seq_len) {
      if (threadIdx.x == 0) report_error(DK_ERR_DEVICE_CHECK, 0x500);
      return false;
    }
    bos = b;
    len = e - b;
  } else {
    bos = static_cast<int64_t>(n) * p.seq_len;
    len = p.seq_len;
  }
  return true;
}

__device__ __forceinline__ float load_any(const void* p, int64_t i, int dtype) {
  if (dtype == DK_F32) return static_cast<const float*>(p)[i];
  if (dtype == DK_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

template <int DK, int DV>
struct Smem {
  static constexpr int kS = DK * DV;           // state
  static constexpr int kKt = DK * kPadC;       // K^T of the chunk
  static constexpr int kQt = DK * kPadC;       // Q^T of the chunk, later the o accumulators [chunk][DV]
  static constexpr int kV = kChunk * DV;       // R, then V'
  static constexpr int kA = kChunk * kChunk;   // A (strict lower)
  static constexpr int kP = kChunk * kChunk;   // scale * decay * q.k (lower incl. diagonal)
  static constexpr int kVec = 4 * kChunk;      // gamma, exp(gamma), beta, exp(gamma_last - gamma)
  static constexpr int kFloats = kS + kKt + kQt + kV + kA + kP + kVec;
  static constexpr size_t kBytes = static_cast<size_t>(kFloats) * 4;
  static_assert(kQt >= kChunk * DV, "o accumulators reuse the Q^T tile");
};

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(kThreads, 1) gdn_chunk_kernel(const Params p) {
  using SM = Smem<DK, DV>;
  extern __shared__ __align__(16) float sm[];
  float* S = sm;
  float* Kt = S + SM::kS;
  float* Qt = Kt + SM::kKt;
  float* Osm = Qt;                 // reused after Q^T is consumed
  float* Vp = Qt + SM::kQt;
  float* Am = Vp + SM::kV;
  float* Pm = Am + SM::kA;
  float* gam = Pm + SM::kP;
  float* egam = gam + kChunk;
  float* bet = egam + kChunk;
  float* wlast = bet + kChunk;

  pdl_wait();
  const int hv = blockIdx.x;
  const int n = blockIdx.y;
  const int HV = p.HV;
  const int hq = hv / (HV / p.H);
  const int tid = threadIdx.x;
  int64_t bos, len;
  if (!seq_range(p, n, bos, len)) return;
  const T* q = static_cast<const T*>(p.q);
  const T* k = static_cast<const T*>(p.k);
  const T* v = static_cast<const T*>(p.v);
  T* o = static_cast<T*>(p.o);

  // initial state
  const int64_t sbase = (static_cast<int64_t>(n) * HV + hv) * DK * DV;
  for (int e = tid; e < DK * DV; e += kThreads) S[e] = p.h0 ? load_any(p.h0, sbase + e, p.h0_dtype) : 0.0f;

  for (int64_t c0 = 0; c0 < len; c0 += p.chunk) {
    const int L = static_cast<int>((len - c0) < p.chunk ? (len - c0) : p.chunk);
    __syncthreads();  // previous chunk done with every tile
    // ---- load the chunk: K^T, Q^T (f32), V, g, beta; rows >= L are zero ----
    // Every thread issues all of its 16-byte loads before using any of them.
    {
      constexpr int KCH = kChunk * DK / 8;   // 16-byte chunks of the K (and Q) tile
      constexpr int VCH = kChunk * DV / 8;
      constexpr int KPT = (KCH + kThreads - 1) / kThreads;
      constexpr int VPT = (VCH + kThreads - 1) / kThreads;
      uint4 kr[KPT], qr[KPT], vr[VPT];
      // K/Q: token index fastest across lanes, so the transposed shared-memory stores
      // (row stride kPadC = 68 floats) fall in 32 different banks
#pragma unroll
      for (int u = 0; u < KPT; ++u) {
        const int e = tid + u * kThreads;
        const int t = e % kChunk, c = e / kChunk;
        kr[u] = qr[u] = make_uint4(0u, 0u, 0u, 0u);
        if (e < KCH && t < L) {
          const int64_t off = ((bos + c0 + t) * p.H + hq) * DK + c * 8;
          kr[u] = *reinterpret_cast<const uint4*>(k + off);
          qr[u] = *reinterpret_cast<const uint4*>(q + off);
        }
      }
#pragma unroll
      for (int u = 0; u < VPT; ++u) {
        const int e = tid + u * kThreads;
        const int t = e / (DV / 8), c = e - t * (DV / 8);
        vr[u] = make_uint4(0u, 0u, 0u, 0u);
        if (e < VCH && t < L) vr[u] = *reinterpret_cast<const uint4*>(v + ((bos + c0 + t) * HV + hv) * DV + c * 8);
      }
      // g and beta of the chunk, one token per thread of the first two warps
      float gt = 0.0f, bt = 0.0f;
      if (tid < kChunk && tid < L) {
        gt = load_any(p.g, (bos + c0 + tid) * HV + hv, p.gb_dtype);
        bt = load_any(p.beta, (bos + c0 + tid) * HV + hv, p.gb_dtype);
      }
#pragma unroll
      for (int u = 0; u < KPT; ++u) {
        const int e = tid + u * kThreads;
        if (e < KCH) {
          const int t = e % kChunk, c = e / kChunk;
          const T* kh = reinterpret_cast<const T*>(&kr[u]);
          const T* qh = reinterpret_cast<const T*>(&qr[u]);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            Kt[(c * 8 + j) * kPadC + t] = to_f32<T>(kh[j]);
            Qt[(c * 8 + j) * kPadC + t] = to_f32<T>(qh[j]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < VPT; ++u) {
        const int e = tid + u * kThreads;
        if (e < VCH) {
          const T* vh = reinterpret_cast<const T*>(&vr[u]);
#pragma unroll
          for (int j = 0; j < 8; ++j) Vp[e * 8 + j] = to_f32<T>(vh[j]);
        }
      }
      // gamma: inclusive prefix sum over the chunk in a fixed order -- a Kogge-Stone scan
      // within each 32-token half, then the first half's total added to the second half
      if (tid < kChunk) {
        const int ln = tid & 31;
        float acc = gt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float up = __shfl_up_sync(0xffffffffu, acc, o);
          if (ln >= o) acc = __fadd_rn(up, acc);
        }
        gam[tid] = acc;
        bet[tid] = bt;
      }
    }
    __syncthreads();
    if (tid >= 32 && tid < kChunk) gam[tid] = __fadd_rn(gam[31], gam[tid]);
    __syncthreads();
    if (tid < kChunk) {
      egam[tid] = expf(gam[tid]);
      wlast[tid] = (tid < L) ? expf(__fsub_rn(gam[L - 1], gam[tid])) : 0.0f;
    }
    __syncthreads();

    // ---- A and P: thread -> row t = tid / 4, columns j in [16 (tid % 4), +16) ----
    {
      const int t = tid >> 2;
      const int j0 = (tid & 3) * 16;
      float gk[16], qk[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) gk[jj] = qk[jj] = 0.0f;
      if (t < L) {
#pragma unroll 4
        for (int i = 0; i < DK; ++i) {
          const float kt = Kt[i * kPadC + t];
          const float qt = Qt[i * kPadC + t];
          const float4* kr = reinterpret_cast<const float4*>(Kt + i * kPadC + j0);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const float4 kj = kr[q4];
            gk[4 * q4 + 0] = __fmaf_rn(kt, kj.x, gk[4 * q4 + 0]);
            gk[4 * q4 + 1] = __fmaf_rn(kt, kj.y, gk[4 * q4 + 1]);
            gk[4 * q4 + 2] = __fmaf_rn(kt, kj.z, gk[4 * q4 + 2]);
            gk[4 * q4 + 3] = __fmaf_rn(kt, kj.w, gk[4 * q4 + 3]);
            qk[4 * q4 + 0] = __fmaf_rn(qt, kj.x, qk[4 * q4 + 0]);
            qk[4 * q4 + 1] = __fmaf_rn(qt, kj.y, qk[4 * q4 + 1]);
            qk[4 * q4 + 2] = __fmaf_rn(qt, kj.z, qk[4 * q4 + 2]);
            qk[4 * q4 + 3] = __fmaf_rn(qt, kj.w, qk[4 * q4 + 3]);
          }
        }
      }
      const float gt = gam[t], bt = bet[t];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = j0 + jj;
        const bool in = (t < L) && (j <= t);
        const float dec = in ? expf(__fsub_rn(gt, gam[j])) : 0.0f;
        Am[t * kChunk + j] = (in && j < t) ? __fmul_rn(__fmul_rn(bt, dec), gk[jj]) : 0.0f;
        Pm[t * kChunk + j] = in ? __fmul_rn(__fmul_rn(p.scale, dec), qk[jj]) : 0.0f;
      }
    }

    // ---- K S0 and Q S0: thread -> column c, a quarter/half of the rows ----
    {
      constexpr int kRowGroups = kThreads / DV;      // 2 (DV 128), 4 (DV 64), 8 (DV 32)
      constexpr int kRows = kChunk / kRowGroups;     // 32, 16, 8
      const int c = tid % DV;
      const int t0 = (tid / DV) * kRows;
      float ks[kRows], qs[kRows];
#pragma unroll
      for (int r = 0; r < kRows; ++r) ks[r] = qs[r] = 0.0f;
      if (t0 < L) {
#pragma unroll 2
        for (int i = 0; i < DK; ++i) {
          const float s = S[i * DV + c];
          const float4* kr = reinterpret_cast<const float4*>(Kt + i * kPadC + t0);
          const float4* qr = reinterpret_cast<const float4*>(Qt + i * kPadC + t0);
#pragma unroll
          for (int r4 = 0; r4 < kRows / 4; ++r4) {
            const float4 a = kr[r4], b = qr[r4];
            ks[4 * r4 + 0] = __fmaf_rn(a.x, s, ks[4 * r4 + 0]);
            ks[4 * r4 + 1] = __fmaf_rn(a.y, s, ks[4 * r4 + 1]);
            ks[4 * r4 + 2] = __fmaf_rn(a.z, s, ks[4 * r4 + 2]);
            ks[4 * r4 + 3] = __fmaf_rn(a.w, s, ks[4 * r4 + 3]);
            qs[4 * r4 + 0] = __fmaf_rn(b.x, s, qs[4 * r4 + 0]);
            qs[4 * r4 + 1] = __fmaf_rn(b.y, s, qs[4 * r4 + 1]);
            qs[4 * r4 + 2] = __fmaf_rn(b.z, s, qs[4 * r4 + 2]);
            qs[4 * r4 + 3] = __fmaf_rn(b.w, s, qs[4 * r4 + 3]);
          }
        }
      }
      __syncthreads();  // every thread is done reading Q^T before it becomes the o tile
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const int t = t0 + r;
        // R_t = beta_t (v_t - exp(gamma_t) (S0^T k_t)); o_t starts at scale exp(gamma_t) (S0^T q_t)
        Vp[t * DV + c] = __fmul_rn(bet[t], __fsub_rn(Vp[t * DV + c], __fmul_rn(egam[t], ks[r])));
        Osm[t * DV + c] = __fmul_rn(__fmul_rn(p.scale, egam[t]), qs[r]);
      }
    }
    __syncthreads();

    // ---- forward substitution (I + A) V' = R and the intra-chunk output, one thread per column ----
    if (tid < DV) {
      const int c = tid;
      float vp[kChunk];
#pragma unroll
      for (int t = 0; t < kChunk; ++t) {
        if (t < L) {
          float acc = Vp[t * DV + c];
          const float* arow = Am + t * kChunk;
#pragma unroll
          for (int j = 0; j < t; ++j) acc = __fmaf_rn(-arow[j], vp[j], acc);
          vp[t] = acc;
          Vp[t * DV + c] = acc;
          float ot = Osm[t * DV + c];
          const float* prow = Pm + t * kChunk;
#pragma unroll
          for (int j = 0; j <= t; ++j) ot = __fmaf_rn(prow[j], vp[j], ot);
          o[((bos + c0 + t) * HV + hv) * DV + c] = from_f32<T>(ot);
        } else {
          vp[t] = 0.0f;
        }
      }
    }
    __syncthreads();

    // ---- state: S = exp(gamma_last) S0 + sum_t exp(gamma_last - gamma_t) k_t v'_t^T ----
    {
      constexpr int kRowGroups = kThreads / DV;
      constexpr int kRows = DK / kRowGroups;
      const int c = tid % DV;
      const int i0 = (tid / DV) * kRows;
      const float el = egam[L - 1];
      float acc[kRows];
#pragma unroll
      for (int r = 0; r < kRows; ++r) acc[r] = __fmul_rn(el, S[(i0 + r) * DV + c]);
      for (int t = 0; t < L; ++t) {
        const float vw = __fmul_rn(wlast[t], Vp[t * DV + c]);
#pragma unroll
        for (int r = 0; r < kRows; ++r) acc[r] = __fmaf_rn(Kt[(i0 + r) * kPadC + t], vw, acc[r]);
      }
#pragma unroll
      for (int r = 0; r < kRows; ++r) S[(i0 + r) * DV + c] = acc[r];
    }
  }
  __syncthreads();
  if (p.ht) {
    for (int e = tid; e < DK * DV; e += kThreads) p.ht[sbase + e] = S[e];
  }
}

// ---------------------------------------------------------------------------
// Token-by-token recurrence (decode; fused_recurrent_gated_delta_rule), in the
// order of the published recurrence: S <- exp(g) S; u = S^T k; v' = beta (v - u);
// S <- S + k v'^T; o = S^T (scale q).  One CTA per (value head, sequence, block of
// 32 value columns); warp w holds rows [w DK/4, (w+1) DK/4) of those columns in
// registers (lane = column), so the state is read and written exactly once per
// call.  Sums over rows: each warp's rows in ascending order, then the four warp
// partials ((w0 + w1) + w2) + w3.
// ---------------------------------------------------------------------------
constexpr int kRecWarps = 4;

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(32 * kRecWarps) gdn_recurrent_kernel(const Params p) {
  constexpr int kRows = DK / kRecWarps;
  __shared__ float kk[DK], qq[DK];
  __shared__ float red[2][kRecWarps][32];
  __shared__ float sc[2];
  pdl_wait();
  const int hv = blockIdx.x;
  const int n = blockIdx.y;
  const int HV = p.HV;
  const int hq = hv / (HV / p.H);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.z * 32 + lane;
  const int row0 = warp * kRows;
  int64_t bos, len;
  if (!seq_range(p, n, bos, len)) return;
  const T* q = static_cast<const T*>(p.q);
  const T* k = static_cast<const T*>(p.k);
  const T* v = static_cast<const T*>(p.v);
  T* o = static_cast<T*>(p.o);
  const int64_t sbase = (static_cast<int64_t>(n) * HV + hv) * DK * DV;
  float s[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r)
    s[r] = p.h0 ? load_any(p.h0, sbase + static_cast<int64_t>(row0 + r) * DV + c, p.h0_dtype) : 0.0f;

  for (int64_t t = 0; t < len; ++t) {
    const int64_t tok = bos + t;
    __syncthreads();  // the previous token is done with kk, qq, red, sc
    for (int i = threadIdx.x; i < DK; i += 32 * kRecWarps) {
      const int64_t off = (tok * p.H + hq) * DK + i;
      kk[i] = to_f32<T>(k[off]);
      qq[i] = __fmul_rn(to_f32<T>(q[off]), p.scale);
    }
    if (threadIdx.x == 0) {
      sc[0] = expf(load_any(p.g, tok * HV + hv, p.gb_dtype));
      sc[1] = load_any(p.beta, tok * HV + hv, p.gb_dtype);
    }
    __syncthreads();
    const float e = sc[0], b = sc[1];
    float u = 0.0f;
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      s[r] = __fmul_rn(s[r], e);
      u = __fmaf_rn(s[r], kk[row0 + r], u);
    }
    red[0][warp][lane] = u;
    __syncthreads();
    const float us = __fadd_rn(__fadd_rn(__fadd_rn(red[0][0][lane], red[0][1][lane]), red[0][2][lane]), red[0][3][lane]);
    const float vp = __fmul_rn(b, __fsub_rn(to_f32<T>(v[(tok * HV + hv) * DV + c]), us));
    float ov = 0.0f;
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      s[r] = __fmaf_rn(kk[row0 + r], vp, s[r]);
      ov = __fmaf_rn(s[r], qq[row0 + r], ov);
    }
    red[1][warp][lane] = ov;
    __syncthreads();
    if (warp == 0) {
      const float os = __fadd_rn(__fadd_rn(__fadd_rn(red[1][0][lane], red[1][1][lane]), red[1][2][lane]), red[1][3][lane]);
      o[(tok * HV + hv) * DV + c] = from_f32<T>(os);
    }
  }
  if (p.ht) {
#pragma unroll
    for (int r = 0; r < kRows; ++r) p.ht[sbase + static_cast<int64_t>(row0 + r) * DV + c] = s[r];
  }
}

}  // namespace gdn
}  // namespace dk
