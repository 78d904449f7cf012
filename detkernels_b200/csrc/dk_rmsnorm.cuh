// RMSNorm kernels.
//
// Invariant kernel (replaces kernels/rmsnorm.py:63-89 _single_block_kernel):
//   one CTA of 256 threads per row, always.  Thread t owns the 16-byte chunks
//   t, t+256, t+512, ... of its row and accumulates x^2 over them in ascending
//   order with fused multiply-adds; the 32 lanes of a warp are combined by an
//   xor butterfly (16, 8, 4, 2, 1) and the 8 warp sums by a second butterfly
//   (4, 2, 1).  Every step depends only on n_cols, so a row's bits never depend
//   on n_rows.  var = sum / n_cols, rstd = 1 / sqrt(var + eps) (IEEE division
//   and square root), y = (x * rstd) * w, rounded to the output dtype (RNE).
//
// Variant kernels (replace kernels/rmsnorm.py:91-138, dispatched as in
//   rmsnorm.py:200-217): for small batches each row is split into n_splits
//   chunks whose partial sums of squares are added with f32 atomics, so the
//   summation order is decided by the scheduler.
#pragma once

#include "dk_common.cuh"

namespace dk {

constexpr int kRmsThreads = DK_RMSNORM_THREADS;

template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

__device__ __forceinline__ float block_sum_256(float acc, float* red) {
  // fixed xor butterfly within the warp
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  float t = (lane < kRmsThreads / 32) ? red[lane] : 0.0f;
  if (warp == 0) {
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
    if (lane == 0) red[8] = t;
  }
  __syncthreads();
  return red[8];
}

// Vectorised path: every row pointer is 16-byte aligned and n_cols % VEC == 0.
// MAXC chunks per thread are kept in registers; longer rows are re-read for the
// normalisation pass (same arithmetic either way).
template <typename T, typename W, int MAXC>
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_inv_vec_kernel(const T* __restrict__ x, int64_t xs,
                                                                       const W* __restrict__ w,
                                                                       T* __restrict__ y, int64_t ys,
                                                                       int64_t n_cols, float eps) {
  pdl_wait();   // x may come from the previous kernel
  if (threadIdx.x == 0) pdl_launch_dependents();
  constexpr int VEC = Vec16<T>::N;
  __shared__ float red[9];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * xs;
  T* yr = y + row * ys;
  const int64_t nchunks = n_cols / VEC;

  Vec16<T> keep[MAXC];
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * kRmsThreads;
    if (c < nchunks) {
      keep[i] = *reinterpret_cast<const Vec16<T>*>(xr + c * VEC);
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = to_f32<T>(keep[i].v[j]);
        acc = __fmaf_rn(f, f, acc);
      }
    }
  }
  for (int64_t c = threadIdx.x + (int64_t)MAXC * kRmsThreads; c < nchunks; c += kRmsThreads) {
    Vec16<T> t = *reinterpret_cast<const Vec16<T>*>(xr + c * VEC);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float f = to_f32<T>(t.v[j]);
      acc = __fmaf_rn(f, f, acc);
    }
  }
  const float total = block_sum_256(acc, red);
  const float var = __fdiv_rn(total, (float)n_cols);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));

#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * kRmsThreads;
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
  for (int64_t c = threadIdx.x + (int64_t)MAXC * kRmsThreads; c < nchunks; c += kRmsThreads) {
    Vec16<T> t = *reinterpret_cast<const Vec16<T>*>(xr + c * VEC);
    Vec16<T> o;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float xn = __fmul_rn(to_f32<T>(t.v[j]), rstd);
      o.v[j] = from_f32<T>(__fmul_rn(xn, to_f32<W>(w[c * VEC + j])));
    }
    *reinterpret_cast<Vec16<T>*>(yr + c * VEC) = o;
  }
}

// Streaming form of rmsnorm_inv_vec_kernel for long row batches (rows of at most MAXC chunks
// per thread): a persistent CTA normalises rows b, b + gridDim.x, ...; every thread loads its
// chunks of the NEXT row into registers (streaming loads) before it reduces and writes the
// current one, so each SM keeps its CTAs' next rows in flight while they compute.  Thread t owns
// chunks t, t + 256, ... of every row, accumulates x^2 in the vector kernel's order and reduces
// with the same butterflies, so the bits are those of the vector kernel.  Measured on B200 at
// 65536 x 4096 f32: 6.66 TB/s at 4 CTAs per SM (a shared-memory ring of bulk copies reached 5.1).
constexpr int kRmsStreamPerSm = 4;

template <typename T, typename W, int MAXC>
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_inv_stream_kernel(const T* __restrict__ x, int64_t xs,
                                                                          const W* __restrict__ w,
                                                                          T* __restrict__ y, int64_t ys,
                                                                          int64_t n_rows, int64_t n_cols, float eps) {
  __shared__ float red[9];
  constexpr int VEC = Vec16<T>::N;
  const int64_t nchunks = n_cols / VEC;
  pdl_wait();   // x may come from the previous kernel
  if (threadIdx.x == 0) pdl_launch_dependents();
  uint4 cur[MAXC], nxt[MAXC];
  int64_t row = blockIdx.x;
  if (row < n_rows) {
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int64_t ch = threadIdx.x + (int64_t)c * kRmsThreads;
      if (ch < nchunks) cur[c] = __ldcs(reinterpret_cast<const uint4*>(x + row * xs) + ch);
    }
  }
  for (; row < n_rows; row += gridDim.x) {
    const int64_t nrow = row + gridDim.x;
    if (nrow < n_rows) {
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int64_t ch = threadIdx.x + (int64_t)c * kRmsThreads;
        if (ch < nchunks) nxt[c] = __ldcs(reinterpret_cast<const uint4*>(x + nrow * xs) + ch);
      }
    }
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int64_t ch = threadIdx.x + (int64_t)c * kRmsThreads;
      if (ch < nchunks) {
        const Vec16<T> v = *reinterpret_cast<const Vec16<T>*>(&cur[c]);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float f = to_f32<T>(v.v[j]);
          acc = __fmaf_rn(f, f, acc);
        }
      }
    }
    const float total = block_sum_256(acc, red);
    const float var = __fdiv_rn(total, (float)n_cols);
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    T* yr = y + row * ys;
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int64_t ch = threadIdx.x + (int64_t)c * kRmsThreads;
      if (ch < nchunks) {
        const Vec16<T> v = *reinterpret_cast<const Vec16<T>*>(&cur[c]);
        Vec16<T> o;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float xn = __fmul_rn(to_f32<T>(v.v[j]), rstd);
          o.v[j] = from_f32<T>(__fmul_rn(xn, to_f32<W>(w[ch * VEC + j])));
        }
        __stcs(reinterpret_cast<uint4*>(yr) + ch, *reinterpret_cast<const uint4*>(&o));
      }
    }
#pragma unroll
    for (int c = 0; c < MAXC; ++c) cur[c] = nxt[c];
  }
}

// Streaming form of rmsnorm_inv_vec_kernel for many short rows (at most 128 16-byte chunks: 1024
// 16-bit or 512 f32 elements): each half of a persistent CTA (128 threads) walks its own rows, one
// chunk per thread, with the chunks of the next two rows loaded before the current row is reduced
// (6 CTAs per SM: 1536 threads, 48 bytes each in flight).  In the
// 256-thread kernel such a row's chunks all belong to threads 0-127, so warps 4-7 contribute exact
// zeros and its cross-warp butterfly (4, 2, 1) reduces to this half's (2, 1) over the same four
// warp sums in the same order: the bits are those of the vector kernel.
constexpr int kRmsHalfPerSm = 6;

// Barrier among the 128 threads of one half of the CTA (named barriers 1 and 2).
__device__ __forceinline__ void half_sync(int half) {
  if (half == 0) {
    asm volatile("bar.sync 1, 128;" ::: "memory");
  } else {
    asm volatile("bar.sync 2, 128;" ::: "memory");
  }
}

template <typename T, typename W>
__global__ void __launch_bounds__(kRmsThreads, kRmsHalfPerSm) rmsnorm_inv_half_kernel(const T* __restrict__ x, int64_t xs,
                                                                        const W* __restrict__ w,
                                                                        T* __restrict__ y, int64_t ys,
                                                                        int64_t n_rows, int64_t n_cols, float eps) {
  __shared__ float red[2][5];
  constexpr int VEC = Vec16<T>::N;
  const int half = threadIdx.x >> 7;
  const int ht = threadIdx.x & 127;
  const int lane = threadIdx.x & 31, hw = ht >> 5;
  const int64_t nchunks = n_cols / VEC;
  const bool mine = ht < nchunks;
  pdl_wait();   // x may come from the previous kernel
  if (threadIdx.x == 0) pdl_launch_dependents();
  const int64_t stride = 2 * static_cast<int64_t>(gridDim.x);
  int64_t row = 2 * static_cast<int64_t>(blockIdx.x) + half;
  uint4 cur = make_uint4(0u, 0u, 0u, 0u), nxt = cur, nxt2 = cur;
  if (row < n_rows && mine) cur = __ldcs(reinterpret_cast<const uint4*>(x + row * xs) + ht);
  if (row + stride < n_rows && mine) nxt = __ldcs(reinterpret_cast<const uint4*>(x + (row + stride) * xs) + ht);
  for (; row < n_rows; row += stride) {
    const int64_t nrow = row + 2 * stride;
    if (nrow < n_rows && mine) nxt2 = __ldcs(reinterpret_cast<const uint4*>(x + nrow * xs) + ht);
    float acc = 0.0f;
    const Vec16<T> v = *reinterpret_cast<const Vec16<T>*>(&cur);
    if (mine) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = to_f32<T>(v.v[j]);
        acc = __fmaf_rn(f, f, acc);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) red[half][hw] = acc;
    half_sync(half);
    if (hw == 0) {
      float t = (lane < 4) ? red[half][lane] : 0.0f;
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      if (lane == 0) red[half][4] = t;
    }
    half_sync(half);
    const float total = red[half][4];
    const float var = __fdiv_rn(total, (float)n_cols);
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    if (mine) {
      Vec16<T> o;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float xn = __fmul_rn(to_f32<T>(v.v[j]), rstd);
        o.v[j] = from_f32<T>(__fmul_rn(xn, to_f32<W>(w[ht * VEC + j])));
      }
      __stcs(reinterpret_cast<uint4*>(y + row * ys) + ht, *reinterpret_cast<const uint4*>(&o));
    }
    cur = nxt;
    nxt = nxt2;
  }
}

// Embedding lookup fused into the invariant RMSNorm: row r reads table row idx[r], copies it
// to x_out (the residual stream) and normalises it with exactly rmsnorm_inv_vec_kernel's
// arithmetic.  An index outside [0, table_rows) records DK_ERR_DEVICE_CHECK and leaves the
// row untouched.  Vector path only: 16-byte aligned rows, n_cols <= MAXC * 256 * VEC.
template <typename T, typename W, int MAXC>
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_gather_vec_kernel(const T* __restrict__ table, int64_t ts,
                                                                          int64_t table_rows,
                                                                          const int64_t* __restrict__ idx,
                                                                          const W* __restrict__ w, T* __restrict__ x,
                                                                          int64_t xs, T* __restrict__ y, int64_t ys,
                                                                          int64_t n_cols, float eps) {
  pdl_wait();   // the indices may come from the previous kernel
  if (threadIdx.x == 0) pdl_launch_dependents();
  constexpr int VEC = Vec16<T>::N;
  __shared__ float red[9];
  const int64_t row = blockIdx.x;
  const int64_t src = idx[row];
  if (src < 0 || src >= table_rows) {
    if (threadIdx.x == 0) report_error(DK_ERR_DEVICE_CHECK, 0x300);
    return;
  }
  const T* tr = table + src * ts;
  T* xr = x + row * xs;
  T* yr = y + row * ys;
  const int64_t nchunks = n_cols / VEC;
  Vec16<T> keep[MAXC];
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * kRmsThreads;
    if (c < nchunks) {
      keep[i] = *reinterpret_cast<const Vec16<T>*>(tr + c * VEC);
      *reinterpret_cast<Vec16<T>*>(xr + c * VEC) = keep[i];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = to_f32<T>(keep[i].v[j]);
        acc = __fmaf_rn(f, f, acc);
      }
    }
  }
  const float total = block_sum_256(acc, red);
  const float var = __fdiv_rn(total, (float)n_cols);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int64_t c = threadIdx.x + (int64_t)i * kRmsThreads;
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

// Scalar path for unaligned rows or n_cols not a multiple of the vector width.
// It walks the same 16-byte chunks in the same per-thread order as the vector
// path (the last chunk may be short), so a row's bits do not depend on which
// path its pointer alignment selected.
template <typename T, typename W>
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_inv_scalar_kernel(const T* __restrict__ x, int64_t xs,
                                                                          const W* __restrict__ w,
                                                                          T* __restrict__ y, int64_t ys,
                                                                          int64_t n_cols, float eps) {
  pdl_wait();   // x may come from the previous kernel
  if (threadIdx.x == 0) pdl_launch_dependents();
  constexpr int VEC = Vec16<T>::N;
  __shared__ float red[9];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * xs;
  T* yr = y + row * ys;
  const int64_t nchunks = (n_cols + VEC - 1) / VEC;
  float acc = 0.0f;
  for (int64_t c = threadIdx.x; c < nchunks; c += kRmsThreads) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const int64_t e = c * VEC + j;
      if (e < n_cols) {
        const float f = to_f32<T>(xr[e]);
        acc = __fmaf_rn(f, f, acc);
      }
    }
  }
  const float total = block_sum_256(acc, red);
  const float var = __fdiv_rn(total, (float)n_cols);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (int64_t e = threadIdx.x; e < n_cols; e += kRmsThreads) {
    const float xn = __fmul_rn(to_f32<T>(xr[e]), rstd);
    yr[e] = from_f32<T>(__fmul_rn(xn, to_f32<W>(w[e])));
  }
}

// Embedding lookup + invariant RMSNorm for rows the vector gather cannot take (unaligned
// table or output rows, n_cols not a multiple of the vector width, or longer than the
// vector kernel keeps in registers): the chunk walk of rmsnorm_inv_scalar_kernel, reading
// table row idx[r] and copying it to x_out, so the bits equal the lookup followed by the
// invariant RMSNorm on either path.
template <typename T, typename W>
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_gather_scalar_kernel(const T* __restrict__ table, int64_t ts,
                                                                             int64_t table_rows,
                                                                             const int64_t* __restrict__ idx,
                                                                             const W* __restrict__ w,
                                                                             T* __restrict__ x, int64_t xs,
                                                                             T* __restrict__ y, int64_t ys,
                                                                             int64_t n_cols, float eps) {
  pdl_wait();   // the indices may come from the previous kernel
  if (threadIdx.x == 0) pdl_launch_dependents();
  constexpr int VEC = Vec16<T>::N;
  __shared__ float red[9];
  const int64_t row = blockIdx.x;
  const int64_t src = idx[row];
  if (src < 0 || src >= table_rows) {
    if (threadIdx.x == 0) report_error(DK_ERR_DEVICE_CHECK, 0x301);
    return;
  }
  const T* tr = table + src * ts;
  T* xr = x + row * xs;
  T* yr = y + row * ys;
  const int64_t nchunks = (n_cols + VEC - 1) / VEC;
  float acc = 0.0f;
  for (int64_t c = threadIdx.x; c < nchunks; c += kRmsThreads) {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const int64_t e = c * VEC + j;
      if (e < n_cols) {
        const T v = tr[e];
        xr[e] = v;
        const float f = to_f32<T>(v);
        acc = __fmaf_rn(f, f, acc);
      }
    }
  }
  const float total = block_sum_256(acc, red);
  const float var = __fdiv_rn(total, (float)n_cols);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (int64_t e = threadIdx.x; e < n_cols; e += kRmsThreads) {
    const float xn = __fmul_rn(to_f32<T>(tr[e]), rstd);
    yr[e] = from_f32<T>(__fmul_rn(xn, to_f32<W>(w[e])));
  }
}

// ---- batch-variant twin: split partial sums combined with atomics ----
template <typename T>
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_var_partial_kernel(const T* __restrict__ x, int64_t xs,
                                                                           float* __restrict__ partial,
                                                                           int64_t n_cols, int n_splits) {
  __shared__ float red[9];
  const int64_t row = blockIdx.x;
  const int split = blockIdx.y;
  const int64_t chunk = (n_cols + n_splits - 1) / n_splits;
  const int64_t lo = split * chunk;
  const int64_t hi = (lo + chunk < n_cols) ? lo + chunk : n_cols;
  const T* xr = x + row * xs;
  float acc = 0.0f;
  for (int64_t e = lo + threadIdx.x; e < hi; e += kRmsThreads) {
    const float f = to_f32<T>(xr[e]);
    acc = __fmaf_rn(f, f, acc);
  }
  const float total = block_sum_256(acc, red);
  if (threadIdx.x == 0) atomicAdd(partial + row, total);
}

template <typename T, typename W>
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_var_finalize_kernel(const T* __restrict__ x, int64_t xs,
                                                                            const W* __restrict__ w,
                                                                            const float* __restrict__ partial,
                                                                            T* __restrict__ y, int64_t ys,
                                                                            int64_t n_cols, float eps) {
  const int64_t row = blockIdx.x;
  const T* xr = x + row * xs;
  T* yr = y + row * ys;
  const float var = __fdiv_rn(partial[row], (float)n_cols);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (int64_t e = threadIdx.x; e < n_cols; e += kRmsThreads) {
    const float xn = __fmul_rn(to_f32<T>(xr[e]), rstd);
    yr[e] = from_f32<T>(__fmul_rn(xn, to_f32<W>(w[e])));
  }
}

}  // namespace dk
