// Deliberately batch-VARIANT decode attention (the "before" baseline).
//
// Replaces kernels/attention.py:145-249 (_attn_split_max_kernel and
// _attn_split_sumacc_kernel) as dispatched by attention_batch_variant
// (attention.py:301-348): the KV sequence of every (batch, head) is cut into a
// fixed COUNT of chunks; pass 1 combines the chunk maxima with an atomic max,
// pass 2 adds each chunk's sum of exp(score - max) and exp-weighted V with f32
// atomics, whose order is decided by the scheduler; pass 3 divides.  CUDA
// cores only -- this path exists to demonstrate non-invariance, not speed.
#pragma once

#include "dk_common.cuh"

namespace dk {
namespace attn_var {

constexpr int kThreads = 128;

struct Params {
  const void* q;
  int64_t q_sb, q_sh;
  const void* k;
  const void* v;
  int64_t kv_sb, kv_sh, kv_ss;
  void* out;
  int64_t o_sb, o_sh;
  int B, H, S, D;
  int n_splits;
  float scale;
  float* m;    // [B*H]
  float* l;    // [B*H]
  float* acc;  // [B*H*D]
};

__device__ __forceinline__ void atomic_max_f32(float* addr, float val) {
  if (val >= 0.0f)
    atomicMax(reinterpret_cast<int*>(addr), __float_as_int(val));
  else
    atomicMin(reinterpret_cast<unsigned int*>(addr), __float_as_uint(val));
}

template <typename T>
__device__ float score_of(const Params& p, const T* q, const T* k, int s) {
  const T* kr = k + static_cast<int64_t>(s) * p.kv_ss;
  float acc = 0.0f;
  for (int d = 0; d < p.D; ++d) acc = fmaf(to_f32<T>(q[d]), to_f32<T>(kr[d]), acc);
  return acc * p.scale;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) var_max_kernel(Params p) {
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const T* q = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
  const T* k = static_cast<const T*>(p.k) + b * p.kv_sb + h * p.kv_sh;
  const int chunk = (p.S + p.n_splits - 1) / p.n_splits;
  const int lo = split * chunk, hi = min(lo + chunk, p.S);
  float mx = -INFINITY;
  for (int s = lo + threadIdx.x; s < hi; s += blockDim.x) mx = fmaxf(mx, score_of<T>(p, q, k, s));
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0 && mx > -INFINITY) atomic_max_f32(p.m + b * p.H + h, mx);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) var_sumacc_kernel(Params p) {
  extern __shared__ float sh[];  // [kThreads/32][D] partial acc, then [kThreads/32] l
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const T* q = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
  const T* k = static_cast<const T*>(p.k) + b * p.kv_sb + h * p.kv_sh;
  const T* v = static_cast<const T*>(p.v) + b * p.kv_sb + h * p.kv_sh;
  const int chunk = (p.S + p.n_splits - 1) / p.n_splits;
  const int lo = split * chunk, hi = min(lo + chunk, p.S);
  const float m = p.m[b * p.H + h];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* wacc = sh + warp * p.D;
  for (int d = lane; d < p.D; d += 32) wacc[d] = 0.0f;
  float lsum = 0.0f;
  __syncwarp();
  // each warp walks tokens lo+warp, lo+warp+4, ...; lanes split the head dimension
  for (int s = lo + warp; s < hi; s += kThreads / 32) {
    const T* kr = k + static_cast<int64_t>(s) * p.kv_ss;
    float part = 0.0f;
    for (int d = lane; d < p.D; d += 32) part = fmaf(to_f32<T>(q[d]), to_f32<T>(kr[d]), part);
    for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    const float pr = expf(part * p.scale - m);
    lsum += pr;
    const T* vr = v + static_cast<int64_t>(s) * p.kv_ss;
    for (int d = lane; d < p.D; d += 32) wacc[d] = fmaf(pr, to_f32<T>(vr[d]), wacc[d]);
  }
  __syncwarp();
  for (int d = lane; d < p.D; d += 32) atomicAdd(p.acc + (static_cast<int64_t>(b) * p.H + h) * p.D + d, wacc[d]);
  if (lane == 0) atomicAdd(p.l + b * p.H + h, lsum);
}

template <typename T>
__global__ void var_finalize_kernel(Params p) {
  const int64_t n = static_cast<int64_t>(p.B) * p.H * p.D;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t bh = i / p.D;
    const int d = static_cast<int>(i - bh * p.D);
    const int b = static_cast<int>(bh / p.H), h = static_cast<int>(bh % p.H);
    T* o = static_cast<T*>(p.out) + b * p.o_sb + h * p.o_sh + d;
    *o = from_f32<T>(p.acc[i] / p.l[bh]);
  }
}

__global__ void var_init_kernel(float* m, float* l, float* acc, int64_t bh, int64_t bhd) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < bhd;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    acc[i] = 0.0f;
    if (i < bh) {
      m[i] = -INFINITY;
      l[i] = 0.0f;
    }
  }
}

}  // namespace attn_var
}  // namespace dk
