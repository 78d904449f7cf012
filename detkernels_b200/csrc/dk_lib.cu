// detkernels_b200 C ABI (see include/detkernels_b200.h).
//
// One translation unit: the kernels live in the dk_*.cuh headers; this file
// holds argument validation, TMA tensor-map encoding, schedule selection and
// the extern "C" entry points.  Nothing here allocates device memory: scratch
// space comes from the caller's workspace.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <utility>

#include "dk_common.cuh"
#include "dk_rmsnorm.cuh"
#include "dk_gemm.cuh"
#include "dk_gemm2.cuh"
#include "dk_gemm_wide.cuh"
#include "dk_attention.cuh"
#include "dk_attention_variant.cuh"
#include "dk_gdn.cuh"
#include "dk_gdn_tc.cuh"
#include "dk_gdn_umma.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return DK_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch with programmatic stream serialization: the kernel may begin (and run
// its preamble) while the previous kernel on the stream finishes; every kernel
// of this library waits for its predecessor (griddepcontrol.wait) before it
// touches global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

constexpr int kMaxDevices = 64;

// Every workspace starts with a fixed area of arrival counters shared by all
// ops.  It must be zero when the workspace is first used; every call leaves it
// zero again.  Non-counter scratch always lives after it, so calls with
// different shapes never see each other's data in a counter.
constexpr size_t kCounterBytes = DK_WORKSPACE_COUNTER_BYTES;
constexpr int64_t kMaxCounters = static_cast<int64_t>(kCounterBytes / sizeof(int32_t));
inline uint8_t* ws_data(void* ws) { return static_cast<uint8_t*>(ws) + kCounterBytes; }

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int sm_count(int device) {
  static int cache[kMaxDevices] = {0};
  if (device < 0 || device >= kMaxDevices) return 148;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cache[device] = n;
  }
  return cache[device];
}

// Raise the dynamic shared-memory limit of `fn` once per device.
template <typename F>
int ensure_smem(F fn, int bytes, bool (&done)[kMaxDevices]) {
  const int dev = current_device();
  if (dev >= 0 && dev < kMaxDevices && done[dev]) return DK_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  if (dev >= 0 && dev < kMaxDevices) done[dev] = true;
  return DK_OK;
}

// ---- TMA tensor maps through the driver entry point (no link-time libcuda dependency) ----
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

int encode_map(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz, const char* what) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DK_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", what);
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) gs[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dt, rank, const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DK_ERR_INVALID_ARGUMENT, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return DK_OK;
}

bool valid_dtype(int d) { return d == DK_F32 || d == DK_F16 || d == DK_BF16; }

// ============================ RMSNorm ============================
// Streaming vector RMSNorm over `rows` rows of at most MAXC * 256 chunks (<= 16 KB): a persistent
// grid of kRmsStreamPerSm CTAs per SM (never more than rows), each walking rows b, b + grid, ...
// with the next row's chunks in flight in registers.
template <typename T, typename W, int MAXC>
cudaError_t rmsnorm_stream(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int64_t cols,
                           float eps, cudaStream_t st) {
  const int64_t cap = static_cast<int64_t>(dk::kRmsStreamPerSm) * sm_count(current_device());
  const unsigned grid = static_cast<unsigned>(rows < cap ? rows : cap);
  return launch_pdl(dk::rmsnorm_inv_stream_kernel<T, W, MAXC>, dim3(grid), dim3(dk::kRmsThreads), 0, st,
                    static_cast<const T*>(x), xs, static_cast<const W*>(w), static_cast<T*>(y), ys, rows, cols, eps);
}

template <typename T, typename W>
int rmsnorm_inv_launch(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int64_t cols,
                       float eps, cudaStream_t st) {
  constexpr int VEC = dk::Vec16<T>::N;
  const bool vec = (cols % VEC == 0) && (xs % VEC == 0) && (ys % VEC == 0) && aligned16(x) && aligned16(y);
  const dim3 grid(static_cast<unsigned>(rows));
  const int64_t per_thread = (cols / VEC + dk::kRmsThreads - 1) / dk::kRmsThreads;   // chunks per thread
  cudaError_t e;
  if (vec && rows > 1 && per_thread >= 3 && per_thread <= 4) {
    // rows of 3-4 chunks per thread (12-16 KB: 4096 f32, 8192 16-bit elements): streamed by
    // persistent CTAs that hold the next row in registers.  Shorter rows keep one CTA per row.
    e = rmsnorm_stream<T, W, 4>(x, xs, w, y, ys, rows, cols, eps, st);
  } else if (vec && cols / VEC <= 128 && rows >= 2LL * dk::kRmsHalfPerSm * sm_count(current_device())) {
    // many short rows (at most 128 chunks): persistent CTAs, a row per 128-thread half
    const int64_t cap = static_cast<int64_t>(dk::kRmsHalfPerSm) * sm_count(current_device());
    const int64_t want = (rows + 1) / 2;
    e = launch_pdl(dk::rmsnorm_inv_half_kernel<T, W>, dim3(static_cast<unsigned>(want < cap ? want : cap)),
                   dim3(dk::kRmsThreads), 0, st, static_cast<const T*>(x), xs, static_cast<const W*>(w),
                   static_cast<T*>(y), ys, rows, cols, eps);
  } else if (vec) {
    constexpr int MAXC = (sizeof(T) == 4) ? 8 : 4;
    e = launch_pdl(dk::rmsnorm_inv_vec_kernel<T, W, MAXC>, grid, dim3(dk::kRmsThreads), 0, st,
                   static_cast<const T*>(x), xs, static_cast<const W*>(w), static_cast<T*>(y), ys, cols, eps);
  } else {
    e = launch_pdl(dk::rmsnorm_inv_scalar_kernel<T, W>, grid, dim3(dk::kRmsThreads), 0, st,
                   static_cast<const T*>(x), xs, static_cast<const W*>(w), static_cast<T*>(y), ys, cols, eps);
  }
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "rmsnorm_batch_invariant: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

template <typename T, typename W>
int rmsnorm_gather_launch(const void* table, int64_t ts, int64_t table_rows, const int64_t* idx, const void* w,
                          void* x, int64_t xs, void* y, int64_t ys, int64_t rows, int64_t cols, float eps,
                          cudaStream_t st) {
  constexpr int VEC = dk::Vec16<T>::N;
  constexpr int MAXC = (sizeof(T) == 4) ? 8 : 4;
  const bool vec = (cols % VEC == 0) && (ts % VEC == 0) && (xs % VEC == 0) && (ys % VEC == 0) && aligned16(table) &&
                   aligned16(x) && aligned16(y) && cols <= static_cast<int64_t>(MAXC) * dk::kRmsThreads * VEC;
  cudaError_t e;
  if (vec)
    e = launch_pdl(dk::rmsnorm_gather_vec_kernel<T, W, MAXC>, dim3(static_cast<unsigned>(rows)),
                   dim3(dk::kRmsThreads), 0, st, static_cast<const T*>(table), ts, table_rows, idx,
                   static_cast<const W*>(w), static_cast<T*>(x), xs, static_cast<T*>(y), ys, cols, eps);
  else
    e = launch_pdl(dk::rmsnorm_gather_scalar_kernel<T, W>, dim3(static_cast<unsigned>(rows)),
                   dim3(dk::kRmsThreads), 0, st, static_cast<const T*>(table), ts, table_rows, idx,
                   static_cast<const W*>(w), static_cast<T*>(x), xs, static_cast<T*>(y), ys, cols, eps);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "rmsnorm_gather: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

template <typename T, typename W>
int rmsnorm_var_launch(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int64_t cols,
                       float eps, int n_splits, float* partial, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(partial, 0, sizeof(float) * rows, st);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "rmsnorm_batch_variant: memset: %s", cudaGetErrorString(e));
  dk::rmsnorm_var_partial_kernel<T><<<dim3(static_cast<unsigned>(rows), n_splits), dk::kRmsThreads, 0, st>>>(
      static_cast<const T*>(x), xs, partial, cols, n_splits);
  dk::rmsnorm_var_finalize_kernel<T, W><<<dim3(static_cast<unsigned>(rows)), dk::kRmsThreads, 0, st>>>(
      static_cast<const T*>(x), xs, static_cast<const W*>(w), partial, static_cast<T*>(y), ys, cols, eps);
  return check_launch("rmsnorm_batch_variant");
}

int rms_validate(const void* x, const void* w, const void* y, int64_t xs, int64_t ys, int64_t rows, int64_t cols,
                 int dtype, int wdtype, const char* what) {
  if (!valid_dtype(dtype) || !valid_dtype(wdtype)) return fail(DK_ERR_UNSUPPORTED, "%s: bad dtype", what);
  if (rows < 0 || cols <= 0) return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad shape [%lld, %lld]", what, (long long)rows,
                                         (long long)cols);
  if (rows > 0x7fffffffLL) return fail(DK_ERR_INVALID_ARGUMENT, "%s: too many rows", what);
  if (rows > 0 && (!x || !w || !y)) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  if (rows > 1 && (xs < cols || ys < cols)) return fail(DK_ERR_INVALID_ARGUMENT, "%s: row stride < n_cols", what);
  return DK_OK;
}

#define DK_DISPATCH_RMS(FN, ...)                                                                          \
  do {                                                                                                    \
    if (dtype == DK_F32) {                                                                                \
      if (wdtype == DK_F32) return FN<float, float>(__VA_ARGS__);                                         \
      if (wdtype == DK_F16) return FN<float, __half>(__VA_ARGS__);                                        \
      return FN<float, __nv_bfloat16>(__VA_ARGS__);                                                       \
    } else if (dtype == DK_F16) {                                                                         \
      if (wdtype == DK_F32) return FN<__half, float>(__VA_ARGS__);                                        \
      if (wdtype == DK_F16) return FN<__half, __half>(__VA_ARGS__);                                       \
      return FN<__half, __nv_bfloat16>(__VA_ARGS__);                                                      \
    } else {                                                                                              \
      if (wdtype == DK_F32) return FN<__nv_bfloat16, float>(__VA_ARGS__);                                 \
      if (wdtype == DK_F16) return FN<__nv_bfloat16, __half>(__VA_ARGS__);                                \
      return FN<__nv_bfloat16, __nv_bfloat16>(__VA_ARGS__);                                               \
    }                                                                                                     \
  } while (0)

// ============================ GEMM ============================
int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

int slice_len_for(int64_t K, int n_slices) {
  int64_t l = ceil_div(K, n_slices);
  l = ceil_div(l, dk::gemm::kUK) * dk::gemm::kUK;
  if (l < dk::gemm::kUK) l = dk::gemm::kUK;
  return static_cast<int>(l);
}

struct GemmPlan {
  int mode;
  int group;
  int kernel;          // 0 one-CTA, 1 CTA pair (256-column tiles), 2 wide CTA pair (256 x 256 tiles)
  int n_tiles, m_tiles;
  size_t ws_bytes;     // workspace bytes this plan needs
  size_t counters_off; // byte offset of the counters region
  size_t partials_off; // byte offset of the partials region
  bool stash;          // the wide kernel with 8-slice units parks the tree's left half in the workspace
  size_t stash_off;    // byte offset of that stash
};

// Schedule choice (never changes the arithmetic): slices per work unit.  A
// small cost model -- per-SM streaming of the unit's operand tiles in waves,
// plus the L2 round trip of the f32 slice partials when slices are spread
// over CTAs -- picks the cheapest of 8 (FOLD), 4, 2, 1 (SPLIT).
// Slices per work unit forced by the test hook dk_matmul_pair_schedule_for_test (0: the cost model).
int g_group_override = 0;

int pick_group(int64_t M, int64_t N, int64_t K, int64_t tiles, int sms, int kernel) {
  if (g_group_override) return g_group_override;
  const int a_rows = (M <= dk::gemm::kTileM) ? static_cast<int>(ceil_div(M, 8) * 8) : dk::gemm::kTileM;
  const int stage_bytes = (kernel == 2) ? dk::gemm::kWideStageBytes
                          : (kernel == 1) ? dk::gemm::kPairStageBytes
                                          : dk::gemm::stage_bytes_for(a_rows);
  const double kSmBytesPerUs = 100e3;   // sustained TMA bytes per SM per microsecond
  const double kL2BytesPerUs = 10e6;    // L2 bytes per microsecond for the partial round trip
  const int64_t kb_per_slice = ceil_div(slice_len_for(K, dk::gemm::kSlices), kernel == 2   ? dk::gemm::kWideBK
                                                                      : kernel == 1 ? dk::gemm::kBK
                                                                                    : dk::gemm::kStageK);
  double best = 1e30;
  int best_g = dk::gemm::kSlices;
  for (int g = dk::gemm::kSlices; g >= 1; g /= 2) {
    const int64_t units = tiles * (dk::gemm::kSlices / g);
    const int64_t waves = ceil_div(units, sms);
    const double load = static_cast<double>(waves) * g * kb_per_slice * stage_bytes / kSmBytesPerUs;
    // each unit writes one subtree sum; the last arriver reads them back
    const double part = (g < dk::gemm::kSlices) ? 2.0 * (dk::gemm::kSlices / g) * M * N * 4 / kL2BytesPerUs : 0.0;
    const double t = load + part;
    if (t < best * 0.97) {
      best = t;
      best_g = g;
    }
  }
  return best_g;
}

// Which GEMM kernel runs an invariant call (never changes the arithmetic): 0 = the planner's
// choice, 1 = always the one-CTA kernel, 2 = always the CTA-pair kernel, 3 = always the wide
// CTA-pair kernel.  Only the test hook dk_matmul_pair_schedule_for_test sets it.
int g_pair_override = 0;

// The CTA-pair kernel with 256 x 128 tiles moves 24 KB per SM per 128 x 128 x 64 of work instead
// of 32 KB, but measured on B200 it is not faster than the one-CTA kernel (M = 2048, N = 4096:
// 147 vs 129 us); it runs only when forced.  The wide kernel (256 x 256 tiles, 16 KB per SM per
// 128 x 128 x 64) runs when the token count fills its 256-token tiles.
int pick_kernel(int64_t M, int64_t N, int64_t K, int sms) {
  if (g_pair_override == 1) return 0;
  if (g_pair_override == 2) return 1;
  if (g_pair_override == 3) return 2;
  // Measured on B200 (CUDA graph, weights beyond L2): above 256 tokens the wide kernel wins; at
  // 129-256 tokens only when there are a wave of 256-column tiles for its 8-slice units (the LM
  // head, N = 32000: 47 vs 61 us); with fewer tiles it needs split-K partials, whose row-wise
  // stores make it slower than the one-CTA kernel (N = 11008, K = 4096: 64 vs 50 us).
  (void)K;
  if (M > 2 * dk::gemm::kTileM) return 2;
  if (M > dk::gemm::kTileM && ceil_div(N, dk::gemm::kWideTileN) >= sms / 2) return 2;
  return 0;
}

GemmPlan plan_invariant(int64_t M, int64_t N, int64_t K, int sms) {
  GemmPlan pl{};
  pl.kernel = pick_kernel(M, N, K, sms);
  const int tile_n = pl.kernel ? dk::gemm::kPairTileN : dk::gemm::kTileN;
  const int tile_m = (pl.kernel == 2) ? dk::gemm::kWideTileM : dk::gemm::kTileM;
  pl.n_tiles = static_cast<int>(ceil_div(N, tile_n));
  pl.m_tiles = static_cast<int>(ceil_div(M, tile_m));
  const int64_t tiles = static_cast<int64_t>(pl.n_tiles) * pl.m_tiles * (pl.kernel ? 2 : 1);   // in CTAs
  const int group = pick_group(M, N, K, tiles, sms, pl.kernel);
  pl.group = group;
  pl.mode = (group == dk::gemm::kSlices) ? dk::gemm::FOLD : dk::gemm::SPLIT;
  size_t end = 0;
  if (pl.mode == dk::gemm::SPLIT) {
    pl.counters_off = 0;
    pl.partials_off = kCounterBytes;
    end = pl.partials_off + sizeof(float) * static_cast<size_t>(dk::gemm::kSlices / group) * M * N;
  }
  if (pl.kernel == 2 && group == dk::gemm::kSlices) {
    // one stash per CTA the launch can hold resident (at most one CTA per SM), after the
    // workspace's arrival counters, which must stay zero for the other entry points
    pl.stash = true;
    pl.stash_off = ((end > kCounterBytes ? end : kCounterBytes) + 255) / 256 * 256;
    end = pl.stash_off + sizeof(float) * static_cast<size_t>(dk::gemm::kWideStashFloats) * sms;
  }
  pl.ws_bytes = end;
  return pl;
}

int gemm_validate(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N, int64_t K, int dtype,
                  const char* what) {
  if (dtype != DK_BF16 && dtype != DK_F16)
    return fail(DK_ERR_UNSUPPORTED, "%s: dtype must be bf16 or f16", what);
  if (M < 0 || N < 0 || K < 0 || M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad shape", what);
  if (M == 0 || N == 0 || K == 0) return DK_OK;
  if (!a || !b) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  if (!aligned16(a) || !aligned16(b)) return fail(DK_ERR_INVALID_ARGUMENT, "%s: A and B must be 16-byte aligned", what);
  if (lda % 8 != 0 || ldb % 8 != 0)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: lda and ldb must be multiples of 8 elements", what);
  if (lda < K || ldb < N) return fail(DK_ERR_INVALID_ARGUMENT, "%s: leading dimension too small", what);
  return DK_OK;
}

template <typename T>
int launch_fold(const float* partials, int n_parts, const dk::gemm::Params& p, cudaStream_t st) {
  const int64_t total = static_cast<int64_t>(p.M) * ceil_div(p.N, 4);
  const int64_t want = ceil_div(total, 256);
  // one resident wave (4 blocks per SM), so every block has issued the early
  // dependent-launch trigger soon after the GEMM completes
  const int64_t cap = 4 * static_cast<int64_t>(sm_count(current_device()));
  const int blocks = static_cast<int>(want < cap ? want : cap);
  cudaError_t e = launch_pdl(dk::gemm::fold_groups_kernel<T>, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, st,
                             partials, n_parts, p);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "matmul fold: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

// The RMSNorm half of DK_EPI_RESIDUAL_RMSNORM (the GEMM itself runs DK_EPI_RESIDUAL).
struct NormSpec {
  const void* w;
  int w_dtype;
  void* out;
  int64_t ld;
  float eps;
};

template <typename T, typename W>
int launch_fold_rmsnorm_t(const float* partials, int n_parts, const dk::gemm::Params& p, const NormSpec& nm,
                          cudaStream_t st) {
  cudaError_t e = launch_pdl(dk::gemm::fold_residual_rmsnorm_kernel<T, W, 4>, dim3(static_cast<unsigned>(p.M)),
                             dim3(dk::kRmsThreads), 0, st, partials, n_parts, p, static_cast<const W*>(nm.w),
                             static_cast<T*>(nm.out), nm.ld, nm.eps);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "matmul fold+rmsnorm: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

// Upper tree levels + residual + RMSNorm in one kernel when a CTA can hold a row in
// 16-byte chunks; otherwise the fold kernel followed by the RMSNorm kernel (same bits).
int launch_fold_norm(int dtype, const float* partials, int n_parts, const dk::gemm::Params& p, const NormSpec& nm,
                     cudaStream_t st) {
  constexpr int kVec = 8;   // 16-bit elements per 16-byte chunk
  const bool fused = (p.N % kVec == 0) && (p.N <= 4 * dk::kRmsThreads * kVec) && (p.ldc % kVec == 0) &&
                     (nm.ld % kVec == 0) && aligned16(p.c) && aligned16(nm.out) &&
                     (nm.w_dtype == dtype || nm.w_dtype == DK_F32);
  if (fused) {
    if (dtype == DK_BF16) {
      if (nm.w_dtype == DK_F32) return launch_fold_rmsnorm_t<__nv_bfloat16, float>(partials, n_parts, p, nm, st);
      return launch_fold_rmsnorm_t<__nv_bfloat16, __nv_bfloat16>(partials, n_parts, p, nm, st);
    }
    if (nm.w_dtype == DK_F32) return launch_fold_rmsnorm_t<__half, float>(partials, n_parts, p, nm, st);
    return launch_fold_rmsnorm_t<__half, __half>(partials, n_parts, p, nm, st);
  }
  int rc = (dtype == DK_BF16) ? launch_fold<__nv_bfloat16>(partials, n_parts, p, st)
                              : launch_fold<__half>(partials, n_parts, p, st);
  if (rc) return rc;
  return dk_rmsnorm_batch_invariant(p.c, p.ldc, nm.w, nm.out, nm.ld, p.M, p.N, dtype, nm.w_dtype, nm.eps, st);
}

// The CTA-pair kernel's launch: clusters of 2, as many pairs as can be resident at once.
template <typename T, int FMT, bool FOLDK>
cudaError_t launch_pair(const CUtensorMap& tmB, const CUtensorMap& tmA, const dk::gemm::Params& p, int64_t units,
                        cudaStream_t st, int* rc) {
  auto fn = dk::gemm::gemm_pair_kernel<T, FMT, FOLDK>;
  static bool done[kMaxDevices] = {};
  static int max_pairs[kMaxDevices] = {};
  *rc = ensure_smem(fn, dk::gemm::kSmemBytes, done);
  if (*rc) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(dk::gemm::kThreads);
  cfg.dynamicSmemBytes = dk::gemm::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const int dev = current_device();
  int pairs = (dev >= 0 && dev < kMaxDevices) ? max_pairs[dev] : 0;
  if (pairs <= 0) {
    cfg.gridDim = dim3(2 * 64);
    if (cudaOccupancyMaxActiveClusters(&pairs, fn, &cfg) != cudaSuccess || pairs <= 0) pairs = sm_count(dev) / 2;
    if (dev >= 0 && dev < kMaxDevices) max_pairs[dev] = pairs;
  }
  const int64_t n = units < pairs ? units : pairs;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * n));
  return cudaLaunchKernelEx(&cfg, fn, tmB, tmA, p);
}

// The wide kernel's launch: clusters of 2, as many pairs as can be resident at once (at most
// one CTA per SM, which the stash is sized for).  Its register split (setmaxnreg) is exact only
// for kWideLaunchRegs registers per thread, so a build with another count is refused.
template <typename T, int FMT, bool FOLDK>
cudaError_t launch_wide(const CUtensorMap& tmB, const CUtensorMap& tmA, const dk::gemm::Params& p, int64_t units,
                        cudaStream_t st, int* rc) {
  auto fn = dk::gemm::gemm_wide_kernel<T, FMT, FOLDK>;
  static bool done[kMaxDevices] = {};
  static int max_pairs[kMaxDevices] = {};
  *rc = ensure_smem(fn, dk::gemm::kSmemBytes, done);
  if (*rc) return cudaSuccess;
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, fn) != cudaSuccess || fa.numRegs != dk::gemm::kWideLaunchRegs) {
    *rc = fail(DK_ERR_UNSUPPORTED, "wide GEMM built with %d registers per thread, %d expected", fa.numRegs,
               dk::gemm::kWideLaunchRegs);
    return cudaSuccess;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(dk::gemm::kWideThreads);
  cfg.dynamicSmemBytes = dk::gemm::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const int dev = current_device();
  int pairs = (dev >= 0 && dev < kMaxDevices) ? max_pairs[dev] : 0;
  if (pairs <= 0) {
    cfg.gridDim = dim3(2 * 64);
    if (cudaOccupancyMaxActiveClusters(&pairs, fn, &cfg) != cudaSuccess || pairs <= 0) pairs = sm_count(dev) / 2;
    if (pairs > sm_count(dev) / 2) pairs = sm_count(dev) / 2;
    if (dev >= 0 && dev < kMaxDevices) max_pairs[dev] = pairs;
  }
  const int64_t n = units < pairs ? units : pairs;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * n));
  return cudaLaunchKernelEx(&cfg, fn, tmB, tmA, p);
}

int gemm_launch(int dtype, const void* a, int64_t lda, const void* b, int64_t ldb, dk::gemm::Params p,
                cudaStream_t st, const char* what, const NormSpec* norm = nullptr) {
  p.a_rows = (p.pair == 2) ? dk::gemm::kWideRows
             : p.pair      ? dk::gemm::kPairRows
                           : ((p.m_tiles == 1) ? static_cast<int>(ceil_div(p.M, 8) * 8) : dk::gemm::kTileM);
  const int64_t k_mem = p.k_extent > 0 ? p.k_extent : p.K;
  CUtensorMap tmB, tmA;
  const uint64_t dimsB[2] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(k_mem)};
  const uint64_t strB[1] = {static_cast<uint64_t>(ldb) * 2};
  const uint32_t boxB[2] = {64, static_cast<uint32_t>(dk::gemm::kBK)};
  const uint64_t dimsA[2] = {static_cast<uint64_t>(k_mem), static_cast<uint64_t>(p.M)};
  const uint64_t strA[1] = {static_cast<uint64_t>(lda) * 2};
  const uint32_t boxA[2] = {static_cast<uint32_t>(dk::gemm::kBK), static_cast<uint32_t>(p.a_rows)};
  const CUtensorMapDataType dt = (dtype == DK_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc = encode_map(&tmB, dt, 2, b, dimsB, strB, boxB, CU_TENSOR_MAP_SWIZZLE_128B, what);
  if (rc) return rc;
  rc = encode_map(&tmA, dt, 2, a, dimsA, strA, boxA, CU_TENSOR_MAP_SWIZZLE_128B, what);
  if (rc) return rc;

  const int n_groups = (p.slice_end - p.slice_begin) / p.group;
  const int64_t units = static_cast<int64_t>(p.n_tiles) * p.m_tiles * n_groups;
  const int sms = sm_count(current_device());
  const int grid = static_cast<int>(units < sms ? units : sms);
  if (grid <= 0) return DK_OK;
  cudaError_t e;
  const bool fold = (p.mode == dk::gemm::FOLD);
  if (p.pair == 2) {
    int lrc = DK_OK;
    if (dtype == DK_BF16)
      e = fold ? launch_wide<__nv_bfloat16, 1, true>(tmB, tmA, p, units, st, &lrc)
               : launch_wide<__nv_bfloat16, 1, false>(tmB, tmA, p, units, st, &lrc);
    else
      e = fold ? launch_wide<__half, 0, true>(tmB, tmA, p, units, st, &lrc)
               : launch_wide<__half, 0, false>(tmB, tmA, p, units, st, &lrc);
    if (lrc) return lrc;
  } else if (p.pair) {
    int lrc = DK_OK;
    if (dtype == DK_BF16)
      e = fold ? launch_pair<__nv_bfloat16, 1, true>(tmB, tmA, p, units, st, &lrc)
               : launch_pair<__nv_bfloat16, 1, false>(tmB, tmA, p, units, st, &lrc);
    else
      e = fold ? launch_pair<__half, 0, true>(tmB, tmA, p, units, st, &lrc)
               : launch_pair<__half, 0, false>(tmB, tmA, p, units, st, &lrc);
    if (lrc) return lrc;
  } else if (dtype == DK_BF16) {
    static bool done[2][kMaxDevices] = {};
    auto fn = fold ? dk::gemm::gemm_kernel<__nv_bfloat16, 1, true> : dk::gemm::gemm_kernel<__nv_bfloat16, 1, false>;
    if ((rc = ensure_smem(fn, dk::gemm::kSmemBytes, done[fold]))) return rc;
    e = launch_pdl(fn, dim3(grid), dim3(dk::gemm::kThreads), dk::gemm::kSmemBytes, st, tmB, tmA, p);
  } else {
    static bool done[2][kMaxDevices] = {};
    auto fn = fold ? dk::gemm::gemm_kernel<__half, 0, true> : dk::gemm::gemm_kernel<__half, 0, false>;
    if ((rc = ensure_smem(fn, dk::gemm::kSmemBytes, done[fold]))) return rc;
    e = launch_pdl(fn, dim3(grid), dim3(dk::gemm::kThreads), dk::gemm::kSmemBytes, st, tmB, tmA, p);
  }
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  if (p.mode == dk::gemm::SPLIT) {
    // the upper tree levels over the groups' subtree sums, as a dependent launch
    const int n_parts = (p.slice_end - p.slice_begin) / p.group;
    if (norm) return launch_fold_norm(dtype, p.ws, n_parts, p, *norm, st);
    if (dtype == DK_BF16) return launch_fold<__nv_bfloat16>(p.ws, n_parts, p, st);
    return launch_fold<__half>(p.ws, n_parts, p, st);
  }
  if (norm) {
    const int rc = check_launch(what);
    if (rc) return rc;
    return dk_rmsnorm_batch_invariant(p.c, p.ldc, norm->w, norm->out, norm->ld, p.M, p.N, dtype, norm->w_dtype,
                                      norm->eps, st);
  }
  return check_launch(what);
}

int zero_output(void* c, int64_t ldc, int64_t M, int64_t N, int elem, cudaStream_t st) {
  if (M == 0 || N == 0) return DK_OK;
  cudaError_t e = cudaMemset2DAsync(c, ldc * elem, 0, N * elem, M, st);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "matmul: memset: %s", cudaGetErrorString(e));
  return DK_OK;
}

template <typename T>
int launch_cast(const float* src, void* c, int64_t ldc, int M, int N, cudaStream_t st) {
  const int64_t MN = static_cast<int64_t>(M) * N;
  const int blocks = static_cast<int>(ceil_div(MN, 256) < 4096 ? ceil_div(MN, 256) : 4096);
  dk::gemm::cast_out_kernel<T><<<blocks, 256, 0, st>>>(src, static_cast<T*>(c), ldc, M, N);
  return check_launch("matmul_batch_variant");
}

// ============================ attention ============================
struct AttnPlan {
  int n_tiles, rows_cap, max_splits, spu, upt;
  size_t o_bytes, ml_bytes, cnt_bytes, total;
};

// Splits per CTA (schedule only; the arithmetic of a row never depends on it):
// enough CTAs to fill the GPU a few times over, at most 8 splits (2048 tokens)
// per CTA so long rows do not leave a tail.
AttnPlan plan_attention(int32_t n_tiles, int32_t rows_per_tile, int32_t hq, int32_t hkv, int32_t D,
                        int32_t max_kv_len) {
  AttnPlan pl{};
  const int G = (hkv > 0) ? hq / hkv : 1;
  pl.n_tiles = n_tiles;
  pl.rows_cap = (rows_per_tile <= 1) ? G : (dk::attn::kRows / G) * G;
  pl.max_splits = static_cast<int>(ceil_div(max_kv_len > 0 ? max_kv_len : 1, dk::attn::kSplit));
  const int64_t pairs = static_cast<int64_t>(n_tiles) * (hkv > 0 ? hkv : 1);
  const int64_t target = 4LL * sm_count(current_device());
  int64_t upt = (pairs >= target) ? 1 : ceil_div(target, pairs);
  if (upt > pl.max_splits) upt = pl.max_splits;
  int spu = static_cast<int>(ceil_div(pl.max_splits, upt));
  if (spu > 8) spu = 8;
  if (spu < 1) spu = 1;
  pl.spu = spu;
  pl.upt = static_cast<int>(ceil_div(pl.max_splits, spu));
  const size_t slots = static_cast<size_t>(n_tiles) * hkv * pl.max_splits * pl.rows_cap;
  pl.o_bytes = ceil_div(slots * D * sizeof(float), 256) * 256;
  pl.ml_bytes = ceil_div(slots * 2 * sizeof(float), 256) * 256;
  pl.cnt_bytes = static_cast<size_t>(n_tiles) * hkv * sizeof(int32_t);
  // scratch only when some tile's splits are spread over several CTAs
  pl.total = (pl.upt > 1) ? (kCounterBytes + pl.o_bytes + pl.ml_bytes) : 0;
  return pl;
}

template <typename T, int D, int KM, bool T1>
int attn_launch_km(const dk::attn::KvMaps& maps, const dk::attn::Params& p, int64_t n_items, cudaStream_t st) {
  using C = dk::attn::Cfg<D, T1>;
  static bool done[kMaxDevices] = {false};
  static int resident[kMaxDevices][dk::attn::kRows + 1] = {};   // CTAs per SM, by rows_cap
  auto fn = dk::attn::attn_kernel<T, D, KM, T1>;
  int rc = ensure_smem(fn, C::smem_bytes(dk::attn::kRows), done);
  if (rc) return rc;
  const int dev = current_device();
  const int smem = C::smem_bytes(p.rows_cap);
  int per_sm = 0;
  if (dev >= 0 && dev < kMaxDevices && p.rows_cap >= 0 && p.rows_cap <= dk::attn::kRows)
    per_sm = resident[dev][p.rows_cap];
  if (per_sm <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, dk::attn::kThreads, smem) != cudaSuccess ||
        per_sm <= 0)
      per_sm = 1;
    if (dev >= 0 && dev < kMaxDevices && p.rows_cap >= 0 && p.rows_cap <= dk::attn::kRows)
      resident[dev][p.rows_cap] = per_sm;
  }
  // persistent grid: every CTA resident at once, each walking items b, b + grid, ...
  const int64_t cap = static_cast<int64_t>(per_sm) * sm_count(dev);
  const int grid = static_cast<int>(n_items < cap ? n_items : cap);
  if (grid <= 0) return DK_OK;
  cudaError_t e = launch_pdl(fn, dim3(grid), dim3(dk::attn::kThreads), smem, st, maps, p);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "attention_batch_invariant: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

template <typename T, int D>
int attn_launch(const dk::attn::KvMaps& maps, const dk::attn::Params& p, int64_t n_items,
                cudaStream_t st) {
  constexpr int kThr = dk::attn::kConsumerWarps * 32;
  constexpr int kNarrow = (4 < dk::attn::Cfg<D>::KMAX) ? 4 : dk::attn::Cfg<D>::KMAX;
  if (p.rows_cap == 1) return attn_launch_km<T, D, 1, true>(maps, p, n_items, st);
  if (p.rows_cap * D <= kNarrow * kThr) return attn_launch_km<T, D, kNarrow, false>(maps, p, n_items, st);
  return attn_launch_km<T, D, dk::attn::Cfg<D>::KMAX, false>(maps, p, n_items, st);
}

template <typename T, int DK, int DV>
int gdn_launch_t(const dk::gdn::Params& p, int64_t n_seqs, cudaStream_t st) {
  if (p.chunk == 1) {
    cudaError_t e = launch_pdl(dk::gdn::gdn_recurrent_kernel<T, DK, DV>,
                               dim3(p.HV, static_cast<unsigned>(n_seqs), DV / 32), dim3(32 * dk::gdn::kRecWarps), 0, st,
                               p);
    if (e != cudaSuccess) return fail(DK_ERR_CUDA, "gdn: launch failed: %s", cudaGetErrorString(e));
    return DK_OK;
  }
  static bool done[kMaxDevices] = {};
  auto fn = dk::gdn::gdn_chunk_kernel<T, DK, DV>;
  const int bytes = static_cast<int>(dk::gdn::Smem<DK, DV>::kBytes);
  int rc = ensure_smem(fn, bytes, done);
  if (rc) return rc;
  cudaError_t e = launch_pdl(fn, dim3(p.HV, static_cast<unsigned>(n_seqs)), dim3(dk::gdn::kThreads), bytes, st, p);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "gdn: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

template <int D>
int gdn_launch_tc(const dk::gdn::Params& p, int64_t n_seqs, cudaStream_t st) {
  static bool done[kMaxDevices] = {};
  auto fn = dk::gdn::gdn_chunk_tc_kernel<D>;
  const int bytes = dk::gdn::TcSmem<D>::kBytes;
  int rc = ensure_smem(fn, bytes, done);
  if (rc) return rc;
  cudaError_t e = launch_pdl(fn, dim3(p.HV, static_cast<unsigned>(n_seqs)), dim3(dk::gdn::kTcThreads), bytes, st, p);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "gdn: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

// Which kernel runs chunked bf16 GDN with head dim 128: 0 = the tcgen05 kernel, 1 = the mma.sync
// kernel.  Only the test hook dk_gdn_kernel_for_test sets it.
int g_gdn_override = 0;

// Chunked bf16, head dim 128, on tcgen05 (gdn_chunk_umma_kernel): K, Q and V chunks by TMA through
// 2-D maps over the packed [tokens, heads x 128] tensors.
int gdn_launch_umma(const dk::gdn::Params& p, int64_t n_seqs, cudaStream_t st) {
  static bool done[kMaxDevices] = {};
  auto fn = dk::gdn::gdn_chunk_umma_kernel;
  int rc = ensure_smem(fn, dk::gdn::kUmSmem, done);
  if (rc) return rc;
  const int64_t rows = p.cu_seqlens ? p.seq_len : n_seqs * p.seq_len;
  if (rows <= 0) return DK_OK;
  if (rows > 0x7fffffffLL) return fail(DK_ERR_UNSUPPORTED, "gdn: more than 2^31 tokens");
  CUtensorMap tk, tq, tv;
  const uint64_t dqk[2] = {static_cast<uint64_t>(p.H) * dk::gdn::kUmD, static_cast<uint64_t>(rows)};
  const uint64_t sqk[1] = {static_cast<uint64_t>(p.H) * dk::gdn::kUmD * 2};
  const uint64_t dvv[2] = {static_cast<uint64_t>(p.HV) * dk::gdn::kUmD, static_cast<uint64_t>(rows)};
  const uint64_t svv[1] = {static_cast<uint64_t>(p.HV) * dk::gdn::kUmD * 2};
  const uint32_t box[2] = {64, static_cast<uint32_t>(dk::gdn::kChunk)};
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if ((rc = encode_map(&tk, dt, 2, p.k, dqk, sqk, box, CU_TENSOR_MAP_SWIZZLE_128B, "gdn"))) return rc;
  if ((rc = encode_map(&tq, dt, 2, p.q, dqk, sqk, box, CU_TENSOR_MAP_SWIZZLE_128B, "gdn"))) return rc;
  if ((rc = encode_map(&tv, dt, 2, p.v, dvv, svv, box, CU_TENSOR_MAP_SWIZZLE_128B, "gdn"))) return rc;
  cudaError_t e = launch_pdl(fn, dim3(p.HV, static_cast<unsigned>(n_seqs)), dim3(dk::gdn::kUmThreads),
                             dk::gdn::kUmSmem, st, tk, tq, tv, p);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "gdn: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

template <typename T>
int gdn_launch_dims(const dk::gdn::Params& p, int dk_, int dv_, int64_t n_seqs, cudaStream_t st) {
  // chunked bf16: head dim 128 on tcgen05, 64 on mma.sync; otherwise the f32 CUDA-core kernel
  if (std::is_same<T, __nv_bfloat16>::value && p.chunk == dk::gdn::kChunk && dk_ == dv_) {
    if (dk_ == 128 && g_gdn_override == 0) return gdn_launch_umma(p, n_seqs, st);
    if (dk_ == 128) return gdn_launch_tc<128>(p, n_seqs, st);
    if (dk_ == 64) return gdn_launch_tc<64>(p, n_seqs, st);
  }
  if (dk_ == 128 && dv_ == 128) return gdn_launch_t<T, 128, 128>(p, n_seqs, st);
  if (dk_ == 64 && dv_ == 64) return gdn_launch_t<T, 64, 64>(p, n_seqs, st);
  if (dk_ == 32 && dv_ == 32) return gdn_launch_t<T, 32, 32>(p, n_seqs, st);
  return fail(DK_ERR_UNSUPPORTED, "gdn: head dims (%d, %d) not built (32/32, 64/64, 128/128)", dk_, dv_);
}

}  // namespace

// Fixed scratch for dk_attention_batch_invariant_noalloc (32 MiB per device, zero at load).
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(32) << 20;
static __device__ __align__(256) unsigned char dk_noalloc_scratch[kNoAllocScratchBytes];

namespace {

std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kMaxDevices] = {nullptr};

// Device address of dk_noalloc_scratch on the current device, looked up on the first call
// per device (with that device current) and cached.
int noalloc_scratch(void** out, const char* what) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(DK_ERR_UNSUPPORTED, "%s: device %d out of range", what, dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, dk_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(DK_ERR_CUDA, "%s: cudaGetSymbolAddress failed: %s", what, cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return DK_OK;
}

}  // namespace

// =====================================================================================
extern "C" {

int dk_abi_version(void) { return DK_ABI_VERSION; }

const char* dk_last_error(void) { return g_last_error.c_str(); }

int dk_device_status(int device, int clear, int* code, int* detail) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return fail(DK_ERR_CUDA, "dk_device_status: no CUDA device");
  if (cudaSetDevice(device) != cudaSuccess) return fail(DK_ERR_INVALID_ARGUMENT, "dk_device_status: bad device");
  int c = 0, d = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&c, dk::g_status_code, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&d, dk::g_status_detail, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int z = 0;
    e = cudaMemcpyToSymbol(dk::g_status_code, &z, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(dk::g_status_detail, &z, sizeof(int));
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "dk_device_status: %s", cudaGetErrorString(e));
  if (code) *code = c;
  if (detail) *detail = d;
  return DK_OK;
}

int dk_kernel_attributes(int which, int* num_regs, int* max_threads, int* local_bytes, int* max_dynamic_smem) {
  cudaFuncAttributes a{};
  cudaError_t e;
  switch (which) {
    case 0: e = cudaFuncGetAttributes(&a, dk::gemm::gemm_kernel<__nv_bfloat16, 1, true>); break;
    case 1: e = cudaFuncGetAttributes(&a, dk::attn::attn_kernel<__nv_bfloat16, 128, 4, false>); break;
    case 2: e = cudaFuncGetAttributes(&a, dk::attn::attn_kernel<__nv_bfloat16, 64, 4, false>); break;
    case 3: e = cudaFuncGetAttributes(&a, dk::rmsnorm_inv_vec_kernel<float, float, 8>); break;
    default: return fail(DK_ERR_INVALID_ARGUMENT, "dk_kernel_attributes: unknown kernel %d", which);
  }
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "dk_kernel_attributes: %s", cudaGetErrorString(e));
  if (num_regs) *num_regs = a.numRegs;
  if (max_threads) *max_threads = a.maxThreadsPerBlock;
  if (local_bytes) *local_bytes = static_cast<int>(a.localSizeBytes);
  if (max_dynamic_smem) *max_dynamic_smem = a.maxDynamicSharedSizeBytes;
  return DK_OK;
}

int dk_test_bounded_wait(int skip_arrive, int64_t limit_ns, void* stream) {
  if (limit_ns <= 0 || limit_ns > 100000000LL)
    return fail(DK_ERR_INVALID_ARGUMENT, "dk_test_bounded_wait: limit_ns must be in (0, 100 ms]");
  dk::bounded_wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      skip_arrive ? 1 : 0, static_cast<unsigned long long>(limit_ns));
  return check_launch("dk_test_bounded_wait");
}

int dk_num_sms(int device, int* out) {
  int n = 0;
  cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "dk_num_sms: %s", cudaGetErrorString(e));
  if (out) *out = n;
  return DK_OK;
}

// ---------------- RMSNorm ----------------
int dk_rmsnorm_batch_invariant(const void* x, int64_t x_row_stride, const void* weight, void* out,
                               int64_t out_row_stride, int64_t n_rows, int64_t n_cols, int dtype, int wdtype,
                               float eps, void* stream) {
  int rc = rms_validate(x, weight, out, x_row_stride, out_row_stride, n_rows, n_cols, dtype, wdtype,
                        "rmsnorm_batch_invariant");
  if (rc) return rc;
  if (n_rows == 0) return DK_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DK_DISPATCH_RMS(rmsnorm_inv_launch, x, x_row_stride, weight, out, out_row_stride, n_rows, n_cols, eps, st);
}

int dk_rmsnorm_gather_batch_invariant(const void* table, int64_t table_row_stride, int64_t table_rows,
                                      const int64_t* row_index, const void* weight, void* x_out, int64_t x_row_stride,
                                      void* out, int64_t out_row_stride, int64_t n_rows, int64_t n_cols, int dtype,
                                      int wdtype, float eps, void* stream) {
  int rc = rms_validate(table, weight, out, table_row_stride, out_row_stride, n_rows, n_cols, dtype, wdtype,
                        "rmsnorm_gather");
  if (rc) return rc;
  if (n_rows == 0) return DK_OK;
  if (!row_index || !x_out || table_rows <= 0 || (n_rows > 1 && x_row_stride < n_cols) ||
      (table_rows > 1 && table_row_stride < n_cols))
    return fail(DK_ERR_INVALID_ARGUMENT, "rmsnorm_gather: bad index, table or x_out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DK_DISPATCH_RMS(rmsnorm_gather_launch, table, table_row_stride, table_rows, row_index, weight, x_out, x_row_stride,
                  out, out_row_stride, n_rows, n_cols, eps, st);
}

size_t dk_rmsnorm_variant_workspace_size(int64_t n_rows) {
  return kCounterBytes + static_cast<size_t>(ceil_div((n_rows > 0 ? n_rows : 1) * 4, 256) * 256);
}

int dk_rmsnorm_batch_variant(const void* x, int64_t x_row_stride, const void* weight, void* out,
                             int64_t out_row_stride, int64_t n_rows, int64_t n_cols, int dtype, int wdtype, float eps,
                             int split_threshold, int n_splits, void* workspace, size_t workspace_bytes,
                             void* stream) {
  int rc = rms_validate(x, weight, out, x_row_stride, out_row_stride, n_rows, n_cols, dtype, wdtype,
                        "rmsnorm_batch_variant");
  if (rc) return rc;
  if (n_rows == 0) return DK_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_rows >= split_threshold) {
    DK_DISPATCH_RMS(rmsnorm_inv_launch, x, x_row_stride, weight, out, out_row_stride, n_rows, n_cols, eps, st);
  }
  if (n_splits < 1 || n_splits > 1024) return fail(DK_ERR_INVALID_ARGUMENT, "rmsnorm_batch_variant: bad n_splits");
  if (!workspace || workspace_bytes < dk_rmsnorm_variant_workspace_size(n_rows))
    return fail(DK_ERR_WORKSPACE, "rmsnorm_batch_variant: workspace too small");
  float* partial = reinterpret_cast<float*>(ws_data(workspace));
  DK_DISPATCH_RMS(rmsnorm_var_launch, x, x_row_stride, weight, out, out_row_stride, n_rows, n_cols, eps, n_splits,
                  partial, st);
}

// ---------------- matmul ----------------
size_t dk_matmul_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0) return 0;
  return plan_invariant(M, N, K, sm_count(current_device())).ws_bytes;
}

size_t dk_matmul_variant_workspace_size(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  return kCounterBytes + static_cast<size_t>(ceil_div(M * N * 4, 256) * 256);
}

int dk_matmul_batch_invariant(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc, int64_t M,
                              int64_t N, int64_t K, int dtype, void* workspace, size_t workspace_bytes,
                              void* stream) {
  return dk_matmul_batch_invariant_ex(a, lda, b, ldb, c, ldc, M, N, K, dtype, nullptr, workspace, workspace_bytes,
                                      stream);
}

int dk_matmul_batch_invariant_ex(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                                 int64_t M, int64_t N, int64_t K, int dtype, const dk_matmul_epilogue* epi,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  const char* what = "matmul_batch_invariant";
  int rc = gemm_validate(a, lda, b, ldb, M, N, K, dtype, what);
  if (rc) return rc;
  if (M == 0 || N == 0) return DK_OK;
  dk_matmul_epilogue e{};
  e.mode = DK_EPI_STORE;
  if (epi) e = *epi;
  int64_t out_cols = N;
  switch (e.mode) {
    case DK_EPI_STORE:
    case DK_EPI_SILU:
      break;
    case DK_EPI_RESIDUAL:
      if (!e.resid || e.ld_resid < N) return fail(DK_ERR_INVALID_ARGUMENT, "%s: residual epilogue needs R", what);
      break;
    case DK_EPI_RESIDUAL_RMSNORM:
      if (!e.resid || e.ld_resid < N) return fail(DK_ERR_INVALID_ARGUMENT, "%s: residual epilogue needs R", what);
      if (!e.norm_w || !e.norm_out || e.norm_ld < N || !valid_dtype(e.norm_w_dtype))
        return fail(DK_ERR_INVALID_ARGUMENT, "%s: RMSNorm epilogue needs a weight, an output and norm_ld >= N", what);
      break;
    case DK_EPI_SILU_MUL:
      if (N % 2) return fail(DK_ERR_INVALID_ARGUMENT, "%s: gate/up epilogue needs an even N", what);
      out_cols = N / 2;
      break;
    case DK_EPI_ARGMAX:
      if (!e.argmax_keys) return fail(DK_ERR_INVALID_ARGUMENT, "%s: argmax epilogue needs keys", what);
      if (N > 0x7fffffffLL) return fail(DK_ERR_UNSUPPORTED, "%s: argmax over more than 2^31 columns", what);
      if (!c) out_cols = 0;
      break;
    case DK_EPI_QKV_CACHE:
      if (e.q_cols < 0 || e.kv_cols <= 0 || e.head_dim <= 0 || e.kv_cols % e.head_dim ||
          static_cast<int64_t>(e.q_cols) + 2LL * e.kv_cols != N || !e.k_cache || !e.v_cache || !e.row_pos)
        return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad QKV cache epilogue", what);
      if (e.block_table && (e.page_size <= 0 || e.blocks_per_seq <= 0 || e.n_blocks <= 0 ||
                            e.block_table_stride < e.blocks_per_seq))
        return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad paged KV fields (page_size, blocks_per_seq, n_blocks)", what);
      out_cols = e.q_cols;
      break;
    default:
      return fail(DK_ERR_INVALID_ARGUMENT, "%s: unknown epilogue mode %d", what, e.mode);
  }
  if (!c && out_cols > 0) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null output", what);
  if (ldc < out_cols) return fail(DK_ERR_INVALID_ARGUMENT, "%s: ldc too small", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    if (e.mode != DK_EPI_STORE) return fail(DK_ERR_UNSUPPORTED, "%s: K == 0 with a fused epilogue", what);
    return zero_output(c, ldc, M, N, 2, st);
  }
  const GemmPlan pl = plan_invariant(M, N, K, sm_count(current_device()));
  dk::gemm::Params p{};
  p.epi = e;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.slice_len = slice_len_for(K, dk::gemm::kSlices);
  p.slice_begin = 0;
  p.slice_end = dk::gemm::kSlices;
  p.group = pl.group;
  p.n_tiles = pl.n_tiles;
  p.m_tiles = pl.m_tiles;
  p.mode = pl.mode;
  p.pair = pl.kernel;
  p.c = c;
  p.ldc = ldc;
  if (pl.ws_bytes > 0) {
    if (!workspace || workspace_bytes < pl.ws_bytes)
      return fail(DK_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", what, pl.ws_bytes,
                  workspace_bytes);
    if (!aligned16(workspace)) return fail(DK_ERR_WORKSPACE, "%s: workspace must be 16-byte aligned", what);
    if (pl.mode == dk::gemm::SPLIT) p.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + pl.partials_off);
    if (pl.stash) p.stash = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + pl.stash_off);
  }
  if (pl.kernel == 2 && pl.group == dk::gemm::kSlices && !p.stash)
    return fail(DK_ERR_WORKSPACE, "%s: the wide schedule needs its stash", what);
  if (e.mode == DK_EPI_RESIDUAL_RMSNORM) {
    const NormSpec nm{e.norm_w, e.norm_w_dtype, e.norm_out, e.norm_ld, e.norm_eps};
    p.epi.mode = DK_EPI_RESIDUAL;   // the GEMM (or its fold) writes C; the norm follows from it
    return gemm_launch(dtype, a, lda, b, ldb, p, st, what, &nm);
  }
  return gemm_launch(dtype, a, lda, b, ldb, p, st, what);
}

int dk_argmax_finish(unsigned long long* keys, int64_t n_rows, int64_t* tokens, int64_t* tokens_copy,
                     int32_t* lens_a, int32_t* lens_b, void* stream) {
  if (n_rows < 0) return fail(DK_ERR_INVALID_ARGUMENT, "argmax_finish: negative row count");
  if (n_rows == 0) return DK_OK;
  if (!keys || !tokens) return fail(DK_ERR_INVALID_ARGUMENT, "argmax_finish: null keys or tokens");
  const int64_t want = ceil_div(n_rows, 256);
  const int blocks = static_cast<int>(want < 1024 ? want : 1024);
  cudaError_t e = launch_pdl(dk::gemm::argmax_finish_kernel, dim3(blocks), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), keys, n_rows, tokens, tokens_copy, lens_a, lens_b);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "argmax_finish: launch failed: %s", cudaGetErrorString(e));
  return DK_OK;
}

int dk_matmul_slice_partials(const void* a, int64_t lda, const void* b, int64_t ldb, float* partials, int64_t M,
                             int64_t N, int64_t K, int slice_begin, int slice_end, int dtype, void* stream) {
  const char* what = "matmul_slice_partials";
  int rc = gemm_validate(a, lda, b, ldb, M, N, K, dtype, what);
  if (rc) return rc;
  const int span = slice_end - slice_begin;
  if (slice_begin < 0 || slice_end > dk::gemm::kSlices || span <= 0 || (span & (span - 1)) != 0 ||
      slice_begin % span != 0)
    return fail(DK_ERR_INVALID_ARGUMENT,
                "%s: slice range [%d, %d) is not an aligned group of 1, 2, 4 or 8 slices", what, slice_begin,
                slice_end);
  if (M == 0 || N == 0) return DK_OK;
  if (!partials) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null partials", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    cudaError_t e = cudaMemsetAsync(partials, 0, sizeof(float) * M * N, st);
    return e == cudaSuccess ? DK_OK : fail(DK_ERR_CUDA, "%s: memset: %s", what, cudaGetErrorString(e));
  }
  dk::gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.slice_len = slice_len_for(K, dk::gemm::kSlices);
  p.slice_begin = slice_begin;
  p.slice_end = slice_end;
  p.group = span;
  p.n_tiles = static_cast<int>(ceil_div(N, dk::gemm::kTileN));
  p.m_tiles = static_cast<int>(ceil_div(M, dk::gemm::kTileM));
  p.mode = dk::gemm::PARTIAL;
  p.ws = partials;
  return gemm_launch(dtype, a, lda, b, ldb, p, st, what);
}

int dk_matmul_shard_partials(const void* a, int64_t lda, const void* b, int64_t ldb, float* partial, int64_t M,
                             int64_t N, int64_t K, int slice_begin, int slice_end, int dtype, void* stream) {
  const char* what = "matmul_shard_partials";
  const int span = slice_end - slice_begin;
  if (slice_begin < 0 || slice_end > dk::gemm::kSlices || span <= 0 || (span & (span - 1)) != 0 ||
      slice_begin % span != 0)
    return fail(DK_ERR_INVALID_ARGUMENT,
                "%s: slice range [%d, %d) is not an aligned group of 1, 2, 4 or 8 slices", what, slice_begin,
                slice_end);
  if (K < 0 || K > 0x7fffffffLL) return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad K", what);
  int64_t k0, k1;
  dk_matmul_shard_range(K, slice_begin, slice_end, &k0, &k1);
  const int64_t k_loc = k1 - k0;
  if (k_loc == 0) {
    if (M == 0 || N == 0) return DK_OK;
    if (!partial) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null partial", what);
    cudaError_t e = cudaMemsetAsync(partial, 0, sizeof(float) * M * N, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? DK_OK : fail(DK_ERR_CUDA, "%s: memset: %s", what, cudaGetErrorString(e));
  }
  int rc = gemm_validate(a, lda, b, ldb, M, N, k_loc, dtype, what);
  if (rc) return rc;
  if (M == 0 || N == 0) return DK_OK;
  if (!partial) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null partial", what);
  dk::gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.k_base = static_cast<int>(k0);
  p.k_extent = static_cast<int>(k_loc);
  p.slice_len = slice_len_for(K, dk::gemm::kSlices);
  p.slice_begin = slice_begin;
  p.slice_end = slice_end;
  p.group = span;
  p.n_tiles = static_cast<int>(ceil_div(N, dk::gemm::kTileN));
  p.m_tiles = static_cast<int>(ceil_div(M, dk::gemm::kTileM));
  p.mode = dk::gemm::PARTIAL;
  p.ws = partial;
  return gemm_launch(dtype, a, lda, b, ldb, p, static_cast<cudaStream_t>(stream), what);
}

void dk_matmul_shard_range(int64_t K, int slice_begin, int slice_end, int64_t* k_begin, int64_t* k_end) {
  const int64_t L = (K <= 0) ? 0 : slice_len_for(K, dk::gemm::kSlices);
  int64_t b = L * slice_begin, e = L * slice_end;
  if (b > K) b = K;
  if (e > K) e = K;
  if (b < 0) b = 0;
  if (e < b) e = b;
  if (k_begin) *k_begin = b;
  if (k_end) *k_end = e;
}

int dk_matmul_fold_slices(const float* partials, int n_parts, void* c, int64_t ldc, int64_t M, int64_t N, int dtype,
                          void* stream) {
  if (dtype != DK_BF16 && dtype != DK_F16) return fail(DK_ERR_UNSUPPORTED, "matmul_fold_slices: bad dtype");
  if (n_parts != 1 && n_parts != 2 && n_parts != 4 && n_parts != 8)
    return fail(DK_ERR_INVALID_ARGUMENT, "matmul_fold_slices: n_parts must be 1, 2, 4 or 8");
  if (M < 0 || N < 0 || M > 0x7fffffffLL || N > 0x7fffffffLL)
    return fail(DK_ERR_INVALID_ARGUMENT, "matmul_fold_slices: bad shape");
  if (M == 0 || N == 0) return DK_OK;
  if (!partials || !c || ldc < N) return fail(DK_ERR_INVALID_ARGUMENT, "matmul_fold_slices: bad pointer/ldc");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dk::gemm::Params p{};
  p.epi.mode = DK_EPI_STORE;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.c = c;
  p.ldc = ldc;
  if (dtype == DK_BF16) return launch_fold<__nv_bfloat16>(partials, n_parts, p, st);
  return launch_fold<__half>(partials, n_parts, p, st);
}

int dk_matmul_fold_slices_ex(const float* partials, int n_parts, void* c, int64_t ldc, int64_t M, int64_t N,
                             int dtype, const dk_matmul_epilogue* epi, void* stream) {
  const char* what = "matmul_fold_slices_ex";
  if (dtype != DK_BF16 && dtype != DK_F16) return fail(DK_ERR_UNSUPPORTED, "%s: bad dtype", what);
  if (n_parts != 1 && n_parts != 2 && n_parts != 4 && n_parts != 8)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: n_parts must be 1, 2, 4 or 8", what);
  if (M < 0 || N < 0 || M > 0x7fffffffLL || N > 0x7fffffffLL) return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad shape", what);
  if (M == 0 || N == 0) return DK_OK;
  if (!partials) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null partials", what);
  dk_matmul_epilogue e{};
  e.mode = DK_EPI_STORE;
  if (epi) e = *epi;
  int64_t out_cols = N;
  switch (e.mode) {
    case DK_EPI_STORE:
    case DK_EPI_SILU:
      break;
    case DK_EPI_RESIDUAL:
    case DK_EPI_RESIDUAL_RMSNORM:
      if (!e.resid || e.ld_resid < N) return fail(DK_ERR_INVALID_ARGUMENT, "%s: residual epilogue needs R", what);
      if (e.mode == DK_EPI_RESIDUAL_RMSNORM && (!e.norm_w || !e.norm_out || e.norm_ld < N || !valid_dtype(e.norm_w_dtype)))
        return fail(DK_ERR_INVALID_ARGUMENT, "%s: RMSNorm epilogue needs a weight, an output and norm_ld >= N", what);
      break;
    case DK_EPI_SILU_MUL:
      if (N % 2) return fail(DK_ERR_INVALID_ARGUMENT, "%s: gate/up epilogue needs an even N", what);
      out_cols = N / 2;
      break;
    case DK_EPI_ARGMAX:
      if (!e.argmax_keys) return fail(DK_ERR_INVALID_ARGUMENT, "%s: argmax epilogue needs keys", what);
      if (!c) out_cols = 0;
      break;
    default:
      return fail(DK_ERR_UNSUPPORTED, "%s: epilogue mode %d is not available after a fold", what, e.mode);
  }
  if (out_cols > 0 && (!c || ldc < out_cols)) return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad output or ldc", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dk::gemm::Params p{};
  p.epi = e;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.c = c;
  p.ldc = ldc;
  if (e.mode == DK_EPI_RESIDUAL_RMSNORM) {
    const NormSpec nm{e.norm_w, e.norm_w_dtype, e.norm_out, e.norm_ld, e.norm_eps};
    p.epi.mode = DK_EPI_RESIDUAL;
    return launch_fold_norm(dtype, partials, n_parts, p, nm, st);
  }
  if (dtype == DK_BF16) return launch_fold<__nv_bfloat16>(partials, n_parts, p, st);
  return launch_fold<__half>(partials, n_parts, p, st);
}

int dk_argmax_finish_parts(const unsigned long long* keys, int n_parts, int64_t part_stride,
                           const int64_t* col_offsets, int64_t n_rows, int64_t* tokens, int64_t* tokens_copy,
                           int32_t* lens_a, int32_t* lens_b, unsigned long long* reset_keys, void* stream) {
  const char* what = "argmax_finish_parts";
  if (n_rows < 0 || n_parts < 1 || n_parts > 8 || part_stride < n_rows)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad sizes (1 <= n_parts <= 8, part_stride >= n_rows)", what);
  if (n_rows == 0) return DK_OK;
  if (!keys || !tokens || !col_offsets) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null keys, tokens or offsets", what);
  dk::gemm::PartOffsets offs{};
  for (int q = 0; q < n_parts; ++q) {
    if (col_offsets[q] < 0 || col_offsets[q] > 0x7fffffffLL)
      return fail(DK_ERR_INVALID_ARGUMENT, "%s: column offset out of range", what);
    offs.v[q] = col_offsets[q];
  }
  const int64_t want = ceil_div(n_rows, 256);
  const int blocks = static_cast<int>(want < 1024 ? want : 1024);
  cudaError_t e = launch_pdl(dk::gemm::argmax_finish_parts_kernel, dim3(blocks), dim3(256), 0,
                             static_cast<cudaStream_t>(stream), keys, n_parts, part_stride, offs, n_rows, tokens,
                             tokens_copy, lens_a, lens_b, reset_keys);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return DK_OK;
}

int dk_matmul_batch_variant(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc, int64_t M,
                            int64_t N, int64_t K, int dtype, int split_m_threshold, int split_k, void* workspace,
                            size_t workspace_bytes, void* stream) {
  const char* what = "matmul_batch_variant";
  if (M >= split_m_threshold)
    return dk_matmul_batch_invariant(a, lda, b, ldb, c, ldc, M, N, K, dtype, workspace, workspace_bytes, stream);
  int rc = gemm_validate(a, lda, b, ldb, M, N, K, dtype, what);
  if (rc) return rc;
  if (M == 0 || N == 0) return DK_OK;
  if (!c || ldc < N) return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad output", what);
  if (split_k < 1 || split_k > 64) return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad split_k", what);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) return zero_output(c, ldc, M, N, 2, st);
  const size_t need = dk_matmul_variant_workspace_size(M, N);
  if (!workspace || workspace_bytes < need)
    return fail(DK_ERR_WORKSPACE, "%s: workspace of %zu bytes needed", what, need);
  float* acc = reinterpret_cast<float*>(ws_data(workspace));
  cudaError_t e = cudaMemsetAsync(acc, 0, sizeof(float) * M * N, st);
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "%s: memset: %s", what, cudaGetErrorString(e));
  dk::gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.slice_len = slice_len_for(K, split_k);
  p.slice_begin = 0;
  p.slice_end = split_k;
  p.group = 1;
  p.n_tiles = static_cast<int>(ceil_div(N, dk::gemm::kTileN));
  p.m_tiles = static_cast<int>(ceil_div(M, dk::gemm::kTileM));
  p.mode = dk::gemm::ATOMIC;
  p.ws = acc;
  rc = gemm_launch(dtype, a, lda, b, ldb, p, st, what);
  if (rc) return rc;
  if (dtype == DK_BF16) return launch_cast<__nv_bfloat16>(acc, c, ldc, (int)M, (int)N, st);
  return launch_cast<__half>(acc, c, ldc, (int)M, (int)N, st);
}

// ---------------- attention ----------------
size_t dk_attention_workspace_size(int32_t n_tiles, int32_t rows_per_tile, int32_t n_q_heads, int32_t n_kv_heads,
                                   int32_t head_dim, int32_t max_kv_len) {
  if (n_tiles <= 0 || n_kv_heads <= 0 || n_q_heads <= 0 || head_dim <= 0) return 0;
  return plan_attention(n_tiles, rows_per_tile, n_q_heads, n_kv_heads, head_dim, max_kv_len).total;
}

}  // extern "C"

namespace {

// Paged KV description (null: a contiguous [n_seq, heads, capacity, d] cache).
struct PagedKV {
  const int32_t* table;
  int64_t table_stride;
  int32_t page;
  int32_t blocks_per_seq;
  int64_t n_blocks;
};

// The invariant decode attention over a contiguous cache (pg == nullptr; kv_stride_seq /
// kv_n_seq / kv_capacity describe it) or a paged one (the strides describe the block pool;
// kv_n_seq is the number of block-table rows and the capacity blocks_per_seq * page).
int attention_invariant_impl(const void* q, int64_t q_stride_row, int64_t q_stride_head, const void* k,
                             const void* v, int64_t kv_stride_seq, int64_t kv_stride_head, int64_t kv_stride_tok,
                             int64_t kv_n_seq, int64_t kv_capacity, void* out, int64_t out_stride_row,
                             int64_t out_stride_head, const int32_t* kv_lens, int32_t uniform_kv_len,
                             const int32_t* row_tiles, int32_t n_tiles, int32_t n_rows, int32_t n_q_heads,
                             int32_t n_kv_heads, int32_t head_dim, int32_t max_kv_len, float scale, int dtype,
                             void* workspace, size_t workspace_bytes, void* stream, const PagedKV* pg,
                             const char* what) {
  if (dtype != DK_BF16 && dtype != DK_F16) return fail(DK_ERR_UNSUPPORTED, "%s: dtype must be bf16 or f16", what);
  if (head_dim != 32 && head_dim != 64 && head_dim != 128)
    return fail(DK_ERR_UNSUPPORTED, "%s: head_dim %d not in {32, 64, 128}", what, head_dim);
  if (n_rows < 0 || n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad head counts", what);
  const int G = n_q_heads / n_kv_heads;
  if (G > dk::attn::kRows) return fail(DK_ERR_UNSUPPORTED, "%s: more than 16 query heads per kv head", what);
  if (n_kv_heads > 65535) return fail(DK_ERR_INVALID_ARGUMENT, "%s: too many kv heads", what);
  if (n_rows == 0) return DK_OK;
  if (!q || !k || !v || !out) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  if (pg) {
    if (!pg->table || pg->page <= 0 || pg->page % dk::attn::kBlock || pg->blocks_per_seq <= 0 ||
        pg->n_blocks <= 0 || pg->n_blocks > 0x7fffffffLL || pg->table_stride < pg->blocks_per_seq)
      return fail(DK_ERR_INVALID_ARGUMENT,
                  "%s: paged KV needs a block table, page_size a multiple of %d, blocks_per_seq > 0, "
                  "n_blocks > 0 and block_table_stride >= blocks_per_seq", what, dk::attn::kBlock);
    kv_capacity = static_cast<int64_t>(pg->page) * pg->blocks_per_seq;
  }
  if (max_kv_len < 0 || kv_capacity <= 0 || kv_n_seq <= 0 || kv_capacity > 0x7fffffffLL || kv_n_seq > 0x7fffffffLL)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad KV extents", what);
  if (!kv_lens && (uniform_kv_len < 0 || uniform_kv_len > max_kv_len || uniform_kv_len > kv_capacity))
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: uniform_kv_len out of range", what);
  if (!row_tiles) {
    n_tiles = n_rows;
    if (kv_n_seq < n_rows) return fail(DK_ERR_INVALID_ARGUMENT, "%s: fewer KV sequences than rows", what);
  } else if (n_tiles <= 0) {
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: n_tiles must be positive with row_tiles", what);
  }
  if (!aligned16(k) || !aligned16(v)) return fail(DK_ERR_INVALID_ARGUMENT, "%s: K/V must be 16-byte aligned", what);
  if ((kv_stride_tok * 2) % 16 || (kv_stride_head * 2) % 16 || (kv_stride_seq * 2) % 16)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: KV strides must be multiples of 8 elements", what);
  if ((reinterpret_cast<uintptr_t>(q) & 3u) || (q_stride_row & 1) || (q_stride_head & 1))
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: q rows must be 4-byte aligned", what);

  const AttnPlan pl = plan_attention(n_tiles, row_tiles ? 2 : 1, n_q_heads, n_kv_heads, head_dim, max_kv_len);
  if (static_cast<int64_t>(pl.n_tiles) * pl.upt > 0x7fffffffLL)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: grid too large", what);
  if (pl.total > 0 && (!workspace || workspace_bytes < pl.total))
    return fail(DK_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", what, pl.total, workspace_bytes);
  if (pl.total > 0 && !aligned16(workspace)) return fail(DK_ERR_WORKSPACE, "%s: workspace alignment", what);

  dk::attn::Params p{};
  p.q = q;
  p.q_sr = q_stride_row;
  p.q_sh = q_stride_head;
  p.out = out;
  p.o_sr = out_stride_row;
  p.o_sh = out_stride_head;
  p.kv_lens = kv_lens;
  p.uniform_len = uniform_kv_len;
  p.tiles = row_tiles;
  p.n_tiles = n_tiles;
  p.rows_cap = pl.rows_cap;
  p.n_rows = n_rows;
  p.hq = n_q_heads;
  p.hkv = n_kv_heads;
  p.G = G;
  p.max_splits = pl.max_splits;
  p.spu = pl.spu;
  p.upt = pl.upt;
  p.kv_capacity = static_cast<int32_t>(kv_capacity);
  p.kv_n_seq = static_cast<int32_t>(kv_n_seq);
  if (pg) {
    p.block_table = pg->table;
    p.bt_stride = pg->table_stride;
    p.page = pg->page;
    p.n_blocks = static_cast<int32_t>(pg->n_blocks);
  }
  p.scale_log2 = scale * 1.4426950408889634f;
  if (pl.total > 0) {
    if (static_cast<int64_t>(n_tiles) * n_kv_heads > kMaxCounters)
      return fail(DK_ERR_INVALID_ARGUMENT, "%s: %d tiles x %d kv heads exceed the workspace counter area", what,
                  n_tiles, n_kv_heads);
    uint8_t* w = ws_data(workspace);
    p.ws_o = reinterpret_cast<float*>(w);
    p.ws_ml = reinterpret_cast<float*>(w + pl.o_bytes);
    p.counters = static_cast<int32_t*>(workspace);
  }

  // K/V tensor maps: 4-D (d, token, kv head, sequence) -- or (d, token in block, kv head, block);
  // 64-token boxes for whole blocks, 16-token boxes for the tail of a split
  dk::attn::KvMaps maps;
  const int boxd = head_dim < 64 ? head_dim : 64;
  const uint64_t dims[4] = {static_cast<uint64_t>(head_dim), static_cast<uint64_t>(pg ? pg->page : kv_capacity),
                            static_cast<uint64_t>(n_kv_heads), static_cast<uint64_t>(pg ? pg->n_blocks : kv_n_seq)};
  const uint64_t strides[3] = {static_cast<uint64_t>(kv_stride_tok) * 2, static_cast<uint64_t>(kv_stride_head) * 2,
                               static_cast<uint64_t>(kv_stride_seq) * 2};
  const uint32_t box[4] = {static_cast<uint32_t>(boxd), static_cast<uint32_t>(dk::attn::kBlock), 1, 1};
  const CUtensorMapSwizzle swz = (boxd == 64) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapDataType dt = (dtype == DK_BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint32_t box16[4] = {static_cast<uint32_t>(boxd), static_cast<uint32_t>(dk::attn::kTailRows), 1, 1};
  int rc = encode_map(&maps.k, dt, 4, k, dims, strides, box, swz, what);
  if (!rc) rc = encode_map(&maps.v, dt, 4, v, dims, strides, box, swz, what);
  if (!rc) rc = encode_map(&maps.k16, dt, 4, k, dims, strides, box16, swz, what);
  if (!rc) rc = encode_map(&maps.v16, dt, 4, v, dims, strides, box16, swz, what);
  if (rc) return rc;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n_items = static_cast<int64_t>(pl.n_tiles) * pl.upt * n_kv_heads;
  if (dtype == DK_BF16) {
    if (head_dim == 32) return attn_launch<__nv_bfloat16, 32>(maps, p, n_items, st);
    if (head_dim == 64) return attn_launch<__nv_bfloat16, 64>(maps, p, n_items, st);
    return attn_launch<__nv_bfloat16, 128>(maps, p, n_items, st);
  }
  if (head_dim == 32) return attn_launch<__half, 32>(maps, p, n_items, st);
  if (head_dim == 64) return attn_launch<__half, 64>(maps, p, n_items, st);
  return attn_launch<__half, 128>(maps, p, n_items, st);
}

}  // namespace

extern "C" {

int dk_attention_batch_invariant(const void* q, int64_t q_stride_row, int64_t q_stride_head, const void* k,
                                 const void* v, int64_t kv_stride_seq, int64_t kv_stride_head, int64_t kv_stride_tok,
                                 int64_t kv_n_seq, int64_t kv_capacity, void* out, int64_t out_stride_row,
                                 int64_t out_stride_head, const int32_t* kv_lens, int32_t uniform_kv_len,
                                 const int32_t* row_tiles, int32_t n_tiles, int32_t n_rows, int32_t n_q_heads,
                                 int32_t n_kv_heads, int32_t head_dim, int32_t max_kv_len, float scale, int dtype,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  return attention_invariant_impl(q, q_stride_row, q_stride_head, k, v, kv_stride_seq, kv_stride_head,
                                  kv_stride_tok, kv_n_seq, kv_capacity, out, out_stride_row, out_stride_head,
                                  kv_lens, uniform_kv_len, row_tiles, n_tiles, n_rows, n_q_heads, n_kv_heads,
                                  head_dim, max_kv_len, scale, dtype, workspace, workspace_bytes, stream, nullptr,
                                  "attention_batch_invariant");
}

int dk_attention_paged_batch_invariant(const void* q, int64_t q_stride_row, int64_t q_stride_head,
                                       const void* k_pool, const void* v_pool, int64_t pool_stride_block,
                                       int64_t pool_stride_head, int64_t pool_stride_tok, int64_t n_blocks,
                                       int32_t page_size, const int32_t* block_table, int64_t block_table_stride,
                                       int64_t kv_n_seq, int32_t blocks_per_seq, void* out, int64_t out_stride_row,
                                       int64_t out_stride_head, const int32_t* kv_lens, int32_t uniform_kv_len,
                                       const int32_t* row_tiles, int32_t n_tiles, int32_t n_rows,
                                       int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_kv_len,
                                       float scale, int dtype, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  const PagedKV pg{block_table, block_table_stride, page_size, blocks_per_seq, n_blocks};
  return attention_invariant_impl(q, q_stride_row, q_stride_head, k_pool, v_pool, pool_stride_block,
                                  pool_stride_head, pool_stride_tok, kv_n_seq, 0, out, out_stride_row,
                                  out_stride_head, kv_lens, uniform_kv_len, row_tiles, n_tiles, n_rows, n_q_heads,
                                  n_kv_heads, head_dim, max_kv_len, scale, dtype, workspace, workspace_bytes, stream,
                                  &pg, "attention_paged_batch_invariant");
}

size_t dk_attention_variant_workspace_size(int32_t batch, int32_t n_heads, int32_t head_dim) {
  if (batch <= 0 || n_heads <= 0 || head_dim <= 0) return 0;
  const int64_t bh = static_cast<int64_t>(batch) * n_heads;
  return kCounterBytes + static_cast<size_t>((2 * bh + bh * head_dim) * sizeof(float));
}

int dk_attention_batch_variant(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k, const void* v,
                               int64_t kv_stride_b, int64_t kv_stride_h, int64_t kv_stride_s, void* out,
                               int64_t out_stride_b, int64_t out_stride_h, int32_t batch, int32_t n_heads,
                               int32_t seq_len, int32_t head_dim, float scale, int32_t split_s, int dtype,
                               void* workspace, size_t workspace_bytes, void* stream) {
  const char* what = "attention_batch_variant";
  if (dtype != DK_BF16 && dtype != DK_F16 && dtype != DK_F32) return fail(DK_ERR_UNSUPPORTED, "%s: bad dtype", what);
  if (batch < 0 || n_heads <= 0 || seq_len <= 0 || head_dim <= 0 || split_s < 1 || batch > 0x7fffffff ||
      n_heads > 65535 || split_s > 65535)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad shape", what);
  if (batch == 0) return DK_OK;
  if (!q || !k || !v || !out) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  const size_t need = dk_attention_variant_workspace_size(batch, n_heads, head_dim);
  if (!workspace || workspace_bytes < need) return fail(DK_ERR_WORKSPACE, "%s: workspace too small", what);
  dk::attn_var::Params p{};
  p.q = q;
  p.q_sb = q_stride_b;
  p.q_sh = q_stride_h;
  p.k = k;
  p.v = v;
  p.kv_sb = kv_stride_b;
  p.kv_sh = kv_stride_h;
  p.kv_ss = kv_stride_s;
  p.out = out;
  p.o_sb = out_stride_b;
  p.o_sh = out_stride_h;
  p.B = batch;
  p.H = n_heads;
  p.S = seq_len;
  p.D = head_dim;
  p.n_splits = split_s;
  p.scale = scale;
  const int64_t bh = static_cast<int64_t>(batch) * n_heads;
  p.m = reinterpret_cast<float*>(ws_data(workspace));
  p.l = p.m + bh;
  p.acc = p.l + bh;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int init_blocks = static_cast<int>(ceil_div(bh * head_dim, 256) < 4096 ? ceil_div(bh * head_dim, 256) : 4096);
  dk::attn_var::var_init_kernel<<<init_blocks, 256, 0, st>>>(p.m, p.l, p.acc, bh, bh * head_dim);
  const dim3 grid(batch, n_heads, split_s);
  const size_t shm = sizeof(float) * (dk::attn_var::kThreads / 32) * head_dim;
  if (shm > 48 * 1024) return fail(DK_ERR_UNSUPPORTED, "%s: head_dim too large", what);
  const int fin_blocks = init_blocks;
#define DK_VAR_LAUNCH(T)                                                                    \
  dk::attn_var::var_max_kernel<T><<<grid, dk::attn_var::kThreads, 0, st>>>(p);              \
  dk::attn_var::var_sumacc_kernel<T><<<grid, dk::attn_var::kThreads, shm, st>>>(p);         \
  dk::attn_var::var_finalize_kernel<T><<<fin_blocks, 256, 0, st>>>(p);
  if (dtype == DK_BF16) {
    DK_VAR_LAUNCH(__nv_bfloat16)
  } else if (dtype == DK_F16) {
    DK_VAR_LAUNCH(__half)
  } else {
    DK_VAR_LAUNCH(float)
  }
#undef DK_VAR_LAUNCH
  return check_launch(what);
}

// ---------------------------------------------------------------------------------------------
// Decode attention without a caller workspace.  Its scratch is a fixed-size array in device
// global memory owned by this library image: each GPU that loads the library holds it until
// the process exits.  In host code the array's name is only a host-side placeholder, so its
// device address is looked up once per device with cudaGetSymbolAddress and cached.
// ---------------------------------------------------------------------------------------------
size_t dk_attention_noalloc_scratch_limit(void) { return kNoAllocScratchBytes; }

// Test hook, deliberately absent from the public header: which kernel runs invariant matmuls
// (low 4 bits: 0 = the planner's choice, 1 = one-CTA kernel, 2 = CTA-pair kernel, 3 = wide CTA-pair
// kernel; bits 4 and up: slices per work unit, 0 = the planner's choice, else 1, 2, 4 or 8), so a
// test can compare the schedules' bits on the same shapes.  Returns the previous setting.
int dk_matmul_pair_schedule_for_test(int mode) {
  const int prev = g_pair_override | (g_group_override << 4);
  const int kernel = mode & 15, group = mode >> 4;
  if (kernel <= 3 && (group == 0 || group == 1 || group == 2 || group == 4 || group == 8)) {
    g_pair_override = kernel;
    g_group_override = group;
  }
  return prev;
}

// Test hook, deliberately absent from the public header: which kernel runs chunked bf16 GDN with
// head dim 128 (0 = the tcgen05 kernel, 1 = the mma.sync kernel).  Returns the previous setting.
int dk_gdn_kernel_for_test(int mode) {
  const int prev = g_gdn_override;
  if (mode == 0 || mode == 1) g_gdn_override = mode;
  return prev;
}

// Test hook, deliberately absent from the public header: writes `value` into the first `bytes`
// bytes of the no-alloc scratch on the current device (synchronously), so a test can show that
// the next no-alloc call clears the arrival counters it relies on.
int dk_noalloc_scratch_fill_for_test(int value, size_t bytes) {
  if (bytes > kNoAllocScratchBytes) return fail(DK_ERR_INVALID_ARGUMENT, "fill beyond the no-alloc scratch");
  void* p = nullptr;
  int rc = noalloc_scratch(&p, "dk_noalloc_scratch_fill_for_test");
  if (rc) return rc;
  cudaError_t e = cudaMemset(p, value & 0xff, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(DK_ERR_CUDA, "dk_noalloc_scratch_fill_for_test: %s", cudaGetErrorString(e));
  return DK_OK;
}

int dk_attention_batch_invariant_noalloc(const void* q, int64_t q_stride_row, int64_t q_stride_head, const void* k,
                                         const void* v, int64_t kv_stride_seq, int64_t kv_stride_head,
                                         int64_t kv_stride_tok, int64_t kv_n_seq, int64_t kv_capacity, void* out,
                                         int64_t out_stride_row, int64_t out_stride_head, const int32_t* kv_lens,
                                         int32_t uniform_kv_len, const int32_t* row_tiles, int32_t n_tiles,
                                         int32_t n_rows, int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                         int32_t max_kv_len, float scale, int dtype, void* stream) {
  const char* what = "attention_batch_invariant_noalloc";
  const int32_t tiles = row_tiles ? n_tiles : n_rows;
  const size_t need = dk_attention_workspace_size(tiles, row_tiles ? 2 : 1, n_q_heads, n_kv_heads, head_dim,
                                                  max_kv_len);
  if (need > kNoAllocScratchBytes)
    return fail(DK_ERR_WORKSPACE,
                "%s: this call needs %zu bytes of scratch but the built-in scratch holds %zu; use "
                "dk_attention_batch_invariant with a caller workspace (or fewer rows / a shorter max_kv_len)",
                what, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    int rc = noalloc_scratch(&scratch, what);
    if (rc) return rc;
    // The arrival counters must start at zero; the previous call on this device may have left
    // them non-zero if it stopped early.  Only the counters this call uses are cleared.
    const size_t counter_bytes = static_cast<size_t>(tiles) * static_cast<size_t>(n_kv_heads) * sizeof(int32_t);
    if (counter_bytes > kCounterBytes)
      return fail(DK_ERR_INVALID_ARGUMENT, "%s: too many tiles x kv heads for the counter area", what);
    cudaError_t e = cudaMemsetAsync(scratch, 0, counter_bytes, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(DK_ERR_CUDA, "%s: clearing counters: %s", what, cudaGetErrorString(e));
  }
  return dk_attention_batch_invariant(q, q_stride_row, q_stride_head, k, v, kv_stride_seq, kv_stride_head,
                                      kv_stride_tok, kv_n_seq, kv_capacity, out, out_stride_row, out_stride_head,
                                      kv_lens, uniform_kv_len, row_tiles, n_tiles, n_rows, n_q_heads, n_kv_heads,
                                      head_dim, max_kv_len, scale, dtype, scratch,
                                      scratch ? kNoAllocScratchBytes : 0, stream);
}

}  // extern "C"

int dk_gdn_forward(const void* q, const void* k, const void* v, const void* g, const void* beta, void* o,
                   const int64_t* cu_seqlens, int64_t n_seqs, int64_t seq_len, int n_heads, int n_v_heads,
                   int head_dim_k, int head_dim_v, int dtype, int gb_dtype, float scale, const void* initial_state,
                   int state_dtype, float* final_state, int chunk_size, void* stream) {
  const char* what = "gdn_forward";
  if (dtype != DK_BF16 && dtype != DK_F16) return fail(DK_ERR_UNSUPPORTED, "%s: q/k/v must be bf16 or f16", what);
  auto ok_dt = [](int d) { return d == DK_F32 || d == DK_BF16 || d == DK_F16; };
  if (!ok_dt(gb_dtype) || (initial_state && !ok_dt(state_dtype)))
    return fail(DK_ERR_UNSUPPORTED, "%s: g/beta and the initial state must be f32, bf16 or f16", what);
  if (n_seqs < 0 || seq_len < 0 || n_heads <= 0 || n_v_heads <= 0 || n_v_heads % n_heads)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: bad sizes (n_v_heads must be a multiple of n_heads)", what);
  if (chunk_size != 1 && chunk_size != dk::gdn::kChunk)
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: chunk_size must be 1 or %d", what, dk::gdn::kChunk);
  if (n_seqs > 65535 || n_v_heads > 65535) return fail(DK_ERR_UNSUPPORTED, "%s: too many sequences or heads", what);
  if (!(scale == scale)) return fail(DK_ERR_INVALID_ARGUMENT, "%s: scale is NaN", what);
  if (n_seqs == 0) return DK_OK;
  if (!q || !k || !v || !g || !beta || !o) return fail(DK_ERR_INVALID_ARGUMENT, "%s: null tensor", what);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v))
    return fail(DK_ERR_INVALID_ARGUMENT, "%s: q, k and v must start on a 16-byte boundary", what);
  dk::gdn::Params p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.g = g;
  p.beta = beta;
  p.o = o;
  p.cu_seqlens = cu_seqlens;
  p.seq_len = seq_len;
  p.h0 = initial_state;
  p.ht = final_state;
  p.H = n_heads;
  p.HV = n_v_heads;
  p.gb_dtype = gb_dtype;
  p.h0_dtype = state_dtype;
  p.chunk = chunk_size;
  p.scale = scale;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DK_BF16) return gdn_launch_dims<__nv_bfloat16>(p, head_dim_k, head_dim_v, n_seqs, st);
  return gdn_launch_dims<__half>(p, head_dim_k, head_dim_v, n_seqs, st);
}
