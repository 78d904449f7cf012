/*
 * detkernels_b200 -- C ABI of the batch-invariant kernel library for NVIDIA B200 (sm_100a).
 *
 * Every entry point takes raw device pointers, element strides, sizes, a CUDA
 * stream (passed as void*, i.e. a cudaStream_t) and, where the kernel needs
 * scratch space, a caller-provided device workspace.  The library never
 * allocates device memory.  Launches are asynchronous on the given stream; the
 * return value reports argument validation and launch errors only.  Errors
 * detected on the device (a bounded wait that expired, an index outside the
 * caller's buffers) are recorded in a per-device status word that
 * dk_device_status() reads and clears.
 *
 * Each compute entry point names the reference interface it replaces
 * (AdityaShome/DetKernels, Python + Triton):
 *   kernels/rmsnorm.py, kernels/matmul.py, kernels/attention.py.
 *
 * Batch invariance contract: for every entry point marked "invariant", the
 * bits written for one output row depend only on that row's inputs (and, for
 * attention, that row's own KV sequence and length) -- never on how many other
 * rows are in the call, what they contain, or which work schedule the library
 * picked for the call.
 */
#ifndef DETKERNELS_B200_H
#define DETKERNELS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define DK_OK 0
#define DK_ERR_INVALID_ARGUMENT 1 /* shape, stride, pointer or alignment rejected */
#define DK_ERR_UNSUPPORTED 2      /* dtype / head_dim / size combination not built */
#define DK_ERR_WORKSPACE 3        /* workspace missing or smaller than *_workspace_size() */
#define DK_ERR_CUDA 4             /* a CUDA runtime or driver call failed */
#define DK_ERR_DEVICE_TIMEOUT 5   /* a bounded device-side wait expired (see detail) */
#define DK_ERR_DEVICE_CHECK 6     /* a device-side index check failed (see detail) */

/* ---- workspaces ----
 * Every workspace starts with DK_WORKSPACE_COUNTER_BYTES of arrival counters shared by all entry
 * points.  Zero that area once when the workspace is created; every call leaves it zero again (after
 * a device-side error, zero it again).  Scratch data always lives after it.  Calls that may overlap
 * on the GPU (different streams) need different workspaces. */
#define DK_WORKSPACE_COUNTER_BYTES (1u << 20)

/* ---- dtype codes ---- */
#define DK_F32 0
#define DK_F16 1
#define DK_BF16 2

/* ---- fixed numerics of the invariant kernels (part of the output definition) ---- */
#define DK_MATMUL_K_SLICES 8        /* K is reduced as 8 fixed slices, summed along a fixed f32 tree */
#define DK_ATTN_KV_SPLIT 256        /* decode attention reduces KV in fixed splits of 256 tokens */
#define DK_RMSNORM_THREADS 256      /* one CTA of 256 threads per row */

/* ---- library / device queries ---- */
/* Layout version of this header's structs and signatures; dk_abi_version() of a library built from it
 * returns the same number.  2: dk_matmul_epilogue gained the DK_EPI_RESIDUAL_RMSNORM fields.
 * 3: dk_matmul_epilogue gained the paged-KV fields (block_table ... n_blocks). */
#define DK_ABI_VERSION 3
int dk_abi_version(void);
/* Message for the last non-zero return code on the calling host thread. */
const char* dk_last_error(void);
/* Reads the device status word of `device` (synchronises that device).  If
 * `clear` is non-zero the word is reset to DK_OK afterwards. */
int dk_device_status(int device, int clear, int* code, int* detail);
int dk_num_sms(int device, int* out);
/* Introspection of the compiled kernels on the current device (registers per thread, the
 * launch-time thread limit, local-memory bytes, dynamic shared-memory limit).  which: 0 = bf16
 * GEMM, 1 = bf16 decode attention d128, 2 = bf16 decode attention d64, 3 = f32 RMSNorm. */
int dk_kernel_attributes(int which, int* num_regs, int* max_threads, int* local_bytes, int* max_dynamic_smem);
/* Self-test of the device-side bounded wait that every kernel of this library uses: one CTA waits on
 * a shared-memory barrier for at most limit_ns (0 < limit_ns <= 100 ms).  A second warp arrives on it
 * unless skip_arrive is non-zero; then the wait runs out, the kernel records DK_ERR_DEVICE_TIMEOUT
 * (detail 0x7E57) in the device status word and returns -- the context stays usable.  No counterpart
 * in the reference (its Triton kernels have no bounded waits). */
int dk_test_bounded_wait(int skip_arrive, int64_t limit_ns, void* stream);

/* ---- RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w, f32 math, y in x's dtype ----
 * x, out: [n_rows, n_cols] with unit column stride and the given row strides
 * (elements).  dtype: DK_F32 / DK_F16 / DK_BF16 for x and out; weight_dtype
 * for w (any of the three). */

/* replaces kernels/rmsnorm.py:155-177 rmsnorm_batch_invariant (+ _single_block_kernel 63-89) */
int dk_rmsnorm_batch_invariant(const void* x, int64_t x_row_stride, const void* weight, void* out,
                               int64_t out_row_stride, int64_t n_rows, int64_t n_cols, int dtype,
                               int weight_dtype, float eps, void* stream);

/* Embedding lookup + invariant RMSNorm: x_out[r, :] = table[row_index[r], :] and out[r, :] =
 * dk_rmsnorm_batch_invariant(x_out[r, :]), the same bits as the lookup followed by that call, in one
 * launch.  row_index: device int64[n_rows]; an index outside [0, table_rows) sets the device status
 * (DK_ERR_DEVICE_CHECK) and leaves its row unwritten.  Any row alignment and n_cols (16-byte aligned rows
 * with n_cols a multiple of 16 bytes take the vector path).  No counterpart in the reference: it fuses the decoder's
 * `self.embed[token_ids]` (kernels/tiny_model.py:110) into the first block's input norm. */
int dk_rmsnorm_gather_batch_invariant(const void* table, int64_t table_row_stride, int64_t table_rows,
                                      const int64_t* row_index, const void* weight, void* x_out, int64_t x_row_stride,
                                      void* out, int64_t out_row_stride, int64_t n_rows, int64_t n_cols, int dtype,
                                      int wdtype, float eps, void* stream);

/* Scratch bytes dk_rmsnorm_batch_variant needs for n_rows rows. */
size_t dk_rmsnorm_variant_workspace_size(int64_t n_rows);
/* replaces kernels/rmsnorm.py:180-218 rmsnorm_batch_variant: when n_rows < split_threshold each row's
 * sum of squares is split into n_splits chunks combined with f32 atomics (order decided by the
 * scheduler: deliberately NOT batch invariant); otherwise identical to the invariant kernel. */
int dk_rmsnorm_batch_variant(const void* x, int64_t x_row_stride, const void* weight, void* out,
                             int64_t out_row_stride, int64_t n_rows, int64_t n_cols, int dtype,
                             int weight_dtype, float eps, int split_threshold, int n_splits,
                             void* workspace, size_t workspace_bytes, void* stream);

/* ---- Matmul: C[M,N] = A[M,K] @ B[K,N] (row-major, unit inner stride), f32 accumulate ----
 * dtype: DK_BF16 or DK_F16 (A, B and C share it).  Row strides (lda, ldb, ldc)
 * in elements; lda and ldb must be multiples of 8 and A, B 16-byte aligned
 * (TMA).  The invariant kernel reduces K as DK_MATMUL_K_SLICES fixed slices of
 * ceil16(K/8) elements, each accumulated by tcgen05 in ascending 16-wide K
 * steps into its own f32 TMEM accumulator (partial p_s), then summed along the
 * fixed tree ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)) and rounded to the dtype. */

/* Scratch bytes the invariant / variant matmul may need for this shape: f32 subtree sums when
 * the schedule splits K over CTAs, and for large token counts (the CTA-pair kernel) a 128 KB
 * stash per resident CTA for the left half of the slice tree.  0 means no workspace is needed. */
size_t dk_matmul_workspace_size(int64_t M, int64_t N, int64_t K);
/* replaces kernels/matmul.py:161-186 matmul_batch_invariant (+ _matmul_kernel 64-100) */
int dk_matmul_batch_invariant(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                              int64_t M, int64_t N, int64_t K, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream);
/* Same numerics for one aligned group of slices [slice_begin, slice_end) (1, 2, 4 or 8 slices,
 * slice_begin a multiple of the group size): writes that group's subtree sum to partial[m * N + n]
 * (f32).  Row-parallel tensor parallelism: rank r of a TP-way split computes group r. */
int dk_matmul_slice_partials(const void* a, int64_t lda, const void* b, int64_t ldb, float* partial,
                             int64_t M, int64_t N, int64_t K, int slice_begin, int slice_end, int dtype,
                             void* stream);
/* Row-parallel tensor parallelism on K shards.  dk_matmul_shard_range gives the K range [k_begin,
 * k_end) of the full K that an aligned slice group [slice_begin, slice_end) covers; a rank holding only
 * that range -- a: [M, k_end - k_begin] (its columns of A), b: [k_end - k_begin, N] (its rows of B) --
 * calls dk_matmul_shard_partials with the FULL K to get the group's f32 subtree sum, bit-identical to
 * dk_matmul_slice_partials on the unsharded operands.  No counterpart in the reference (its matmul has
 * no tensor parallelism, kernels/matmul.py:161-186). */
void dk_matmul_shard_range(int64_t K, int slice_begin, int slice_end, int64_t* k_begin, int64_t* k_end);
int dk_matmul_shard_partials(const void* a, int64_t lda, const void* b, int64_t ldb, float* partial, int64_t M,
                             int64_t N, int64_t K, int slice_begin, int slice_end, int dtype, void* stream);
/* out[m,n] = the upper tree levels over n_parts (1, 2, 4 or 8) subtree sums in group order,
 * partials[j * M * N + m * N + n], rounded to dtype: reproduces dk_matmul_batch_invariant bit for bit. */
int dk_matmul_fold_slices(const float* partials, int n_parts, void* c, int64_t ldc, int64_t M, int64_t N,
                          int dtype, void* stream);
/* Scratch bytes dk_matmul_batch_variant needs on its split-K path. */
size_t dk_matmul_variant_workspace_size(int64_t M, int64_t N);
/* replaces kernels/matmul.py:189-228 matmul_batch_variant: when M < split_m_threshold, K is split
 * into split_k chunks whose f32 partials are combined with atomics (deliberately NOT batch
 * invariant); otherwise the invariant kernel runs. */
int dk_matmul_batch_variant(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                            int64_t M, int64_t N, int64_t K, int dtype, int split_m_threshold, int split_k,
                            void* workspace, size_t workspace_bytes, void* stream);

/* ---- Matmul with a fused epilogue ----
 * What happens to each output element's f32 tree sum v(m, n) before it is stored.  Every step rounds
 * exactly where the unfused torch ops of a decoder block round (matmul output, residual add, SiLU,
 * product), so a fused call returns the bits of the unfused sequence. */
#define DK_EPI_STORE 0     /* C[m,n] = round(v) */
#define DK_EPI_RESIDUAL 1  /* C[m,n] = round(R[m,n] + round(v)); R may be C itself */
#define DK_EPI_SILU 2      /* C[m,n] = round(silu(round(v))), silu(x) = x / (1 + exp(-x)) */
#define DK_EPI_SILU_MUL 3  /* B's columns hold gate/up pairs (2j, 2j+1); C is [M, N/2]:
                              C[m,j] = round(round(silu(round(v(m,2j)))) * round(v(m,2j+1))) */
#define DK_EPI_QKV_CACHE 4 /* columns [0, q_cols) -> C[m, n]; the next kv_cols -> K cache, the next kv_cols ->
                              V cache, at (row_seq[m], n' / head_dim, row_pos[m], n' % head_dim) */
#define DK_EPI_ARGMAX 5    /* per row, the first column holding the largest round(v) (NaN above all, -0 == +0),
                              torch.argmax's answer, folded into argmax_keys[m] with 64-bit atomicMax of
                              (ordered value << 32 | ~n): order-free, so deterministic.  C is optional
                              (NULL: logits are not stored).  argmax_keys must be 0 before the call;
                              dk_argmax_finish reads and re-zeroes them. */
#define DK_EPI_RESIDUAL_RMSNORM 6 /* C = round(R + round(v)) as DK_EPI_RESIDUAL, then norm_out[m, :] =
                                 * dk_rmsnorm_batch_invariant(C[m, :], norm_w, eps): the same bits as the two
                                 * calls, with the norm computed while C is folded (one launch fewer) */
typedef struct dk_matmul_epilogue {
  int mode;
  const void* resid;       /* DK_EPI_RESIDUAL: R, same dtype as C */
  int64_t ld_resid;
  int32_t q_cols, kv_cols, head_dim;  /* DK_EPI_QKV_CACHE */
  void* k_cache;
  void* v_cache;
  int64_t cache_stride_seq, cache_stride_head, cache_stride_tok;  /* elements; unit stride along d */
  const int32_t* row_seq;  /* device int32[M]; NULL: row m writes cache sequence m */
  const int32_t* row_pos;  /* device int32[M]: token position written by row m */
  unsigned long long* argmax_keys;  /* DK_EPI_ARGMAX: device uint64[M] */
  const void* norm_w;      /* DK_EPI_RESIDUAL_RMSNORM: weight [N] of norm_w_dtype */
  int norm_w_dtype;
  void* norm_out;          /* [M, N] rows norm_ld apart, dtype of C */
  int64_t norm_ld;
  float norm_eps;
  /* DK_EPI_QKV_CACHE into a paged cache (block_table non-NULL): k_cache / v_cache are block pools
   * [n_blocks, heads, page_size, head_dim] (cache_stride_seq = the block stride), and position pos of
   * sequence s goes to block block_table[s * block_table_stride + pos / page_size], token pos %
   * page_size.  A position past blocks_per_seq blocks or an entry outside [0, n_blocks) is recorded as
   * DK_ERR_DEVICE_CHECK and not stored. */
  const int32_t* block_table;
  int64_t block_table_stride;
  int32_t page_size;
  int32_t blocks_per_seq;
  int64_t n_blocks;
} dk_matmul_epilogue;

/* dk_matmul_batch_invariant followed by the epilogue `epi` (same K numerics; NULL epi = DK_EPI_STORE).
 * No counterpart in the reference: it fuses the reference decoder's element-wise torch ops
 * (tiny_model.py:110-139) into the matmul that produces their input. */
int dk_matmul_batch_invariant_ex(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                                 int64_t M, int64_t N, int64_t K, int dtype, const dk_matmul_epilogue* epi,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* End of a greedy decode step after a DK_EPI_ARGMAX matmul, one thread per row: tokens[r] = the row's
 * argmax column (also into tokens_copy[r] when non-NULL), keys[r] = 0, and lens_a[r] += 1,
 * lens_b[r] += 1 for the non-NULL ones.  No counterpart in the reference: it replaces the
 * `logits.argmax(-1)` and cache-length bookkeeping of tiny_model.py:150-157. */
int dk_argmax_finish(unsigned long long* keys, int64_t n_rows, int64_t* tokens, int64_t* tokens_copy,
                     int32_t* lens_a, int32_t* lens_b, void* stream);

/* ---- Tensor-parallel decoder layers (no counterpart in the reference: its TinyModel runs on one
 * device, kernels/tiny_model.py:99-140) ---- */
/* Row-parallel layer output: the fold of dk_matmul_fold_slices (n_parts = 1, 2, 4 or 8 subtree sums in
 * group order, partials[j * M * N + m * N + n]) followed by the epilogue `epi` exactly as
 * dk_matmul_batch_invariant_ex applies it (DK_EPI_STORE, _RESIDUAL, _RESIDUAL_RMSNORM, _SILU, _SILU_MUL
 * or _ARGMAX; NULL = DK_EPI_STORE), so a layer split over ranks returns the one-GPU fused bits. */
int dk_matmul_fold_slices_ex(const float* partials, int n_parts, void* c, int64_t ldc, int64_t M, int64_t N,
                             int dtype, const dk_matmul_epilogue* epi, void* stream);
/* Greedy step end for a column-parallel LM head: keys[p * part_stride + r] (p < n_parts <= 8) are part
 * p's DK_EPI_ARGMAX keys over its own columns, which start at column col_offsets[p] (host array) of the
 * full vocabulary.  tokens[r] = the global argmax (largest value, then smallest column: the one-GPU
 * answer); then as dk_argmax_finish, with reset_keys[r] = 0 for the caller's local key buffer (optional). */
int dk_argmax_finish_parts(const unsigned long long* keys, int n_parts, int64_t part_stride,
                           const int64_t* col_offsets, int64_t n_rows, int64_t* tokens, int64_t* tokens_copy,
                           int32_t* lens_a, int32_t* lens_b, unsigned long long* reset_keys, void* stream);

/* ---- Decode attention (one query per row, split-KV with a fixed split size) ----
 * q:   [n_rows, n_q_heads, head_dim], strides (q_stride_row, q_stride_head), unit d stride.
 * k,v: KV cache viewed as [kv_n_seq, n_kv_heads, kv_capacity, head_dim] with element strides
 *      (kv_stride_seq, kv_stride_head, kv_stride_tok), unit d stride; k and v share strides.
 * out: [n_rows, n_q_heads, head_dim], strides (out_stride_row, out_stride_head).
 * Row r attends to tokens [0, kv_len_r) of KV sequence seq_r, q head h uses kv head
 * h / (n_q_heads / n_kv_heads).  kv_lens (device int32[n_rows]) may be NULL, then every row
 * uses uniform_kv_len.  row_tiles (device int32[3 * n_tiles]: first row, row count, seq) groups
 * consecutive rows that read the same KV sequence (at most 16 / group rows per tile); when NULL,
 * row r is its own tile reading sequence r.  max_kv_len bounds every kv_len_r (sizes the grid).
 * head_dim in {32, 64, 128}; dtype DK_BF16 or DK_F16; scale multiplies q.k. */
/* Scratch bytes for a call with n_tiles tiles (n_rows when row_tiles is NULL) of up to rows_per_tile rows
 * (1 without row_tiles); 0 when no row needs more than one split. */
size_t dk_attention_workspace_size(int32_t n_tiles, int32_t rows_per_tile, int32_t n_q_heads, int32_t n_kv_heads,
                                   int32_t head_dim, int32_t max_kv_len);
/* replaces kernels/attention.py:289-298 attention_batch_invariant (+ _attn_direct_kernel 86-143,
 * _run_direct 266-286), extended with GQA, per-row KV lengths and row tiles */
int dk_attention_batch_invariant(const void* q, int64_t q_stride_row, int64_t q_stride_head, const void* k,
                                 const void* v, int64_t kv_stride_seq, int64_t kv_stride_head,
                                 int64_t kv_stride_tok, int64_t kv_n_seq, int64_t kv_capacity, void* out,
                                 int64_t out_stride_row, int64_t out_stride_head, const int32_t* kv_lens,
                                 int32_t uniform_kv_len, const int32_t* row_tiles, int32_t n_tiles,
                                 int32_t n_rows, int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                 int32_t max_kv_len, float scale, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Decode attention over a paged KV cache: the arithmetic, arguments and bits of
 * dk_attention_batch_invariant, with the K/V cache given as block pools k_pool / v_pool
 * [n_blocks, n_kv_heads, page_size, head_dim] (element strides pool_stride_block, pool_stride_head,
 * pool_stride_tok; unit d stride) and a block table: token t of KV sequence s is token t % page_size
 * of block block_table[s * block_table_stride + t / page_size] (device int32 [kv_n_seq][...], at least
 * blocks_per_seq entries per row).  page_size must be a multiple of 64; kv lengths may reach
 * blocks_per_seq * page_size.  A table entry outside [0, n_blocks) is recorded as DK_ERR_DEVICE_CHECK
 * (detail 0x212).  Workspace as dk_attention_workspace_size.  No counterpart in the reference: its
 * cache is one contiguous tensor grown by torch.cat (kernels/tiny_model.py:119-125) and it lists
 * paging as a simplification (kernels/attention.py:35-40). */
int dk_attention_paged_batch_invariant(const void* q, int64_t q_stride_row, int64_t q_stride_head,
                                       const void* k_pool, const void* v_pool, int64_t pool_stride_block,
                                       int64_t pool_stride_head, int64_t pool_stride_tok, int64_t n_blocks,
                                       int32_t page_size, const int32_t* block_table, int64_t block_table_stride,
                                       int64_t kv_n_seq, int32_t blocks_per_seq, void* out, int64_t out_stride_row,
                                       int64_t out_stride_head, const int32_t* kv_lens, int32_t uniform_kv_len,
                                       const int32_t* row_tiles, int32_t n_tiles, int32_t n_rows,
                                       int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim, int32_t max_kv_len,
                                       float scale, int dtype, void* workspace, size_t workspace_bytes,
                                       void* stream);

/* Scratch bytes dk_attention_batch_variant needs. */
size_t dk_attention_variant_workspace_size(int32_t batch, int32_t n_heads, int32_t head_dim);
/* replaces kernels/attention.py:145-249 (_attn_split_max_kernel, _attn_split_sumacc_kernel) as dispatched by
 * attention_batch_variant (attention.py:301-348): q [batch, n_heads, head_dim], k/v [batch, n_heads, seq_len,
 * head_dim] (unit d stride), KV cut into split_s chunks combined with f32 atomics -- deliberately NOT
 * batch invariant.  dtype DK_F32 / DK_F16 / DK_BF16. */
int dk_attention_batch_variant(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k, const void* v,
                               int64_t kv_stride_b, int64_t kv_stride_h, int64_t kv_stride_s, void* out,
                               int64_t out_stride_b, int64_t out_stride_h, int32_t batch, int32_t n_heads,
                               int32_t seq_len, int32_t head_dim, float scale, int32_t split_s, int dtype,
                               void* workspace, size_t workspace_bytes, void* stream);

/* ---- decode attention for callers that cannot allocate device memory ----
 * No counterpart in the reference.  Some callers cannot hand this library a workspace: code that
 * runs inside another runtime's allocator or memory-pool callbacks, plugins whose host owns every
 * device allocation, or paths where a cudaMalloc would synchronise the device at the wrong time.
 * This entry point takes the same arguments as dk_attention_batch_invariant minus the workspace,
 * and produces the same bits.  Its scratch is a 32 MiB array in device memory that belongs to the
 * library (dk_attention_noalloc_scratch_limit() returns the size): every GPU that loads the library
 * keeps it until the process exits.  Calls whose multi-split scratch would exceed it are rejected
 * with DK_ERR_WORKSPACE.  It never allocates: the first call on a device looks up the array's
 * device address with that device current (cudaGetSymbolAddress) and caches it, so make that first
 * call before any stream capture on the device.  Each call clears the arrival counters it uses on
 * `stream`.  All calls share the one array, so calls on one device that may overlap on the GPU (for
 * example on different streams without ordering) race and give wrong results; order them. */
size_t dk_attention_noalloc_scratch_limit(void);
int dk_attention_batch_invariant_noalloc(const void* q, int64_t q_stride_row, int64_t q_stride_head, const void* k,
                                         const void* v, int64_t kv_stride_seq, int64_t kv_stride_head,
                                         int64_t kv_stride_tok, int64_t kv_n_seq, int64_t kv_capacity, void* out,
                                         int64_t out_stride_row, int64_t out_stride_head, const int32_t* kv_lens,
                                         int32_t uniform_kv_len, const int32_t* row_tiles, int32_t n_tiles,
                                         int32_t n_rows, int32_t n_q_heads, int32_t n_kv_heads, int32_t head_dim,
                                         int32_t max_kv_len, float scale, int dtype, void* stream);

/* ---- Gated delta rule (Gated DeltaNet linear attention), forward ----
 * replaces the FLA `chunk_gated_delta_rule` / `fused_recurrent_gated_delta_rule` calls of the
 * reference's gdn/repro.py:76,161-162,293-294 (fla 0.5.1 API, [B, T, heads, dim] layout).
 * q, k: [tokens, n_heads, head_dim_k]; v: [tokens, n_v_heads, head_dim_v]; g (log decay), beta:
 * [tokens, n_v_heads]; o: [tokens, n_v_heads, head_dim_v] in q's dtype, all contiguous, q/k/v
 * starting on a 16-byte boundary.  Value head j
 * uses query/key head j / (n_v_heads / n_heads).  Sequences: cu_seqlens (device int64[n_seqs + 1])
 * with seq_len = the packed length T of q/k/v/g/beta/o (a sequence whose pair falls outside [0, T] or
 * decreases is skipped and recorded as DK_ERR_DEVICE_CHECK, detail 0x500), or, when cu_seqlens is
 * NULL, n_seqs rows of seq_len tokens each.  initial_state / final_state: [n_seqs,
 * n_v_heads, head_dim_k, head_dim_v] (final in f32), either may be NULL.  chunk_size 64 computes
 * 64-token chunks from each sequence's start (chunked form); 1 steps token by token in the order of
 * the recurrence (decode path; FLA's fused_recurrent_gated_delta_rule).  A sequence's
 * result never depends on the other sequences of the call.  Head dims: 32/32, 64/64, 128/128. */
int dk_gdn_forward(const void* q, const void* k, const void* v, const void* g, const void* beta, void* o,
                   const int64_t* cu_seqlens, int64_t n_seqs, int64_t seq_len, int n_heads, int n_v_heads,
                   int head_dim_k, int head_dim_v, int dtype, int gb_dtype, float scale, const void* initial_state,
                   int state_dtype, float* final_state, int chunk_size, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DETKERNELS_B200_H */
