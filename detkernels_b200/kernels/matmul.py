"""Batch-invariant matmul on B200 tensor cores, and its deliberately batch-variant twin.

Drop-in for the reference's ``kernels/matmul.py``:

* ``matmul_reference`` (matmul.py:42-49): f32 ``a @ b`` cast back to a's dtype.
* ``matmul_batch_invariant`` (matmul.py:161-186): tcgen05/TMEM GEMM fed by
  TMA with one tile shape for every M and K reduced as 8 fixed slices folded
  along a fixed tree -- a row's bits never depend on M.  ``block_m/n/k`` are
  accepted for signature compatibility; the tile shape is fixed.
* ``matmul_batch_variant`` (matmul.py:189-228): split-K with f32 atomics when
  ``M < split_m_threshold``.

The 8 K-slice partials are summed along the fixed tree
((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)).  Extensions used by tensor parallelism:
``matmul_slice_partials`` (f32 subtree sum of one aligned group of slices) and
``matmul_fold_slices`` (the upper tree levels over the groups' sums), which
together reproduce ``matmul_batch_invariant`` bit for bit.

A and B must be bf16 or f16 (same dtype); the output has a's dtype.
"""
from __future__ import annotations

from detkernels_b200 import _lib

K_SLICES = _lib.MATMUL_K_SLICES


def matmul_reference(a, b):
    """Plain PyTorch eager matmul, float32 accumulation (reference matmul.py:42-49)."""
    import torch

    orig_dtype = a.dtype
    out = a.to(torch.float32) @ b.to(torch.float32)
    return out.to(orig_dtype)


def _tma_ready(t):
    """Return t, or a copy whose rows are 16-byte aligned (unit inner stride,
    row stride a multiple of 8 elements) as TMA requires.  Values are unchanged,
    so the result bits are unchanged."""
    import torch

    rows, cols = t.shape
    if t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.stride(0) >= cols and t.data_ptr() % 16 == 0:
        return t
    ld = (cols + 7) // 8 * 8
    buf = torch.zeros((rows, ld), dtype=t.dtype, device=t.device)
    buf[:, :cols].copy_(t)
    return buf[:, :cols]


def _check_inputs(a, b, name):
    assert a.is_cuda and b.is_cuda, "%s requires CUDA tensors" % name
    assert a.dim() == 2 and b.dim() == 2, "%s expects 2-D operands" % name
    M, K = a.shape
    K2, N = b.shape
    assert K == K2, f"inner dims must match, got {K} and {K2}"
    if a.dtype != b.dtype:
        raise TypeError("%s: a and b must share a dtype, got %s and %s" % (name, a.dtype, b.dtype))
    _lib.dtype_code(a.dtype)
    return M, K, N


def matmul_batch_invariant(a, b, block_m: int = 64, block_n: int = 64, block_k: int = 32):
    """Batch-invariant matmul: fixed tile shape, fixed 8-slice K reduction."""
    import torch

    M, K, N = _check_inputs(a, b, "matmul_batch_invariant")
    c = torch.empty((M, N), device=a.device, dtype=a.dtype)
    if M == 0 or N == 0:
        return c
    a2, b2 = _tma_ready(a), _tma_ready(b)
    lib = _lib.load()
    stream = _lib.stream_ptr(a.device)
    nbytes = lib.dk_matmul_workspace_size(M, N, K)
    ws = _lib.workspace(nbytes, a.device, stream)
    rc = lib.dk_matmul_batch_invariant(
        a2.data_ptr(), a2.stride(0), b2.data_ptr(), b2.stride(0), c.data_ptr(), c.stride(0), M, N, K,
        _lib.dtype_code(a.dtype), ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        stream)
    _lib.check(rc, "matmul_batch_invariant")
    _lib.count_launch()
    return c


def matmul_batch_variant(a, b, split_m_threshold: int = 64, split_k: int = 4,
                         block_m: int = 64, block_n: int = 64, block_k: int = 32):
    """Deliberately batch-variant matmul: split-K with f32 atomics when M < split_m_threshold."""
    import torch

    M, K, N = _check_inputs(a, b, "matmul_batch_variant")
    c = torch.empty((M, N), device=a.device, dtype=a.dtype)
    if M == 0 or N == 0:
        return c
    a2, b2 = _tma_ready(a), _tma_ready(b)
    lib = _lib.load()
    stream = _lib.stream_ptr(a.device)
    if M >= split_m_threshold:
        nbytes = lib.dk_matmul_workspace_size(M, N, K)
    else:
        nbytes = lib.dk_matmul_variant_workspace_size(M, N)
    ws = _lib.workspace(nbytes, a.device, stream)
    rc = lib.dk_matmul_batch_variant(
        a2.data_ptr(), a2.stride(0), b2.data_ptr(), b2.stride(0), c.data_ptr(), c.stride(0), M, N, K,
        _lib.dtype_code(a.dtype), int(split_m_threshold), int(split_k),
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, stream)
    _lib.check(rc, "matmul_batch_variant")
    return c


def matmul_slice_partials(a, b, slice_begin: int, slice_end: int, out=None):
    """f32 [M, N] subtree sum of the aligned slice group [slice_begin, slice_end)
    (1, 2, 4 or 8 of the 8 K slices; slice_begin a multiple of the group size)."""
    import torch

    M, K, N = _check_inputs(a, b, "matmul_slice_partials")
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=torch.float32)
    assert out.shape == (M, N) and out.dtype == torch.float32 and out.is_contiguous()
    if M == 0 or N == 0:
        return out
    a2, b2 = _tma_ready(a), _tma_ready(b)
    rc = _lib.load().dk_matmul_slice_partials(
        a2.data_ptr(), a2.stride(0), b2.data_ptr(), b2.stride(0), out.data_ptr(), M, N, K, int(slice_begin),
        int(slice_end), _lib.dtype_code(a.dtype), _lib.stream_ptr(a.device))
    _lib.check(rc, "matmul_slice_partials")
    _lib.count_launch()
    return out


def matmul_fold_slices(partials, dtype, out=None):
    """Sum [n, M, N] f32 subtree sums of n equal aligned slice groups (n in 1, 2, 4, 8, in
    group order) along the upper levels of the slice tree and round to ``dtype``."""
    import torch

    assert partials.is_cuda and partials.dtype == torch.float32 and partials.is_contiguous()
    n_parts, M, N = partials.shape
    if out is None:
        out = torch.empty((M, N), device=partials.device, dtype=dtype)
    if M == 0 or N == 0:
        return out
    rc = _lib.load().dk_matmul_fold_slices(partials.data_ptr(), int(n_parts), out.data_ptr(), out.stride(0), M, N,
                                           _lib.dtype_code(dtype), _lib.stream_ptr(partials.device))
    _lib.check(rc, "matmul_fold_slices")
    _lib.count_launch()
    return out


_EPILOGUES = {"store": _lib.DK_EPI_STORE, "residual": _lib.DK_EPI_RESIDUAL, "silu": _lib.DK_EPI_SILU,
              "silu_mul": _lib.DK_EPI_SILU_MUL, "qkv_cache": _lib.DK_EPI_QKV_CACHE, "argmax": _lib.DK_EPI_ARGMAX,
              "residual_rmsnorm": _lib.DK_EPI_RESIDUAL_RMSNORM}


def matmul_fused(a, b, epilogue: str = "store", out=None, workspace=None, residual=None, q_cols: int = 0,
                 head_dim: int = 0, k_cache=None, v_cache=None, row_seq=None, row_pos=None, argmax_keys=None,
                 norm_weight=None, norm_out=None, eps: float = 1e-6, block_table=None):
    """``matmul_batch_invariant`` (same K numerics) with the decoder's next element-wise op fused
    into the store; every step rounds where the unfused torch sequence rounds, so the result bits
    equal that sequence's.  Epilogues:

    * ``"store"``: ``a @ b``.
    * ``"residual"``: ``residual + a @ b`` (``residual`` [M, N]; may be ``out`` itself).
    * ``"silu"``: ``silu(a @ b)``.
    * ``"silu_mul"``: b's columns are (gate, up) pairs; returns ``silu(g) * u``, [M, N/2].
    * ``"qkv_cache"``: the first ``q_cols`` columns are returned ([M, q_cols]); the next
      (N - q_cols)/2 are K, the last (N - q_cols)/2 are V, written into ``k_cache``/``v_cache``
      ([n_seq, H_kv, capacity, head_dim]) at sequence ``row_seq[m]`` (int32; None: m) and position
      ``row_pos[m]`` (int32).  With ``block_table`` (int32 [n_seq, blocks_per_seq]) the caches are
      block pools [n_blocks, H_kv, page, head_dim] and position p of sequence s goes to block
      ``block_table[s, p // page]``, token ``p % page``.
    * ``"argmax"``: folds each row's first maximal column into ``argmax_keys`` (int64 [M] used as
      uint64, zero before the call; ``argmax_finish`` reads and re-zeroes them).  Logits are stored
      only when ``out`` is given.
    * ``"residual_rmsnorm"``: ``"residual"``, and ``norm_out`` ([M, N]) receives
      ``rmsnorm_batch_invariant(result, norm_weight, eps)`` -- the bits of the two calls, with the
      norm computed while the split-K sums are folded.
    """
    import ctypes

    import torch

    M, K, N = _check_inputs(a, b, "matmul_fused")
    epi, out_cols = _epilogue_struct(epilogue, M, N, a.dtype, residual, q_cols, head_dim, k_cache, v_cache, row_seq,
                                     row_pos, argmax_keys, norm_weight, norm_out, eps, block_table)
    if out is None and epilogue != "argmax":
        out = torch.empty((M, out_cols), device=a.device, dtype=a.dtype)
    if out is not None:
        assert out.shape == (M, out_cols) and out.dtype == a.dtype and out.stride(1) == 1
    if M == 0 or N == 0:
        return out
    a2, b2 = _tma_ready(a), _tma_ready(b)
    lib = _lib.load()
    stream = _lib.stream_ptr(a.device)
    if workspace is None:
        workspace = _lib.workspace(lib.dk_matmul_workspace_size(M, N, K), a.device, stream)
    rc = lib.dk_matmul_batch_invariant_ex(
        a2.data_ptr(), a2.stride(0), b2.data_ptr(), b2.stride(0), out.data_ptr() if out is not None else None,
        out.stride(0) if out is not None else out_cols, M, N, K, _lib.dtype_code(a.dtype), ctypes.byref(epi),
        workspace.data_ptr() if workspace is not None else None, workspace.numel() if workspace is not None else 0,
        stream)
    _lib.check(rc, "matmul_fused")
    _lib.count_launch()
    return out


def _epilogue_struct(epilogue, M, N, dtype, residual=None, q_cols=0, head_dim=0, k_cache=None, v_cache=None,
                     row_seq=None, row_pos=None, argmax_keys=None, norm_weight=None, norm_out=None, eps=1e-6,
                     block_table=None):
    """(dk_matmul_epilogue, output columns) for an [M, N] product of ``dtype`` with ``epilogue``."""
    import torch

    if epilogue not in _EPILOGUES:
        raise ValueError("unknown epilogue %r" % (epilogue,))
    epi = _lib.MatmulEpilogue()
    epi.mode = _EPILOGUES[epilogue]
    out_cols = N
    if epilogue in ("residual", "residual_rmsnorm"):
        assert residual is not None and residual.shape == (M, N) and residual.dtype == dtype
        assert residual.is_cuda and residual.stride(1) == 1
        epi.resid, epi.ld_resid = residual.data_ptr(), residual.stride(0)
        if epilogue == "residual_rmsnorm":
            assert norm_weight is not None and norm_weight.is_cuda and norm_weight.is_contiguous()
            assert norm_weight.numel() == N
            assert norm_out is not None and norm_out.shape == (M, N) and norm_out.dtype == dtype
            assert norm_out.stride(1) == 1
            epi.norm_w, epi.norm_w_dtype = norm_weight.data_ptr(), _lib.dtype_code(norm_weight.dtype)
            epi.norm_out, epi.norm_ld, epi.norm_eps = norm_out.data_ptr(), norm_out.stride(0), float(eps)
    elif epilogue == "silu_mul":
        if N % 2:
            raise ValueError("silu_mul needs an even number of columns")
        out_cols = N // 2
    elif epilogue == "qkv_cache":
        kv_cols = (N - q_cols) // 2
        assert k_cache is not None and v_cache is not None and row_pos is not None
        assert k_cache.shape == v_cache.shape and k_cache.stride() == v_cache.stride()
        assert k_cache.dtype == dtype and k_cache.stride(3) == 1 and k_cache.shape[3] == head_dim
        assert row_pos.dtype == torch.int32 and row_pos.numel() >= M
        assert row_seq is None or (row_seq.dtype == torch.int32 and row_seq.numel() >= M)
        epi.q_cols, epi.kv_cols, epi.head_dim = int(q_cols), int(kv_cols), int(head_dim)
        epi.k_cache, epi.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
        epi.cache_stride_seq, epi.cache_stride_head, epi.cache_stride_tok = k_cache.stride(0), k_cache.stride(1), \
            k_cache.stride(2)
        epi.row_seq = row_seq.data_ptr() if row_seq is not None else None
        epi.row_pos = row_pos.data_ptr()
        if block_table is not None:
            assert block_table.dtype == torch.int32 and block_table.is_cuda and block_table.dim() == 2
            assert block_table.stride(1) == 1
            epi.block_table, epi.block_table_stride = block_table.data_ptr(), block_table.stride(0)
            epi.page_size, epi.blocks_per_seq = k_cache.shape[2], block_table.shape[1]
            epi.n_blocks = k_cache.shape[0]
        out_cols = q_cols
    elif epilogue == "argmax":
        assert argmax_keys is not None and argmax_keys.dtype == torch.int64 and argmax_keys.numel() >= M
        epi.argmax_keys = argmax_keys.data_ptr()
    return epi, out_cols


def matmul_fold_fused(partials, dtype, epilogue: str = "store", out=None, residual=None, argmax_keys=None,
                      norm_weight=None, norm_out=None, eps: float = 1e-6):
    """``matmul_fold_slices`` followed by a fused epilogue (``"store"``, ``"residual"``,
    ``"residual_rmsnorm"``, ``"silu"``, ``"silu_mul"`` or ``"argmax"``), applied as
    ``matmul_fused`` applies it: a row-parallel layer whose ranks' subtree sums were gathered
    gets the one-GPU fused layer's bits."""
    import ctypes

    import torch

    assert partials.is_cuda and partials.dtype == torch.float32 and partials.is_contiguous()
    n_parts, M, N = partials.shape
    if epilogue == "qkv_cache":
        raise ValueError("the qkv_cache epilogue is not available after a fold")
    epi, out_cols = _epilogue_struct(epilogue, M, N, dtype, residual, argmax_keys=argmax_keys,
                                     norm_weight=norm_weight, norm_out=norm_out, eps=eps)
    if out is None and epilogue != "argmax":
        out = torch.empty((M, out_cols), device=partials.device, dtype=dtype)
    if out is not None:
        assert out.shape == (M, out_cols) and out.dtype == dtype and out.stride(1) == 1
    if M == 0 or N == 0:
        return out
    rc = _lib.load().dk_matmul_fold_slices_ex(
        partials.data_ptr(), int(n_parts), out.data_ptr() if out is not None else None,
        out.stride(0) if out is not None else out_cols, M, N, _lib.dtype_code(dtype), ctypes.byref(epi),
        _lib.stream_ptr(partials.device))
    _lib.check(rc, "matmul_fold_fused")
    _lib.count_launch()
    return out


def argmax_finish(argmax_keys, tokens, tokens_copy=None, lens_a=None, lens_b=None):
    """After an ``"argmax"`` matmul over n rows: tokens[r] (int64) = row r's argmax column (also
    into tokens_copy), keys re-zeroed, lens_a/lens_b (int32) advanced by one."""
    import torch

    n = tokens.numel()
    assert argmax_keys.numel() >= n and tokens.dtype == torch.int64 and tokens.is_contiguous()
    for t in (lens_a, lens_b):
        assert t is None or (t.dtype == torch.int32 and t.numel() >= n)
    assert tokens_copy is None or (tokens_copy.dtype == torch.int64 and tokens_copy.numel() >= n)
    rc = _lib.load().dk_argmax_finish(
        argmax_keys.data_ptr(), n, tokens.data_ptr(), tokens_copy.data_ptr() if tokens_copy is not None else None,
        lens_a.data_ptr() if lens_a is not None else None, lens_b.data_ptr() if lens_b is not None else None,
        _lib.stream_ptr(tokens.device))
    _lib.check(rc, "argmax_finish")
    _lib.count_launch()
    return tokens


def argmax_finish_parts(gathered_keys, col_offsets, tokens, tokens_copy=None, lens_a=None, lens_b=None,
                        reset_keys=None):
    """End of a greedy step for a column-parallel LM head: gathered_keys [n_parts, n] (int64 used as
    uint64) hold each part's ``"argmax"`` keys over its own columns, which start at col_offsets[p] of
    the vocabulary.  tokens[r] = the global argmax (the one-GPU answer); tokens_copy, lens and
    reset_keys as in ``argmax_finish``."""
    import ctypes

    import torch

    n_parts, n = gathered_keys.shape
    assert gathered_keys.dtype == torch.int64 and gathered_keys.is_contiguous() and gathered_keys.is_cuda
    assert len(col_offsets) == n_parts and tokens.dtype == torch.int64 and tokens.numel() >= n, (
        "argmax_finish_parts: %d parts with %d column offsets, %d keys per part, tokens %s of %d elements"
        % (n_parts, len(col_offsets), n, tokens.dtype, tokens.numel()))
    for t in (lens_a, lens_b):
        assert t is None or (t.dtype == torch.int32 and t.numel() >= n)
    for t in (tokens_copy, reset_keys):
        assert t is None or (t.dtype == torch.int64 and t.numel() >= n)
    offs = (ctypes.c_int64 * n_parts)(*[int(o) for o in col_offsets])
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    rc = _lib.load().dk_argmax_finish_parts(
        gathered_keys.data_ptr(), int(n_parts), n, offs, n, tokens.data_ptr(), ptr(tokens_copy), ptr(lens_a),
        ptr(lens_b), ptr(reset_keys), _lib.stream_ptr(tokens.device))
    _lib.check(rc, "argmax_finish_parts")
    _lib.count_launch()
    return tokens
