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
