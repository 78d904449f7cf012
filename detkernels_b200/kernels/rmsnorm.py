"""Batch-invariant RMSNorm, and its deliberately batch-variant twin.

Drop-in for the reference's ``kernels/rmsnorm.py`` (same names, arguments,
return values and preconditions):

* ``rmsnorm_reference`` (rmsnorm.py:39-48): plain torch, f32 math, runs on any
  device.  Ground truth for tolerance checks.
* ``rmsnorm_batch_invariant`` (rmsnorm.py:155-177): one CTA of 256 threads per
  row on the B200, fixed per-thread chunk order and a fixed shuffle tree, so a
  row's bits never depend on how many rows are in the call.
* ``rmsnorm_batch_variant`` (rmsnorm.py:180-218): below ``split_threshold``
  rows, each row's sum of squares is split into ``n_splits`` chunks combined
  with f32 atomics -- the scheduler-dependent order the invariant kernel
  removes.

The CUDA ops raise if the library is not built; there is no CPU fallback.
"""
from __future__ import annotations

from detkernels_b200 import _lib


def rmsnorm_reference(x, weight, eps: float = 1e-6):
    """Plain PyTorch eager RMSNorm, float32 accumulation (reference rmsnorm.py:39-48)."""
    import torch

    orig_dtype = x.dtype
    x_f32 = x.to(torch.float32)
    var = x_f32.pow(2).mean(dim=-1, keepdim=True)
    x_norm = x_f32 * torch.rsqrt(var + eps)
    return (x_norm * weight.to(torch.float32)).to(orig_dtype)


def _prepare(x, weight, name):
    import torch

    assert x.is_cuda, "%s requires a CUDA tensor" % name
    assert weight.is_cuda and weight.device == x.device, "%s: weight must be on x's device" % name
    orig_shape = x.shape
    n_cols = orig_shape[-1]
    assert weight.numel() == n_cols, "%s: weight has %d elements, expected %d" % (name, weight.numel(), n_cols)
    x2d = x.reshape(-1, n_cols)
    if x2d.stride(-1) != 1:
        x2d = x2d.contiguous()
    w = weight.reshape(-1)
    if w.stride(0) != 1:
        w = w.contiguous()
    out = torch.empty((x2d.shape[0], n_cols), dtype=x.dtype, device=x.device)
    return orig_shape, x2d, w, out


def rmsnorm_batch_invariant(x, weight, eps: float = 1e-6):
    """Batch-invariant RMSNorm: one CTA per row, fixed reduction order."""
    orig_shape, x2d, w, out = _prepare(x, weight, "rmsnorm_batch_invariant")
    n_rows, n_cols = x2d.shape
    if n_rows == 0:
        return out.reshape(orig_shape)
    lib = _lib.load()
    rc = lib.dk_rmsnorm_batch_invariant(
        x2d.data_ptr(), x2d.stride(0), w.data_ptr(), out.data_ptr(), out.stride(0), n_rows, n_cols,
        _lib.dtype_code(x.dtype), _lib.dtype_code(w.dtype), float(eps), _lib.stream_ptr(x.device))
    _lib.check(rc, "rmsnorm_batch_invariant")
    _lib.count_launch()
    return out.reshape(orig_shape)


def rmsnorm_gather(table, index, weight, eps: float = 1e-6, x_out=None, out=None):
    """Embedding lookup fused into the batch-invariant RMSNorm: returns (x, y) with
    x = table[index] and y = rmsnorm_batch_invariant(x, weight, eps), bit for bit, from one
    launch.  index: int64 CUDA tensor [n]; an index outside the table sets the device status."""
    import torch

    assert table.is_cuda and index.is_cuda and weight.is_cuda, "rmsnorm_gather requires CUDA tensors"
    assert table.dim() == 2 and table.stride(1) == 1 and index.dtype == torch.int64 and index.dim() == 1
    n, h = index.numel(), table.shape[1]
    assert weight.numel() == h
    w = weight.reshape(-1).contiguous()
    idx = index.contiguous()
    if x_out is None:
        x_out = torch.empty((n, h), dtype=table.dtype, device=table.device)
    if out is None:
        out = torch.empty((n, h), dtype=table.dtype, device=table.device)
    assert x_out.shape == (n, h) and out.shape == (n, h) and x_out.stride(1) == 1 and out.stride(1) == 1
    if n == 0:
        return x_out, out
    rc = _lib.load().dk_rmsnorm_gather_batch_invariant(
        table.data_ptr(), table.stride(0), table.shape[0], idx.data_ptr(), w.data_ptr(), x_out.data_ptr(),
        x_out.stride(0), out.data_ptr(), out.stride(0), n, h, _lib.dtype_code(table.dtype), _lib.dtype_code(w.dtype),
        float(eps), _lib.stream_ptr(table.device))
    _lib.check(rc, "rmsnorm_gather")
    _lib.count_launch()
    return x_out, out


def rmsnorm_batch_variant(x, weight, eps: float = 1e-6, split_threshold: int = 16, n_splits: int = 4):
    """Deliberately batch-variant RMSNorm: split + f32 atomics when n_rows < split_threshold."""
    orig_shape, x2d, w, out = _prepare(x, weight, "rmsnorm_batch_variant")
    n_rows, n_cols = x2d.shape
    if n_rows == 0:
        return out.reshape(orig_shape)
    lib = _lib.load()
    stream = _lib.stream_ptr(x.device)
    nbytes = lib.dk_rmsnorm_variant_workspace_size(n_rows)
    ws = _lib.workspace(nbytes, x.device, stream)
    rc = lib.dk_rmsnorm_batch_variant(
        x2d.data_ptr(), x2d.stride(0), w.data_ptr(), out.data_ptr(), out.stride(0), n_rows, n_cols,
        _lib.dtype_code(x.dtype), _lib.dtype_code(w.dtype), float(eps), int(split_threshold), int(n_splits),
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, stream)
    _lib.check(rc, "rmsnorm_batch_variant")
    return out.reshape(orig_shape)
