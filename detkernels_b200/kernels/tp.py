"""Tensor parallelism for the batch-invariant matmul, bitwise equal to one GPU.

No counterpart in the reference (its matmul has no tensor parallelism,
kernels/matmul.py:161-186); this is the multi-GPU decomposition of the same
invariant numerics:

* Row-parallel (attention output and MLP down projections): K is cut into the
  matmul's 8 fixed slices and rank r of a TP-way group (TP in 1, 2, 4, 8) holds
  the aligned slice group [r*8/TP, (r+1)*8/TP) -- the K range
  ``shard_k_range(K, tp, r)`` of A's columns and B's rows.  Each rank computes
  its group's f32 subtree sum (``dk_matmul_shard_partials``), the sums are
  all-gathered in rank order (NCCL), and every rank adds them along the upper
  levels of the slice tree (``dk_matmul_fold_slices``): the same f32 operations
  as the one-GPU kernel, so the result is bit-identical for every TP.
* Column-parallel (QKV, gate/up, LM head): N is split; output columns are
  independent, so each rank's columns equal the one-GPU columns bit for bit.

The compute steps are parameters (``partial_fn``, ``fold_fn``) so the host-side
bookkeeping can be exercised on CPU processes; the defaults are the CUDA
kernels and nothing here falls back to another implementation.
"""
from __future__ import annotations

from detkernels_b200 import _lib

K_SLICES = _lib.MATMUL_K_SLICES


def _check_tp(tp: int):
    if tp not in (1, 2, 4, 8):
        raise ValueError("tensor-parallel size must be 1, 2, 4 or 8, got %d" % tp)


def slice_group(tp: int, rank: int):
    """The aligned K-slice group [begin, end) owned by rank ``rank`` of a ``tp``-way split."""
    _check_tp(tp)
    if not 0 <= rank < tp:
        raise ValueError("rank %d outside a %d-way group" % (rank, tp))
    span = K_SLICES // tp
    return rank * span, (rank + 1) * span


def shard_k_range(K: int, tp: int, rank: int):
    """[k_begin, k_end) of the full K held by ``rank`` (A's columns, B's rows)."""
    import ctypes
    b, e = slice_group(tp, rank)
    k0, k1 = ctypes.c_int64(), ctypes.c_int64()
    _lib.load().dk_matmul_shard_range(int(K), b, e, ctypes.byref(k0), ctypes.byref(k1))
    return k0.value, k1.value


def shard_n_range(N: int, tp: int, rank: int):
    """[n_begin, n_end) of a column-parallel split (contiguous, ceil(N / tp) per rank)."""
    _check_tp(tp)
    per = -(-N // tp)
    return min(rank * per, N), min((rank + 1) * per, N)


def shard_partial(a_shard, b_shard, K: int, tp: int, rank: int, out=None):
    """f32 [M, N] subtree sum of ``rank``'s slice group from its K shard of A ([M, k1-k0]) and B."""
    import torch

    assert a_shard.is_cuda and b_shard.is_cuda, "shard_partial requires CUDA tensors"
    from .matmul import _tma_ready
    M, N = a_shard.shape[0], b_shard.shape[1]
    k0, k1 = shard_k_range(K, tp, rank)
    if a_shard.shape[1] != k1 - k0 or b_shard.shape[0] != k1 - k0:
        raise ValueError("rank %d of TP=%d holds K[%d:%d] (%d columns), got A %s and B %s"
                         % (rank, tp, k0, k1, k1 - k0, tuple(a_shard.shape), tuple(b_shard.shape)))
    if out is None:
        out = torch.empty((M, N), device=a_shard.device, dtype=torch.float32)
    if M == 0 or N == 0:
        return out
    b0, b1 = slice_group(tp, rank)
    a2 = _tma_ready(a_shard) if k1 > k0 else a_shard
    w2 = _tma_ready(b_shard) if k1 > k0 else b_shard
    rc = _lib.load().dk_matmul_shard_partials(
        a2.data_ptr(), a2.stride(0) if k1 > k0 else 0, w2.data_ptr(), w2.stride(0) if k1 > k0 else 0,
        out.data_ptr(), M, N, int(K), b0, b1, _lib.dtype_code(a_shard.dtype), _lib.stream_ptr(a_shard.device))
    _lib.check(rc, "matmul_shard_partials")
    _lib.count_launch()
    return out


def _fold(gathered, dtype):
    from .matmul import matmul_fold_slices
    return matmul_fold_slices(gathered, dtype)


def check_agreement(group=None, **fields):
    """Every rank of ``group`` must pass equal ``fields`` (TP size, shard counts, shapes ...):
    one all_gather_object, then ValueError on every rank if any rank differs, so a rank with a
    different split fails before its first data exchange instead of hanging it."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    got = [None] * world
    dist.all_gather_object(got, fields, group=group)
    if any(g != got[0] for g in got):
        raise ValueError("tensor-parallel ranks disagree: %s" % got)
    return got[0]


def all_gather_ranks(t, group=None):
    """[world, *t.shape] stack of every rank's tensor, in rank order."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(t.shape), device=t.device, dtype=t.dtype)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t.contiguous(), group=group)
    return out


def row_parallel_matmul(a_shard, b_shard, K: int, group=None, out_dtype=None, partial_fn=None, fold_fn=None):
    """Row-parallel ``A @ B`` over the process group: every rank passes its K shard of A and B
    (``shard_k_range``) and receives the full [M, N] product, bit-identical to
    ``matmul_batch_invariant`` on the unsharded operands."""
    import torch.distributed as dist

    tp = dist.get_world_size(group)
    rank = dist.get_rank(group)
    _check_tp(tp)
    partial_fn = partial_fn or shard_partial
    fold_fn = fold_fn or _fold
    part = partial_fn(a_shard, b_shard, K, tp, rank)
    gathered = all_gather_ranks(part, group)
    return fold_fn(gathered, out_dtype or a_shard.dtype)


def column_parallel_matmul(a, b_shard, group=None, gather: bool = False, matmul_fn=None):
    """Column-parallel ``A @ B``: each rank multiplies by its column shard of B
    (``shard_n_range``); with ``gather`` the [M, N] result is assembled on every rank."""
    import torch

    if matmul_fn is None:
        from .matmul import matmul_batch_invariant as matmul_fn
    part = matmul_fn(a, b_shard)
    if not gather:
        return part
    import torch.distributed as dist
    tp = dist.get_world_size(group)
    width = part.shape[1]
    sizes = [None] * tp
    dist.all_gather_object(sizes, width, group=group)
    if len(set(sizes)) != 1:
        raise ValueError("column shards must be equal for gather (got widths %s)" % sizes)
    stacked = all_gather_ranks(part, group)          # [tp, M, width]
    return torch.cat(list(stacked.unbind(0)), dim=1)
