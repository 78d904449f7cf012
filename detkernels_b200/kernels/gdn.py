"""Gated delta rule (Gated DeltaNet linear attention) forward on B200.

Replaces the third-party call the reference makes through FLA
(``fla.ops.gated_delta_rule.chunk_gated_delta_rule``, fla 0.5.1; reference
gdn/repro.py:76, 161-162, 293-294) with the same calling convention:

* ``chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None,
  output_final_state=False, cu_seqlens=None)`` -> ``(o, final_state)``
* ``fused_recurrent_gated_delta_rule(...)`` -- same arguments, token-by-token.

Shapes (FLA's ``[B, T, heads, dim]`` layout): q, k ``[B, T, H, K]``; v
``[B, T, HV, V]`` with ``HV % H == 0`` (value head j reads query/key head
``j // (HV // H)``); g (log-space decay) and beta ``[B, T, HV]``; with
``cu_seqlens`` (int64, ``[N + 1]``) B must be 1 and the sequences are packed
along T.  ``initial_state`` ``[N, HV, K, V]`` (any float dtype, read as f32);
``final_state`` is f32.  ``o`` has q's dtype.

Batch invariance: each (sequence, value head) is computed by one CTA that cuts
64-token chunks from the sequence's own start and reduces in a fixed order, so
a sequence's output and final state do not depend on the other sequences of
the call, its position in a packed batch, or the call's total size.
"""
from __future__ import annotations

from detkernels_b200 import _lib

CHUNK = 64
HEAD_DIMS = ((32, 32), (64, 64), (128, 128))


def _gb_dtype(t):
    import torch
    return {torch.float32: _lib.DK_F32, torch.bfloat16: _lib.DK_BF16, torch.float16: _lib.DK_F16}[t.dtype]


def _forward(q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens, chunk, name):
    import torch

    assert q.is_cuda and k.is_cuda and v.is_cuda and g.is_cuda and beta.is_cuda, "%s requires CUDA tensors" % name
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("%s: q, k, v must be [B, T, heads, dim]" % name)
    if q.shape[2] != k.shape[2]:
        raise ValueError("q and k must have the same number of heads, but got q.shape[2]=%d and k.shape[2]=%d"
                         % (q.shape[2], k.shape[2]))
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    if HV % H != 0:
        raise ValueError("For GVA, num_v_heads (HV=%d) must be evenly divisible by num_heads (H=%d), but got "
                         "HV %% H = %d" % (HV, H, HV % H))
    if k.shape != q.shape or v.shape[:2] != (B, T) or g.shape != (B, T, HV) or beta.shape != (B, T, HV):
        raise ValueError("%s: inconsistent shapes q %s k %s v %s g %s beta %s"
                         % (name, tuple(q.shape), tuple(k.shape), tuple(v.shape), tuple(g.shape),
                            tuple(beta.shape)))
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise TypeError("%s: q, k, v must share a dtype" % name)
    if (K, V) not in HEAD_DIMS:
        raise NotImplementedError("%s: head dims (%d, %d) not built; supported %s" % (name, K, V, HEAD_DIMS))
    if cu_seqlens is not None:
        if B != 1:
            raise ValueError("The batch size is expected to be 1 rather than %d when using `cu_seqlens`."
                             "Please flatten variable-length inputs before processing." % B)
        if cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1:
            raise ValueError("cu_seqlens must be a 1-D tensor of N + 1 offsets")
        if not cu_seqlens.is_cuda:
            # host offsets are checked here; device offsets are checked by the kernels, which skip
            # a bad sequence and record DK_ERR_DEVICE_CHECK instead of reading outside the inputs
            host = cu_seqlens.to(torch.int64)
            if bool((host < 0).any()) or bool((host[1:] < host[:-1]).any()) or int(host[-1]) > T:
                raise ValueError("cu_seqlens must be non-decreasing offsets within [0, T=%d], got %s"
                                 % (T, host.tolist()))
        cu = cu_seqlens.to(device=q.device, dtype=torch.int64).contiguous()
        N = cu.numel() - 1
        seq_len = T   # the packed length: the bound the kernels check cu_seqlens against
    else:
        cu = None
        N = B
        seq_len = T
    if initial_state is not None:
        if initial_state.shape != (N, HV, K, V):
            raise ValueError("The number of initial states is expected to be equal to the number of input "
                             "sequences, i.e., %d rather than %d." % (N, initial_state.shape[0]))
        initial_state = initial_state.contiguous()
    if scale is None:
        scale = K ** -0.5
    # contiguous, starting on a 16-byte boundary (a fresh copy when a view is not)
    q, k, v = (t.contiguous() for t in (q, k, v))
    q, k, v = (t if t.data_ptr() % 16 == 0 else t.clone() for t in (q, k, v))
    gb = g.dtype if g.dtype == beta.dtype else torch.float32
    g, beta = g.to(gb).contiguous(), beta.to(gb).contiguous()
    o = torch.empty((B, T, HV, V), device=q.device, dtype=q.dtype)
    final = torch.empty((N, HV, K, V), device=q.device, dtype=torch.float32) if output_final_state else None
    if N == 0 or (T == 0 and final is None):
        return o, final
    rc = _lib.load().dk_gdn_forward(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), o.data_ptr(),
        cu.data_ptr() if cu is not None else None, N, seq_len, H, HV, K, V, _lib.dtype_code(q.dtype),
        _gb_dtype(g), float(scale), initial_state.data_ptr() if initial_state is not None else None,
        _gb_dtype(initial_state) if initial_state is not None else _lib.DK_F32,
        final.data_ptr() if final is not None else None, chunk, _lib.stream_ptr(q.device))
    _lib.check(rc, name)
    _lib.count_launch()
    return o, final


def chunk_gated_delta_rule(q, k, v, g, beta, scale: float | None = None, initial_state=None,
                           output_final_state: bool = False, cu_seqlens=None, **kwargs):
    """Chunked (64-token) gated delta rule forward: returns (o, final_state or None)."""
    if kwargs.get("use_qk_l2norm_in_kernel") or kwargs.get("use_gate_in_kernel"):
        raise NotImplementedError("in-kernel q/k normalisation and gate computation are not built")
    if "head_first" in kwargs:
        raise DeprecationWarning("head_first has been removed. Inputs must be in `[B, T, H, ...]` format.")
    return _forward(q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens, CHUNK,
                    "chunk_gated_delta_rule")


def fused_recurrent_gated_delta_rule(q, k, v, g, beta, scale: float | None = None, initial_state=None,
                                     output_final_state: bool = False, cu_seqlens=None, **kwargs):
    """Token-by-token gated delta rule forward (decode): returns (o, final_state or None)."""
    if kwargs.get("use_qk_l2norm_in_kernel"):
        raise NotImplementedError("in-kernel q/k normalisation is not built")
    return _forward(q, k, v, g, beta, scale, initial_state, output_final_state, cu_seqlens, 1,
                    "fused_recurrent_gated_delta_rule")
