"""Batch-invariant single-query (decode-step) attention.

Drop-in for the reference's ``kernels/attention.py``:

* ``attention_reference`` (attention.py:49-71): einsum scores, softmax, einsum
  with V, all f32.  Extended (keyword-only) with GQA -- k/v may carry fewer
  heads than q, query head h reading kv head h // (H / H_kv) -- and per-row KV
  lengths ``kv_lens``.
* ``attention_batch_invariant`` (attention.py:289-298): split-KV decode
  attention with a fixed split SIZE of 256 tokens, a fixed in-split order and a
  fixed-order combine, so a row's output bits depend only on its own q, KV and
  length.  ``block_s`` is accepted for signature compatibility.
* ``attention_batch_variant`` (attention.py:301-348): the deliberately variant
  twin -- a fixed split COUNT with f32 atomics when B*H < split_bh_threshold.

Shapes: q [B, H, D]; k, v [B, H_kv, S, D]; out like q.
"""
from __future__ import annotations

from detkernels_b200 import _lib

KV_SPLIT = _lib.ATTN_KV_SPLIT


def attention_reference(q, k, v, scale: float | None = None, *, kv_lens=None):
    """Plain PyTorch eager decode-step attention, f32 (reference attention.py:49-71).

    q: (B, H, D); k, v: (B, H_kv, S, D) with H % H_kv == 0; kv_lens: optional
    per-row valid lengths (row b attends to k[b, :, :kv_lens[b]])."""
    import torch

    orig_dtype = q.dtype
    d = q.shape[-1]
    if scale is None:
        scale = 1.0 / (d ** 0.5)
    q32 = q.to(torch.float32)
    H, Hkv = q.shape[1], k.shape[1]
    if kv_lens is None:
        k32 = k.to(torch.float32)
        v32 = v.to(torch.float32)
        if Hkv != H:
            k32 = k32.repeat_interleave(H // Hkv, dim=1)
            v32 = v32.repeat_interleave(H // Hkv, dim=1)
        scores = torch.einsum("bhd,bhsd->bhs", q32, k32) * scale
        probs = torch.softmax(scores, dim=-1)
        out = torch.einsum("bhs,bhsd->bhd", probs, v32)
        return out.to(orig_dtype)
    # ragged rows: each row's own prefix of the cache, converted and expanded alone (the padding
    # beyond a row's length is never touched)
    outs = []
    for b in range(q.shape[0]):
        L = int(kv_lens[b])
        if L == 0:
            outs.append(torch.zeros_like(q32[b]))
            continue
        kb = k[b, :, :L].to(torch.float32)
        vb = v[b, :, :L].to(torch.float32)
        if Hkv != H:
            kb = kb.repeat_interleave(H // Hkv, dim=0)
            vb = vb.repeat_interleave(H // Hkv, dim=0)
        s = torch.einsum("hd,hsd->hs", q32[b], kb) * scale
        outs.append(torch.einsum("hs,hsd->hd", torch.softmax(s, dim=-1), vb))
    return torch.stack(outs).to(orig_dtype)


def attention_decode(q, k_cache, v_cache, kv_lens, *, scale=None, row_tiles=None, max_kv_len=None, out=None,
                     workspace=None, block_table=None):
    """General entry: q [R, H, D] rows over a KV cache [N_seq, H_kv, capacity, D].

    kv_lens: int32 CUDA tensor [R] (or an int for every row).  row_tiles:
    optional int32 CUDA tensor [T, 3] (first row, row count, sequence) grouping
    consecutive rows of one sequence; without it row r reads sequence r.
    max_kv_len: host-side bound on every kv_len (defaults to the capacity).
    block_table: optional int32 CUDA tensor [N_seq, blocks_per_seq] for a paged cache: k_cache /
    v_cache are then block pools [n_blocks, H_kv, page, D] (page a multiple of 64) and token t of
    sequence s lives at block_table[s, t // page], token t % page.  Same bits as a contiguous cache.
    """
    import torch

    assert q.is_cuda and k_cache.is_cuda and v_cache.is_cuda, "attention requires CUDA tensors"
    R, H, D = q.shape
    n_seq, Hkv, cap, D2 = k_cache.shape
    if block_table is not None:
        assert block_table.dtype == torch.int32 and block_table.is_cuda and block_table.dim() == 2
        assert block_table.stride(1) == 1
        n_blocks, page = n_seq, cap
        n_seq, cap = block_table.shape[0], block_table.shape[1] * page
    assert D2 == D and v_cache.shape == k_cache.shape, "q/k/v shape mismatch"
    assert k_cache.stride() == v_cache.stride(), "k and v caches must share strides"
    assert k_cache.stride(3) == 1 and q.stride(2) == 1, "unit stride along head_dim required"
    if q.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype:
        raise TypeError("attention: q, k, v must share a dtype")
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    if out is None:
        out = torch.empty((R, H, D), dtype=q.dtype, device=q.device)
    if R == 0:
        return out
    if max_kv_len is None:
        max_kv_len = cap
    lens_ptr, uniform = None, 0
    if isinstance(kv_lens, int):
        uniform = kv_lens
    else:
        assert kv_lens.dtype == torch.int32 and kv_lens.is_cuda and kv_lens.numel() == R
        lens_ptr = kv_lens.data_ptr()
    tiles_ptr, n_tiles, rows_per_tile = None, R, 1
    if row_tiles is not None:
        assert row_tiles.dtype == torch.int32 and row_tiles.is_cuda and row_tiles.is_contiguous()
        tiles_ptr, n_tiles, rows_per_tile = row_tiles.data_ptr(), row_tiles.shape[0], 2
    lib = _lib.load()
    stream = _lib.stream_ptr(q.device)
    if workspace is None:
        nbytes = lib.dk_attention_workspace_size(n_tiles, rows_per_tile, H, Hkv, D, int(max_kv_len))
        workspace = _lib.workspace(nbytes, q.device, stream)
    if block_table is not None:
        rc = lib.dk_attention_paged_batch_invariant(
            q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0),
            k_cache.stride(1), k_cache.stride(2), n_blocks, page, block_table.data_ptr(), block_table.stride(0),
            n_seq, block_table.shape[1], out.data_ptr(), out.stride(0), out.stride(1), lens_ptr, int(uniform),
            tiles_ptr, int(n_tiles), R, H, Hkv, D, int(max_kv_len), float(scale), _lib.dtype_code(q.dtype),
            workspace.data_ptr() if workspace is not None else None,
            workspace.numel() if workspace is not None else 0, stream)
        _lib.check(rc, "attention_paged_batch_invariant")
        _lib.count_launch()
        return out
    rc = lib.dk_attention_batch_invariant(
        q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0),
        k_cache.stride(1), k_cache.stride(2), n_seq, cap, out.data_ptr(), out.stride(0), out.stride(1),
        lens_ptr, int(uniform), tiles_ptr, int(n_tiles), R, H, Hkv, D, int(max_kv_len), float(scale),
        _lib.dtype_code(q.dtype), workspace.data_ptr() if workspace is not None else None,
        workspace.numel() if workspace is not None else 0, stream)
    _lib.check(rc, "attention_batch_invariant")
    _lib.count_launch()
    return out


def _kv_ready(t):
    # TMA needs a unit stride along D and 16-byte aligned strides elsewhere
    if t.stride(3) == 1 and all((s * t.element_size()) % 16 == 0 for s in t.stride()[:3]) \
            and t.data_ptr() % 16 == 0:
        return t
    return t.contiguous()


def attention_batch_invariant(q, k, v, scale: float | None = None, block_s: int = 64, *, kv_lens=None):
    """Batch-invariant decode-step attention (fixed split size, fixed-order combine)."""
    import torch

    assert q.is_cuda and k.is_cuda and v.is_cuda, "attention_batch_invariant requires CUDA tensors"
    B, H, D = q.shape
    Bk, Hkv, S, Dk = k.shape
    assert Bk == B and Dk == D and v.shape == k.shape, "q/k/v shape mismatch"
    assert H % Hkv == 0, "query heads must be a multiple of kv heads"
    q2 = q if q.stride(2) == 1 and q.stride(0) % 2 == 0 and q.stride(1) % 2 == 0 else q.contiguous()
    k2, v2 = _kv_ready(k), _kv_ready(v)
    if k2.stride() != v2.stride():
        k2, v2 = k2.contiguous(), v2.contiguous()
    if kv_lens is None:
        lens = S
    else:
        lens = torch.as_tensor(kv_lens, device=q.device).to(torch.int32).contiguous()
    out = torch.empty((B, H, D), dtype=q.dtype, device=q.device)
    return attention_decode(q2, k2, v2, lens, scale=scale, max_kv_len=S, out=out)


def attention_batch_variant(q, k, v, scale: float | None = None, split_bh_threshold: int = 32, split_s: int = 4,
                            block_s: int = 64):
    """Deliberately batch-variant decode attention (reference attention.py:301-348): a fixed split COUNT
    combined with f32 atomics when B * H < split_bh_threshold, else the invariant kernel."""
    import torch

    assert q.is_cuda and k.is_cuda and v.is_cuda, "attention_batch_variant requires CUDA tensors"
    B, H, D = q.shape
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    if B * H >= split_bh_threshold:
        return attention_batch_invariant(q, k, v, scale)
    S = k.shape[2]
    if k.shape[1] != H:
        k = k.repeat_interleave(H // k.shape[1], dim=1)
        v = v.repeat_interleave(H // v.shape[1], dim=1)
    if k.stride(3) != 1 or k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    q2 = q if q.stride(2) == 1 else q.contiguous()
    out = torch.empty((B, H, D), dtype=q.dtype, device=q.device)
    lib = _lib.load()
    stream = _lib.stream_ptr(q.device)
    ws = _lib.workspace(lib.dk_attention_variant_workspace_size(B, H, D), q.device, stream)
    rc = lib.dk_attention_batch_variant(
        q2.data_ptr(), q2.stride(0), q2.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
        k.stride(2), out.data_ptr(), out.stride(0), out.stride(1), B, H, S, D, float(scale), int(split_s),
        _lib.dtype_code(q.dtype), ws.data_ptr(), ws.numel(), stream)
    _lib.check(rc, "attention_batch_variant")
    return out
