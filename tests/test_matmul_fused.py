"""Fused matmul epilogues: each equals, bit for bit, the unfused torch sequence it
replaces in the decoder (matmul_batch_invariant, then the torch element-wise op),
on shapes that take the one-CTA fold schedule and the split schedule."""
import pytest

pytestmark = pytest.mark.gpu

# (M, K, N): the first two are many-tile shapes (one CTA folds all slices), the
# others have few tiles (slices spread over CTAs and folded by a second kernel)
SHAPES = [(256, 1024, 4096), (300, 512, 2304), (1, 1024, 256), (7, 2816, 640), (64, 128, 96)]


def _inputs(dev, m, k, n, dtype, seed=0):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    a = torch.randn(m, k, device=dev, dtype=dtype, generator=g)
    b = (0.05 * torch.randn(k, n, device=dev, generator=g)).to(dtype)
    return a, b


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16"])
@pytest.mark.parametrize("mkn", SHAPES)
def test_store_residual_silu(dev, dtype_name, mkn):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant, matmul_fused
    dtype = getattr(torch, dtype_name)
    m, k, n = mkn
    a, b = _inputs(dev, m, k, n, dtype)
    plain = matmul_batch_invariant(a, b)
    assert torch.equal(matmul_fused(a, b, "store"), plain)
    r = torch.randn(m, n, device=dev, dtype=dtype)
    assert torch.equal(matmul_fused(a, b, "residual", residual=r), r + plain)
    inplace = r.clone()
    matmul_fused(a, b, "residual", residual=inplace, out=inplace)
    assert torch.equal(inplace, r + plain)
    assert torch.equal(matmul_fused(a, b, "silu"), torch.nn.functional.silu(plain))


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16"])
@pytest.mark.parametrize("mkn", SHAPES)
def test_silu_mul_on_interleaved_gate_up(dev, dtype_name, mkn):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant, matmul_fused
    dtype = getattr(torch, dtype_name)
    m, k, n = mkn
    a, wg = _inputs(dev, m, k, n, dtype, seed=1)
    _, wu = _inputs(dev, m, k, n, dtype, seed=2)
    w = torch.stack([wg, wu], dim=2).reshape(k, 2 * n).contiguous()
    want = torch.nn.functional.silu(matmul_batch_invariant(a, wg)) * matmul_batch_invariant(a, wu)
    assert torch.equal(matmul_fused(a, w, "silu_mul"), want)


@pytest.mark.parametrize("mkn", [(256, 1024, 1024), (5, 512, 256), (40, 256, 128)])
def test_qkv_cache_writes_k_and_v_where_index_put_would(dev, mkn):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant, matmul_fused
    m, k, hq_d = mkn
    D, Hkv, n_seq, cap = 64, 2, 9, 50
    n = hq_d + 2 * Hkv * D
    a, w = _inputs(dev, m, k, n, torch.bfloat16, seed=3)
    g = torch.Generator().manual_seed(4)
    seq = torch.randint(0, n_seq, (m,), generator=g)
    pos = torch.randperm(n_seq * cap, generator=g)[:m] % cap   # rows may share a sequence
    # distinct (seq, pos) pairs so the expected cache is well defined
    pairs = {}
    for i in range(m):
        pairs[(int(seq[i]), int(pos[i]))] = i
    keep = torch.tensor(sorted(pairs.values()))
    a = a[keep.to(dev)].contiguous()
    seq, pos = seq[keep], pos[keep]
    m = a.shape[0]
    kc = torch.full((n_seq, Hkv, cap, D), 7.0, device=dev, dtype=torch.bfloat16)
    vc = torch.full_like(kc, -3.0)
    q = matmul_fused(a, w, "qkv_cache", q_cols=hq_d, head_dim=D, k_cache=kc, v_cache=vc,
                     row_seq=seq.to(dev, torch.int32), row_pos=pos.to(dev, torch.int32))
    full = matmul_batch_invariant(a, w)
    kc2 = torch.full_like(kc, 7.0)
    vc2 = torch.full_like(kc, -3.0)
    kc2[seq.to(dev), :, pos.to(dev), :] = full[:, hq_d:hq_d + Hkv * D].view(m, Hkv, D)
    vc2[seq.to(dev), :, pos.to(dev), :] = full[:, hq_d + Hkv * D:].view(m, Hkv, D)
    assert torch.equal(q, full[:, :hq_d])
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16"])
@pytest.mark.parametrize("mkn", [(256, 1024, 32000), (3, 1024, 32000), (64, 256, 64), (9, 128, 1000)])
def test_argmax_matches_torch_argmax_including_ties(dev, dtype_name, mkn):
    import torch
    from detkernels_b200.kernels.matmul import argmax_finish, matmul_batch_invariant, matmul_fused
    dtype = getattr(torch, dtype_name)
    m, k, n = mkn
    a, w = _inputs(dev, m, k, n, dtype, seed=5)
    # exact ties: duplicated weight columns, an all-zero row (every logit 0 -> column 0),
    # a row whose maximum sits in two tiles
    w[:, n - 1] = w[:, 3]
    w[:, n // 2] = w[:, 3]
    a[m // 2] = 0
    logits = matmul_batch_invariant(a, w)
    keys = torch.zeros(m, dtype=torch.int64, device=dev)
    out = torch.empty_like(logits)
    matmul_fused(a, w, "argmax", argmax_keys=keys, out=out)
    assert torch.equal(out, logits)
    tok = torch.empty(m, dtype=torch.int64, device=dev)
    copy = torch.empty_like(tok)
    la = torch.arange(m, dtype=torch.int32, device=dev)
    lb = la + 1
    argmax_finish(keys, tok, copy, la, lb)
    want = logits.argmax(dim=-1)
    assert torch.equal(tok, want) and torch.equal(copy, want)
    assert torch.equal(keys, torch.zeros_like(keys))
    assert torch.equal(la, torch.arange(m, dtype=torch.int32, device=dev) + 1)
    assert torch.equal(lb, la + 1)
    # without logits, twice in a row (keys were re-zeroed)
    for _ in range(2):
        matmul_fused(a, w, "argmax", argmax_keys=keys)
        argmax_finish(keys, tok)
        assert torch.equal(tok, want)


@pytest.mark.parametrize("mkn", [(256, 1024, 32000), (7, 512, 1000), (300, 256, 4096)])
def test_argmax_ties_inside_one_32_column_chunk(dev, mkn):
    """Equal maxima at columns 7 and 8 (one 32-column chunk, different running maxima of the
    chunk reduction) and 40 (the next chunk): the smallest column wins, as torch.argmax."""
    import torch
    from detkernels_b200.kernels.matmul import argmax_finish, matmul_batch_invariant, matmul_fused
    m, k, n = mkn
    a, w = _inputs(dev, m, k, n, torch.bfloat16, seed=9)
    a = a.abs()
    for col in (8, 7, 40):
        w[:, col] = 0.25
    logits = matmul_batch_invariant(a, w)
    keys = torch.zeros(m, dtype=torch.int64, device=dev)
    tok = torch.empty(m, dtype=torch.int64, device=dev)
    matmul_fused(a, w, "argmax", argmax_keys=keys)
    argmax_finish(keys, tok)
    want = logits.argmax(dim=-1)
    assert torch.equal(tok, want)
    assert bool((want == 7).all())


def test_fused_rows_are_batch_invariant(dev):
    """A row's fused result does not depend on the other rows (M = 1 vs 256)."""
    import torch
    from detkernels_b200.kernels.matmul import argmax_finish, matmul_fused
    a, wg = _inputs(dev, 256, 1024, 2816, torch.bfloat16, seed=6)
    w = torch.stack([wg, wg.flip(1)], dim=2).reshape(1024, -1).contiguous()
    full = matmul_fused(a, w, "silu_mul")
    solo = matmul_fused(a[:1].contiguous(), w, "silu_mul")
    assert torch.equal(full[:1], solo)
    keys = torch.zeros(256, dtype=torch.int64, device=dev)
    tok = torch.empty(256, dtype=torch.int64, device=dev)
    matmul_fused(a, wg, "argmax", argmax_keys=keys)
    argmax_finish(keys, tok)
    tok1 = torch.empty(1, dtype=torch.int64, device=dev)
    matmul_fused(a[:1].contiguous(), wg, "argmax", argmax_keys=keys)
    argmax_finish(keys, tok1)
    assert tok1.item() == tok[0].item()


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16"])
@pytest.mark.parametrize("mkn", SHAPES + [(256, 1024, 1024), (256, 2816, 1024), (5, 4096, 1000)])
def test_residual_rmsnorm_equals_residual_then_rmsnorm(dev, dtype_name, mkn):
    """The fused residual + RMSNorm epilogue gives the bits of the residual matmul followed by
    rmsnorm_batch_invariant, with the residual in place or not and either weight dtype (the
    split shapes take the one-kernel fold + norm; N = 1000 and the fold-schedule shapes take
    the separate RMSNorm kernel)."""
    import torch
    from detkernels_b200.kernels.matmul import matmul_fused
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    dtype = getattr(torch, dtype_name)
    m, k, n = mkn
    a, b = _inputs(dev, m, k, n, dtype, seed=m + n)
    r = torch.randn(m, n, device=dev, dtype=dtype)
    for w_dtype in (dtype, torch.float32):
        w = (1.0 + 0.1 * torch.randn(n, device=dev)).to(w_dtype)
        h_ref = matmul_fused(a, b, "residual", residual=r)
        y_ref = rmsnorm_batch_invariant(h_ref, w, 1e-6)
        y = torch.empty_like(r)
        h = matmul_fused(a, b, "residual_rmsnorm", residual=r, norm_weight=w, norm_out=y, eps=1e-6)
        assert torch.equal(h, h_ref) and torch.equal(y, y_ref), (mkn, w_dtype)
        inplace = r.clone()
        y2 = torch.full_like(r, float("nan"))
        matmul_fused(a, b, "residual_rmsnorm", residual=inplace, out=inplace, norm_weight=w, norm_out=y2, eps=1e-6)
        assert torch.equal(inplace, h_ref) and torch.equal(y2, y_ref), (mkn, w_dtype)
