"""RMSNorm: the reference's test pattern (kernels tests/test_rmsnorm.py) on the
B200 kernels, plus oracle parity and the headline invariance sweep (row 0 fixed, B in
{1, 64}, 100 runs, bitwise)."""
import numpy as np
import pytest

from oracle import ops as oracle

pytestmark = pytest.mark.gpu


def _random_input(dev, n_rows, n_cols, dtype, seed=0):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(n_rows, n_cols, device=dev, dtype=dtype, generator=g)
    weight = torch.randn(n_cols, device=dev, dtype=dtype, generator=g)
    return x, weight


def test_batch_invariant_matches_reference(dev):
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant, rmsnorm_reference
    x, weight = _random_input(dev, 8, 4096, torch.float16)
    got = rmsnorm_batch_invariant(x, weight)
    want = rmsnorm_reference(x, weight)
    torch.testing.assert_close(got, want, atol=2e-2, rtol=2e-2)


def test_batch_variant_matches_reference(dev):
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_variant, rmsnorm_reference
    x_small, weight = _random_input(dev, 4, 4096, torch.float16, seed=1)
    x_large, _ = _random_input(dev, 32, 4096, torch.float16, seed=1)
    for x in (x_small, x_large):
        torch.testing.assert_close(rmsnorm_batch_variant(x, weight), rmsnorm_reference(x, weight),
                                   atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("dtype_name", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("shape", [(1, 4096), (64, 4096), (3, 1000), (5, 37), (2, 12288), (7, 1)])
def test_matches_oracle(dev, dtype_name, shape):
    """f32 math: vs the oracle within a few f32 ulps before rounding (f32 out),
    or at most one ulp of the 16-bit output type."""
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    dtype = getattr(torch, dtype_name)
    x, _ = _random_input(dev, *shape, dtype=dtype, seed=3)
    g = torch.Generator(device=dev).manual_seed(4)
    w = (1.0 + 0.1 * torch.randn(shape[1], device=dev, generator=g)).to(dtype)
    got = rmsnorm_batch_invariant(x, w, eps=1e-6).float().cpu().numpy()
    want = oracle.rmsnorm(x.float().cpu().numpy(), w.float().cpu().numpy(), 1e-6, dtype_name)
    if dtype_name == "float32":
        np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-6)
    else:
        tol = 2 ** -7 if dtype_name == "bfloat16" else 2 ** -10
        np.testing.assert_allclose(got, want, rtol=tol, atol=tol)


def test_batch_invariant_row_is_identical_regardless_of_batch_size(dev):
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    n_cols = 4096
    torch.manual_seed(0)
    row = torch.randn(1, n_cols, device=dev, dtype=torch.float16)
    weight = torch.randn(n_cols, device=dev, dtype=torch.float16)
    solo_out = rmsnorm_batch_invariant(row, weight)
    batch = torch.randn(64, n_cols, device=dev, dtype=torch.float16)
    batch[0] = row[0]
    batch_out = rmsnorm_batch_invariant(batch, weight)
    assert torch.equal(solo_out[0], batch_out[0])


def test_baseline_config_row0_bitwise_over_100_runs(dev):
    """x f32 [B, 4096], B in {1, 64}, x ~ N(0,1), w = 1 + 0.1 N(0,1), eps 1e-6;
    row 0 fixed, other rows redrawn from seed 1000 + run; row 0 bitwise equal."""
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    g = torch.Generator(device=dev).manual_seed(0)
    row0 = torch.randn(1, 4096, device=dev, generator=g)
    w = 1.0 + 0.1 * torch.randn(4096, device=dev, generator=g)
    ref = rmsnorm_batch_invariant(row0, w, eps=1e-6)[0].clone()
    for run in range(100):
        for B in (1, 64):
            gr = torch.Generator(device=dev).manual_seed(1000 + run)
            x = torch.randn(B, 4096, device=dev, generator=gr)
            x[0] = row0[0]
            out = rmsnorm_batch_invariant(x, w, eps=1e-6)
            assert torch.equal(out[0], ref), (run, B)


def test_row_bits_do_not_depend_on_alignment_or_position(dev):
    """An unaligned view takes the scalar path, which walks the same chunks in the
    same per-thread order as the vectorised path: identical bits."""
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    torch.manual_seed(1)
    flat = torch.randn(3 * 4096 + 1, device=dev, dtype=torch.bfloat16)
    w = torch.randn(4096, device=dev, dtype=torch.bfloat16)
    raw = flat[1:].view(3, 4096)                  # 2-byte offset: scalar path
    assert raw.data_ptr() % 16 != 0
    assert torch.equal(rmsnorm_batch_invariant(raw, w), rmsnorm_batch_invariant(raw.clone(), w))
    shifted = torch.cat([torch.zeros(1, 4096, device=dev, dtype=torch.bfloat16), raw])
    assert torch.equal(rmsnorm_batch_invariant(shifted, w)[1:], rmsnorm_batch_invariant(raw, w))


def test_empty_and_3d_input(dev):
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant, rmsnorm_reference
    w = torch.randn(64, device=dev)
    assert rmsnorm_batch_invariant(torch.empty(0, 64, device=dev), w).shape == (0, 64)
    x = torch.randn(2, 3, 64, device=dev)
    torch.testing.assert_close(rmsnorm_batch_invariant(x, w), rmsnorm_reference(x, w), rtol=1e-5, atol=1e-5)


def test_batch_variant_row_can_diverge_across_batch_sizes(dev):
    """Documents (not asserts) the failure mode, as the reference does."""
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_variant
    torch.manual_seed(0)
    row = torch.randn(1, 4096, device=dev, dtype=torch.float16)
    weight = torch.randn(4096, device=dev, dtype=torch.float16)
    solo_out = rmsnorm_batch_variant(row, weight)
    batch = torch.randn(64, 4096, device=dev, dtype=torch.float16)
    batch[0] = row[0]
    batch_out = rmsnorm_batch_variant(batch, weight)
    assert not torch.isnan(solo_out).any()
    assert not torch.isnan(batch_out).any()


def test_requires_cuda_tensor():
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    with pytest.raises(AssertionError):
        rmsnorm_batch_invariant(torch.randn(2, 8), torch.randn(8))


@pytest.mark.parametrize("dtype_name,w_name", [("bfloat16", "bfloat16"), ("float16", "float32"), ("float32", "float32")])
def test_gather_equals_lookup_then_rmsnorm(dev, dtype_name, w_name):
    """The fused embedding lookup + RMSNorm gives the bits of table[index] followed by
    rmsnorm_batch_invariant, for repeated and arbitrary indices; an index outside the
    table is caught by the kernel's check (status DK_ERR_DEVICE_CHECK, nothing written)."""
    import torch
    from detkernels_b200 import _lib
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant, rmsnorm_gather
    dtype, w_dtype = getattr(torch, dtype_name), getattr(torch, w_name)
    g = torch.Generator(device=dev).manual_seed(11)
    table = torch.randn(1000, 1024, device=dev, generator=g).to(dtype)
    w = (1.0 + 0.1 * torch.randn(1024, device=dev, generator=g)).to(w_dtype)
    for n in (1, 7, 256):
        idx = torch.randint(0, 1000, (n,), device=dev, generator=g)
        idx[0] = idx[-1]
        x, y = rmsnorm_gather(table, idx, w, 1e-6)
        assert torch.equal(x, table[idx])
        assert torch.equal(y, rmsnorm_batch_invariant(table[idx], w, 1e-6))
    bad = torch.tensor([3, 1000], device=dev, dtype=torch.int64)
    x = torch.zeros(2, 1024, device=dev, dtype=dtype)
    y = torch.zeros(2, 1024, device=dev, dtype=dtype)
    rmsnorm_gather(table, bad, w, 1e-6, x_out=x, out=y)
    code, _ = _lib.device_status(torch.cuda.current_device(), clear=True)
    assert code == _lib.DK_ERR_DEVICE_CHECK
    assert torch.equal(x[0], table[3]) and int(x[1].count_nonzero()) == 0 and int(y[1].count_nonzero()) == 0


@pytest.mark.parametrize("n_cols,offset", [(1001, 0), (12000, 0), (1024, 1)])
def test_gather_scalar_path_equals_lookup_then_rmsnorm(dev, n_cols, offset):
    """Rows the vector gather cannot take -- an odd hidden size, a row longer than the
    vector kernel keeps in registers, an unaligned table view -- go through the scalar
    gather, which walks the scalar RMSNorm's chunks: same bits as lookup + RMSNorm."""
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant, rmsnorm_gather
    g = torch.Generator(device=dev).manual_seed(5)
    full = torch.randn(300, n_cols + offset, device=dev, generator=g).to(torch.bfloat16)
    table = full[:, offset:]
    w = (1.0 + 0.1 * torch.randn(n_cols, device=dev, generator=g)).to(torch.bfloat16)
    idx = torch.randint(0, 300, (37,), device=dev, generator=g)
    x, y = rmsnorm_gather(table, idx, w, 1e-6)
    assert torch.equal(x, table[idx])
    assert torch.equal(y, rmsnorm_batch_invariant(table[idx].contiguous(), w, 1e-6))


def test_batch_variant_row_diverges_while_invariant_row_does_not(dev):
    """The variant twin splits a row's sum of squares over CTAs when the batch is small and not
    when it is large, so a row's bits change with the batch size; the invariant kernel's do not.
    Sixteen random rows: at least one must differ."""
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant, rmsnorm_batch_variant
    g = torch.Generator(device=dev).manual_seed(22)
    weight = (1 + 0.1 * torch.randn(4096, device=dev, generator=g)).to(torch.float32)
    batch = torch.randn(64, 4096, device=dev, generator=g).to(torch.float32)
    diverged = 0
    for r in range(16):
        row = batch[r:r + 1].contiguous()
        diverged += int(not torch.equal(rmsnorm_batch_variant(row, weight)[0], rmsnorm_batch_variant(batch, weight)[r]))
        assert torch.equal(rmsnorm_batch_invariant(row, weight)[0], rmsnorm_batch_invariant(batch, weight)[r])
    assert diverged > 0


@pytest.mark.parametrize("dtype_name,w_name,cols", [("bfloat16", "bfloat16", 1024), ("float16", "float32", 1000),
                                                    ("float32", "float32", 512), ("bfloat16", "float32", 8)])
def test_many_short_rows_equal_the_one_row_per_cta_bits(dev, dtype_name, w_name, cols):
    """A large batch of short rows (at most 128 16-byte chunks) runs on persistent CTAs, a row per
    128-thread half; a batch below the size threshold runs one CTA per row.  The same rows give
    the same bits on both paths."""
    import torch
    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant
    dt, wt = getattr(torch, dtype_name), getattr(torch, w_name)
    g = torch.Generator(device=dev).manual_seed(cols)
    x = (3 * torch.randn(5001, cols, device=dev, generator=g)).to(dt)
    w = (1 + 0.1 * torch.randn(cols, device=dev, generator=g)).to(wt)
    many = rmsnorm_batch_invariant(x, w)
    few = rmsnorm_batch_invariant(x[:1000].contiguous(), w)
    torch.cuda.synchronize()
    assert torch.equal(many[:1000], few)
    want = oracle.rmsnorm(x.float().cpu().numpy(), w.float().cpu().numpy(), 1e-6, dtype_name)
    tol = {"float32": (2e-6, 1e-6), "bfloat16": (2 ** -7, 2 ** -7), "float16": (2 ** -10, 2 ** -10)}[dtype_name]
    np.testing.assert_allclose(many.float().cpu().numpy(), want, rtol=tol[0], atol=tol[1])
