"""Matmul: the reference's test pattern (tests/test_matmul.py) on the tcgen05
GEMM, oracle parity, the headline invariance sweep (row 0 across M in
{1, 8, 64, 256, 2048}, N in {4096, 11008}) and the slice/fold decomposition
used by tensor parallelism."""
import numpy as np
import pytest

from oracle import ops as oracle
from oracle.numerics import ulp_distance_bf16

pytestmark = pytest.mark.gpu


def _random_input(dev, m, k, n, dtype, seed=0, wscale=1.0):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    a = torch.randn(m, k, device=dev, dtype=dtype, generator=g)
    b = (wscale * torch.randn(k, n, device=dev, dtype=torch.float32, generator=g)).to(dtype)
    return a, b


def test_batch_invariant_matches_reference(dev):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant, matmul_reference
    a, b = _random_input(dev, 128, 256, 128, torch.float16)
    torch.testing.assert_close(matmul_batch_invariant(a, b), matmul_reference(a, b), atol=2e-2, rtol=2e-2)


def test_batch_variant_matches_reference(dev):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_variant, matmul_reference
    a_small, b = _random_input(dev, 8, 256, 128, torch.float16, seed=1)
    a_large, _ = _random_input(dev, 128, 256, 128, torch.float16, seed=1)
    for a in (a_small, a_large):
        torch.testing.assert_close(matmul_batch_variant(a, b), matmul_reference(a, b), atol=2e-2, rtol=2e-2)


def _assert_close_to_exact(got, a, b, dtype_name):
    """|got - exact| <= 1 output ulp + f32 accumulation error bound."""
    exact = oracle.matmul_f64(a.float().cpu().numpy(), b.float().cpu().numpy())
    absprod = oracle.matmul_f64(np.abs(a.float().cpu().numpy()), np.abs(b.float().cpu().numpy()))
    k = a.shape[1]
    ulp = 2.0 ** -8 if dtype_name == "bfloat16" else 2.0 ** -11
    bound = ulp * np.abs(exact) + (k * 2.0 ** -23) * absprod + 1e-30
    err = np.abs(got.float().cpu().numpy().astype(np.float64) - exact)
    worst = np.max(err / bound)
    assert worst <= 1.0, "error %.3g of the bound" % worst


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16"])
@pytest.mark.parametrize("mkn", [(1, 4096, 4096), (8, 4096, 4096), (64, 1024, 2816), (256, 2816, 1024),
                                 (3, 100, 40), (130, 200, 136), (2048, 4096, 4096), (17, 11008, 256),
                                 (5, 16, 8), (1, 8, 4096)])
def test_matches_oracle(dev, dtype_name, mkn):
    """Within one output ulp plus the f32 accumulation bound of the exact product
    (rtol 1e-2 of the config is far looser)."""
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    m, k, n = mkn
    dtype = getattr(torch, dtype_name)
    a, b = _random_input(dev, m, k, n, dtype, seed=m + k + n, wscale=0.02)
    got = matmul_batch_invariant(a, b)
    _assert_close_to_exact(got, a, b, dtype_name)
    want = oracle.matmul(a.float().cpu().numpy(), b.float().cpu().numpy(), dtype_name)
    np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=1e-2, atol=1e-2)


def test_batch_invariant_row_is_identical_regardless_of_batch_size(dev):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    k, n = 256, 128
    torch.manual_seed(0)
    row = torch.randn(1, k, device=dev, dtype=torch.float16)
    weight = torch.randn(k, n, device=dev, dtype=torch.float16)
    solo_out = matmul_batch_invariant(row, weight)
    batch = torch.randn(128, k, device=dev, dtype=torch.float16)
    batch[0] = row[0]
    batch_out = matmul_batch_invariant(batch, weight)
    assert torch.equal(solo_out[0], batch_out[0])


@pytest.mark.parametrize("N", [4096, 11008])
def test_baseline_config_row0_bitwise_across_M(dev, N):
    """A bf16 [M, 4096] ~ N(0,1), W bf16 [4096, N] ~ 0.02 N(0,1); tracked row 0
    bitwise equal for M in {1, 8, 64, 256, 2048} (these M use both the SPLIT
    and the FOLD schedule) and across co-batch contents."""
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    g = torch.Generator(device=dev).manual_seed(0)
    w = (0.02 * torch.randn(4096, N, device=dev, generator=g)).to(torch.bfloat16)
    row0 = torch.randn(1, 4096, device=dev, generator=g).to(torch.bfloat16)
    ref = matmul_batch_invariant(row0, w)[0].clone()
    for rep in range(3):
        for M in (1, 8, 64, 256, 2048):
            gr = torch.Generator(device=dev).manual_seed(1000 + 10 * rep + M)
            a = torch.randn(M, 4096, device=dev, generator=gr).to(torch.bfloat16)
            a[0] = row0[0]
            out = matmul_batch_invariant(a, w)
            assert torch.equal(out[0], ref), (rep, M)
            # the tracked row at a different position gives the same bits too
            if M > 1:
                a2 = a.roll(M // 2 + 1, dims=0)
                assert torch.equal(matmul_batch_invariant(a2, w)[(M // 2 + 1) % M], ref), (rep, M)


def test_slice_partials_fold_reproduce_invariant_output(dev):
    """TP decomposition: for every TP degree (1, 2, 4, 8 aligned slice groups) the
    groups' subtree sums folded along the upper tree equal the single call bit for bit."""
    import torch
    from detkernels_b200.kernels.matmul import (matmul_batch_invariant, matmul_fold_slices,
                                                matmul_slice_partials)
    for (m, k, n) in [(5, 4096, 1024), (300, 2816, 1024), (1, 1024, 2816), (2048, 1024, 256)]:
        a, b = _random_input(dev, m, k, n, torch.bfloat16, seed=7, wscale=0.02)
        ref = matmul_batch_invariant(a, b)
        for tp in (1, 2, 4, 8):
            g = 8 // tp
            parts = torch.stack([matmul_slice_partials(a, b, r * g, (r + 1) * g) for r in range(tp)])
            assert torch.equal(matmul_fold_slices(parts, torch.bfloat16), ref), (m, k, n, tp)
        # a single slice's sum is the product over that K range (f32 tolerance)
        L = ((k + 7) // 8 + 15) // 16 * 16
        p3 = a[:, 3 * L:4 * L].float() @ b[3 * L:4 * L].float()
        torch.testing.assert_close(matmul_slice_partials(a, b, 3, 4), p3, rtol=1e-4, atol=1e-4)
    with pytest.raises(ValueError):
        matmul_slice_partials(a, b, 1, 3)   # not an aligned group


def test_strided_and_unaligned_operands(dev):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    a_big, b_big = _random_input(dev, 70, 300, 260, torch.bfloat16, seed=9)
    a = a_big[3:, 7:7 + 200]    # unaligned, strided view
    b = b_big[:200, 5:5 + 130]
    got = matmul_batch_invariant(a, b)
    assert torch.equal(got, matmul_batch_invariant(a.contiguous(), b.contiguous()))
    _assert_close_to_exact(got, a, b, "bfloat16")


def test_empty_and_zero_k(dev):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    a = torch.randn(0, 64, device=dev, dtype=torch.bfloat16)
    b = torch.randn(64, 32, device=dev, dtype=torch.bfloat16)
    assert matmul_batch_invariant(a, b).shape == (0, 32)
    z = matmul_batch_invariant(torch.randn(4, 0, device=dev, dtype=torch.bfloat16),
                               torch.randn(0, 16, device=dev, dtype=torch.bfloat16))
    assert z.shape == (4, 16) and (z == 0).all()


def test_rejects_mixed_or_f32_dtypes(dev):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    with pytest.raises(TypeError):
        matmul_batch_invariant(torch.randn(2, 8, device=dev, dtype=torch.bfloat16),
                               torch.randn(8, 8, device=dev, dtype=torch.float16))
    with pytest.raises(NotImplementedError):
        matmul_batch_invariant(torch.randn(2, 8, device=dev), torch.randn(8, 8, device=dev))


def test_batch_variant_row_can_diverge_across_batch_sizes(dev):
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_variant
    torch.manual_seed(0)
    row = torch.randn(1, 256, device=dev, dtype=torch.float16)
    weight = torch.randn(256, 128, device=dev, dtype=torch.float16)
    solo_out = matmul_batch_variant(row, weight)
    batch = torch.randn(128, 256, device=dev, dtype=torch.float16)
    batch[0] = row[0]
    batch_out = matmul_batch_variant(batch, weight)
    assert not torch.isnan(solo_out).any()
    assert not torch.isnan(batch_out).any()


def test_matches_cublas_within_bf16_rounding(dev):
    """Same math as torch.matmul (cuBLAS) up to f32 summation order: at most a
    couple of bf16 ulps apart."""
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    a, b = _random_input(dev, 256, 4096, 4096, torch.bfloat16, seed=11, wscale=0.02)
    got = matmul_batch_invariant(a, b)
    cub = a @ b
    torch.testing.assert_close(got.float(), cub.float(), rtol=2 ** -7, atol=1e-3)
    big = cub.float().abs() > 0.05
    assert np.max(ulp_distance_bf16(got.float()[big].cpu().numpy(), cub.float()[big].cpu().numpy())) <= 2


def test_batch_variant_row_diverges_while_invariant_row_does_not(dev):
    """The failure mode the invariant kernel removes, shown on B200: the variant twin takes a
    split-K path for a lone row and a direct path inside a 128-row batch, so the same row's
    bits change with the batch; the invariant kernel's do not.  Several random rows: at least
    one must differ (the two paths sum 4096 products in different orders)."""
    import torch
    from detkernels_b200.kernels.matmul import matmul_batch_invariant, matmul_batch_variant
    g = torch.Generator(device=dev).manual_seed(21)
    weight = torch.randn(4096, 512, device=dev, generator=g).to(torch.float16)
    batch = torch.randn(128, 4096, device=dev, generator=g).to(torch.float16)
    diverged = 0
    for r in range(8):
        row = batch[r:r + 1].contiguous()
        diverged += int(not torch.equal(matmul_batch_variant(row, weight)[0], matmul_batch_variant(batch, weight)[r]))
        assert torch.equal(matmul_batch_invariant(row, weight)[0], matmul_batch_invariant(batch, weight)[r])
    assert diverged > 0
