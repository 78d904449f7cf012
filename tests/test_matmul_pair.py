"""The CTA-pair GEMMs (tcgen05.mma.cta_group::2: 256 weight columns x 128 tokens per pair,
and the wide kernel's 256 x 256) against the one-CTA GEMM: the same bits on the same shapes,
for plain stores, every split-K schedule and fused epilogues.  A test hook that is not part
of the public header forces the kernel (low 4 bits: 1 one-CTA, 2 pair, 3 wide) and the
slices per work unit (bits 4 and up: 1, 2, 4 or 8; 0 = the planner's choice)."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(300, 512, 1024), (1000, 4096, 4096), (2048, 11008, 4096), (129, 256, 64), (513, 1000, 200),
          (4096, 1024, 2816), (257, 3072, 1024), (7, 768, 96)]


def _force(mode):
    from detkernels_b200 import _lib
    fn = _lib.load().dk_matmul_pair_schedule_for_test
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int]
    return fn(mode)


@pytest.fixture
def restore_schedule():
    yield
    _force(0)


@pytest.mark.parametrize("kernel", [2, 3])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_pair_kernel_equals_one_cta_kernel(dev, restore_schedule, M, N, K, kernel):
    import torch

    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    a = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(K, N, device=dev, generator=g)).to(torch.bfloat16)
    _force(1)
    want = matmul_batch_invariant(a, b)
    _force(kernel)
    got = matmul_batch_invariant(a, b)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # f16 too
    a16, b16 = a.to(torch.float16), b.to(torch.float16)
    _force(1)
    want16 = matmul_batch_invariant(a16, b16)
    _force(kernel)
    assert torch.equal(matmul_batch_invariant(a16, b16), want16)


@pytest.mark.parametrize("group", [1, 2, 4, 8])
@pytest.mark.parametrize("M,N,K", [(700, 1000, 4096), (257, 3072, 1024), (40, 512, 200)])
def test_wide_kernel_every_group_equals_one_cta_kernel(dev, restore_schedule, M, N, K, group):
    """Every slice grouping of the wide kernel (SPLIT launches for 1, 2 and 4 slices per unit, the
    stash for 8) against the one-CTA kernel with the planner's grouping."""
    import torch

    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    g = torch.Generator(device=dev).manual_seed(M * 7 + N + K + group)
    a = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(K, N, device=dev, generator=g)).to(torch.bfloat16)
    _force(1)
    want = matmul_batch_invariant(a, b)
    _force(3 | (group << 4))
    got = matmul_batch_invariant(a, b)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("kernel", [2, 3])
@pytest.mark.parametrize("epilogue", ["residual_rmsnorm", "silu_mul", "argmax", "silu", "residual"])
def test_pair_kernel_fused_epilogues(dev, restore_schedule, epilogue, kernel):
    import torch

    from detkernels_b200.kernels.matmul import matmul_fused
    g = torch.Generator(device=dev).manual_seed(9)
    M, K, N = 700, 1024, 2048
    a = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(K, N, device=dev, generator=g)).to(torch.bfloat16)
    r = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(N, device=dev, generator=g)).to(torch.bfloat16)
    outs = []
    for mode in (1, kernel):
        _force(mode)
        if epilogue == "residual_rmsnorm":
            nrm = torch.empty_like(r)
            y = matmul_fused(a, b, "residual_rmsnorm", residual=r, norm_weight=w, norm_out=nrm)
            outs.append((y, nrm))
        elif epilogue == "residual":
            outs.append((matmul_fused(a, b, "residual", residual=r),))
        elif epilogue == "argmax":
            keys = torch.zeros(M, dtype=torch.int64, device=dev)
            matmul_fused(a, b, "argmax", argmax_keys=keys)
            outs.append((keys,))
        else:
            outs.append((matmul_fused(a, b, epilogue),))
    torch.cuda.synchronize()
    for x, y in zip(*outs):
        assert torch.equal(x, y)


def test_pair_kernel_rows_equal_one_cta_rows_at_other_m(dev, restore_schedule):
    """Row 0 of a 2048-token product on the pair kernel equals the same row at M = 1, 64 and
    256 on the one-CTA kernel."""
    import torch

    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    _force(2)
    g = torch.Generator(device=dev).manual_seed(3)
    a = torch.randn(2048, 4096, device=dev, generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(4096, 4096, device=dev, generator=g)).to(torch.bfloat16)
    big = matmul_batch_invariant(a, b)
    _force(1)
    for m in (1, 64, 256):
        assert torch.equal(matmul_batch_invariant(a[:m].contiguous(), b)[0], big[0]), m


@pytest.mark.parametrize("group", [0, 1, 8])
def test_wide_kernel_leaves_the_workspace_counters_zero(dev, restore_schedule, group):
    """The workspace a stream shares between entry points starts with arrival counters that must
    stay zero between calls; the wide kernel's stash and split partials live after them."""
    import torch

    from detkernels_b200 import _lib
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    g = torch.Generator(device=dev).manual_seed(77 + group)
    a = torch.randn(1024, 2048, device=dev, generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(2048, 1536, device=dev, generator=g)).to(torch.bfloat16)
    _force(3 | (group << 4))
    matmul_batch_invariant(a, b)
    torch.cuda.synchronize()
    ws = _lib.workspace(1, a.device, _lib.stream_ptr(a.device))
    assert int(ws[: 1 << 20].count_nonzero()) == 0      # DK_WORKSPACE_COUNTER_BYTES
