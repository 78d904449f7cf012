"""Tensor-parallel matmul: host bookkeeping on CPU ranks (gloo) against the oracle,
the CUDA shard/fold path against the one-GPU kernel bit for bit, and (with two or
more GPUs) the NCCL path end to end."""
import os
import socket

import numpy as np
import pytest

from _ranks import collect
from oracle import ops as oracle
from oracle.numerics import round_to


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ---------------------------------------------------------------- CPU (gloo) ----
def _oracle_partial(a_shard, b_shard, K, tp, rank):
    """The rank's subtree sum from its K shard, by the oracle's slice split."""
    import torch
    from detkernels_b200.kernels import tp as tpm
    b0, b1 = tpm.slice_group(tp, rank)
    k0, _ = tpm.shard_k_range(K, tp, rank)
    L = oracle.slice_len(K)
    a = a_shard.numpy()
    b = b_shard.numpy()
    parts = []
    for s in range(b0, b1):
        lo, hi = min(s * L, K) - k0, min((s + 1) * L, K) - k0
        parts.append((a[:, lo:hi] @ b[lo:hi]).astype(np.float32) if hi > lo
                     else np.zeros((a.shape[0], b.shape[1]), np.float32))
    return torch.from_numpy(oracle.fold_tree(parts))


def _oracle_fold(gathered, dtype):
    import torch
    return torch.from_numpy(round_to(oracle.fold_tree(list(gathered.numpy())), "bfloat16"))


def _gloo_worker(rank, world, port, K, q):
    import torch
    import torch.distributed as dist
    from detkernels_b200.kernels import tp as tpm
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        M, N = 5, 24
        a = torch.randn(M, K, generator=g)
        b = 0.1 * torch.randn(K, N, generator=g)
        k0, k1 = tpm.shard_k_range(K, world, rank)
        out = tpm.row_parallel_matmul(a[:, k0:k1], b[k0:k1], K, partial_fn=_oracle_partial,
                                      fold_fn=_oracle_fold, out_dtype=torch.bfloat16)
        n0, n1 = tpm.shard_n_range(N, world, rank)
        col = tpm.column_parallel_matmul(a, b[:, n0:n1], gather=True, matmul_fn=lambda x, y: x @ y)
        q.put((rank, out.numpy(), col.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,K", [(2, 1024), (4, 2816), (2, 100)])
def test_row_and_column_parallel_bookkeeping_on_cpu_ranks(world, K):
    import torch
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = collect(q, procs, world, 120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(0)
    a = torch.randn(5, K, generator=g).numpy()
    b = (0.1 * torch.randn(K, 24, generator=g)).numpy()
    want = round_to(oracle.fold_tree(oracle.matmul_slice_partials(a, b)), "bfloat16")
    for rank, out, col in results:
        assert np.array_equal(out, want), rank            # same tree, same bits, every rank
        np.testing.assert_allclose(col, a @ b, rtol=1e-5, atol=1e-5)


def test_slice_groups_cover_k_once():
    from detkernels_b200.kernels import tp as tpm
    for K in (1, 7, 100, 1024, 2816, 4096, 11008):
        for world in (1, 2, 4, 8):
            ranges = [tpm.shard_k_range(K, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == K
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
    with pytest.raises(ValueError):
        tpm.slice_group(3, 0)


# ---------------------------------------------------------------- one GPU ----
@pytest.mark.gpu
@pytest.mark.parametrize("mkn", [(1, 1024, 1024), (256, 2816, 1024), (7, 1000, 200), (300, 512, 768)])
def test_shard_partials_fold_to_the_one_gpu_bits(dev, mkn):
    import torch
    from detkernels_b200.kernels import tp as tpm
    from detkernels_b200.kernels.matmul import matmul_batch_invariant, matmul_fold_slices
    M, K, N = mkn
    g = torch.Generator(device=dev).manual_seed(1)
    a = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(K, N, device=dev, generator=g)).to(torch.bfloat16)
    want = matmul_batch_invariant(a, b)
    for world in (1, 2, 4, 8):
        parts = []
        for r in range(world):
            k0, k1 = tpm.shard_k_range(K, world, r)
            # each rank holds only its columns of A and rows of B (fresh contiguous copies)
            parts.append(tpm.shard_partial(a[:, k0:k1].contiguous(), b[k0:k1].contiguous(), K, world, r))
        got = matmul_fold_slices(torch.stack(parts), torch.bfloat16)
        assert torch.equal(got, want), world


# ---------------------------------------------------------------- NCCL ----
def _nccl_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from detkernels_b200.kernels import tp as tpm
    from detkernels_b200.kernels.matmul import matmul_batch_invariant
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        g = torch.Generator(device=dev).manual_seed(2)
        M, K, N = 256, 2816, 1024
        a = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        b = (0.02 * torch.randn(K, N, device=dev, generator=g)).to(torch.bfloat16)
        k0, k1 = tpm.shard_k_range(K, world, rank)
        out = tpm.row_parallel_matmul(a[:, k0:k1].contiguous(), b[k0:k1].contiguous(), K)
        want = matmul_batch_invariant(a, b)
        q.put((rank, bool(torch.equal(out, want))))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_row_parallel_matches_one_gpu():
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    world = 1 << (world.bit_length() - 1) if world else 0
    if world < 2:
        pytest.skip("needs two or more GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = collect(q, procs, world, 300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok in res)
