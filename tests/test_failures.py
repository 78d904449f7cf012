"""Failure detection on the host, never by faulting a GPU.

CPU ranks (gloo, child processes, a short process-group timeout):
* a rank with a different tensor-parallel split fails the agreement check on
  every rank before any data moves;
* a rank that hands its row-parallel matmul the wrong K shard raises on that
  rank, and the rank left waiting in the exchange gets an error from the short
  process-group timeout instead of hanging;
* a rank that dies before an exchange, and a peer that never joins, end the
  other rank's collective / rendezvous with an error.
GPU: a cu_seqlens pair outside the packed tokens is refused on the host (host
offsets) or skipped by the kernel with DK_ERR_DEVICE_CHECK (device offsets).
"""
import datetime
import os
import socket
import time

import numpy as np
import pytest

from _ranks import collect

TIMEOUT = datetime.timedelta(seconds=6)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=TIMEOUT)


def _spawn(target, world, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    return q, procs


def _finish(procs):
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()


# ---------------------------------------------------------------- mismatched shard count ----
def _agreement_worker(rank, world, port, q):
    import torch.distributed as dist

    from detkernels_b200.kernels import tp as tpm
    _init(rank, world, port)
    try:
        tp = 2 if rank == 0 else 4          # rank 1 was configured for a 4-way split
        try:
            tpm.check_agreement(tp=tp, k_slices=tpm.K_SLICES)
            q.put((rank, "ok"))
        except ValueError as e:
            q.put((rank, "ValueError: " + str(e)[:80]))
    finally:
        dist.destroy_process_group()


def test_mismatched_shard_count_fails_on_every_rank():
    q, procs = _spawn(_agreement_worker, 2)
    res = collect(q, procs, 2, 120)
    _finish(procs)
    assert sorted(r for r, _ in res) == [0, 1]
    assert all(msg.startswith("ValueError: tensor-parallel ranks disagree") for _, msg in res), res


# ---------------------------------------------------------------- wrong K shard ----
def _oracle_partial(a_shard, b_shard, K, tp, rank):
    import torch

    from detkernels_b200.kernels import tp as tpm
    k0, k1 = tpm.shard_k_range(K, tp, rank)
    if a_shard.shape[1] != k1 - k0:
        raise ValueError("rank %d of TP=%d holds K[%d:%d], got %d columns" % (rank, tp, k0, k1, a_shard.shape[1]))
    return a_shard.float() @ b_shard.float()


def _wrong_shard_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from detkernels_b200.kernels import tp as tpm
    _init(rank, world, port)
    K = 1024
    a = torch.randn(3, K)
    b = torch.randn(K, 8)
    k0, k1 = tpm.shard_k_range(K, world, rank)
    if rank == 1:
        k1 -= 16                              # a shard that lost its last 16 columns
    t0 = time.monotonic()
    try:
        tpm.row_parallel_matmul(a[:, k0:k1], b[k0:k1], K, partial_fn=_oracle_partial,
                                fold_fn=lambda g, dt: g.sum(0))
        q.put((rank, "ok", time.monotonic() - t0))
    except ValueError as e:
        q.put((rank, "ValueError", time.monotonic() - t0))
    except RuntimeError as e:
        q.put((rank, "RuntimeError", time.monotonic() - t0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_wrong_shard_raises_and_the_waiting_rank_times_out():
    q, procs = _spawn(_wrong_shard_worker, 2)
    res = dict((r, (kind, dt)) for r, kind, dt in collect(q, procs, 2, 120))
    _finish(procs)
    assert res[1][0] == "ValueError"
    assert res[0][0] == "RuntimeError" and res[0][1] < 60, res


# ---------------------------------------------------------------- killed rank / missing peer ----
def _killed_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    _init(rank, world, port)
    if rank == 1:
        os._exit(3)                           # dies between steps, nothing in flight
    t0 = time.monotonic()
    try:
        out = [torch.zeros(4) for _ in range(world)]
        dist.all_gather(out, torch.ones(4))
        q.put((rank, "ok", time.monotonic() - t0))
    except RuntimeError:
        q.put((rank, "RuntimeError", time.monotonic() - t0))


def test_a_killed_rank_ends_the_survivors_collective_with_an_error():
    q, procs = _spawn(_killed_worker, 2)
    res = []
    deadline = time.monotonic() + 120
    while not res and time.monotonic() < deadline:
        try:
            res.append(q.get(timeout=1.0))
        except Exception:
            pass
    _finish(procs)
    assert res and res[0][0] == 0 and res[0][1] == "RuntimeError" and res[0][2] < 60, res
    assert procs[1].exitcode == 3


def _lonely_worker(rank, world, port, q):
    t0 = time.monotonic()
    try:
        _init(rank, world, port)
        q.put((rank, "ok", time.monotonic() - t0))
    except (RuntimeError, TimeoutError) as e:
        q.put((rank, type(e).__name__, time.monotonic() - t0))


def test_a_peer_that_never_joins_ends_the_rendezvous_with_an_error():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_worker, args=(0, 2, _free_port(), q))
    p.start()
    res = collect(q, [p], 1, 120)
    _finish([p])
    assert res[0][1] in ("RuntimeError", "TimeoutError", "DistStoreError") and res[0][2] < 60, res


# ---------------------------------------------------------------- bad cu_seqlens ----
def _gdn_inputs(dev, T, H=2, HV=4, D=64):
    import torch
    import torch.nn.functional as F
    g = torch.Generator(device=dev).manual_seed(9)
    q = torch.randn(1, T, H, D, device=dev, generator=g).to(torch.bfloat16)
    k = F.normalize(torch.randn(1, T, H, D, device=dev, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(1, T, HV, D, device=dev, generator=g).to(torch.bfloat16)
    gate = F.logsigmoid(torch.randn(1, T, HV, device=dev, generator=g))
    beta = torch.sigmoid(torch.randn(1, T, HV, device=dev, generator=g))
    return q, k, v, gate, beta


@pytest.mark.gpu
def test_bad_host_cu_seqlens_is_refused(dev):
    import torch

    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule
    q, k, v, g, b = _gdn_inputs(dev, 200)
    for bad in ([0, 120, 100, 200], [0, 100, 260], [-5, 100, 200]):
        with pytest.raises(ValueError, match="cu_seqlens"):
            chunk_gated_delta_rule(q, k, v, g, b, cu_seqlens=torch.tensor(bad))


@pytest.mark.gpu
@pytest.mark.parametrize("fn_name", ["chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule"])
def test_bad_device_cu_seqlens_is_skipped_and_reported(dev, fn_name):
    """Sequence 1's end lies beyond the packed tokens: the kernel records DK_ERR_DEVICE_CHECK and
    skips it; the valid sequences keep their bits."""
    import torch

    from detkernels_b200 import _lib
    from detkernels_b200.kernels import gdn
    fn = getattr(gdn, fn_name)
    q, k, v, g, b = _gdn_inputs(dev, 200)
    good = torch.tensor([0, 80, 150, 200], device=dev)
    bad = torch.tensor([0, 80, 5000, 200], device=dev)     # sequence 1 ends past T, sequence 2 decreases
    o_good, _ = fn(q, k, v, g, b, cu_seqlens=good)
    torch.cuda.synchronize()
    assert _lib.device_status(dev.index, clear=True) == (0, 0)
    o_bad, _ = fn(q, k, v, g, b, cu_seqlens=bad)
    code, detail = _lib.device_status(dev.index, clear=True)
    assert code == _lib.DK_ERR_DEVICE_CHECK and detail == 0x500
    assert torch.equal(o_bad[:, :80], o_good[:, :80])
