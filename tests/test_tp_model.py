"""Tensor-parallel TinyModel decoding: bitwise equal to one GPU at TP = 2, 4, 8.

* CPU (gloo ranks): the sharding bookkeeping -- which heads, K slice groups and
  vocabulary columns each rank owns, the rank-order gather and the cross-rank
  argmax -- reproduces the one-process oracle step bit for bit.
* GPU, one process: every rank of a TP group held in one process on one GPU
  (the exchange is a stack), against the TP=1 engine, on ragged prompts and on
  the benchmark model (4 layers, d 1024, 16 x 64, SwiGLU 2816, vocab 32000) for
  128 greedy tokens.
* GPU, NCCL: one process per GPU when two or more GPUs are present.
"""
import os
import socket

import numpy as np
import pytest

from _ranks import collect
from oracle import ops as oracle
from oracle.numerics import round_to

SMALL = dict(vocab_size=1000, num_layers=2, num_heads=8, head_dim=64, mlp_hidden=512, mlp="swiglu",
             dtype="bfloat16", seed=3)
BENCH_MODEL = dict(vocab_size=32000, num_layers=4, num_heads=16, head_dim=64, mlp_hidden=2816, mlp="swiglu",
                   dtype="bfloat16", seed=0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ------------------------------------------------------------------ oracle TP step (CPU) ----
def _f(t):
    return np.ascontiguousarray(t.float().numpy())


def _tree_matmul(a, b):
    """The invariant matmul's f32 arithmetic: 8 K slices, fixed tree, then bf16."""
    parts = [np.ascontiguousarray(p) for p in oracle.matmul_slice_partials(a, b)]
    return round_to(oracle.fold_tree(parts), "bfloat16")


def _group_partial(a_shard, b_shard, K, tp, rank):
    """f32 subtree sum of rank's slice group from its K shard (contiguous slice operands)."""
    from detkernels_b200.kernels import tp as tpm
    b0, b1 = tpm.slice_group(tp, rank)
    k0, _ = tpm.shard_k_range(K, tp, rank)
    L = oracle.slice_len(K)
    parts = []
    for s in range(b0, b1):
        lo, hi = min(s * L, K) - k0, min((s + 1) * L, K) - k0
        if hi > lo:
            parts.append(np.ascontiguousarray(a_shard[:, lo:hi]) @ np.ascontiguousarray(b_shard[lo:hi]))
        else:
            parts.append(np.zeros((a_shard.shape[0], b_shard.shape[1]), np.float32))
    return oracle.fold_tree(parts)


def _full_partial(a, b):
    """The same subtree sums of the full operands (slices cut from the full matrices)."""
    K = a.shape[1]
    L = oracle.slice_len(K)
    parts = []
    for s in range(8):
        lo, hi = min(s * L, K), min((s + 1) * L, K)
        parts.append(np.ascontiguousarray(a[:, lo:hi]) @ np.ascontiguousarray(b[lo:hi]) if hi > lo
                     else np.zeros((a.shape[0], b.shape[1]), np.float32))
    return round_to(oracle.fold_tree(parts), "bfloat16")


def _argmax_key(row, col_offset):
    """(value, -global column) of a row's first maximum: larger is better across ranks."""
    j = int(np.argmax(row))
    return (float(row[j]), -(j + col_offset))


def _step(model, tokens, shard=None, gather=None):
    """One decode step from empty caches over the oracle; shard=(layout, rank) runs one
    rank's part of every layer with ``gather`` exchanging its partials in rank order."""
    from detkernels_b200.kernels.tp_model import shard_weights
    cfg = model.config
    H, D, eps = cfg.num_heads, cfg.head_dim, cfg.eps
    x = _f(model.embed)[np.asarray(tokens)]
    B = len(tokens)
    if shard is not None:
        layout, rank = shard
        sw = shard_weights(model, layout, rank)
        Hl = layout.Hl
    for li, L in enumerate(model.layers):
        xn = oracle.rmsnorm(x, _f(L["norm1_w"]), eps, "bfloat16")
        if shard is None:
            q = _tree_matmul(xn, _f(L["w_q"])).reshape(B, H, D)
            v = _tree_matmul(xn, _f(L["w_v"])).reshape(B, cfg.kv_heads, D)
            # one token per sequence: attention of a length-1 cache returns v (per kv head)
            attn = np.repeat(v, H // cfg.kv_heads, axis=1).reshape(B, H * D)
            o = _full_partial(attn, _f(L["w_o"]))
        else:
            w = sw["layers"][li]
            qkv = _tree_matmul(xn, _f(w["w_qkv"]))
            Hkvl = layout.Hkvl
            v = qkv[:, (Hl + Hkvl) * D:].reshape(B, Hkvl, D)
            attn = np.repeat(v, Hl // Hkvl, axis=1).reshape(B, Hl * D)
            part = _group_partial(attn, _f(w["w_o"]), layout.h, layout.tp, rank)
            o = round_to(oracle.fold_tree(gather(part)), "bfloat16")
        x = round_to(x + o, "bfloat16")
        xn2 = oracle.rmsnorm(x, _f(L["norm2_w"]), eps, "bfloat16")
        if shard is None:
            g = round_to(oracle.silu(_tree_matmul(xn2, _f(L["w_gate"]))), "bfloat16")
            hid = round_to(g * _tree_matmul(xn2, _f(L["w_up"])), "bfloat16")
            down = _full_partial(hid, _f(L["w_mlp2"]))
        else:
            gu = _tree_matmul(xn2, _f(w["w_gu"]))
            hid = round_to(round_to(oracle.silu(gu[:, 0::2]), "bfloat16") * gu[:, 1::2], "bfloat16")
            part = _group_partial(hid, _f(w["w_mlp2"]), layout.F, layout.tp, rank)
            down = round_to(oracle.fold_tree(gather(part)), "bfloat16")
        x = round_to(x + down, "bfloat16")
    xf = oracle.rmsnorm(x, _f(model.norm_f_w), eps, "bfloat16")
    if shard is None:
        logits = _tree_matmul(xf, _f(model.w_lm_head))
        return x, [int(np.argmax(r)) for r in logits]
    logits = _tree_matmul(xf, _f(sw["w_lm_head"]))
    off = layout.vocab_offsets[rank]
    keys = [_argmax_key(r, off) for r in logits]
    every = gather(keys)                       # [tp][B] keys in rank order
    toks = [-max(every[p][b] for p in range(layout.tp))[1] for b in range(B)]
    return x, toks


def _gloo_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    from detkernels_b200.kernels.tp_model import TPLayout
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        model = TinyModel(TinyModelConfig(**SMALL), device="cpu")
        layout = TPLayout(model.config, world)

        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        tokens = [5, 999, 0, 321, 321]
        x, toks = _step(model, tokens, (layout, rank), gather)
        q.put((rank, x, toks))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_reproduce_the_one_process_step(world):
    import torch.multiprocessing as mp

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(collect(q, procs, world, 240), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    model = TinyModel(TinyModelConfig(**SMALL), device="cpu")
    x1, toks1 = _step(model, [5, 999, 0, 321, 321])
    for rank, x, toks in res:
        assert np.array_equal(x, x1), rank
        assert toks == toks1, rank


def test_layout_rejects_sizes_that_miss_the_slice_groups():
    from detkernels_b200.kernels.tiny_model import TinyModelConfig
    from detkernels_b200.kernels.tp_model import TPLayout
    with pytest.raises(ValueError):
        TPLayout(TinyModelConfig(**dict(SMALL, num_heads=6)), 4)     # heads not divisible
    with pytest.raises(ValueError):
        TPLayout(TinyModelConfig(**dict(SMALL, num_heads=12, head_dim=40)), 8)  # K slices cut heads
    with pytest.raises(ValueError):
        TPLayout(TinyModelConfig(**SMALL), 3)
    lay = TPLayout(TinyModelConfig(**BENCH_MODEL), 8)
    assert lay.hidden(7) == (7 * 352, 2816) and lay.vocab_offsets == [4000 * r for r in range(8)]


# ------------------------------------------------------------------ GPU, one process ----
def _prompts(n, vocab, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, int(rng.integers(1, 70))).tolist() for _ in range(n)]


@pytest.mark.gpu
@pytest.mark.parametrize("use_graph", [False, True])
def test_emulated_tp_equals_one_gpu(dev, use_graph):
    import torch

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    model = TinyModel(TinyModelConfig(**SMALL), device=str(dev))
    prompts = _prompts(9, SMALL["vocab_size"], 1)
    want = model.engine(9, 100, use_graph=use_graph).generate(prompts, 20)
    for tp in (2, 4, 8):
        got = model.tp_engine(tp, 9, 100, use_graph=use_graph).generate(prompts, 20)
        torch.cuda.synchronize()
        assert torch.equal(got, want), tp


@pytest.mark.gpu
def test_emulated_tp_with_spare_batch_capacity(dev):
    """An engine built for more rows than the call's prompts (the serving case): the prefill's
    greedy step gathers only the prompts' argmax keys and the tokens equal one GPU's."""
    import torch

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    model = TinyModel(TinyModelConfig(**SMALL), device=str(dev))
    prompts = _prompts(5, SMALL["vocab_size"], 3)
    want = model.engine(5, 100).generate(prompts, 12)
    for tp in (2, 4):
        got = model.tp_engine(tp, 11, 100).generate(prompts, 12)
        torch.cuda.synchronize()
        assert torch.equal(got, want), tp


@pytest.mark.gpu
def test_emulated_tp_on_the_benchmark_model_128_tokens(dev):
    """The benchmark model's tracked 32-token prompt among 7 ragged prompts: 128 greedy tokens
    at TP = 2, 4, 8 equal TP = 1's for every row."""
    import torch

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    model = TinyModel(TinyModelConfig(**BENCH_MODEL), device=str(dev))
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 32000, 32).tolist()] + [rng.integers(0, 32000, int(rng.integers(16, 513))).tolist()
                                                       for _ in range(7)]
    want = model.generate(prompts, 128, "batch_invariant")
    for tp in (2, 4, 8):
        got = model.generate(prompts, 128, "batch_invariant", tp=tp)
        torch.cuda.synchronize()
        assert torch.equal(got, want), tp


@pytest.mark.gpu
def test_fold_fused_epilogues_match_the_fused_gemm(dev):
    """Gathered shard partials folded with an epilogue == the one-GPU fused matmul's bits."""
    import torch

    from detkernels_b200.kernels import tp as tpm
    from detkernels_b200.kernels.matmul import argmax_finish, argmax_finish_parts, matmul_fold_fused, matmul_fused
    g = torch.Generator(device=dev).manual_seed(4)
    M, K, N = 37, 2816, 1024
    a = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(K, N, device=dev, generator=g)).to(torch.bfloat16)
    r = torch.randn(M, N, device=dev, generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(N, device=dev, generator=g)).to(torch.bfloat16)
    want_n = torch.empty_like(r)
    want = matmul_fused(a, b, "residual_rmsnorm", residual=r, norm_weight=nw, norm_out=want_n)
    for tp in (1, 2, 4, 8):
        parts = []
        for rk in range(tp):
            k0, k1 = tpm.shard_k_range(K, tp, rk)
            parts.append(tpm.shard_partial(a[:, k0:k1].contiguous(), b[k0:k1].contiguous(), K, tp, rk))
        got_n = torch.empty_like(r)
        got = matmul_fold_fused(torch.stack(parts), torch.bfloat16, "residual_rmsnorm", residual=r, norm_weight=nw,
                                norm_out=got_n)
        assert torch.equal(got, want) and torch.equal(got_n, want_n), tp
    # column-parallel argmax: vocabulary split over parts, ties broken toward the lowest column
    V = 1000
    w = (0.02 * torch.randn(K, V, device=dev, generator=g)).to(torch.bfloat16)
    w[:, 600] = w[:, 100]            # an exact tie across two parts
    keys = torch.zeros(M, dtype=torch.int64, device=dev)
    matmul_fused(a, w, "argmax", argmax_keys=keys)
    want_t = torch.empty(M, dtype=torch.int64, device=dev)
    argmax_finish(keys, want_t)
    assert torch.equal(want_t, matmul_fused(a, w).argmax(dim=-1))
    for tp in (2, 4, 8):
        offs = [tpm.shard_n_range(V, tp, rk)[0] for rk in range(tp)]
        ks = []
        for rk in range(tp):
            n0, n1 = tpm.shard_n_range(V, tp, rk)
            kk = torch.zeros(M, dtype=torch.int64, device=dev)
            matmul_fused(a, w[:, n0:n1].contiguous(), "argmax", argmax_keys=kk)
            ks.append(kk)
        got_t = torch.empty(M, dtype=torch.int64, device=dev)
        argmax_finish_parts(torch.stack(ks), offs, got_t, reset_keys=ks[0])
        assert torch.equal(got_t, want_t), tp
        assert int(ks[0].count_nonzero()) == 0


# ------------------------------------------------------------------ NCCL ----
def _nccl_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    try:
        dev = torch.device("cuda", rank)
        model = TinyModel(TinyModelConfig(**BENCH_MODEL), device=str(dev))
        rng = np.random.default_rng(0)
        prompts = [rng.integers(0, 32000, 32).tolist()] + [rng.integers(0, 32000, int(rng.integers(16, 513))).tolist()
                                                           for _ in range(7)]
        got = model.generate(prompts, 128, "batch_invariant", tp=world, group=dist.group.WORLD).cpu()
        want = model.generate(prompts, 128, "batch_invariant").cpu()
        model._engines.clear()   # release graphs holding NCCL calls before the group goes
        torch.cuda.synchronize()
        q.put((rank, bool(torch.equal(got, want))))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_tp_decode_equals_one_gpu():
    import torch
    import torch.multiprocessing as mp
    n = min(torch.cuda.device_count(), 8)
    world = 1 << (n.bit_length() - 1) if n else 0
    if world < 2:
        pytest.skip("needs two or more GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = collect(q, procs, world, 600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok in res), res
