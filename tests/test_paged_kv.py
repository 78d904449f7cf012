"""Paged KV cache: decode attention and the serving engine over a block pool with a
block table give the bits of the contiguous cache, for every page size.

No counterpart in the reference, which grows one contiguous KV tensor per layer
with torch.cat (kernels/tiny_model.py:119-125) and lists paging as a
simplification (kernels/attention.py:35-40).
"""
import numpy as np
import pytest


def test_block_allocator_hands_out_distinct_blocks_and_reports_exhaustion():
    from detkernels_b200.kernels.tiny_model import BlockAllocator
    al = BlockAllocator(n_blocks=40, max_slots=6, blocks_per_seq=8)
    table = al.assign([1, 64, 65, 300, 0], 64)
    used = [int(x) for row, n in zip(table, [1, 1, 2, 5, 0]) for x in row[:n]]
    assert len(used) == len(set(used)) == 9 and 0 not in used
    assert (table[4] == 0).all() and (table[5] == 0).all()       # no tokens / no sequence: block 0
    assert max(used) < 40
    with pytest.raises(RuntimeError, match="exhausted"):
        al.assign([512] * 5, 64)                                  # 40 blocks needed, 39 available
    with pytest.raises(ValueError):
        al.assign([600], 64)                                      # more than 8 blocks per sequence


def _to_pages(k, lens, page, rng):
    """[n_seq, Hkv, S, D] -> (pool [n_blocks, Hkv, page, D], table [n_seq, S // page]) with the
    blocks of all sequences scattered in a random order and unused blocks filled with noise."""
    import torch
    n_seq, hkv, S, D = k.shape
    per = S // page
    n_blocks = n_seq * per + 3
    order = rng.permutation(n_blocks)
    table = torch.tensor(order[:n_seq * per].reshape(n_seq, per), dtype=torch.int32, device=k.device)
    pool = torch.randn(n_blocks, hkv, page, D, device=k.device).to(k.dtype)   # noise where nothing lives
    for s in range(n_seq):
        for b in range(per):
            pool[table[s, b]] = k[s, :, b * page:(b + 1) * page]
    return pool, table


@pytest.mark.gpu
@pytest.mark.parametrize("page", [64, 128, 256, 512])
@pytest.mark.parametrize("H,Hkv,D", [(32, 8, 128), (16, 16, 64)])
def test_paged_attention_equals_contiguous(dev, page, H, Hkv, D):
    import torch

    from detkernels_b200.kernels.attention import attention_decode
    rng = np.random.default_rng(page + D)
    g = torch.Generator(device=dev).manual_seed(page)
    n_seq, S = 6, 2048
    q = torch.randn(n_seq, H, D, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(n_seq, Hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(n_seq, Hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
    lens = torch.tensor([1, 63, 64, 257, 1500, 2048], dtype=torch.int32, device=dev)
    want = attention_decode(q, k, v, lens, max_kv_len=S)
    kp, table = _to_pages(k, lens, page, rng)
    vp = torch.empty_like(kp)
    vp.copy_(kp)
    for s in range(n_seq):
        for b in range(S // page):
            vp[table[s, b]] = v[s, :, b * page:(b + 1) * page]
    got = attention_decode(q, kp, vp, lens, max_kv_len=S, block_table=table)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_paged_attention_rejects_a_page_that_is_not_a_multiple_of_64(dev):
    import torch

    from detkernels_b200.kernels.attention import attention_decode
    q = torch.zeros(1, 8, 64, device=dev, dtype=torch.bfloat16)
    pool = torch.zeros(4, 8, 96, 64, device=dev, dtype=torch.bfloat16)
    table = torch.zeros(1, 2, dtype=torch.int32, device=dev)
    with pytest.raises(ValueError, match="multiple of 64"):
        attention_decode(q, pool, pool, torch.ones(1, dtype=torch.int32, device=dev), block_table=table)


@pytest.mark.gpu
def test_paged_attention_reports_a_table_entry_outside_the_pool(dev):
    import torch

    from detkernels_b200 import _lib
    from detkernels_b200.kernels.attention import attention_decode
    q = torch.randn(1, 8, 64, device=dev).to(torch.bfloat16)
    pool = torch.randn(4, 8, 64, 64, device=dev).to(torch.bfloat16)
    table = torch.tensor([[1, 9]], dtype=torch.int32, device=dev)      # block 9 is not in the pool
    attention_decode(q, pool, pool, torch.tensor([100], dtype=torch.int32, device=dev), block_table=table)
    code, detail = _lib.device_status(dev.index, clear=True)
    assert code == _lib.DK_ERR_DEVICE_CHECK and detail == 0x212


@pytest.mark.gpu
@pytest.mark.parametrize("page", [64, 256])
def test_paged_engine_equals_contiguous_engine(dev, page):
    """The serving engine with a paged pool (blocks scattered by the allocator) generates the
    contiguous engine's tokens for ragged prompts, with and without CUDA graphs."""
    import torch

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    cfg = TinyModelConfig(vocab_size=2000, num_layers=2, num_heads=8, head_dim=64, mlp_hidden=512, mlp="swiglu",
                          dtype="bfloat16", seed=5, num_kv_heads=2)
    model = TinyModel(cfg, device=str(dev))
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 2000, int(rng.integers(1, 400))).tolist() for _ in range(11)]
    want = model.generate(prompts, 40, "batch_invariant")
    got = model.generate(prompts, 40, "batch_invariant", kv_page_size=page)
    assert torch.equal(got, want)
    eng = model.engine(11, 440, use_graph=False, page_size=page)
    assert torch.equal(eng.generate(prompts, 40), want)
    # a second batch through the same engine reuses the pool
    prompts2 = [rng.integers(0, 2000, int(rng.integers(1, 300))).tolist() for _ in range(5)]
    assert torch.equal(model.generate(prompts2, 40, "batch_invariant", kv_page_size=page),
                       model.generate(prompts2, 40, "batch_invariant"))


@pytest.mark.gpu
def test_paged_engine_on_the_benchmark_model(dev):
    """The benchmark model's tracked prompt among 255 ragged prompts: 128 tokens, paged (64-token
    blocks) == contiguous for every row."""
    import torch

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    cfg = TinyModelConfig(vocab_size=32000, num_layers=4, num_heads=16, head_dim=64, mlp_hidden=2816, mlp="swiglu",
                          dtype="bfloat16", seed=0)
    model = TinyModel(cfg, device=str(dev))
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 32000, 32).tolist()] + [rng.integers(0, 32000, int(rng.integers(16, 513))).tolist()
                                                       for _ in range(255)]
    want = model.generate(prompts, 128, "batch_invariant")
    got = model.generate(prompts, 128, "batch_invariant", kv_page_size=64)
    assert torch.equal(got, want)
