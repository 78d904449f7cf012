"""Decode attention: the reference's test pattern (tests/test_attention.py),
oracle parity with GQA and ragged KV lengths, the headline invariance config
(q [B, 32, 128], 8 kv heads, L ~ U[128, 8192], B in {1, 8, 64, 256}), and
prefill row tiles reproducing decode rows bit for bit."""
import numpy as np
import pytest

from oracle import ops as oracle

pytestmark = pytest.mark.gpu


def _random_qkv(dev, b, h, s, d, dtype, seed=0, hkv=None):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    hkv = h if hkv is None else hkv
    q = torch.randn(b, h, d, device=dev, dtype=dtype, generator=g)
    k = torch.randn(b, hkv, s, d, device=dev, dtype=dtype, generator=g)
    v = torch.randn(b, hkv, s, d, device=dev, dtype=dtype, generator=g)
    return q, k, v


def test_batch_invariant_matches_reference(dev):
    import torch
    from detkernels_b200.kernels.attention import attention_batch_invariant, attention_reference
    q, k, v = _random_qkv(dev, 8, 4, 128, 64, torch.float16)
    torch.testing.assert_close(attention_batch_invariant(q, k, v), attention_reference(q, k, v),
                               atol=2e-2, rtol=2e-2)


def test_batch_variant_matches_reference(dev):
    import torch
    from detkernels_b200.kernels.attention import attention_batch_variant, attention_reference
    for (b, h) in ((1, 1), (8, 4)):
        q, k, v = _random_qkv(dev, b, h, 128, 64, torch.float16, seed=1)
        torch.testing.assert_close(attention_batch_variant(q, k, v), attention_reference(q, k, v),
                                   atol=2e-2, rtol=2e-2)


def _oracle(q, k, v, kv_lens=None, dtype_name="bfloat16"):
    lens = None if kv_lens is None else kv_lens.cpu().numpy()
    return oracle.attention(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                            kv_lens=lens, dtype=dtype_name)


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16"])
@pytest.mark.parametrize("cfg", [
    # (B, H, Hkv, S, D)
    (2, 32, 8, 1000, 128),
    (3, 16, 16, 300, 64),
    (4, 4, 4, 129, 32),
    (1, 8, 1, 2049, 128),
    (5, 16, 4, 64, 64),
    (2, 2, 2, 1, 32),
])
def test_matches_oracle(dev, dtype_name, cfg):
    """Error vs the f32 oracle below 2 output ulps of the output scale (the
    kernel rounds probabilities to the input type for P.V, like FlashAttention)."""
    import torch
    from detkernels_b200.kernels.attention import attention_batch_invariant
    B, H, Hkv, S, D = cfg
    dtype = getattr(torch, dtype_name)
    q, k, v = _random_qkv(dev, B, H, S, D, dtype, seed=S + D, hkv=Hkv)
    got = attention_batch_invariant(q, k, v).float().cpu().numpy()
    want = _oracle(q, k, v, dtype_name=dtype_name)
    tol = 2 ** -6 if dtype_name == "bfloat16" else 2 ** -8
    np.testing.assert_allclose(got, want, rtol=tol, atol=tol)


@pytest.mark.parametrize("D,H,Hkv", [(128, 32, 8), (64, 16, 16)])
def test_ragged_lengths_match_oracle(dev, D, H, Hkv):
    import torch
    from detkernels_b200.kernels.attention import attention_batch_invariant
    B, S = 6, 1300
    q, k, v = _random_qkv(dev, B, H, S, D, torch.bfloat16, seed=5, hkv=Hkv)
    lens = torch.tensor([1, 255, 256, 257, 1300, 700], dtype=torch.int32, device=dev)
    # poison the cache beyond each row's length: it must never be read into the result
    for b in range(B):
        k[b, :, int(lens[b]):] = float("nan")
        v[b, :, int(lens[b]):] = float("nan")
    got = attention_batch_invariant(q, k, v, kv_lens=lens)
    assert not torch.isnan(got).any()
    kk, vv = k.clone(), v.clone()
    kk[torch.isnan(kk)] = 0
    vv[torch.isnan(vv)] = 0
    want = _oracle(q, kk, vv, kv_lens=lens)
    np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=2 ** -6, atol=2 ** -6)


def test_zero_length_rows_give_zeros(dev):
    import torch
    from detkernels_b200.kernels.attention import attention_batch_invariant
    q, k, v = _random_qkv(dev, 3, 8, 600, 64, torch.bfloat16, seed=2)
    lens = torch.tensor([0, 600, 0], dtype=torch.int32, device=dev)
    out = attention_batch_invariant(q, k, v, kv_lens=lens)
    assert (out[0] == 0).all() and (out[2] == 0).all()
    assert not torch.isnan(out[1]).any()


def test_batch_invariant_row_is_identical_regardless_of_batch_size(dev):
    import torch
    from detkernels_b200.kernels.attention import attention_batch_invariant
    s, d = 128, 64
    torch.manual_seed(0)
    q_row = torch.randn(1, 1, d, device=dev, dtype=torch.float16)
    k_row = torch.randn(1, 1, s, d, device=dev, dtype=torch.float16)
    v_row = torch.randn(1, 1, s, d, device=dev, dtype=torch.float16)
    solo_out = attention_batch_invariant(q_row, k_row, v_row)
    q_batch = torch.randn(64, 1, d, device=dev, dtype=torch.float16)
    k_batch = torch.randn(64, 1, s, d, device=dev, dtype=torch.float16)
    v_batch = torch.randn(64, 1, s, d, device=dev, dtype=torch.float16)
    q_batch[0], k_batch[0], v_batch[0] = q_row[0], k_row[0], v_row[0]
    batch_out = attention_batch_invariant(q_batch, k_batch, v_batch)
    assert torch.equal(solo_out[0], batch_out[0])


def test_baseline_config_tracked_sequence_bitwise(dev):
    """q bf16 [B, 32, 128], K/V 8 kv heads x 128, per-sequence L ~ U[128, 8192],
    scale 1/sqrt(128); the tracked sequence's output is bitwise equal whatever
    is co-batched (B in {1, 8, 64, 256}) and wherever it sits."""
    import torch
    from detkernels_b200.kernels.attention import attention_decode
    D, H, Hkv, S = 128, 32, 8, 8192
    g = torch.Generator(device=dev).manual_seed(0)
    L0 = 5000
    q0 = torch.randn(1, H, D, device=dev, generator=g).to(torch.bfloat16)
    k0 = torch.randn(Hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
    v0 = torch.randn(Hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
    ref = None
    for B in (1, 8, 64, 256):
        gb = torch.Generator(device=dev).manual_seed(100 + B)
        q = torch.randn(B, H, D, device=dev, generator=gb).to(torch.bfloat16)
        kc = torch.randn(B, Hkv, S, D, device=dev, generator=gb).to(torch.bfloat16)
        vc = torch.randn(B, Hkv, S, D, device=dev, generator=gb).to(torch.bfloat16)
        lens = torch.randint(128, 8193, (B,), generator=gb, device=dev).to(torch.int32)
        pos = (B * 7) // 11
        q[pos], kc[pos], vc[pos], lens[pos] = q0[0], k0, v0, L0
        out = attention_decode(q, kc, vc, lens, max_kv_len=S)
        if ref is None:
            ref = out[pos].clone()
        assert torch.equal(out[pos], ref), B
        del kc, vc


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float16"])
def test_prefill_row_tiles_reproduce_decode_rows(dev, dtype_name):
    """Rows of one sequence processed as a multi-row tile (prefill) give exactly
    the bits of the same rows processed one per tile (decode).  Without grouped
    query heads the decode launch takes the single-row (transposed) kernel, so this
    also pins that kernel to the 16-row form at d 32, 64 and 128."""
    import torch
    from detkernels_b200.kernels.attention import attention_decode
    dtype = getattr(torch, dtype_name)
    for (H, Hkv, D) in ((16, 16, 64), (32, 8, 128), (8, 8, 32), (8, 8, 128)):
        G = H // Hkv
        rows_per_tile = 16 // G
        S = 700
        g = torch.Generator(device=dev).manual_seed(H + D)
        kc = torch.randn(2, Hkv, S, D, device=dev, generator=g).to(dtype)
        vc = torch.randn(2, Hkv, S, D, device=dev, generator=g).to(dtype)
        # sequence 0: prompt positions 0..299 ; sequence 1: positions 0..S-1 at stride 7
        pos = [list(range(300)), list(range(0, S, 7))]
        rows_seq, rows_len, tiles = [], [], []
        for sq, pl in enumerate(pos):
            for t0 in range(0, len(pl), rows_per_tile):
                chunk = pl[t0:t0 + rows_per_tile]
                tiles.append([len(rows_seq), len(chunk), sq])
                rows_seq += [sq] * len(chunk)
                rows_len += [p + 1 for p in chunk]
        R = len(rows_seq)
        q = torch.randn(R, H, D, device=dev, generator=g).to(dtype)
        lens = torch.tensor(rows_len, dtype=torch.int32, device=dev)
        tiles_t = torch.tensor(tiles, dtype=torch.int32, device=dev)
        out_tiled = attention_decode(q, kc, vc, lens, row_tiles=tiles_t, max_kv_len=S)
        # decode: one row per tile, each reading its own copy of the sequence's cache
        seq_idx = torch.tensor(rows_seq, device=dev)
        k_rows, v_rows = kc[seq_idx].contiguous(), vc[seq_idx].contiguous()
        out_rows = attention_decode(q, k_rows, v_rows, lens, max_kv_len=S)
        assert torch.equal(out_tiled, out_rows), (H, Hkv, D)
        want = oracle.attention(q.float().cpu().numpy(), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                                kv_lens=rows_len, row_seq=rows_seq)
        tol = 2 ** -6 if dtype == torch.bfloat16 else 2 ** -8
        np.testing.assert_allclose(out_tiled.float().cpu().numpy(), want, rtol=tol, atol=tol)


def test_batch_variant_row_can_diverge_across_batch_sizes(dev):
    import torch
    from detkernels_b200.kernels.attention import attention_batch_variant
    torch.manual_seed(0)
    q_row = torch.randn(1, 1, 64, device=dev, dtype=torch.float16)
    k_row = torch.randn(1, 1, 128, 64, device=dev, dtype=torch.float16)
    v_row = torch.randn(1, 1, 128, 64, device=dev, dtype=torch.float16)
    solo_out = attention_batch_variant(q_row, k_row, v_row)
    q_batch = torch.randn(64, 1, 64, device=dev, dtype=torch.float16)
    k_batch = torch.randn(64, 1, 128, 64, device=dev, dtype=torch.float16)
    v_batch = torch.randn(64, 1, 128, 64, device=dev, dtype=torch.float16)
    q_batch[0], k_batch[0], v_batch[0] = q_row[0], k_row[0], v_row[0]
    batch_out = attention_batch_variant(q_batch, k_batch, v_batch)
    assert not torch.isnan(solo_out).any()
    assert not torch.isnan(batch_out).any()


def test_batch_variant_row_diverges_while_invariant_row_does_not(dev):
    """The variant twin splits a lone sequence's KV over four CTAs but not a sequence inside a
    64-sequence batch, so the row's bits change with the batch; the invariant kernel's do not.
    Eight random rows: at least one must differ."""
    import torch
    from detkernels_b200.kernels.attention import attention_batch_invariant, attention_batch_variant
    g = torch.Generator(device=dev).manual_seed(23)
    q = torch.randn(64, 1, 64, device=dev, generator=g).to(torch.float16)
    k = torch.randn(64, 1, 1024, 64, device=dev, generator=g).to(torch.float16)
    v = torch.randn(64, 1, 1024, 64, device=dev, generator=g).to(torch.float16)
    batch_var = attention_batch_variant(q, k, v)
    batch_inv = attention_batch_invariant(q, k, v)
    diverged = 0
    for r in range(8):
        one = [x[r:r + 1].contiguous() for x in (q, k, v)]
        diverged += int(not torch.equal(attention_batch_variant(*one)[0], batch_var[r]))
        assert torch.equal(attention_batch_invariant(*one)[0], batch_inv[r])
    assert diverged > 0
