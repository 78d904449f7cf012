"""Gated delta rule: the CUDA kernel against the f32 oracle (a restatement of
FLA's naive recurrence) and the FLA-generated golden fixture; the invariance
harness (the reference's gdn/repro.py checks, now asserting bitwise identity);
chunked vs token-by-token agreement."""
import os

import numpy as np
import pytest

from oracle import ops as oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# o is bf16 (one rounding of a value of size ~1) after f32 arithmetic in another
# order than the oracle's: 2^-7 relative plus a small absolute term
O_RTOL, O_ATOL = 2 ** -7, 1e-2
S_RTOL, S_ATOL = 1e-4, 1e-4


def _inputs(dev, lens, H, HV, D, dtype, seed=0, h0=False):
    import torch
    import torch.nn.functional as F
    g = torch.Generator(device=dev).manual_seed(seed)
    T = sum(lens)
    q = torch.randn(1, T, H, D, device=dev, generator=g).to(dtype)
    k = F.normalize(torch.randn(1, T, H, D, device=dev, generator=g), p=2, dim=-1).to(dtype)
    v = torch.randn(1, T, HV, D, device=dev, generator=g).to(dtype)
    gate = F.logsigmoid(torch.randn(1, T, HV, device=dev, generator=g)).to(dtype)
    beta = torch.sigmoid(torch.randn(1, T, HV, device=dev, generator=g)).to(dtype)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), device=dev, dtype=torch.long)
    s0 = 0.1 * torch.randn(len(lens), HV, D, D, device=dev, generator=g) if h0 else None
    return q, k, v, gate, beta, cu, s0


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("mode", ["chunk", "recurrent"])
@pytest.mark.parametrize("D,H,HV,lens", [(32, 2, 4, [1, 7, 63, 64, 65, 130]), (64, 1, 2, [100, 37]),
                                         (128, 2, 4, [129, 5])])
def test_matches_oracle(dev, mode, D, H, HV, lens):
    import torch
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule
    fn = chunk_gated_delta_rule if mode == "chunk" else fused_recurrent_gated_delta_rule
    q, k, v, gate, beta, cu, s0 = _inputs(dev, lens, H, HV, D, torch.bfloat16, seed=D, h0=True)
    o, final = fn(q, k, v, gate, beta, initial_state=s0, output_final_state=True, cu_seqlens=cu)
    want_o, want_s = oracle.gdn_recurrent(_np(q[0]), _np(k[0]), _np(v[0]), _np(gate[0]), _np(beta[0]),
                                          initial_state=_np(s0), cu_seqlens=cu.cpu().numpy(), dtype="float32")
    np.testing.assert_allclose(_np(o[0]), want_o, rtol=O_RTOL, atol=O_ATOL)
    np.testing.assert_allclose(_np(final), want_s, rtol=S_RTOL, atol=S_ATOL)


def test_matches_fla_naive_golden_fixture(dev):
    import torch
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule
    d = np.load(os.path.join(GOLDEN, "gdn.npz"))
    t = {key: torch.from_numpy(d[key]).to(dev) for key in ("q", "k", "v", "g", "beta")}
    bf = {key: t[key].to(torch.bfloat16)[None] for key in t}
    o, final = chunk_gated_delta_rule(bf["q"], bf["k"], bf["v"], bf["g"], bf["beta"],
                                      initial_state=torch.from_numpy(d["h0"]).to(dev), output_final_state=True,
                                      cu_seqlens=torch.from_numpy(d["cu_seqlens"]).to(dev))
    np.testing.assert_allclose(_np(o[0]), d["o"], rtol=O_RTOL, atol=O_ATOL)
    np.testing.assert_allclose(_np(final), d["final"], rtol=S_RTOL, atol=S_ATOL)


@pytest.mark.parametrize("D", [64, 128])
def test_rectangular_batch_equals_packed_bitwise(dev, D):
    """The same sequences as B rows of length T or packed with cu_seqlens: same bits."""
    import torch
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule
    q, k, v, gate, beta, cu, s0 = _inputs(dev, [100] * 3, 2, 4, D, torch.bfloat16, seed=5, h0=True)
    o_p, f_p = chunk_gated_delta_rule(q, k, v, gate, beta, initial_state=s0, output_final_state=True, cu_seqlens=cu)
    r = [x.view(3, 100, *x.shape[2:]) for x in (q, k, v, gate, beta)]
    o_r, f_r = chunk_gated_delta_rule(*r[:3], r[3], r[4], initial_state=s0, output_final_state=True)
    assert torch.equal(o_p.view_as(o_r), o_r) and torch.equal(f_p, f_r)


def test_zero_length_sequences_pass_the_state_through(dev):
    import torch
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule
    q, k, v, gate, beta, cu, s0 = _inputs(dev, [0, 9, 0], 2, 2, 32, torch.bfloat16, seed=6, h0=True)
    o, final = chunk_gated_delta_rule(q, k, v, gate, beta, initial_state=s0, output_final_state=True, cu_seqlens=cu)
    assert torch.equal(final[0], s0[0].float()) and torch.equal(final[2], s0[2].float())


def test_pack_position_does_not_change_a_sequences_bits_d128(dev):
    """A 200-token sequence alone, first in a pack and last in a pack of ragged neighbours (whose
    tokens sit right after / before it in memory): the same output and state bits."""
    import torch
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule
    q, k, v, gate, beta, cu, s0 = _inputs(dev, [37, 200, 131], 2, 4, 128, torch.bfloat16, seed=11, h0=True)
    o, f = chunk_gated_delta_rule(q, k, v, gate, beta, initial_state=s0, output_final_state=True, cu_seqlens=cu)
    sl = slice(37, 237)
    alone = [x[:, sl].contiguous() for x in (q, k, v, gate, beta)]
    o1, f1 = chunk_gated_delta_rule(*alone, initial_state=s0[1:2], output_final_state=True,
                                    cu_seqlens=torch.tensor([0, 200], device=dev))
    assert torch.equal(o1[0], o[0, sl]) and torch.equal(f1[0], f[1])
    # the same sequence moved to the front of another pack
    perm = [x[:, list(range(37, 237)) + list(range(0, 37))].contiguous() for x in (q, k, v, gate, beta)]
    o2, f2 = chunk_gated_delta_rule(*perm, initial_state=torch.stack([s0[1], s0[0]]), output_final_state=True,
                                    cu_seqlens=torch.tensor([0, 200, 237], device=dev))
    assert torch.equal(o2[0, :200], o[0, sl]) and torch.equal(f2[0], f[1])


def test_tcgen05_and_mma_sync_chunk_kernels_agree(dev):
    """The tcgen05 chunk kernel (head dim 128) against the mma.sync one it replaced, both within the
    oracle tolerance of each other (their f32 sums run in different orders)."""
    import ctypes

    import torch

    from detkernels_b200 import _lib
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule
    hook = _lib.load().dk_gdn_kernel_for_test   # a test hook outside the public header
    hook.restype, hook.argtypes = ctypes.c_int, [ctypes.c_int]
    q, k, v, gate, beta, cu, s0 = _inputs(dev, [1, 64, 65, 700, 2000], 4, 8, 128, torch.bfloat16, seed=12, h0=True)
    try:
        hook(1)
        o_old, f_old = chunk_gated_delta_rule(q, k, v, gate, beta, initial_state=s0, output_final_state=True,
                                              cu_seqlens=cu)
    finally:
        hook(0)
    o_new, f_new = chunk_gated_delta_rule(q, k, v, gate, beta, initial_state=s0, output_final_state=True,
                                          cu_seqlens=cu)
    torch.testing.assert_close(o_new.float(), o_old.float(), rtol=O_RTOL, atol=O_ATOL)
    torch.testing.assert_close(f_new, f_old, rtol=S_RTOL, atol=S_ATOL)


def test_chunked_and_recurrent_agree(dev):
    import torch
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule
    q, k, v, gate, beta, cu, _ = _inputs(dev, [300, 77], 4, 8, 128, torch.bfloat16, seed=7)
    o1, s1 = chunk_gated_delta_rule(q, k, v, gate, beta, output_final_state=True, cu_seqlens=cu)
    o2, s2 = fused_recurrent_gated_delta_rule(q, k, v, gate, beta, output_final_state=True, cu_seqlens=cu)
    torch.testing.assert_close(o1.float(), o2.float(), rtol=O_RTOL, atol=O_ATOL)
    torch.testing.assert_close(s1, s2, rtol=1e-3, atol=1e-3)


def test_repro_checks_are_all_bitwise_identical(dev):
    from detkernels_b200.gdn import repro
    dv = str(dev)
    res = repro.check_row_invariance([1, 8, 33], seq_len=80, h=2, hv=4, k_dim=32, v_dim=32, device=dv)
    assert all(c["identical"] and c["max_abs_diff"] == 0.0 for c in res["comparisons"])
    res = repro.check_packing_position_invariance(tracked_seq_len=48, other_seq_lens=(37, 53, 29, 61), device=dv)
    assert len(res["comparisons"]) == 4 and all(c["identical"] for c in res["comparisons"])
    res = repro.check_geometry_invariance(tracked_seq_len=50, other_totals=(0, 500, 2000), device=dv)
    assert all(c["identical"] for c in res["comparisons"])
    res = repro.check_decode_state_drift(n_steps=40, n_other_seqs_options=(0, 7, 63), device=dv)
    assert all(c["identical"] and c["first_diverging_step"] is None for c in res["comparisons"])


def test_repro_cli_writes_the_reference_report(dev, tmp_path):
    import json
    from detkernels_b200.gdn.repro import main
    out = tmp_path / "gdn.json"
    main(["--mode", "all", "--batch-sizes", "1,4", "--seq-len", "40", "--tracked-seq-len", "16",
          "--other-seq-lens", "12,20", "--n-steps", "5", "--n-other-seqs", "0,3", "--other-totals", "0,100",
          "--output", str(out)])
    rep = json.loads(out.read_text())
    for key in ("row_results", "packing_results", "decode_results", "geometry_results"):
        assert rep[key] and all(c["identical"] for r in rep[key] for c in r["comparisons"])


@pytest.mark.parametrize("D", [64, 128])
def test_f16_inputs_match_oracle(dev, D):
    """f16 inputs (the f32 CUDA-core chunk kernel) against the oracle."""
    import torch
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule
    q, k, v, gate, beta, cu, s0 = _inputs(dev, [70, 129], 2, 4, D, torch.float16, seed=11, h0=True)
    o, final = chunk_gated_delta_rule(q, k, v, gate, beta, initial_state=s0, output_final_state=True, cu_seqlens=cu)
    want_o, want_s = oracle.gdn_recurrent(_np(q[0]), _np(k[0]), _np(v[0]), _np(gate[0]), _np(beta[0]),
                                          initial_state=_np(s0), cu_seqlens=cu.cpu().numpy(), dtype="float32")
    np.testing.assert_allclose(_np(o[0]), want_o, rtol=2 ** -9, atol=4e-3)
    np.testing.assert_allclose(_np(final), want_s, rtol=S_RTOL, atol=S_ATOL)
