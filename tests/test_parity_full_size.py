"""Parity with the oracle at the configured (full) sizes, not only small cases.

* Gated delta rule: 4 packed sequences of 2048-4096 tokens, 16 q/k heads and 32
  value heads of dim 128 through the chunked kernel (64 chained chunks of state
  for the longest), against the f64 recurrence on a subset of value heads; then
  300 token-by-token decode steps from the kernel's own final state against the
  oracle continuing from its own.
* Decode attention: 8 rows, 32 query / 8 kv heads of dim 128, KV lengths up to
  8192 (32 splits of 256 merged online) against the f32 oracle.
* TinyModel: the benchmark model (4 layers, d 1024, 16 x 64, SwiGLU 2816, vocab
  32000, bf16) decoding 128 greedy tokens for the tracked 32-token prompt and 7
  ragged prompts of 16-512 tokens.  The oracle is teacher-forced with the
  kernel's tokens: at every one of the 1024 steps the kernel's token must be
  within NEAR_TIE of the oracle's largest logit (its argmax up to a near-tie),
  so each row equals the free-running oracle up to its first near-tie.  With
  32000 bf16 logits such ties are common (margins of 0 or 1 ulp were seen at the
  first difference of every row), so rows may part after one.
"""
import numpy as np
import pytest

from oracle import ops as oracle

pytestmark = pytest.mark.gpu

# gdn: o is bf16 (2^-7 relative plus an absolute term for values near zero); the f32 state
# against the f64 recurrence after up to 4096 tokens
O_RTOL, O_ATOL = 2 ** -7, 1e-2
S_RTOL, S_ATOL = 1e-4, 1e-4
# attention output is bf16: 2^-6 relative and absolute
A_TOL = 2 ** -6
# a greedy step whose oracle top-2 logits differ by less than this (4 bf16 ulps at 2.0) is a near-tie
NEAR_TIE = 4 * 2 ** -6


def _np(t):
    return t.float().cpu().numpy()


def test_gdn_chunked_4096_tokens_and_300_decode_steps(dev):
    import torch
    import torch.nn.functional as F

    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule
    lens = [4096, 2048, 3000, 2500]
    H, HV, D = 16, 32, 128
    heads = [0, 9, 22, 31]
    T = sum(lens)
    g = torch.Generator(device=dev).manual_seed(17)
    q = F.normalize(torch.randn(1, T, H, D, device=dev, generator=g), p=2, dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(1, T, H, D, device=dev, generator=g), p=2, dim=-1).to(torch.bfloat16)
    v = torch.randn(1, T, HV, D, device=dev, generator=g).to(torch.bfloat16)
    gate = F.logsigmoid(torch.randn(1, T, HV, device=dev, generator=g)).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(1, T, HV, device=dev, generator=g)).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), device=dev, dtype=torch.long)
    o, final = chunk_gated_delta_rule(q, k, v, gate, beta, output_final_state=True, cu_seqlens=cu)
    want_o, want_s = oracle.gdn_recurrent(_np(q[0]), _np(k[0]), _np(v[0]), _np(gate[0]), _np(beta[0]),
                                          cu_seqlens=cu.cpu().numpy(), dtype="float32", acc=np.float64,
                                          v_heads=heads)
    got_o = _np(o[0])[:, heads]
    got_s = _np(final)[:, heads]
    err_o = np.abs(got_o - want_o[:, heads]).max()
    err_s = np.abs(got_s - want_s[:, heads]).max()
    np.testing.assert_allclose(got_o, want_o[:, heads], rtol=O_RTOL, atol=O_ATOL, err_msg="o, max err %g" % err_o)
    np.testing.assert_allclose(got_s, want_s[:, heads], rtol=S_RTOL, atol=S_ATOL,
                               err_msg="state, max err %g" % err_s)

    # 300 decode steps of the same 4 sequences, each from its own state
    N, steps = len(lens), 300
    dq = F.normalize(torch.randn(steps, N, 1, H, D, device=dev, generator=g), p=2, dim=-1).to(torch.bfloat16)
    dk = F.normalize(torch.randn(steps, N, 1, H, D, device=dev, generator=g), p=2, dim=-1).to(torch.bfloat16)
    dv = torch.randn(steps, N, 1, HV, D, device=dev, generator=g).to(torch.bfloat16)
    dg = F.logsigmoid(torch.randn(steps, N, 1, HV, device=dev, generator=g)).to(torch.bfloat16)
    db = torch.sigmoid(torch.randn(steps, N, 1, HV, device=dev, generator=g)).to(torch.bfloat16)
    state = final
    outs = []
    for t in range(steps):
        o_t, state = fused_recurrent_gated_delta_rule(dq[t], dk[t], dv[t], dg[t], db[t], initial_state=state,
                                                      output_final_state=True)
        outs.append(o_t[:, 0])
    got_dec = _np(torch.stack(outs))[:, :, heads]             # [steps, N, heads, D]
    o_state = want_s
    cu_step = np.arange(N + 1)
    worst = 0.0
    for t in range(steps):
        o_ref, o_state = oracle.gdn_recurrent(_np(dq[t, :, 0]), _np(dk[t, :, 0]), _np(dv[t, :, 0]),
                                              _np(dg[t, :, 0]), _np(db[t, :, 0]), initial_state=o_state,
                                              cu_seqlens=cu_step, dtype="float32", acc=np.float64, v_heads=heads)
        worst = max(worst, float(np.abs(got_dec[t] - o_ref[:, heads]).max()))
        np.testing.assert_allclose(got_dec[t], o_ref[:, heads], rtol=O_RTOL, atol=O_ATOL,
                                   err_msg="decode step %d" % t)
    np.testing.assert_allclose(_np(state)[:, heads], o_state[:, heads], rtol=S_RTOL, atol=S_ATOL,
                               err_msg="state after %d decode steps (max o err %g)" % (steps, worst))


def test_decode_attention_to_8192_tokens(dev):
    import torch

    from detkernels_b200.kernels.attention import attention_batch_invariant
    B, H, Hkv, D, S = 8, 32, 8, 128, 8192
    g = torch.Generator(device=dev).manual_seed(23)
    q = torch.randn(B, H, D, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, device=dev, generator=g).to(torch.bfloat16)
    lens = torch.randint(128, S + 1, (B,), device=dev, generator=g)
    lens[0] = S
    lens[1] = 128
    lens[2] = 257
    got = attention_batch_invariant(q, k, v, kv_lens=lens)
    want = oracle.attention(_np(q), _np(k), _np(v), kv_lens=lens.cpu().numpy())
    np.testing.assert_allclose(_np(got), want, rtol=A_TOL, atol=A_TOL)


def test_tinymodel_128_token_decode_matches_the_oracle_to_the_first_near_tie(dev):
    import torch

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    cfg = TinyModelConfig(vocab_size=32000, num_layers=4, num_heads=16, head_dim=64, mlp_hidden=2816, mlp="swiglu",
                          dtype="bfloat16", seed=0)
    model = TinyModel(cfg, device=str(dev))
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 32000, 32).tolist()] + [rng.integers(0, 32000, int(rng.integers(16, 513))).tolist()
                                                       for _ in range(7)]
    got = model.generate(prompts, 128, "batch_invariant").cpu().numpy()

    def f(t):
        return t.float().cpu().numpy()

    w = {"embed": f(model.embed), "layers": [{kk: f(vv) for kk, vv in L.items()} for L in model.layers],
         "norm_f_w": f(model.norm_f_w), "w_lm_head": f(model.w_lm_head)}
    orc = oracle.TinyModelOracle(w, 16, 16, 64, mlp="swiglu", dtype="bfloat16")
    regrets = []
    want, _ = orc.generate(prompts, 128, follow=got, regrets=regrets)
    regrets = np.asarray(regrets)
    agree = got == want
    first = [int(np.argmin(np.append(row, False))) for row in agree]
    print("kernel token == oracle argmax at %d of %d teacher-forced steps; worst regret %g; first difference "
          "per row %s with regrets %s" % (int(agree.sum()), agree.size, float(regrets.max()), first,
                                          [float(regrets[b, t]) if t < 128 else None for b, t in enumerate(first)]))
    assert regrets.max() < NEAR_TIE, (regrets.max(), np.argwhere(regrets >= NEAR_TIE)[:10])
    assert agree[0, :first[0]].all() and first[0] >= 1
