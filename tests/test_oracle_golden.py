"""CPU: the oracle against golden fixtures produced by the reference's own code
(tests/golden/make_golden.py), and this library's drop-in TinyModel against
the reference's TinyModel on the same fixtures."""
import os

import numpy as np
import pytest

from oracle import ops as oracle
from oracle.numerics import round_to, ulp_distance_bf16

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def _close_16bit(got, want, dtype):
    """At most one unit in the last place of the 16-bit type apart."""
    if dtype == "bfloat16":
        assert np.max(ulp_distance_bf16(got, want)) <= 1
    elif dtype == "float16":
        g16 = got.astype(np.float16).view(np.int16).astype(np.int64)
        w16 = want.astype(np.float16).view(np.int16).astype(np.int64)
        assert np.max(np.abs(g16 - w16)) <= 1
    else:
        np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-6)


def test_rmsnorm_oracle_matches_reference_fixtures():
    d = load("rmsnorm")
    for i in range(4):
        dt = str(d["dtype%d" % i])
        got = oracle.rmsnorm(d["x%d" % i], d["w%d" % i], 1e-6, dt)
        _close_16bit(got, d["y%d" % i], dt)


def test_matmul_oracle_matches_reference_fixtures():
    d = load("matmul")
    for i in range(4):
        dt = str(d["dtype%d" % i])
        got = oracle.matmul(d["a%d" % i], d["b%d" % i], dt)
        _close_16bit(got, d["c%d" % i], dt)


def test_attention_oracle_matches_reference_fixtures():
    d = load("attention")
    for i in range(3):
        dt = str(d["dtype%d" % i])
        got = oracle.attention(d["q%d" % i], d["k%d" % i], d["v%d" % i], dtype=dt)
        _close_16bit(got, d["o%d" % i], dt)


def _tiny_weights(d, n_layers=2):
    layers = []
    for li in range(n_layers):
        layers.append({key.split("_", 1)[1]: d[key] for key in d.files if key.startswith("L%d_" % li)})
    return {"embed": d["embed"], "layers": layers, "norm_f_w": d["norm_f_w"], "w_lm_head": d["w_lm_head"]}


def test_tiny_model_oracle_matches_reference_fixture():
    d = load("tiny_model")
    orc = oracle.TinyModelOracle(_tiny_weights(d), 2, 2, 32, mlp="silu", dtype="float16")
    caches = orc.empty_caches(3)
    for step in range(3):
        logits = orc.step(d["tokens%d" % step], caches)
        np.testing.assert_allclose(logits, d["logits%d" % step], rtol=2e-3, atol=2e-4)
        assert np.array_equal(np.argmax(logits, -1), np.argmax(d["logits%d" % step], -1))


def test_drop_in_tiny_model_weights_and_reference_path_match_fixture():
    """Same config and seed -> the reference's weights; forward_step with the
    torch reference formulas reproduces the reference's logits bit for bit."""
    import torch

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig

    d = load("tiny_model")
    cfg = TinyModelConfig(vocab_size=64, num_layers=2, num_heads=2, head_dim=32, mlp_hidden=128, seed=0)
    model = TinyModel(cfg, device="cpu")
    assert np.array_equal(model.embed.float().numpy(), d["embed"])
    for li, layer in enumerate(model.layers):
        for key, val in layer.items():
            assert np.array_equal(val.float().numpy(), d["L%d_%s" % (li, key)]), (li, key)
    kv = [None] * cfg.num_layers
    for step in range(3):
        logits, kv = model.forward_step(torch.as_tensor(d["tokens%d" % step]), kv, "reference")
        assert np.array_equal(logits.float().numpy(), d["logits%d" % step])


def test_gdn_oracle_matches_fla_naive_fixture():
    d = load("gdn")
    o, final = oracle.gdn_recurrent(d["q"], d["k"], d["v"], d["g"], d["beta"], initial_state=d["h0"],
                                    cu_seqlens=d["cu_seqlens"], dtype="float32")
    np.testing.assert_allclose(o, d["o"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(final, d["final"], rtol=1e-4, atol=1e-5)


def test_round_bf16_is_round_to_nearest_even():
    import torch
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    x[:4] = [1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -0.0, 65504.0]
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(round_to(x, "bfloat16"), want)
