"""Host-side arithmetic of bench.py's report tables (CPU only): the in-graph decode matmul
table turns per-launch event times into µs per launch, weight bytes streamed and the fraction
of the HBM peak."""
import os
import sys
import types

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _fake_engine(torch, h=1024, qkv=3072, ff=2816, vocab=4096):
    layer = {"w_qkv": torch.zeros(h, qkv, dtype=torch.bfloat16), "w_o": torch.zeros(h, h, dtype=torch.bfloat16),
             "w_gu": torch.zeros(h, 2 * ff, dtype=torch.bfloat16), "w_mlp2": torch.zeros(ff, h, dtype=torch.bfloat16)}
    model = types.SimpleNamespace(w_lm_head=torch.zeros(h, vocab, dtype=torch.bfloat16))
    return types.SimpleNamespace(layers=[layer], model=model)


def test_decode_gemm_table_arithmetic():
    torch = pytest.importorskip("torch")
    import bench
    eng = _fake_engine(torch)
    steps = bench.NEW_TOKENS - 1
    layers = 4
    times = {"qkv": [0.010] * (layers * steps), "o": [0.005] * (layers * steps),
             "gate_up": [0.020] * (layers * steps), "down": [0.008] * (layers * steps),
             "lm_head": [0.050] * steps}
    peaks = {"hbm_gbs": 6650.0}
    t = bench.decode_gemm_table(times, eng, 256, peaks)
    assert set(t) == {"qkv", "o", "gate_up", "down", "lm_head", "per_decode_step_us"}
    q = t["qkv"]
    assert q["launches_per_step"] == layers and q["us"] == 10.0
    assert q["weight_bytes"] == 1024 * 3072 * 2
    assert q["achieved_gbs"] == pytest.approx(1024 * 3072 * 2 / 10e-6 / 1e9, abs=0.05)
    assert q["frac_hbm"] == pytest.approx(q["achieved_gbs"] / 6650.0, abs=1e-4)
    assert q["tflops"] == pytest.approx(2.0 * 256 * 1024 * 3072 / 10e-6 / 1e12, abs=0.05)
    assert t["lm_head"]["launches_per_step"] == 1
    assert t["per_decode_step_us"] == pytest.approx(layers * (10 + 5 + 20 + 8) + 50, rel=1e-3)


def test_decode_gemm_table_skips_unknown_labels_and_empty_lists():
    torch = pytest.importorskip("torch")
    import bench
    t = bench.decode_gemm_table({"qkv": [], "other": [1.0]}, _fake_engine(torch), 256, {"hbm_gbs": 1.0})
    assert t == {"per_decode_step_us": 0.0}
