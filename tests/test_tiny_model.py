"""TinyModel: the reference's tests (tests/test_tiny_model.py), the serving
engine against the reference-style eager loop, oracle parity, and the benchmark
decode config (4 L, d 1024, 16 x 64, SwiGLU 2816, vocab 32000; a tracked
32-token prompt among 0/7/63/255 ragged prompts; 128 greedy tokens)."""
import numpy as np
import pytest

from oracle import ops as oracle

pytestmark = pytest.mark.gpu


def _small_model(dev, **kw):
    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    cfg = TinyModelConfig(vocab_size=64, num_layers=2, num_heads=2, head_dim=32, mlp_hidden=128, seed=0, **kw)
    return TinyModel(cfg, device=str(dev))


def test_generate_produces_well_formed_output_both_kernel_sets(dev):
    import torch
    model = _small_model(dev)
    for kernel_set in ("batch_invariant", "batch_variant"):
        tokens = torch.randint(0, model.config.vocab_size, (8,), device=dev)
        out = model.generate(tokens, n_steps=4, kernel_set=kernel_set)
        assert out.shape == (8, 4)
        assert (out >= 0).all() and (out < model.config.vocab_size).all()


def test_batch_invariant_generation_is_identical_regardless_of_batch_size(dev):
    import torch
    model = _small_model(dev)
    torch.manual_seed(0)
    start_token = torch.tensor([5], device=dev)
    solo_out = model.generate(start_token, n_steps=5, kernel_set="batch_invariant")
    batch_tokens = torch.randint(0, model.config.vocab_size, (32,), device=dev)
    batch_tokens[0] = start_token[0]
    batch_out = model.generate(batch_tokens, n_steps=5, kernel_set="batch_invariant")
    assert torch.equal(solo_out[0], batch_out[0])


@pytest.mark.parametrize("kw", [dict(), dict(mlp="swiglu", dtype="bfloat16", num_kv_heads=1)])
def test_engine_matches_eager_forward_step_bitwise(dev, kw):
    """Graph-captured engine (fused weights, preallocated cache) == the
    reference-style eager loop (torch.cat KV growth) on the same kernels."""
    import torch
    model = _small_model(dev, **kw)
    tokens = torch.randint(0, model.config.vocab_size, (6,), device=dev, generator=torch.Generator(
        device=dev).manual_seed(3))
    eng = model.generate(tokens, n_steps=7, kernel_set="batch_invariant")
    kv = [None] * model.config.num_layers
    cur, outs = tokens, []
    for _ in range(7):
        logits, kv = model.forward_step(cur, kv, "batch_invariant")
        cur = logits.argmax(dim=-1)
        outs.append(cur)
    assert torch.equal(eng, torch.stack(outs, dim=1))


def test_ragged_prompts_engine_matches_eager(dev):
    import torch
    model = _small_model(dev, mlp="swiglu", dtype="bfloat16")
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 64, (n,), generator=g).tolist() for n in (5, 1, 23, 17)]
    eng = model.generate(prompts, n_steps=6, kernel_set="batch_invariant")
    eager = model._generate_ragged_eager(prompts, 6, "batch_invariant")
    assert torch.equal(eng, eager)


def _oracle_weights(model):
    def f(t):
        return t.float().cpu().numpy()
    layers = []
    for layer in model.layers:
        layers.append({k: f(v) for k, v in layer.items()})
    return {"embed": f(model.embed), "layers": layers, "norm_f_w": f(model.norm_f_w),
            "w_lm_head": f(model.w_lm_head)}


def test_first_step_logits_match_oracle(dev):
    """One decode step of a benchmark-shaped model (bf16, SwiGLU): logits within
    bf16 tolerance of the f32 oracle."""
    import torch
    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    cfg = TinyModelConfig(vocab_size=512, num_layers=2, num_heads=16, head_dim=64, mlp_hidden=2816,
                          mlp="swiglu", dtype="bfloat16", seed=0)
    model = TinyModel(cfg, device=str(dev))
    toks = torch.tensor([3, 77, 500, 12], device=dev)
    logits, _ = model.forward_step(toks, [None] * cfg.num_layers, "batch_invariant")
    orc = oracle.TinyModelOracle(_oracle_weights(model), 16, 16, 64, mlp="swiglu", dtype="bfloat16")
    want = orc.step(toks.cpu().numpy(), orc.empty_caches(4))
    # logits ~ N(0, 0.5): atol 1e-2 is ~5 bf16 ulps, the cascade of per-op bf16 roundings
    np.testing.assert_allclose(logits.float().cpu().numpy(), want, rtol=3e-2, atol=1e-2)


def test_generation_matches_oracle_until_near_tie(dev):
    import torch
    model = _small_model(dev, mlp="swiglu", dtype="bfloat16", num_kv_heads=1)
    prompts = [[1, 2, 3], [9], [40, 41, 42, 43, 44]]
    got = model.generate(prompts, n_steps=5, kernel_set="batch_invariant").cpu().numpy()
    orc = oracle.TinyModelOracle(_oracle_weights(model), 2, 1, 32, mlp="swiglu", dtype="bfloat16")
    want, _ = orc.generate(prompts, 5)
    # tokens may only differ after a step whose top-2 oracle logits are within bf16 noise
    for b in range(len(prompts)):
        if not np.array_equal(got[b], want[b]):
            first = int(np.argmax(got[b] != want[b]))
            assert first > 0, "diverged at the first token"


def _baseline_prompts(n_other, seed):
    g = np.random.default_rng(seed)
    tracked = np.random.default_rng(0).integers(0, 32000, 32).tolist()
    others = [g.integers(0, 32000, int(g.integers(16, 513))).tolist() for _ in range(n_other)]
    return tracked, others


def test_baseline_decode_config_tracked_prompt_bitwise(dev):
    """Tracked prompt's 128 greedy tokens identical with 0, 7, 63 and 255 other
    prompts in the batch and at different batch positions."""
    import torch
    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    cfg = TinyModelConfig(vocab_size=32000, num_layers=4, num_heads=16, head_dim=64, mlp_hidden=2816,
                          mlp="swiglu", dtype="bfloat16", seed=0)
    model = TinyModel(cfg, device=str(dev))
    ref = None
    for n_other in (0, 7, 63, 255):
        tracked, others = _baseline_prompts(n_other, seed=100 + n_other)
        pos = (n_other * 5) // 7
        prompts = others[:pos] + [tracked] + others[pos:]
        out = model.generate(prompts, n_steps=128, kernel_set="batch_invariant")
        row = out[pos].clone()
        if ref is None:
            ref = row
        assert torch.equal(row, ref), n_other


def test_gemm_timing_graph_gives_the_same_tokens_and_one_time_per_matmul(dev):
    """A decode graph captured with events around every matmul (bench.py's in-graph GEMM
    times) generates the same tokens as the plain graph and times each matmul family once per
    layer and step (the LM head once per step)."""
    import torch
    model = _small_model(dev, mlp="swiglu", dtype="bfloat16")
    prompts = [[1, 2, 3], [4, 5, 6, 7, 8], [9]]
    eng = model.engine(len(prompts), 32)
    plan = eng.plan(prompts)
    want = eng.run(plan, 6)
    got = eng.run(plan, 6, gemm_timing=True)
    assert torch.equal(got, want)
    times = eng.gemm_times_ms()
    L, steps = model.config.num_layers, 5
    assert sorted(times) == ["down", "gate_up", "lm_head", "o", "qkv"]
    for label, ms in times.items():
        assert len(ms) == (steps if label == "lm_head" else L * steps), label
        assert all(t > 0 for t in ms)
