"""The kernel-check and kernel-bench CLIs on the GPU (small configurations)."""
import pytest

pytestmark = pytest.mark.gpu


def test_kernel_check_invariant_set_has_no_divergence(dev, tmp_path):
    import json

    from detkernels_b200.kernels.integration import main
    out = tmp_path / "r.json"
    main(["--kernel-set", "batch_invariant", "--batch-sizes", "1,64", "--runs", "6", "--steps", "6",
          "--output", str(out)])
    rep = json.loads(out.read_text())
    for r in rep["batch_size_results"]:
        assert r["all_identical"] and r["n_diverging"] == 0


def test_kernel_check_ragged_prompts_bf16_swiglu(dev):
    from detkernels_b200.kernels.integration import main
    rep = main(["--batch-sizes", "1,33", "--runs", "4", "--steps", "5", "--prompt-len", "9", "--mlp", "swiglu",
                "--dtype", "bfloat16", "--num-kv-heads", "2"])
    assert all(r["all_identical"] for r in rep["batch_size_results"])


def test_kernel_bench_runs(dev):
    from detkernels_b200.kernels.benchmark import main
    rep = main(["--batch-sizes", "1,8", "--iters", "3"])
    for section in ("rmsnorm", "matmul", "attention"):
        assert len(rep[section]) == 2
        for row in rep[section]:
            assert row["batch_invariant_ms"] > 0


BENCH_MODEL_ARGS = ["--vocab-size", "32000", "--num-layers", "4", "--num-heads", "16", "--head-dim", "64",
                    "--mlp-hidden", "2816", "--mlp", "swiglu", "--dtype", "bfloat16", "--prompt-len", "32",
                    "--other-len", "16,512", "--steps", "128"]


def test_kernel_check_benchmark_model_10_runs(dev):
    """The benchmark model: the tracked 32-token prompt among freshly drawn co-batches of 16-512
    token prompts, 128 greedy tokens, 10 runs at each batch size 1, 8, 64, 256."""
    from detkernels_b200.kernels.integration import main
    rep = main(BENCH_MODEL_ARGS + ["--batch-sizes", "1,8,64,256", "--runs", "10"])
    assert all(r["all_identical"] and r["n_diverging"] == 0 for r in rep["batch_size_results"]), rep
    assert rep["across_batch_sizes_and_tp"]["all_identical"], rep


def test_kernel_check_benchmark_model_across_tp(dev):
    """The same tracked tokens at TP 1, 2, 4, 8 (ranks held in this process) and batch 8 / 64."""
    from detkernels_b200.kernels.integration import main
    rep = main(BENCH_MODEL_ARGS + ["--batch-sizes", "8,64", "--runs", "3", "--tp", "1,2,4,8"])
    assert rep["across_batch_sizes_and_tp"]["all_identical"], rep
