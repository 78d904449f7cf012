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
