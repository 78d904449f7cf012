"""``detkernels-kernel-bench``: CUDA-event timing of the invariant kernels
against their batch-variant twins and the eager torch / cuBLAS baselines.

Mirrors the reference's kernels/benchmark.py:23-123 (same shapes, fields and
fp16 default); ``--dtype bfloat16`` is an extension.

    detkernels-kernel-bench --batch-sizes 1,8,64 --iters 50 --output bench.json
"""
from __future__ import annotations

import argparse
import json
from datetime import datetime, timezone


def _time_cuda(fn, n_iters: int = 50, n_warmup: int = 10) -> float:
    """Mean milliseconds per call, one CUDA event pair around n_iters calls."""
    import torch

    for _ in range(n_warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(n_iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / n_iters


def _pct(a, b):
    return (a / b - 1) * 100 if b > 0 else None


def bench_rmsnorm(batch_sizes, n_cols: int = 4096, n_iters: int = 50, dtype=None):
    import torch

    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant, rmsnorm_batch_variant, rmsnorm_reference

    dtype = dtype or torch.float16
    out = []
    for bs in batch_sizes:
        x = torch.randn(bs, n_cols, device="cuda", dtype=dtype)
        w = torch.randn(n_cols, device="cuda", dtype=dtype)
        t_ref = _time_cuda(lambda: rmsnorm_reference(x, w), n_iters)
        t_inv = _time_cuda(lambda: rmsnorm_batch_invariant(x, w), n_iters)
        t_var = _time_cuda(lambda: rmsnorm_batch_variant(x, w), n_iters)
        out.append({"batch_size": bs, "reference_eager_ms": t_ref, "batch_invariant_ms": t_inv,
                    "batch_variant_ms": t_var, "invariant_overhead_vs_eager_pct": _pct(t_inv, t_ref)})
    return out


def bench_matmul(batch_sizes, k: int = 4096, n: int = 4096, n_iters: int = 50, dtype=None):
    import torch

    from detkernels_b200.kernels.matmul import matmul_batch_invariant, matmul_batch_variant

    dtype = dtype or torch.float16
    out = []
    for bs in batch_sizes:
        a = torch.randn(bs, k, device="cuda", dtype=dtype)
        b = torch.randn(k, n, device="cuda", dtype=dtype)
        t_cublas = _time_cuda(lambda: a @ b, n_iters)
        t_inv = _time_cuda(lambda: matmul_batch_invariant(a, b), n_iters)
        t_var = _time_cuda(lambda: matmul_batch_variant(a, b), n_iters)
        out.append({"batch_size": bs, "cublas_ms": t_cublas, "batch_invariant_ms": t_inv,
                    "batch_variant_ms": t_var, "invariant_overhead_vs_cublas_pct": _pct(t_inv, t_cublas)})
    return out


def bench_attention(batch_sizes, num_heads: int = 8, head_dim: int = 64, seq_len: int = 2048, n_iters: int = 50,
                    dtype=None):
    import torch

    from detkernels_b200.kernels.attention import (attention_batch_invariant, attention_batch_variant,
                                                   attention_reference)

    dtype = dtype or torch.float16
    out = []
    for bs in batch_sizes:
        q = torch.randn(bs, num_heads, head_dim, device="cuda", dtype=dtype)
        k = torch.randn(bs, num_heads, seq_len, head_dim, device="cuda", dtype=dtype)
        v = torch.randn(bs, num_heads, seq_len, head_dim, device="cuda", dtype=dtype)
        t_ref = _time_cuda(lambda: attention_reference(q, k, v), n_iters)
        t_inv = _time_cuda(lambda: attention_batch_invariant(q, k, v), n_iters)
        t_var = _time_cuda(lambda: attention_batch_variant(q, k, v), n_iters)
        out.append({"batch_size": bs, "reference_eager_ms": t_ref, "batch_invariant_ms": t_inv,
                    "batch_variant_ms": t_var, "invariant_overhead_vs_eager_pct": _pct(t_inv, t_ref)})
    return out


def main(argv=None):
    import torch

    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--batch-sizes", default="1,8,64", help="Comma-separated batch sizes to sweep.")
    parser.add_argument("--iters", type=int, default=50)
    parser.add_argument("--dtype", choices=["float16", "bfloat16"], default="float16")
    parser.add_argument("--output", default=None)
    args = parser.parse_args(argv)
    batch_sizes = [int(x) for x in args.batch_sizes.split(",")]
    dtype = getattr(torch, args.dtype)
    report = {
        "timestamp": datetime.now(timezone.utc).isoformat(),
        "n_iters": args.iters,
        "batch_sizes": batch_sizes,
        "dtype": args.dtype,
        "rmsnorm": bench_rmsnorm(batch_sizes, n_iters=args.iters, dtype=dtype),
        "matmul": bench_matmul(batch_sizes, n_iters=args.iters, dtype=dtype),
        "attention": bench_attention(batch_sizes, n_iters=args.iters, dtype=dtype),
    }
    if args.output:
        with open(args.output, "w") as f:
            json.dump(report, f, indent=2)
    else:
        print(json.dumps(report, indent=2))
    return report


if __name__ == "__main__":
    main()
