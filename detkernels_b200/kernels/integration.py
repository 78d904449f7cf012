"""``detkernels-kernel-check``: repeat-run bitwise check of the TinyModel decode.

Mirrors the reference's kernels/integration.py:33-111: for each batch size, N
repeats; row 0 always starts from the same tracked token while every other row
gets fresh random tokens (seed ``seed_base + repeat``); row 0's generated
tokens are compared across repeats with ``summarize_batch_results``.

Extensions (all optional): ``--kernel-set reference``, ``--num-kv-heads``,
``--mlp swiglu``, ``--dtype bfloat16`` and ``--prompt-len L`` (row 0 gets a
fixed L-token prompt and the other rows ragged prompts of 1..2L tokens).

    detkernels-kernel-check --kernel-set batch_invariant --batch-sizes 1,64 --runs 100 --steps 8
"""
from __future__ import annotations

import argparse
import json
from datetime import datetime, timezone

from detkernels_b200.harness.sweep import summarize_batch_results
from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig


def run_repeats(model, kernel_set: str, batch_size: int, n_steps: int, n_repeats: int, tracked_token: int = 0,
                seed_base: int = 1000, prompt_len: int = 0):
    """Row 0's generated tokens for each repeat, summarised (reference integration.py:33-45)."""
    import torch

    runs = []
    vocab = model.config.vocab_size
    for i in range(n_repeats):
        g = torch.Generator(device=model.device).manual_seed(seed_base + i)
        if prompt_len <= 0:
            tokens = torch.randint(0, vocab, (batch_size,), device=model.device, generator=g)
            tokens[0] = tracked_token
            out = model.generate(tokens, n_steps=n_steps, kernel_set=kernel_set)
        else:
            gc = torch.Generator().manual_seed(seed_base + i)
            tracked = torch.randint(0, vocab, (prompt_len,), generator=torch.Generator().manual_seed(7)).tolist()
            prompts = [tracked] + [torch.randint(0, vocab, (int(torch.randint(1, 2 * prompt_len + 1, (1,),
                                                                                generator=gc)),),
                                                 generator=gc).tolist() for _ in range(batch_size - 1)]
            out = model.generate(prompts, n_steps=n_steps, kernel_set=kernel_set)
        runs.append(tuple(out[0].tolist()))
    return summarize_batch_results(batch_size, runs)


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--kernel-set", choices=["batch_invariant", "batch_variant", "reference"],
                        default="batch_invariant")
    parser.add_argument("--batch-sizes", default="1,64", help="Comma-separated batch sizes to sweep.")
    parser.add_argument("--runs", type=int, default=100)
    parser.add_argument("--steps", type=int, default=8)
    parser.add_argument("--vocab-size", type=int, default=256)
    parser.add_argument("--num-layers", type=int, default=4)
    parser.add_argument("--num-heads", type=int, default=4)
    parser.add_argument("--head-dim", type=int, default=32)
    parser.add_argument("--mlp-hidden", type=int, default=256)
    parser.add_argument("--seed", type=int, default=0, help="Model weight init seed.")
    parser.add_argument("--num-kv-heads", type=int, default=None)
    parser.add_argument("--mlp", choices=["silu", "swiglu"], default="silu")
    parser.add_argument("--dtype", choices=["float16", "bfloat16"], default="float16")
    parser.add_argument("--prompt-len", type=int, default=0)
    parser.add_argument("--device", default="cuda")
    parser.add_argument("--output", default=None)
    args = parser.parse_args(argv)

    batch_sizes = [int(x) for x in args.batch_sizes.split(",")]
    cfg = TinyModelConfig(vocab_size=args.vocab_size, num_layers=args.num_layers, num_heads=args.num_heads,
                          head_dim=args.head_dim, mlp_hidden=args.mlp_hidden, seed=args.seed,
                          num_kv_heads=args.num_kv_heads, mlp=args.mlp, dtype=args.dtype)
    model = TinyModel(cfg, device=args.device)

    results = []
    for bs in batch_sizes:
        r = run_repeats(model, args.kernel_set, bs, args.steps, args.runs, prompt_len=args.prompt_len)
        print(f"batch_size={bs}: all_identical={r.all_identical} n_diverging={r.n_diverging}/{args.runs - 1} "
              f"divergence_indices={r.divergence_indices}")
        results.append(r)

    report = {
        "kernel_set": args.kernel_set,
        "model_config": {"vocab_size": cfg.vocab_size, "num_layers": cfg.num_layers, "num_heads": cfg.num_heads,
                         "head_dim": cfg.head_dim, "mlp_hidden": cfg.mlp_hidden, "seed": cfg.seed,
                         "num_kv_heads": cfg.kv_heads, "mlp": cfg.mlp, "dtype": cfg.dtype},
        "n_repeats": args.runs,
        "n_steps": args.steps,
        "prompt_len": args.prompt_len,
        "timestamp": datetime.now(timezone.utc).isoformat(),
        "batch_size_results": [{"batch_size": r.batch_size, "all_identical": r.all_identical,
                                "n_diverging": r.n_diverging, "divergence_indices": r.divergence_indices}
                               for r in results],
    }
    if args.output:
        with open(args.output, "w") as f:
            json.dump(report, f, indent=2)
    else:
        print(json.dumps(report, indent=2))
    return report


if __name__ == "__main__":
    main()
