"""``detkernels-kernel-check``: repeat-run bitwise check of the TinyModel decode.

Mirrors the reference's kernels/integration.py:33-111: for each batch size, N
repeats; row 0 always starts from the same tracked token while every other row
gets fresh random tokens (seed ``seed_base + repeat``); row 0's generated
tokens are compared across repeats with ``summarize_batch_results``.

Extensions (all optional): ``--kernel-set reference``, ``--num-kv-heads``,
``--mlp swiglu``, ``--dtype bfloat16``, ``--prompt-len L`` (row 0 gets a
fixed L-token prompt and the other rows ragged prompts of 1..2L tokens, or of
``--other-len MIN,MAX`` tokens) and ``--tp 1,2,4,8`` (the sweep is repeated
with the model split over that many tensor-parallel ranks -- the ranks of a
torchrun job when launched with one, else all ranks in this process on one
GPU -- and every run at every TP is compared with the first run at the first
TP).

    detkernels-kernel-check --kernel-set batch_invariant --batch-sizes 1,64 --runs 100 --steps 8
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import datetime, timezone

from detkernels_b200.harness.sweep import summarize_batch_results
from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig


def run_repeats(model, kernel_set: str, batch_size: int, n_steps: int, n_repeats: int, tracked_token: int = 0,
                seed_base: int = 1000, prompt_len: int = 0, other_len=None, tp: int = 1, group=None,
                return_runs: bool = False):
    """Row 0's generated tokens for each repeat, summarised (reference integration.py:33-45).
    With return_runs the list of row-0 token tuples is returned as well."""
    import torch

    runs = []
    vocab = model.config.vocab_size
    gen_kw = {"tp": tp, "group": group} if (tp != 1 or group is not None) else {}
    lo, hi = other_len if other_len else (1, 2 * max(prompt_len, 1))
    for i in range(n_repeats):
        g = torch.Generator(device=model.device).manual_seed(seed_base + i)
        if prompt_len <= 0:
            tokens = torch.randint(0, vocab, (batch_size,), device=model.device, generator=g)
            tokens[0] = tracked_token
            out = model.generate(tokens, n_steps=n_steps, kernel_set=kernel_set, **gen_kw)
        else:
            gc = torch.Generator().manual_seed(seed_base + i)
            tracked = torch.randint(0, vocab, (prompt_len,), generator=torch.Generator().manual_seed(7)).tolist()
            prompts = [tracked] + [torch.randint(0, vocab, (int(torch.randint(lo, hi + 1, (1,), generator=gc)),),
                                                 generator=gc).tolist() for _ in range(batch_size - 1)]
            out = model.generate(prompts, n_steps=n_steps, kernel_set=kernel_set, **gen_kw)
        runs.append(tuple(out[0].tolist()))
    res = summarize_batch_results(batch_size, runs)
    return (res, runs) if return_runs else res


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
    parser.add_argument("--other-len", default=None,
                        help="MIN,MAX token count of the co-batched prompts (with --prompt-len; default 1,2L)")
    parser.add_argument("--tp", default="1", help="Comma-separated tensor-parallel sizes (1, 2, 4, 8).")
    parser.add_argument("--device", default="cuda")
    parser.add_argument("--output", default=None)
    args = parser.parse_args(argv)

    batch_sizes = [int(x) for x in args.batch_sizes.split(",")]
    tps = [int(x) for x in args.tp.split(",")]
    other_len = tuple(int(x) for x in args.other_len.split(",")) if args.other_len else None
    group = None
    if any(t > 1 for t in tps) and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # launched by torchrun: the ranks of the job are the tensor-parallel ranks
        import torch
        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        if not dist.is_initialized():
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        group = dist.group.WORLD
        args.device = "cuda:%d" % local
    cfg = TinyModelConfig(vocab_size=args.vocab_size, num_layers=args.num_layers, num_heads=args.num_heads,
                          head_dim=args.head_dim, mlp_hidden=args.mlp_hidden, seed=args.seed,
                          num_kv_heads=args.num_kv_heads, mlp=args.mlp, dtype=args.dtype)
    model = TinyModel(cfg, device=args.device)

    results = []
    first_run = None
    across = []
    for tp in tps:
        grp = group if (group is not None and tp == group.size()) else None
        if tp > 1 and group is not None and grp is None:
            raise SystemExit("--tp %d under torchrun needs %d ranks" % (tp, tp))
        for bs in batch_sizes:
            r, runs = run_repeats(model, args.kernel_set, bs, args.steps, args.runs, prompt_len=args.prompt_len,
                                  other_len=other_len, tp=tp, group=grp, return_runs=True)
            if first_run is None:
                first_run = runs[0]
            n_off = sum(1 for run in runs if tuple(run) != tuple(first_run))
            across.append({"tp": tp, "batch_size": bs, "n_runs_differing_from_first": n_off})
            print(f"tp={tp} batch_size={bs}: all_identical={r.all_identical} "
                  f"n_diverging={r.n_diverging}/{args.runs - 1} divergence_indices={r.divergence_indices} "
                  f"runs_differing_from_first_tp_first_batch={n_off}")
            results.append((tp, r))
        model._engines.clear()

    report = {
        "kernel_set": args.kernel_set,
        "model_config": {"vocab_size": cfg.vocab_size, "num_layers": cfg.num_layers, "num_heads": cfg.num_heads,
                         "head_dim": cfg.head_dim, "mlp_hidden": cfg.mlp_hidden, "seed": cfg.seed,
                         "num_kv_heads": cfg.kv_heads, "mlp": cfg.mlp, "dtype": cfg.dtype},
        "n_repeats": args.runs,
        "n_steps": args.steps,
        "prompt_len": args.prompt_len,
        "other_len": list(other_len) if other_len else None,
        "tp": tps,
        "timestamp": datetime.now(timezone.utc).isoformat(),
        "batch_size_results": [{"tp": tp, "batch_size": r.batch_size, "all_identical": r.all_identical,
                                "n_diverging": r.n_diverging, "divergence_indices": r.divergence_indices}
                               for tp, r in results],
        "across_batch_sizes_and_tp": {"all_identical": all(a["n_runs_differing_from_first"] == 0 for a in across),
                                      "per_setting": across},
    }
    if group is not None:
        import torch.distributed as dist
        dist.destroy_process_group()
    if args.output and (group is None or int(os.environ.get("RANK", "0")) == 0):
        with open(args.output, "w") as f:
            json.dump(report, f, indent=2)
    elif not args.output:
        print(json.dumps(report, indent=2))
    return report


if __name__ == "__main__":
    main()
