"""Batch-invariance harness for the gated delta rule, run on this library's kernel.

Drop-in for the reference's gdn/repro.py (check functions 80-342, CLI
345-442): the same four experiments, argument names, defaults and JSON report
fields, with ``detkernels_b200.kernels.gdn.chunk_gated_delta_rule`` in place of
FLA's.  Each experiment holds one sequence's (q, k, v, beta, gate) fixed,
changes only what is computed alongside it, and compares the tracked output
bit for bit:

* ``row``: rectangular batches of different sizes (tracked row 0);
* ``packing``: the tracked sequence at every position of a cu_seqlens pack;
* ``decode``: T=1 steps with the state carried between calls in bf16, with 0
  vs N other sequences decoding beside it;
* ``geometry``: the tracked sequence first in packs of growing total size.

Inputs follow the reference's generator: q ~ N(0,1), k = L2-normalised
N(0,1), v ~ N(0,1), beta = sigmoid(U[0,1)), gate = logsigmoid(U[0,1)), drawn
from a seeded torch.Generator on the device in the reference's order.
"""
from __future__ import annotations

import argparse
import json
from datetime import datetime, timezone


def _gdn():
    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule
    return chunk_gated_delta_rule


def _draw(shape_qk, shape_v, shape_gb, device, dtype, seed):
    """(q, k, v, beta, gate) from one generator, in the reference's draw order."""
    import torch
    import torch.nn.functional as F

    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(*shape_qk, device=device, dtype=dtype, generator=gen)
    k = F.normalize(torch.randn(*shape_qk, device=device, dtype=dtype, generator=gen), p=2, dim=-1)
    v = torch.randn(*shape_v, device=device, dtype=dtype, generator=gen)
    beta = torch.rand(*shape_gb, device=device, dtype=dtype, generator=gen).sigmoid()
    gate = F.logsigmoid(torch.rand(*shape_gb, device=device, dtype=dtype, generator=gen))
    return q, k, v, beta, gate


def _make_inputs(batch, seq_len, h, hv, k_dim, v_dim, device, dtype, seed):
    return _draw((batch, seq_len, h, k_dim), (batch, seq_len, hv, v_dim), (batch, seq_len, hv), device, dtype,
                 seed)


def _make_seq(seq_len, h, hv, k_dim, v_dim, device, dtype, seed):
    return _draw((seq_len, h, k_dim), (seq_len, hv, v_dim), (seq_len, hv), device, dtype, seed)


def _diff(a, b):
    import torch
    return bool(torch.equal(a, b)), float((a.float() - b.float()).abs().max().item()) if a.numel() else 0.0


def _compare(outputs, keys, key_name, ref_name):
    ref = outputs[keys[0]]
    comparisons = []
    for key in keys[1:]:
        identical, max_abs = _diff(ref, outputs[key])
        comparisons.append({key_name: key, ref_name: keys[0], "identical": identical, "max_abs_diff": max_abs})
    return comparisons


def _run_row(tracked, batch_size, other_rows_seed, seq_len, h, hv, k_dim, v_dim, device, dtype):
    """Tracked sequence at row 0 of a rectangular batch of batch_size rows."""
    import torch

    if batch_size == 1:
        q, k, v, beta, gate = tracked
    else:
        others = _make_inputs(batch_size - 1, seq_len, h, hv, k_dim, v_dim, device, dtype, other_rows_seed)
        q, k, v, beta, gate = (torch.cat([a, b], dim=0) for a, b in zip(tracked, others))
    o, _ = _gdn()(q, k, v, gate, beta, output_final_state=False)
    return o[0]


def check_row_invariance(batch_sizes, seq_len: int = 128, h: int = 2, hv: int = 4, k_dim: int = 64,
                         v_dim: int = 64, device: str = "cuda", dtype=None, seed: int = 0):
    """Tracked row's output across rectangular batch sizes (reference gdn/repro.py:80-119)."""
    import torch

    dtype = torch.bfloat16 if dtype is None else dtype
    tracked = _make_inputs(1, seq_len, h, hv, k_dim, v_dim, device, dtype, seed)
    outputs = {bs: _run_row(tracked, bs, 1000 + bs, seq_len, h, hv, k_dim, v_dim, device, dtype)
               for bs in batch_sizes}
    return {"reference_batch_size": batch_sizes[0],
            "comparisons": _compare(outputs, list(batch_sizes), "batch_size", "reference_batch_size")}


def _run_packed(tracked_seq, other_seqs, tracked_position, device):
    """Pack the sequences along T with cu_seqlens (tracked one at tracked_position);
    returns the tracked sequence's output slice."""
    import torch

    seqs = list(other_seqs)
    seqs.insert(tracked_position, tracked_seq)
    lens = [s[0].shape[0] for s in seqs]
    bounds = [0]
    for n in lens:
        bounds.append(bounds[-1] + n)
    cu_seqlens = torch.tensor(bounds, device=device, dtype=torch.long)
    q, k, v, beta, gate = (torch.cat([s[i] for s in seqs], dim=0).unsqueeze(0) for i in range(5))
    o, _ = _gdn()(q, k, v, gate, beta, output_final_state=False, cu_seqlens=cu_seqlens)
    return o[0, bounds[tracked_position]:bounds[tracked_position + 1]]


def check_packing_position_invariance(tracked_seq_len: int = 48, other_seq_lens=(37, 53, 29, 61), h: int = 2,
                                      hv: int = 4, k_dim: int = 64, v_dim: int = 64, device: str = "cuda",
                                      dtype=None, seed: int = 0):
    """Tracked sequence's output at every position of a fixed-size pack (reference 162-199)."""
    import torch

    dtype = torch.bfloat16 if dtype is None else dtype
    tracked = _make_seq(tracked_seq_len, h, hv, k_dim, v_dim, device, dtype, seed)
    others = [_make_seq(n, h, hv, k_dim, v_dim, device, dtype, seed=100 + i) for i, n in enumerate(other_seq_lens)]
    positions = list(range(len(others) + 1))
    outputs = {pos: _run_packed(tracked, others, pos, device) for pos in positions}
    return {"reference_position": positions[0],
            "comparisons": _compare(outputs, positions, "tracked_position", "reference_position")}


def check_geometry_invariance(tracked_seq_len: int = 50, other_totals=(0, 500, 2000), filler_seq_len: int = 47,
                              h: int = 2, hv: int = 4, k_dim: int = 64, v_dim: int = 64, device: str = "cuda",
                              dtype=None, seed: int = 0):
    """Tracked sequence (first in the pack) against packs of growing total size (reference 202-249)."""
    import torch

    dtype = torch.bfloat16 if dtype is None else dtype
    tracked = _make_seq(tracked_seq_len, h, hv, k_dim, v_dim, device, dtype, seed)
    outputs = {}
    for i, total in enumerate(other_totals):
        fillers = [_make_seq(filler_seq_len, h, hv, k_dim, v_dim, device, dtype, seed=200_000 + i * 1000 + j)
                   for j in range(total // filler_seq_len)]
        outputs[total] = _run_packed(tracked, fillers, 0, device)
    return {"reference_other_tokens_total": other_totals[0],
            "comparisons": _compare(outputs, list(other_totals), "other_tokens_total",
                                    "reference_other_tokens_total")}


def _decode_loop(n_other, n_steps, h, hv, k_dim, v_dim, device, dtype, state_dtype, seed_base):
    """n_steps single-token calls for 1 tracked + n_other rows, the state carried
    between calls in state_dtype; the tracked row's tokens never depend on n_other."""
    import torch

    state = None
    traj = []
    for step in range(n_steps):
        q, k, v, beta, gate = _make_inputs(1 + n_other, 1, h, hv, k_dim, v_dim, device, dtype, seed_base + step)
        tracked = _make_inputs(1, 1, h, hv, k_dim, v_dim, device, dtype, seed=999_000 + step)
        for dst, src in zip((q, k, v, beta, gate), tracked):
            dst[0:1] = src
        o, new_state = _gdn()(q, k, v, gate, beta, initial_state=state, output_final_state=True)
        state = new_state.to(state_dtype)
        traj.append(o[0, 0].clone())
    return torch.stack(traj, dim=0)


def check_decode_state_drift(n_steps: int = 300, n_other_seqs_options=(0, 63), h: int = 2, hv: int = 4,
                             k_dim: int = 64, v_dim: int = 64, device: str = "cuda", dtype=None, state_dtype=None,
                             seed: int = 0):
    """Tracked row's decode trajectory with 0 vs N co-decoding rows (reference 294-342)."""
    import torch

    dtype = torch.bfloat16 if dtype is None else dtype
    state_dtype = torch.bfloat16 if state_dtype is None else state_dtype
    trajs = {n: _decode_loop(n, n_steps, h, hv, k_dim, v_dim, device, dtype, state_dtype, seed * 100_000)
             for n in n_other_seqs_options}
    ref_n = n_other_seqs_options[0]
    comparisons = []
    for n in n_other_seqs_options[1:]:
        per_step = (trajs[ref_n].float() - trajs[n].float()).abs().amax(dim=(1, 2)).tolist()
        first = next((i for i, d in enumerate(per_step) if d > 0), None)
        comparisons.append({"n_other_sequences": n, "reference_n_other_sequences": ref_n,
                            "identical": first is None, "first_diverging_step": first,
                            "max_abs_diff": max(per_step) if per_step else 0.0})
    return {"n_steps": n_steps, "reference_n_other_sequences": ref_n, "comparisons": comparisons}


def _ints(s):
    return [int(x) for x in s.split(",") if x.strip()]


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--mode", choices=["row", "packing", "decode", "geometry", "all"], default="geometry")
    parser.add_argument("--batch-sizes", default="1,64", help="For --mode row.")
    parser.add_argument("--seq-len", type=int, default=128, help="For --mode row.")
    parser.add_argument("--tracked-seq-len", type=int, default=48, help="For --mode packing.")
    parser.add_argument("--other-seq-lens", default="37,53,29,61", help="For --mode packing.")
    parser.add_argument("--n-steps", type=int, default=300, help="For --mode decode.")
    parser.add_argument("--n-other-seqs", default="0,63", help="For --mode decode.")
    parser.add_argument("--geo-tracked-len", type=int, default=50, help="For --mode geometry.")
    parser.add_argument("--geo-filler-len", type=int, default=47, help="For --mode geometry.")
    parser.add_argument("--other-totals", default="0,500,2000", help="For --mode geometry.")
    parser.add_argument("--repeats", type=int, default=1)
    parser.add_argument("--output", default=None)
    args = parser.parse_args(argv)
    batch_sizes = _ints(args.batch_sizes)
    other_seq_lens = tuple(_ints(args.other_seq_lens))
    n_other = tuple(_ints(args.n_other_seqs))
    other_totals = tuple(_ints(args.other_totals))
    modes = ("row", "packing", "decode", "geometry") if args.mode == "all" else (args.mode,)

    results = {m: [] for m in ("row", "packing", "decode", "geometry")}
    for r in range(args.repeats):
        if "row" in modes:
            res = check_row_invariance(batch_sizes, seq_len=args.seq_len, seed=r)
            results["row"].append(res)
            for c in res["comparisons"]:
                print("[row]     repeat=%d batch_size=%d vs ref_bs=%d: identical=%s max_abs_diff=%.6g"
                      % (r, c["batch_size"], c["reference_batch_size"], c["identical"], c["max_abs_diff"]))
        if "packing" in modes:
            res = check_packing_position_invariance(tracked_seq_len=args.tracked_seq_len,
                                                    other_seq_lens=other_seq_lens, seed=r)
            results["packing"].append(res)
            for c in res["comparisons"]:
                print("[packing] repeat=%d tracked_position=%d vs ref_pos=%d: identical=%s max_abs_diff=%.6g"
                      % (r, c["tracked_position"], c["reference_position"], c["identical"], c["max_abs_diff"]))
        if "decode" in modes:
            res = check_decode_state_drift(n_steps=args.n_steps, n_other_seqs_options=n_other, seed=r)
            results["decode"].append(res)
            for c in res["comparisons"]:
                print("[decode]  repeat=%d n_other=%d vs ref_n_other=%d: identical=%s first_diverging_step=%s "
                      "max_abs_diff=%.6g" % (r, c["n_other_sequences"], c["reference_n_other_sequences"],
                                             c["identical"], c["first_diverging_step"], c["max_abs_diff"]))
        if "geometry" in modes:
            res = check_geometry_invariance(tracked_seq_len=args.geo_tracked_len,
                                            filler_seq_len=args.geo_filler_len, other_totals=other_totals, seed=r)
            results["geometry"].append(res)
            for c in res["comparisons"]:
                print("[geometry] repeat=%d other_tokens_total=%d vs ref_total=%d: identical=%s max_abs_diff=%.6g"
                      % (r, c["other_tokens_total"], c["reference_other_tokens_total"], c["identical"],
                         c["max_abs_diff"]))

    report = {
        "timestamp": datetime.now(timezone.utc).isoformat(),
        "mode": args.mode,
        "batch_sizes": batch_sizes,
        "seq_len": args.seq_len,
        "tracked_seq_len": args.tracked_seq_len,
        "other_seq_lens": list(other_seq_lens),
        "geo_tracked_len": args.geo_tracked_len,
        "geo_filler_len": args.geo_filler_len,
        "other_totals": list(other_totals),
        "n_steps": args.n_steps,
        "n_other_seqs_options": list(n_other),
        "repeats": args.repeats,
        "row_results": results["row"],
        "packing_results": results["packing"],
        "decode_results": results["decode"],
        "geometry_results": results["geometry"],
    }
    if args.output:
        with open(args.output, "w") as f:
            json.dump(report, f, indent=2)
    else:
        print(json.dumps(report, indent=2))
    return report


if __name__ == "__main__":
    main()
