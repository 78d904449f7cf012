#!/usr/bin/env python
"""Benchmark of the batch-invariant decode path on B200: prints ONE JSON line.

Workload (one "step"): greedy decoding of 128 tokens for 256 prompts per GPU
with a random-init TinyModel (4 layers, d_model 1024, 16 heads x 64, SwiGLU
2816, vocab 32000, bf16): one tracked 32-token prompt (rank 0) among prompts of
U[16, 512] random tokens, prefilled as rows and decoded through the invariant
RMSNorm / tcgen05 GEMM / split-KV attention kernels with the decode steps in
one CUDA graph.  Multi-GPU runs shard independent requests (weak scaling, no
collective in the data path); the device-timed max over ranks is reported.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the reference's decode step (its eager torch
formulas) on the host cores over the same 256 sequences, for the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

MODEL = dict(vocab_size=32000, num_layers=4, num_heads=16, head_dim=64, mlp_hidden=2816, mlp="swiglu",
             dtype="bfloat16", seed=0)
BATCH_PER_GPU = 256
TRACKED_LEN = 32
OTHER_LEN = (16, 512)
NEW_TOKENS = 128
WORKLOAD_NAME = ("tinymodel-decode: 4L d1024 16x64 SwiGLU2816 vocab32000 bf16, 256 prompts/GPU "
                 "(tracked 32 tok + 255 of U[16,512] tok), 128 greedy tokens")
# inputs vs L2: the KV cache (4 layers x 256 seq x 16 heads x 640 tokens x 64 x bf16 x K,V = 2.7 GB)
# and the weights (168 MB) both exceed the 126 MB L2, so no flush is needed between steps
L2_NOTE = "inputs larger than L2 (KV cache 2.7 GB/GPU, weights 168 MB)"
GEMM_SHAPES = [(m, n) for n in (4096, 11008) for m in (1, 8, 64, 256, 2048)]


def workload_config(world: int = 1):
    """The `config` object of both arms' JSON lines (same keys and values at one GPU)."""
    return {"workload": WORKLOAD_NAME, "global_batch": BATCH_PER_GPU * world, "new_tokens": NEW_TOKENS,
            "l2": L2_NOTE}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ----------------------------------------------------------------------------- inputs
def make_prompts(rank: int, batch: int):
    import numpy as np

    vocab = MODEL["vocab_size"]
    tracked = np.random.default_rng(0).integers(0, vocab, TRACKED_LEN).tolist()
    rng = np.random.default_rng(10_000 + rank)
    n_other = batch - 1 if rank == 0 else batch
    others = [rng.integers(0, vocab, int(rng.integers(OTHER_LEN[0], OTHER_LEN[1] + 1))).tolist()
              for _ in range(n_other)]
    return ([tracked] + others) if rank == 0 else others


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(str(g) for g in self.gpus)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for nm, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed
def dist_setup(n_gpus):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU baseline (oracle)
def cpu_sample(prompts, n_tokens, model=None):
    """Time the oracle's decode (numpy, all host threads) on a bounded sample,
    with the weights of `model` (a CPU TinyModel of the workload by default)."""
    from threadpoolctl import threadpool_limits

    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig
    from oracle import ops as oracle

    cores = len(os.sched_getaffinity(0))
    if model is None:
        model = TinyModel(TinyModelConfig(**MODEL), device="cpu")

    def f(t):
        return t.float().cpu().numpy()

    w = {"embed": f(model.embed), "layers": [{k: f(v) for k, v in L.items()} for L in model.layers],
         "norm_f_w": f(model.norm_f_w), "w_lm_head": f(model.w_lm_head)}
    orc = oracle.TinyModelOracle(w, MODEL["num_heads"], MODEL["num_heads"], MODEL["head_dim"], mlp="swiglu",
                                 dtype="bfloat16")
    with threadpool_limits(limits=cores):
        t0 = time.perf_counter()
        toks, _ = orc.generate(prompts, n_tokens)
        dt = time.perf_counter() - t0
    n = len(prompts) * n_tokens
    return {"value": n / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": "numpy oracle decode of %d prompts (lengths %s), %d greedy tokens each, %.1f s"
                      % (len(prompts), [len(p) for p in prompts], n_tokens, dt)}, toks


def cpu_sample_prompts():
    """Small parity sample for the oracle check: the tracked prompt and 7 co-batched prompts cut to 48 tokens."""
    p = make_prompts(0, 8)
    return [p[0]] + [q[:48] for q in p[1:]]


class ReferenceDecodeCPU:
    """The reference's decode step on the host cores, at the workload's batch and KV lengths.

    Each step is the reference's ``TinyModel.forward_step`` (kernels/tiny_model.py:99-140) built
    from its eager formulas (``rmsnorm_reference``, ``matmul_reference``, ``attention_reference``;
    kernels/rmsnorm.py:39-48, kernels/matmul.py:42-49, kernels/attention.py:49-71) with the
    workload's SwiGLU MLP, over all 256 sequences at once.  The reference grows one KV tensor per
    layer with ``torch.cat`` and has no ragged batches, so here each sequence keeps its own
    unpadded [H, len, D] cache (preallocated for the steps that run) and attention is the
    reference formula on that sequence's cache.  The caches start at the prompt lengths of the
    workload, filled with seeded N(0,1) values: the reference has no prefill, so the prompts'
    prefill is not part of this arm (the GPU arm's steps include it).
    """

    def __init__(self, model, prompts, max_steps, threads):
        import numpy as np
        import torch

        self.model, self.threads = model, threads
        cfg = model.config
        self.B = len(prompts)
        self.H, self.Hkv, self.D = cfg.num_heads, cfg.kv_heads, cfg.head_dim
        self.lens0 = np.array([len(p) for p in prompts], dtype=np.int64)
        g = torch.Generator().manual_seed(1234)
        self.k = [[torch.randn(self.Hkv, int(L) + max_steps, self.D, generator=g).to(model.dtype)
                   for L in self.lens0] for _ in range(cfg.num_layers)]
        self.v = [[torch.randn(self.Hkv, int(L) + max_steps, self.D, generator=g).to(model.dtype)
                   for L in self.lens0] for _ in range(cfg.num_layers)]
        self.max_steps = max_steps
        self.first = torch.tensor([p[-1] for p in prompts], dtype=torch.long)

    def _step(self, tok, lens):
        import torch

        from detkernels_b200.kernels.attention import attention_reference
        from detkernels_b200.kernels.matmul import matmul_reference as mm
        from detkernels_b200.kernels.rmsnorm import rmsnorm_reference as rms

        m, cfg = self.model, self.model.config
        B, H, Hkv, D = self.B, self.H, self.Hkv, self.D
        x = m.embed[tok]
        for li, L in enumerate(m.layers):
            xn = rms(x, L["norm1_w"], cfg.eps)
            q = mm(xn, L["w_q"]).view(B, H, D)
            kn = mm(xn, L["w_k"]).view(B, Hkv, D)
            vn = mm(xn, L["w_v"]).view(B, Hkv, D)
            outs = []
            for b in range(B):
                n = int(lens[b])
                kb, vb = self.k[li][b], self.v[li][b]
                kb[:, n] = kn[b]
                vb[:, n] = vn[b]
                outs.append(attention_reference(q[b:b + 1], kb[None, :, :n + 1], vb[None, :, :n + 1]))
            a = torch.cat(outs).reshape(B, H * D)
            x = x + mm(a, L["w_o"])
            xn = rms(x, L["norm2_w"], cfg.eps)
            if cfg.mlp == "swiglu":
                hid = torch.nn.functional.silu(mm(xn, L["w_gate"])) * mm(xn, L["w_up"])
            else:
                hid = torch.nn.functional.silu(mm(xn, L["w_mlp1"]))
            x = x + mm(hid, L["w_mlp2"])
        logits = mm(rms(x, m.norm_f_w, cfg.eps), m.w_lm_head)
        return logits.argmax(dim=-1)

    def run(self, n_steps):
        """n_steps greedy decode steps over all sequences from the prompt lengths; returns seconds."""
        import torch

        assert n_steps <= self.max_steps
        torch.set_num_threads(self.threads)
        lens = self.lens0.copy()
        tok = self.first.clone()
        t0 = time.perf_counter()
        with torch.inference_mode():
            for _ in range(n_steps):
                tok = self._step(tok, lens)
                lens += 1
        return time.perf_counter() - t0

    def describe(self, n_steps):
        return ("reference eager formulas (torch, %d host threads): %d greedy decode steps x %d sequences "
                "from KV lengths %d..%d (prefill excluded)" % (self.threads, n_steps, self.B, int(self.lens0.min()),
                                                               int(self.lens0.max())))


def cpu_baseline_sample(model=None, n_steps=32):
    """cpu_baseline of the GPU line: one bounded sample (~10-30 s) of ReferenceDecodeCPU."""
    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig

    threads = len(os.sched_getaffinity(0))
    cpu_model = TinyModel(TinyModelConfig(**MODEL), device="cpu")
    ref = ReferenceDecodeCPU(cpu_model, make_prompts(0, BATCH_PER_GPU), n_steps, threads)
    ref.run(1)   # warm-up
    dt = ref.run(n_steps)
    return {"value": ref.B * n_steps / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": ref.describe(n_steps) + ", %.1f s" % dt}


# ----------------------------------------------------------------------------- GEMM vs cuBLAS
def gemm_vs_cublas(iters=10):
    import torch

    from detkernels_b200.kernels.matmul import matmul_batch_invariant

    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    res = {}
    g = torch.Generator(device=dev).manual_seed(0)
    w_cache = {}
    for (m, n) in GEMM_SHAPES:
        if n not in w_cache:
            w_cache[n] = (0.02 * torch.randn(4096, n, device=dev, generator=g)).to(torch.bfloat16)
        w = w_cache[n]
        a = torch.randn(m, 4096, device=dev, generator=g).to(torch.bfloat16)

        def timed(fn):
            for _ in range(3):
                fn()
            ts = []
            for _ in range(iters):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                fn()
                e.record()
                e.synchronize()
                ts.append(s.elapsed_time(e))
            return statistics.median(ts)

        t_ours = timed(lambda: matmul_batch_invariant(a, w))
        t_cub = timed(lambda: torch.matmul(a, w))
        flops = 2.0 * m * n * 4096
        res["M=%d,N=%d" % (m, n)] = {"ours_tflops": round(flops / t_ours / 1e9, 2),
                                     "cublas_tflops": round(flops / t_cub / 1e9, 2),
                                     "ratio": round(t_cub / t_ours, 3),
                                     "ours_us": round(t_ours * 1e3, 2), "cublas_us": round(t_cub * 1e3, 2)}
    del flush
    return res


# ----------------------------------------------------------------------------- RMSNorm roofline
RMS_ROWS = (4096, 65536)
RMS_COLS = 4096


def rmsnorm_roofline(peaks, iters=10):
    """rmsnorm_batch_invariant on x f32 [B, 4096] for B in RMS_ROWS: achieved GB/s of the
    algorithmic bytes 2*B*4096*4 + 4096*4 (read x and w, write y) against the measured HBM copy
    peak.  B = 65536 moves 2.1 GB per call (no L2 reuse); B = 4096 (134 MB) flushes L2 first."""
    import torch

    from detkernels_b200.kernels.rmsnorm import rmsnorm_batch_invariant

    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    w = 1 + 0.1 * torch.randn(RMS_COLS, device=dev, generator=g)
    res = {}
    for B in RMS_ROWS:
        x = torch.randn(B, RMS_COLS, device=dev, generator=g)
        out = rmsnorm_batch_invariant(x, w)
        ts = []
        for i in range(iters + 3):
            if B * RMS_COLS * 4 < 2 * flush.numel():
                flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = rmsnorm_batch_invariant(x, w)
            e.record()
            e.synchronize()
            if i >= 3:
                ts.append(s.elapsed_time(e))
        ms = statistics.median(ts)
        nbytes = 2 * B * RMS_COLS * 4 + RMS_COLS * 4
        gbs = nbytes / ms / 1e6
        res["B=%d" % B] = {"us": round(ms * 1e3, 2), "achieved_gbs": round(gbs, 1),
                           "frac_hbm": round(gbs / peaks["hbm_gbs"], 4), "algorithmic_bytes": nbytes}
        del x, out
    del flush
    return res


# DRAM bytes (read + write) per algorithmic byte of the single-row decode attention kernel, from
# one ncu capture of a launch at this workload's shape (256 rows, 16 heads, d 64, KV lengths of a
# mid-decode step: 363.12 MB read + 4.16 MB written for 355.68 MB algorithmic); the kernel reads
# each KV byte once plus each row's last 16-token group in full, so traffic scales with the
# algorithmic bytes of a launch.
ATTN_DRAM_PER_ALGO_BYTE = (363124480 + 4161024) / 355680256


# ----------------------------------------------------------------------------- gated delta rule
GDN = dict(n_seqs=64, min_len=256, max_len=4096, H=16, HV=32, D=128, decode_steps=300)


def gdn_bench(peaks, iters=3):
    """Chunked prefill of 64 packed sequences (lengths U{256..4096}) and 300 single-token
    decode steps of the same 64 sequences, GVA 16 q/k heads / 32 v heads, d = 128, bf16
    inputs, f32 state.  Inputs exceed L2 (prefill q/k/v ~2 GB, decode state 134 MB x 2)."""
    import numpy as np
    import torch
    import torch.nn.functional as F

    from detkernels_b200.kernels.gdn import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule

    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = GDN
    rng = np.random.default_rng(7)
    lens = rng.integers(cfg["min_len"], cfg["max_len"] + 1, cfg["n_seqs"])
    T = int(lens.sum())
    H, HV, D = cfg["H"], cfg["HV"], cfg["D"]
    g = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(1, T, H, D, device=dev, generator=g).to(torch.bfloat16)
    k = F.normalize(torch.randn(1, T, H, D, device=dev, generator=g), p=2, dim=-1).to(torch.bfloat16)
    v = torch.randn(1, T, HV, D, device=dev, generator=g).to(torch.bfloat16)
    gate = F.logsigmoid(torch.randn(1, T, HV, device=dev, generator=g)).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(1, T, HV, device=dev, generator=g)).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), device=dev, dtype=torch.long)

    def timed(fn, n):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(n):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            ts.append(s.elapsed_time(e))
        return statistics.median(ts)

    state = {}

    def prefill():
        state["o"], state["h"] = chunk_gated_delta_rule(q, k, v, gate, beta, output_final_state=True, cu_seqlens=cu)

    t_pre = timed(prefill, iters)
    # algorithmic work of the chunked form (per v-head, 64-token chunk, d = 128)
    bytes_tok = (H * D * 2) * 2 + (HV * D * 2) * 2 + HV * 2 * 2
    flops_chunk = 6 * 64 * D * D + 10 * 64 * 64 * D + (2 / 3) * 64 ** 3
    pre_bytes = bytes_tok * T + cfg["n_seqs"] * HV * D * D * 4
    pre_flops = flops_chunk * HV * T / 64

    n = cfg["n_seqs"]
    steps = cfg["decode_steps"]
    dq = torch.randn(steps, n, 1, H, D, device=dev, generator=g).to(torch.bfloat16)
    dk = F.normalize(torch.randn(steps, n, 1, H, D, device=dev, generator=g), p=2, dim=-1).to(torch.bfloat16)
    dv = torch.randn(steps, n, 1, HV, D, device=dev, generator=g).to(torch.bfloat16)
    dg = F.logsigmoid(torch.randn(steps, n, 1, HV, device=dev, generator=g)).to(torch.bfloat16)
    db = torch.sigmoid(torch.randn(steps, n, 1, HV, device=dev, generator=g)).to(torch.bfloat16)

    def decode():
        h = state["h"]
        for t in range(steps):
            _, h = fused_recurrent_gated_delta_rule(dq[t], dk[t], dv[t], dg[t], db[t], initial_state=h,
                                                    output_final_state=True)

    t_dec = timed(decode, 1)
    dec_bytes = steps * (2 * n * HV * D * D * 4 + n * ((H * D * 2) * 2 + (HV * D * 2) * 2 + HV * 4))
    hbm = peaks["hbm_gbs"]
    return {
        "workload": "GDN: %d seqs x U{%d..%d} tok (T=%d), H %d / HV %d, d %d, bf16, f32 state; then %d decode steps"
                    % (n, cfg["min_len"], cfg["max_len"], T, H, HV, D, steps),
        "prefill": {"tok_per_s": round(T / t_pre * 1e3, 1), "ms": round(t_pre, 3),
                    "achieved_gbs": round(pre_bytes / t_pre / 1e6, 1),
                    "frac_hbm": round(pre_bytes / t_pre / 1e6 / hbm, 4),
                    "achieved_tflops": round(pre_flops / t_pre / 1e9, 2),
                    "frac_bf16_peak": round(pre_flops / t_pre / 1e9 / peaks["bf16_tflops"], 4)},
        "decode": {"steps_per_s": round(steps / t_dec * 1e3, 1), "us_per_step": round(t_dec / steps * 1e3, 2),
                   "achieved_gbs": round(dec_bytes / t_dec / 1e6, 1),
                   "frac_hbm": round(dec_bytes / t_dec / 1e6 / hbm, 4)},
    }


# ----------------------------------------------------------------------------- main arms
REF_DECODE_STEPS = 4   # decode steps per timed step of the reference arm (B = 256 each)


def run_reference(args, rank, world):
    """The reference's decode step on the host cores (ReferenceDecodeCPU), rank 0 only: each
    step is REF_DECODE_STEPS greedy decode steps of the 256 workload sequences."""
    if rank != 0:
        return 0
    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig

    threads = len(os.sched_getaffinity(0))
    model = TinyModel(TinyModelConfig(**MODEL), device="cpu")
    ref = ReferenceDecodeCPU(model, make_prompts(0, BATCH_PER_GPU), REF_DECODE_STEPS, threads)
    secs = []
    for i in range(args.warmup + args.steps):
        dt = ref.run(REF_DECODE_STEPS)
        if i >= args.warmup:
            secs.append(dt)
    total = sum(secs)
    value = ref.B * REF_DECODE_STEPS * len(secs) / total
    sample = ref.describe(REF_DECODE_STEPS) + " per step"
    line = {"impl": "reference", "metric": "BI decode tok/s", "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total / len(secs) * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random prompts, random-init weights)",
            "config": workload_config(1), "parallelism": "host cores (%d threads)" % threads, "sample": sample,
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, rank, world, local):
    import numpy as np
    import torch

    from detkernels_b200 import _lib
    from detkernels_b200.kernels.tiny_model import TinyModel, TinyModelConfig

    dev = torch.device("cuda", local)
    model = TinyModel(TinyModelConfig(**MODEL), device=str(dev))
    tp = args.tp
    group = None
    if tp > 1:
        # tensor parallel: every rank serves the same 256 prompts with 1/tp of every layer
        import torch.distributed as dist
        if world != tp:
            raise SystemExit("--tp %d needs %d ranks (torchrun --nproc-per-node %d), got %d" % (tp, tp, tp, world))
        group = dist.group.WORLD
        prompts = make_prompts(0, BATCH_PER_GPU)
    else:
        prompts = make_prompts(rank, BATCH_PER_GPU)
    gen_kw = {"tp": tp, "group": group} if tp > 1 else {}
    cap = max(len(p) for p in prompts) + NEW_TOKENS
    if tp > 1:
        eng = model.tp_engine(tp, BATCH_PER_GPU, max(cap, OTHER_LEN[1] + NEW_TOKENS), group)
    else:
        eng = model.engine(BATCH_PER_GPU, max(cap, OTHER_LEN[1] + NEW_TOKENS))
    plan = eng.plan(prompts)

    # solo reference for the tracked prompt (divergence check); a TP solo run is collective
    solo = None
    if rank == 0 or tp > 1:
        solo = model.generate([prompts[0]], NEW_TOKENS, "batch_invariant", **gen_kw)[0].clone()

    for _ in range(args.warmup):
        eng.run(plan, NEW_TOKENS, timing=False)
    eng.run(plan, NEW_TOKENS, timing=True)   # capture the event-carrying graph outside the timed region
    torch.cuda.synchronize(dev)

    sampler = ClockSampler(list(range(world)) if world > 1 else [torch.cuda.current_device()])
    if rank == 0:
        sampler.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    n0 = _lib.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    acc = {"ms": 0.0, "n": 0, "pending": False}

    def collect():
        # attention launch durations of the previous step, from events recorded inside
        # its decode graph; read while this step's prefill already occupies the GPU
        if acc["pending"]:
            times = eng.attention_times_ms()
            acc["ms"] += sum(times)
            acc["n"] += len(times)
            acc["pending"] = False

    # Per-launch attention times come from external events recorded inside the decode graph
    # of the LAST timed step only: an event between two kernels ends their programmatic
    # overlap, so recording them in every step would slow the step it measures.
    outs = []
    start.record()
    for i in range(args.steps):
        last = (i == args.steps - 1)
        outs.append(eng.run(plan, NEW_TOKENS, timing=last))
        acc["pending"] = last
    end.record()
    torch.cuda.synchronize(dev)
    collect()
    attn_ms, attn_n = acc["ms"], acc["n"]
    barrier(world)
    clocks = sampler.stop() if rank == 0 else None
    launches = _lib.launch_count() - n0
    ms_total = start.elapsed_time(end)
    ms_max = max_over_ranks(ms_total, world)
    ms_per_step = ms_max / args.steps
    tokens_all = float(len(prompts) * NEW_TOKENS * args.steps)
    if tp == 1:
        tokens_all = sum_over_ranks(tokens_all, world)
    value = tokens_all / (ms_max / 1e3)

    # divergences: tracked row identical in every timed step and to its solo run
    divergences = 0
    if rank == 0:
        for o in outs:
            if not torch.equal(o[0], solo):
                divergences += 1

    # ---- in-graph decode matmul times: one more run, untimed, whose decode graph brackets every
    # matmul (with its split-K fold) by events; the events end those launches' programmatic
    # overlap, which is why the timed steps carry none ----
    gemm_times = None
    if tp == 1:
        eng.run(plan, NEW_TOKENS, gemm_timing=True)
        gemm_times = eng.gemm_times_ms()

    # ---- end-to-end through the public API with host buffers ----
    for _ in range(0 if args.skip_e2e else 2):   # warm the public path (graph captured on first use)
        model.generate(prompts, NEW_TOKENS, "batch_invariant", **gen_kw).cpu()
    barrier(world)
    torch.cuda.synchronize(dev)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d = 0
    d2h = 0
    e_start.record()
    for _ in range(0 if args.skip_e2e else args.steps):
        res = model.generate(prompts, NEW_TOKENS, "batch_invariant", **gen_kw)
        host = res.cpu()
        d2h = host.numel() * host.element_size()
    e_end.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    h2d = eng.plan(prompts)["h2d_bytes"]
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
    e2e_value = None if args.skip_e2e else tokens_all / (e2e_ms / 1e3)
    if tp > 1:
        # CUDA graphs that hold NCCL calls go before the process group does
        del eng
        model._engines.clear()
        torch.cuda.synchronize(dev)
        barrier(world)

    if rank != 0:
        return 0

    # ---- roofline of the dominant kernel (decode attention, HBM bound) ----
    peaks, peak_kind = load_peaks()
    lens = np.array([len(p) for p in prompts], dtype=np.int64)
    H, D = MODEL["num_heads"] // tp, MODEL["head_dim"]     # one rank's heads
    steps_dec = NEW_TOKENS - 1
    kv_bytes = 0
    for t in range(steps_dec):
        kv_bytes += int((lens + t + 1).sum()) * H * D * 2 * 2  # K and V, bf16
    qo_bytes = len(prompts) * H * D * 2 * 2
    per_step_bytes = (kv_bytes + steps_dec * qo_bytes) * MODEL["num_layers"]
    launches_per_step = steps_dec * MODEL["num_layers"]
    avg_bytes = per_step_bytes / launches_per_step
    avg_ms = attn_ms / max(attn_n, 1)
    achieved = avg_bytes / (avg_ms / 1e3) / 1e9
    roofline = {"kernel": "attn_kernel<bf16,64> (decode attention)", "bound": "hbm",
                "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peak_kind,
                "traffic": int(avg_bytes * ATTN_DRAM_PER_ALGO_BYTE), "avg_launch_us": round(avg_ms * 1e3, 2),
                "algorithmic_bytes_per_launch": int(avg_bytes),
                "share_of_step": round(attn_ms / ms_per_step, 3)}

    decode_gemm = decode_gemm_table(gemm_times, eng, len(prompts), peaks) if gemm_times else None

    cpu = cpu_baseline_sample() if world == 1 and not args.skip_cpu else None
    _, cpu_toks = (cpu_sample(cpu_sample_prompts(), 16, model) if world == 1 and not args.skip_cpu
                   else (None, None))
    parity = None
    if cpu_toks is not None:
        ours_small = model.generate(cpu_sample_prompts(), 16, "batch_invariant").cpu().numpy()
        parity = {"oracle_token_match": float((ours_small == cpu_toks).mean()),
                  "tracked_prefix_match": int(np.argmin(np.append(ours_small[0] == cpu_toks[0], False)))}

    gemm = gemm_vs_cublas() if not args.skip_gemm and world == 1 else None
    rms = rmsnorm_roofline(peaks) if world == 1 else None
    gdn = gdn_bench(peaks) if not args.skip_gdn and world == 1 else None

    line = {
        "metric": "BI decode tok/s", "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": True, "scaling": "strong" if tp > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random prompts, random-init weights)",
        "config": workload_config(1 if tp > 1 else world),
        "parallelism": ("tp%d (every layer split over %d ranks, NCCL all-gather of f32 slice sums)" % (tp, tp)
                        if tp > 1 else "dp%d (request-sharded, no collective)" % world),
        "e2e": {"value": e2e_value and round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "clocks": clocks,
        "divergences": divergences,
        "parity": parity,
        "gemm_vs_cublas": gemm,
        "decode_gemm": decode_gemm,
        "rmsnorm_roofline": rms,
        "gdn": gdn,
    }
    print(json.dumps(line), flush=True)
    return 0


def decode_gemm_table(times, eng, rows, peaks):
    """Per matmul family of the decode step (times from events inside the decode graph, each
    launch with its split-K fold): mean µs per launch, the weight bytes it streams, and those
    bytes per second against the HBM peak (the weights are the matmul's algorithmic bytes: the
    activations of 256 rows are < 6 % of them)."""
    weights = {"qkv": eng.layers[0]["w_qkv"], "o": eng.layers[0]["w_o"],
               "gate_up": eng.layers[0].get("w_gu", eng.layers[0].get("w_mlp1")), "down": eng.layers[0]["w_mlp2"],
               "lm_head": eng.model.w_lm_head}
    out = {}
    step_us = 0.0
    n_steps = NEW_TOKENS - 1
    for label, ms in times.items():
        w = weights.get(label)
        if w is None or not ms:
            continue
        us = 1e3 * sum(ms) / len(ms)
        wb = w.numel() * w.element_size()
        out[label] = {"launches_per_step": round(len(ms) / n_steps, 2), "us": round(us, 2), "weight_bytes": int(wb),
                      "achieved_gbs": round(wb / (us * 1e-6) / 1e9, 1),
                      "frac_hbm": round(wb / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 4),
                      "tflops": round(2.0 * rows * w.numel() / (us * 1e-6) / 1e12, 1)}
        step_us += us * len(ms) / n_steps
    out["per_decode_step_us"] = round(step_us, 1)
    return out


def main(argv=None):
    global NEW_TOKENS
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-gemm", action="store_true", help="skip the GEMM-vs-cuBLAS table")
    ap.add_argument("--skip-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--skip-e2e", action="store_true", help="skip the end-to-end public-API timing")
    ap.add_argument("--skip-gdn", action="store_true", help="skip the gated-delta-rule section")
    ap.add_argument("--gdn-only", action="store_true", help="run and print only the gated-delta-rule section")
    ap.add_argument("--rmsnorm-only", action="store_true", help="run and print only the RMSNorm roofline section")
    ap.add_argument("--gemm-only", default=None, metavar="M,N",
                    help="run and print only matmul_batch_invariant [M,4096] x [4096,N] against cuBLAS (profiling)")
    ap.add_argument("--gemm-kernel", choices=["auto", "one", "pair", "wide"], default="auto",
                    help="with --gemm-only: the planner's kernel, the one-CTA kernel, the CTA-pair kernel "
                         "(256 x 128 tiles) or the wide CTA-pair kernel (256 x 256 tiles)")
    ap.add_argument("--tp", type=int, default=1, choices=[1, 2, 4, 8],
                    help="tensor-parallel decode over the torchrun ranks (needs --nproc-per-node TP)")
    ap.add_argument("--new-tokens", type=int, default=NEW_TOKENS,
                    help="tokens generated per prompt (the workload is 128; smaller only for profiling)")
    args = ap.parse_args(argv)
    NEW_TOKENS = args.new_tokens
    if args.gemm_only:
        import torch
        torch.cuda.set_device(0)
        m, n = (int(v) for v in args.gemm_only.split(","))
        if args.gemm_kernel != "auto":
            import ctypes

            from detkernels_b200 import _lib
            hook = _lib.load().dk_matmul_pair_schedule_for_test   # not in the public header
            hook.restype, hook.argtypes = ctypes.c_int, [ctypes.c_int]
            hook({"one": 1, "pair": 2, "wide": 3}[args.gemm_kernel])
        global GEMM_SHAPES
        GEMM_SHAPES = [(m, n)]
        print(json.dumps({"gemm_vs_cublas": gemm_vs_cublas(iters=5)}), flush=True)
        return 0
    if args.gdn_only or args.rmsnorm_only:
        import torch
        torch.cuda.set_device(0)
        peaks, _ = load_peaks()
        section = {"gdn": gdn_bench(peaks)} if args.gdn_only else {"rmsnorm_roofline": rmsnorm_roofline(peaks)}
        print(json.dumps(section), flush=True)
        return 0
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, rank, int(os.environ.get("WORLD_SIZE", "1")))
    rank, world, local = dist_setup(args.gpus)
    try:
        return run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
