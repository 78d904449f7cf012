"""Generate the golden fixtures in this directory from the REFERENCE's own code.

Run where a checkout of the reference exists (the path is an argument or
$DETKERNELS_REFERENCE; nothing on the GPU side runs it):

    python tests/golden/make_golden.py <path to the reference checkout>

* rmsnorm / matmul / attention: the reference's eager ``*_reference`` functions
  (kernels/rmsnorm.py:39-48, kernels/matmul.py:42-49, kernels/attention.py:49-71)
  on seeded CPU inputs.
* tiny_model: the reference's ``TinyModel`` (kernels/tiny_model.py:64-157) on
  CPU, with its ``_KERNEL_SETS`` given a set made of the same ``*_reference``
  functions (the reference ships only GPU kernel sets); its weights and the
  logits of three decode steps are stored.
* gdn: FLA's pure-torch ``naive_recurrent_gated_delta_rule`` (fla 0.5.1, the
  reference's GDN call sites' third-party dependency; gdn/repro.py:76) on
  per-sequence slices of a packed batch, q/k heads repeated to the value heads.

Fixtures are small .npz files; 16-bit tensors are stored as their float32
values plus a dtype tag.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def f32(t):
    return t.detach().float().cpu().numpy()


def main(ref_root):
    import torch

    sys.path.insert(0, ref_root)
    from kernels.attention import attention_reference
    from kernels.matmul import matmul_reference
    from kernels.rmsnorm import rmsnorm_reference
    import kernels.tiny_model as tm

    g = torch.Generator().manual_seed(1234)

    # ---- rmsnorm: several shapes / dtypes ----
    out = {}
    for i, (rows, cols, dt) in enumerate([(4, 4096, torch.float32), (3, 1000, torch.float16),
                                          (2, 37, torch.bfloat16), (64, 256, torch.float32)]):
        x = torch.randn(rows, cols, generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(cols, generator=g)).to(dt)
        y = rmsnorm_reference(x, w, 1e-6)
        out["x%d" % i], out["w%d" % i], out["y%d" % i] = f32(x), f32(w), f32(y)
        out["dtype%d" % i] = np.array(str(dt).split(".")[-1])
    np.savez_compressed(os.path.join(HERE, "rmsnorm.npz"), **out)

    # ---- matmul ----
    out = {}
    for i, (m, k, n, dt) in enumerate([(3, 256, 128, torch.bfloat16), (8, 1024, 64, torch.float16),
                                       (1, 4096, 32, torch.bfloat16), (17, 100, 40, torch.bfloat16)]):
        a = torch.randn(m, k, generator=g).to(dt)
        b = (0.02 * torch.randn(k, n, generator=g)).to(dt)
        c = matmul_reference(a, b)
        out["a%d" % i], out["b%d" % i], out["c%d" % i] = f32(a), f32(b), f32(c)
        out["dtype%d" % i] = np.array(str(dt).split(".")[-1])
    np.savez_compressed(os.path.join(HERE, "matmul.npz"), **out)

    # ---- attention (reference shapes: q [B,H,D], k/v [B,H,S,D]) ----
    out = {}
    for i, (bsz, h, s, d, dt) in enumerate([(2, 4, 128, 64, torch.float16), (3, 2, 300, 32, torch.bfloat16),
                                            (1, 8, 1, 128, torch.bfloat16)]):
        q = torch.randn(bsz, h, d, generator=g).to(dt)
        k = torch.randn(bsz, h, s, d, generator=g).to(dt)
        v = torch.randn(bsz, h, s, d, generator=g).to(dt)
        o = attention_reference(q, k, v)
        out["q%d" % i], out["k%d" % i], out["v%d" % i], out["o%d" % i] = f32(q), f32(k), f32(v), f32(o)
        out["dtype%d" % i] = np.array(str(dt).split(".")[-1])
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)

    # ---- TinyModel (reference code, reference formulas, CPU) ----
    tm._KERNEL_SETS["golden_reference"] = {"rmsnorm": rmsnorm_reference, "matmul": matmul_reference,
                                           "attention": attention_reference}
    cfg = tm.TinyModelConfig(vocab_size=64, num_layers=2, num_heads=2, head_dim=32, mlp_hidden=128, seed=0)
    model = tm.TinyModel(cfg, device="cpu")
    out = {"embed": f32(model.embed), "norm_f_w": f32(model.norm_f_w), "w_lm_head": f32(model.w_lm_head)}
    for li, layer in enumerate(model.layers):
        for key, val in layer.items():
            out["L%d_%s" % (li, key)] = f32(val)
    tokens = torch.tensor([5, 17, 63])
    kv = [None] * cfg.num_layers
    cur = tokens
    for step in range(3):
        logits, kv = model.forward_step(cur, kv, "golden_reference")
        out["tokens%d" % step] = cur.numpy()
        out["logits%d" % step] = f32(logits)
        cur = logits.argmax(dim=-1)
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), **out)

    # ---- GDN (FLA naive recurrent, fp32) ----
    from fla.ops.gated_delta_rule.naive import naive_recurrent_gated_delta_rule
    import torch.nn.functional as F

    H, HV, K, V = 2, 4, 32, 32
    lens = [7, 40, 13]
    T = sum(lens)
    cu = np.concatenate([[0], np.cumsum(lens)])
    q = torch.randn(T, H, K, generator=g).to(torch.bfloat16)
    k = F.normalize(torch.randn(T, H, K, generator=g), p=2, dim=-1).to(torch.bfloat16)
    v = torch.randn(T, HV, V, generator=g).to(torch.bfloat16)
    gate = F.logsigmoid(torch.randn(T, HV, generator=g)).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn(T, HV, generator=g)).to(torch.bfloat16)
    h0 = 0.1 * torch.randn(len(lens), HV, K, V, generator=g)
    o_all = torch.zeros(T, HV, V)
    finals = []
    rep = HV // H
    for n in range(len(lens)):
        sl = slice(int(cu[n]), int(cu[n + 1]))
        qq = q[sl].float().repeat_interleave(rep, dim=1)[None]
        kk = k[sl].float().repeat_interleave(rep, dim=1)[None]
        o, ht = naive_recurrent_gated_delta_rule(qq, kk, v[sl].float()[None], beta[sl].float()[None],
                                                 gate[sl].float()[None], initial_state=h0[n:n + 1],
                                                 output_final_state=True)
        o_all[sl] = o[0]
        finals.append(ht[0])
    np.savez_compressed(os.path.join(HERE, "gdn.npz"), q=f32(q), k=f32(k), v=f32(v), g=f32(gate), beta=f32(beta),
                        h0=f32(h0), cu_seqlens=cu.astype(np.int64), o=f32(o_all), final=f32(torch.stack(finals)))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DETKERNELS_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py <reference checkout> (or set DETKERNELS_REFERENCE)")
    main(ref)
