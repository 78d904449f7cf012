"""numpy restatement of the reference's eager formulas (the oracle).

All arithmetic is float32 unless stated; bf16/f16 tensors are carried as the
float32 values they hold, and every op ends with the reference's cast back to
the storage dtype (``round_to``).
"""
from __future__ import annotations

import numpy as np

from .numerics import round_to


# --------------------------------------------------------------------------
# kernels/rmsnorm.py:39-48  rmsnorm_reference
#   x32 = x.float(); var = mean(x32^2); y = x32 * rsqrt(var + eps) * w; cast back
# --------------------------------------------------------------------------
def rmsnorm(x, w, eps=1e-6, dtype="float32"):
    x32 = np.asarray(x, dtype=np.float32)
    var = np.mean(x32 * x32, axis=-1, keepdims=True, dtype=np.float32)
    rstd = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    y = (x32 * rstd).astype(np.float32) * np.asarray(w, dtype=np.float32)
    return round_to(y, dtype)


# --------------------------------------------------------------------------
# kernels/matmul.py:42-49  matmul_reference:  (a.float() @ b.float()).to(a.dtype)
# --------------------------------------------------------------------------
def matmul(a, b, dtype="bfloat16"):
    a32 = np.asarray(a, dtype=np.float32)
    b32 = np.asarray(b, dtype=np.float32)
    return round_to(a32 @ b32, dtype)


def slice_len(K, n_slices=8):
    """Slice length of the batch-invariant matmul's K split: ceil16(ceil(K / 8))."""
    per = -(-K // n_slices)
    return -(-per // 16) * 16


def matmul_slice_partials(a, b, slice_begin=0, slice_end=8):
    """f32 partial products of K slices [slice_begin, slice_end) of a @ b, each [M, N]
    (the split that detkernels_b200's invariant matmul folds; tolerance oracle for its
    per-slice sums, exact bookkeeping oracle for sharding and fold order)."""
    a32 = np.asarray(a, dtype=np.float32)
    b32 = np.asarray(b, dtype=np.float32)
    K = a32.shape[1]
    L = slice_len(K)
    out = []
    for s in range(slice_begin, slice_end):
        k0, k1 = min(s * L, K), min((s + 1) * L, K)
        out.append(a32[:, k0:k1] @ b32[k0:k1] if k1 > k0 else np.zeros((a32.shape[0], b32.shape[1]), np.float32))
    return out


def fold_tree(parts):
    """Pairwise tree over 1, 2, 4 or 8 f32 partials in order: ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7))."""
    parts = [np.asarray(p, dtype=np.float32) for p in parts]
    while len(parts) > 1:
        parts = [(parts[i] + parts[i + 1]).astype(np.float32) for i in range(0, len(parts), 2)]
    return parts[0]


def matmul_f64(a, b):
    """Exact-ish f64 product of the operand values (for error bounds)."""
    return np.asarray(a, dtype=np.float64) @ np.asarray(b, dtype=np.float64)


# --------------------------------------------------------------------------
# kernels/attention.py:49-71  attention_reference (einsum, softmax, einsum; f32),
# extended with grouped kv heads (q head h reads kv head h // (H / H_kv)),
# per-row KV lengths and a row -> KV-sequence map.
# --------------------------------------------------------------------------
def _softmax(s):
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def attention(q, k, v, scale=None, kv_lens=None, row_seq=None, dtype="bfloat16"):
    """q [R, H, D]; k, v [N, H_kv, S, D]; returns [R, H, D] rounded to dtype."""
    q32 = np.asarray(q, dtype=np.float32)
    k32 = np.asarray(k, dtype=np.float32)
    v32 = np.asarray(v, dtype=np.float32)
    R, H, D = q32.shape
    Hkv = k32.shape[1]
    G = H // Hkv
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    out = np.zeros((R, H, D), dtype=np.float32)
    for r in range(R):
        n = r if row_seq is None else int(row_seq[r])
        L = k32.shape[2] if kv_lens is None else int(kv_lens[r])
        if L == 0:
            continue
        kk = np.repeat(k32[n, :, :L], G, axis=0)  # [H, L, D]
        vv = np.repeat(v32[n, :, :L], G, axis=0)
        s = np.einsum("hd,hsd->hs", q32[r], kk).astype(np.float32) * np.float32(scale)
        p = _softmax(s).astype(np.float32)
        out[r] = np.einsum("hs,hsd->hd", p, vv)
    return round_to(out, dtype)


# --------------------------------------------------------------------------
# kernels/tiny_model.py:99-140  TinyModel.forward_step (pre-norm residual blocks),
# with the SwiGLU and grouped-kv-head options of this library's TinyModelConfig.
# --------------------------------------------------------------------------
def silu(x):
    x32 = np.asarray(x, dtype=np.float32)
    return x32 / (np.float32(1.0) + np.exp(-x32))


class _SeqCache:
    """One sequence's K or V cache of one layer: [Hkv, n, D] f32 in a buffer that doubles when full
    (appending is O(1) amortised, where concatenating every step is O(n))."""

    def __init__(self, hkv, d):
        self.k = np.zeros((hkv, 16, d), dtype=np.float32)
        self.v = np.zeros((hkv, 16, d), dtype=np.float32)
        self.n = 0

    def append(self, k, v):
        if self.n == self.k.shape[1]:
            grow = lambda a: np.concatenate([a, np.zeros_like(a)], axis=1)  # noqa: E731
            self.k, self.v = grow(self.k), grow(self.v)
        self.k[:, self.n] = k
        self.v[:, self.n] = v
        self.n += 1
        return self.k[:, :self.n], self.v[:, :self.n]


class TinyModelOracle:
    """Decode loop over numpy copies of a TinyModel's weights.

    weights: dict with 'embed', 'layers' (list of dicts), 'norm_f_w', 'w_lm_head'
    as float32 arrays holding the model's storage-dtype values."""

    def __init__(self, weights, num_heads, num_kv_heads, head_dim, eps=1e-6, mlp="silu", dtype="bfloat16"):
        self.w = weights
        self.H, self.Hkv, self.D = num_heads, num_kv_heads, head_dim
        self.eps, self.mlp, self.dtype = eps, mlp, dtype

    def step(self, tokens, caches):
        """tokens: [B] ints; caches: per layer list of per-sequence caches (``empty_caches``; mutated)."""
        dt = self.dtype
        H, Hkv, D = self.H, self.Hkv, self.D
        B = len(tokens)
        x = self.w["embed"][np.asarray(tokens)]
        for li, layer in enumerate(self.w["layers"]):
            xn = rmsnorm(x, layer["norm1_w"], self.eps, dt)
            q = matmul(xn, layer["w_q"], dt).reshape(B, H, D)
            k = matmul(xn, layer["w_k"], dt).reshape(B, Hkv, D)
            v = matmul(xn, layer["w_v"], dt).reshape(B, Hkv, D)
            attn = np.zeros((B, H, D), dtype=np.float32)
            for b in range(B):
                kc, vc = caches[li][b].append(k[b], v[b])
                attn[b] = attention(q[b:b + 1], kc[None], vc[None], dtype=dt)[0]
            o = matmul(attn.reshape(B, H * D), layer["w_o"], dt)
            x = round_to(x + o, dt)
            xn2 = rmsnorm(x, layer["norm2_w"], self.eps, dt)
            if self.mlp == "swiglu":
                gte = round_to(silu(matmul(xn2, layer["w_gate"], dt)), dt)
                up = matmul(xn2, layer["w_up"], dt)
                h = round_to(gte * up, dt)
            else:
                h = round_to(silu(matmul(xn2, layer["w_mlp1"], dt)), dt)
            x = round_to(x + matmul(h, layer["w_mlp2"], dt), dt)
        xf = rmsnorm(x, self.w["norm_f_w"], self.eps, dt)
        return matmul(xf, self.w["w_lm_head"], dt)

    def empty_caches(self, batch):
        return [[_SeqCache(self.Hkv, self.D) for _ in range(batch)] for _ in self.w["layers"]]

    def generate(self, prompts, n_steps, margins=None, follow=None, regrets=None):
        """Greedy decode; prompts: list of token lists. Returns (tokens [B, n_steps], last logits).
        margins (optional list): receives per row the top-1 minus top-2 logit of every generated
        token's step, so a caller can tell a near-tie from a real disagreement.
        follow (optional [B][n_steps] tokens, teacher forcing): the sequence continues with these
        tokens instead of the oracle's choice (the oracle's argmax is still returned), and regrets
        (optional list) receives per row max(logits) - logits[follow token] at every step."""
        B = len(prompts)
        if margins is not None:
            margins[:] = [[] for _ in range(B)]
        if regrets is not None:
            regrets[:] = [[] for _ in range(B)]
        caches = self.empty_caches(B)
        maxp = max(len(p) for p in prompts)
        # feed prompts token by token; a row whose prompt is exhausted starts generating
        out = [[] for _ in range(B)]
        cur = [p[0] for p in prompts]
        pos = [0] * B
        logits = None
        total_steps = maxp + n_steps
        for _ in range(total_steps):
            active = [b for b in range(B) if len(out[b]) < n_steps]
            if not active:
                break
            sub_caches = [[caches[li][b] for b in active] for li in range(len(caches))]
            logits = self.step([cur[b] for b in active], sub_caches)
            for i, b in enumerate(active):
                for li in range(len(caches)):
                    caches[li][b] = sub_caches[li][i]
                pos[b] += 1
                if pos[b] < len(prompts[b]):
                    cur[b] = prompts[b][pos[b]]
                else:
                    nxt = int(np.argmax(logits[i]))
                    if follow is not None:
                        forced = int(follow[b][len(out[b])])
                        if regrets is not None:
                            regrets[b].append(float(logits[i][nxt] - logits[i][forced]))
                        out[b].append(nxt)
                        cur[b] = forced
                    else:
                        out[b].append(nxt)
                        cur[b] = nxt
                    if margins is not None:
                        top2 = np.partition(logits[i], -2)[-2:]
                        margins[b].append(float(top2[1] - top2[0]))
        return np.asarray(out, dtype=np.int64), logits


# --------------------------------------------------------------------------
# Gated Delta Rule recurrence -- the math of FLA's naive_recurrent_gated_delta_rule
# (fla 0.5.1, fla/ops/gated_delta_rule/naive.py), the third-party function behind the
# reference's GDN call sites (gdn/repro.py:76, 161-162, 293-294).  Per head, per token:
#   S <- S * exp(g_t)
#   u  = beta_t * (v_t - S^T k_t)
#   S <- S + k_t u^T
#   o_t = S^T (scale * q_t)
# Value head j reads query/key head j // (HV / H).  State S is [K, V], f32.
# --------------------------------------------------------------------------
def gdn_recurrent(q, k, v, g, beta, scale=None, initial_state=None, cu_seqlens=None, dtype="bfloat16",
                  acc=np.float32, v_heads=None):
    """q, k [T, H, K]; v [T, HV, V]; g, beta [T, HV]; initial_state [N, HV, K, V].

    Returns (o [T, HV, V] rounded to dtype, final_state [N, HV, K, V] f32).  v_heads (optional):
    compute only these value heads (the others stay zero) -- for long sequences."""
    q = np.asarray(q, dtype=acc)
    k = np.asarray(k, dtype=acc)
    v = np.asarray(v, dtype=acc)
    g = np.asarray(g, dtype=acc)
    beta = np.asarray(beta, dtype=acc)
    T, H, K = q.shape
    HV, V = v.shape[1], v.shape[2]
    grp = HV // H
    if scale is None:
        scale = 1.0 / (K ** 0.5)
    if cu_seqlens is None:
        cu_seqlens = [0, T]
    N = len(cu_seqlens) - 1
    o = np.zeros((T, HV, V), dtype=acc)
    final = np.zeros((N, HV, K, V), dtype=acc)
    for n in range(N):
        bos, eos = int(cu_seqlens[n]), int(cu_seqlens[n + 1])
        for j in (range(HV) if v_heads is None else v_heads):
            hq = j // grp
            S = np.zeros((K, V), dtype=acc) if initial_state is None else np.asarray(
                initial_state[n, j], dtype=acc).copy()
            for t in range(bos, eos):
                S = S * np.exp(g[t, j])
                u = beta[t, j] * (v[t, j] - k[t, hq] @ S)
                S = S + np.outer(k[t, hq], u)
                o[t, j] = (q[t, hq] * acc(scale)) @ S
            final[n, j] = S
    return round_to(o.astype(np.float32), dtype), final.astype(np.float32)
