"""Random-weight decode-only transformer over the batch-invariant kernels.

Drop-in for the reference's ``kernels/tiny_model.py``:

* ``TinyModelConfig`` (tiny_model.py:50-62) with the same fields and defaults,
  plus keyword extensions: ``num_kv_heads`` (grouped KV heads), ``mlp``
  (``"silu"``: the reference's ``silu(x W1) W2``; ``"swiglu"``:
  ``(silu(x Wg) * x Wu) W2``) and ``dtype`` (the reference's float16 by default).
* ``TinyModel.__init__`` (tiny_model.py:70-97) draws the weights in the
  reference's order from a seeded generator on the model's device, so the same
  config and seed give the same weights.
* ``TinyModel.forward_step`` (tiny_model.py:99-140) and ``TinyModel.generate``
  (tiny_model.py:142-157) keep the reference's signatures and semantics
  (growing KV dicts, greedy argmax).  ``generate`` also accepts a list of
  token-id lists as ragged prompts.
* ``_KERNEL_SETS`` (tiny_model.py:36-47): ``batch_invariant``,
  ``batch_variant``, plus ``reference`` (the eager torch formulas, any device).

``DecodeEngine`` is the serving path used by ``generate`` for the invariant
kernel set on CUDA: a preallocated (zeroed) KV cache, prompts prefilled as
rows through the same per-row kernels (attention row tiles give exactly the
bits of token-by-token decoding), fused QKV and gate/up weights (every output
column is computed exactly as by the separate matmul), the element-wise ops
fused into the matmul that produces their input (K/V written straight into the
cache, residual adds, SiLU and SiLU*up, the greedy argmax) with the rounding of
the unfused torch ops, and the decode step captured once in a CUDA graph.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

from .attention import attention_batch_invariant, attention_batch_variant, attention_decode, attention_reference
from .matmul import argmax_finish, matmul_batch_invariant, matmul_batch_variant, matmul_fused, matmul_reference
from .rmsnorm import rmsnorm_batch_invariant, rmsnorm_batch_variant, rmsnorm_gather, rmsnorm_reference

_KERNEL_SETS = {
    "batch_invariant": {
        "rmsnorm": rmsnorm_batch_invariant,
        "matmul": matmul_batch_invariant,
        "attention": attention_batch_invariant,
    },
    "batch_variant": {
        "rmsnorm": rmsnorm_batch_variant,
        "matmul": matmul_batch_variant,
        "attention": attention_batch_variant,
    },
    "reference": {
        "rmsnorm": rmsnorm_reference,
        "matmul": matmul_reference,
        "attention": attention_reference,
    },
}


@dataclass
class TinyModelConfig:
    vocab_size: int = 256
    num_layers: int = 4
    num_heads: int = 4
    head_dim: int = 32
    mlp_hidden: int = 256
    eps: float = 1e-6
    seed: int = 0
    num_kv_heads: Optional[int] = None
    mlp: str = "silu"
    dtype: str = "float16"

    @property
    def hidden_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_heads(self) -> int:
        return self.num_heads if self.num_kv_heads is None else self.num_kv_heads


def _torch_dtype(name):
    import torch
    return {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[name]


class TinyModel:
    """Random-weight decode-only transformer (reference tiny_model.py:64-157)."""

    def __init__(self, config: TinyModelConfig, device: str = "cuda"):
        import torch

        if config.mlp not in ("silu", "swiglu"):
            raise ValueError("mlp must be 'silu' or 'swiglu'")
        if config.num_heads % config.kv_heads != 0:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.config = config
        self.device = device
        self.dtype = _torch_dtype(config.dtype)

        h = config.hidden_size
        hkv = config.kv_heads * config.head_dim
        g = torch.Generator(device=device).manual_seed(config.seed)

        def randn(*shape):
            return 0.02 * torch.randn(*shape, device=device, dtype=self.dtype, generator=g)

        self.embed = randn(config.vocab_size, h)
        self.layers = []
        for _ in range(config.num_layers):
            layer = {
                "norm1_w": randn(h) + 1.0,
                "w_q": randn(h, h),
                "w_k": randn(h, hkv),
                "w_v": randn(h, hkv),
                "w_o": randn(h, h),
                "norm2_w": randn(h) + 1.0,
            }
            if config.mlp == "swiglu":
                layer["w_gate"] = randn(h, config.mlp_hidden)
                layer["w_up"] = randn(h, config.mlp_hidden)
            else:
                layer["w_mlp1"] = randn(h, config.mlp_hidden)
            layer["w_mlp2"] = randn(config.mlp_hidden, h)
            self.layers.append(layer)
        self.norm_f_w = randn(h) + 1.0
        self.w_lm_head = randn(h, config.vocab_size)
        self._engines = {}

    # ---- fused weights for the serving path (same bits per output column) ----
    def fused_layer_weights(self):
        """Per layer: w_qkv = [w_q | w_k | w_v]; for SwiGLU, w_gu with gate and up columns
        interleaved (2j = gate j, 2j+1 = up j) for the fused SiLU*up epilogue."""
        import torch

        fused = []
        for layer in self.layers:
            f = {"norm1_w": layer["norm1_w"], "norm2_w": layer["norm2_w"], "w_o": layer["w_o"],
                 "w_mlp2": layer["w_mlp2"],
                 "w_qkv": torch.cat([layer["w_q"], layer["w_k"], layer["w_v"]], dim=1).contiguous()}
            if self.config.mlp == "swiglu":
                f["w_gu"] = torch.stack([layer["w_gate"], layer["w_up"]], dim=2).reshape(
                    layer["w_gate"].shape[0], -1).contiguous()
            else:
                f["w_mlp1"] = layer["w_mlp1"]
            fused.append(f)
        return fused

    def _mlp(self, layer, xn, matmul):
        import torch

        if self.config.mlp == "swiglu":
            gte = torch.nn.functional.silu(matmul(xn, layer["w_gate"]))
            return matmul(gte * matmul(xn, layer["w_up"]), layer["w_mlp2"])
        return matmul(torch.nn.functional.silu(matmul(xn, layer["w_mlp1"])), layer["w_mlp2"])

    def forward_step(self, token_ids, kv_cache, kernel_set: str):
        """One decode step: token_ids (B,) int64 -> next-token logits (B, vocab_size),
        and the updated per-layer KV cache (list of {"k", "v"}: [B, H_kv, S, D])."""
        import torch

        fns = _KERNEL_SETS[kernel_set]
        rmsnorm, matmul, attention = fns["rmsnorm"], fns["matmul"], fns["attention"]
        cfg = self.config
        B = token_ids.shape[0]
        H, Hkv, D = cfg.num_heads, cfg.kv_heads, cfg.head_dim

        x = self.embed[token_ids]
        new_kv_cache = []
        for i, layer in enumerate(self.layers):
            residual = x
            xn = rmsnorm(x, layer["norm1_w"], cfg.eps)
            q = matmul(xn, layer["w_q"]).view(B, H, D)
            k_new = matmul(xn, layer["w_k"]).view(B, Hkv, 1, D)
            v_new = matmul(xn, layer["w_v"]).view(B, Hkv, 1, D)
            prev = kv_cache[i]
            if prev is None:
                k_cache, v_cache = k_new, v_new
            else:
                k_cache = torch.cat([prev["k"], k_new], dim=2)
                v_cache = torch.cat([prev["v"], v_new], dim=2)
            new_kv_cache.append({"k": k_cache, "v": v_cache})
            attn_out = attention(q, k_cache, v_cache).reshape(B, H * D)
            x = residual + matmul(attn_out, layer["w_o"])
            residual2 = x
            x = residual2 + self._mlp(layer, rmsnorm(x, layer["norm2_w"], cfg.eps), matmul)
        logits = matmul(rmsnorm(x, self.norm_f_w, cfg.eps), self.w_lm_head)
        return logits, new_kv_cache

    def generate(self, prompt_token_ids, n_steps: int, kernel_set: str, *, tp: int = 1, group=None,
                 kv_page_size: Optional[int] = None):
        """Greedy decoding.  prompt_token_ids: (B,) int64 start tokens (the
        reference's form) or a list of B token-id lists (ragged prompts).
        Returns (B, n_steps) generated token ids.

        tp / group (keyword-only, invariant kernel set on CUDA): decode with every layer split
        over ``tp`` tensor-parallel ranks -- the ranks of ``group`` (a torch.distributed group of
        ``tp`` processes, each calling generate with the same prompts), or, with ``group=None``,
        all ``tp`` ranks in this process on this model's GPU.  The tokens equal TP=1's bit for bit.
        kv_page_size (keyword-only, invariant set on CUDA): keep the KV cache in blocks of that many
        tokens (a multiple of 64) behind a block table; the tokens are the same bits."""
        import torch

        ragged = isinstance(prompt_token_ids, (list, tuple))
        if kv_page_size is not None and (kernel_set != "batch_invariant" or not str(self.device).startswith("cuda")
                                         or tp != 1 or group is not None):
            raise ValueError("a paged KV cache is served by the one-GPU batch_invariant engine on CUDA")
        if tp != 1 or group is not None:
            if kernel_set != "batch_invariant" or not str(self.device).startswith("cuda"):
                raise ValueError("tensor-parallel decoding runs the batch_invariant kernel set on CUDA")
            prompts = (list(prompt_token_ids) if ragged else [[int(t)] for t in prompt_token_ids.tolist()])
            cap = max(len(p) for p in prompts) + n_steps
            return self.tp_engine(tp, len(prompts), cap, group).generate(prompts, n_steps)
        if kernel_set == "batch_invariant" and str(self.device).startswith("cuda"):
            # ragged prompts go to the engine as given (any int sequence; the plan reads them
            # with numpy); a (B,) tensor becomes B one-token prompts
            prompts = (list(prompt_token_ids) if ragged else [[int(t)] for t in prompt_token_ids.tolist()])
            cap = max(len(p) for p in prompts) + n_steps
            eng = self.engine(len(prompts), cap, page_size=kv_page_size)
            return eng.generate(prompts, n_steps)
        if ragged:
            return self._generate_ragged_eager(prompt_token_ids, n_steps, kernel_set)
        kv_cache = [None] * self.config.num_layers
        current = prompt_token_ids
        generated = []
        for _ in range(n_steps):
            logits, kv_cache = self.forward_step(current, kv_cache, kernel_set)
            current = logits.argmax(dim=-1)
            generated.append(current)
        return torch.stack(generated, dim=1)

    def _generate_ragged_eager(self, prompts, n_steps, kernel_set):
        """Ragged prompts on the eager path: each sequence is decoded alone."""
        import torch

        outs = []
        for p in prompts:
            kv_cache = [None] * self.config.num_layers
            ids = torch.tensor(list(p), device=self.device, dtype=torch.long)
            logits = None
            for t in range(len(p)):
                logits, kv_cache = self.forward_step(ids[t:t + 1], kv_cache, kernel_set)
            seq = []
            cur = logits.argmax(dim=-1)
            for s in range(n_steps):
                seq.append(cur)
                if s + 1 < n_steps:
                    logits, kv_cache = self.forward_step(cur, kv_cache, kernel_set)
                    cur = logits.argmax(dim=-1)
            outs.append(torch.cat(seq))
        return torch.stack(outs)

    def tp_engine(self, tp: int, max_batch: int, max_seq_len: int, group=None, use_graph: bool = True):
        """A cached tensor-parallel engine (see ``tp_model.TPDecodeEngine``)."""
        from .tp_model import TPDecodeEngine

        gid = id(group) if group is not None else None
        for (kind, t, g_id, b, s, g), eng in self._engines.items():
            if kind == "tp" and t == tp and g_id == gid and b >= max_batch and s >= max_seq_len and g == use_graph:
                return eng
        eng = TPDecodeEngine(self, tp, max_batch, max_seq_len, group=group, use_graph=use_graph)
        self._engines[("tp", tp, gid, max_batch, max_seq_len, use_graph)] = eng
        return eng

    def engine(self, max_batch: int, max_seq_len: int, use_graph: bool = True,
               page_size: Optional[int] = None) -> "DecodeEngine":
        """A cached DecodeEngine whose capacity covers (max_batch, max_seq_len); page_size: a paged
        KV cache of blocks of that many tokens (a multiple of 64) instead of one slab per sequence."""
        kind = "dp" if page_size is None else ("paged", int(page_size))
        for (k, _, _, b, s, g), eng in self._engines.items():
            if k == kind and b >= max_batch and s >= max_seq_len and g == use_graph:
                return eng
        eng = DecodeEngine(self, max_batch, max_seq_len, use_graph=use_graph, page_size=page_size)
        self._engines[(kind, 1, None, max_batch, max_seq_len, use_graph)] = eng
        return eng


class BlockAllocator:
    """Host-side owner of a paged KV pool's blocks.  Block 0 is never handed out: padding rows
    and unused table entries point at it.  ``assign`` starts from a free pool and gives slot b
    ceil(tokens[b] / page) blocks in a seeded shuffled order, so neighbouring sequences do not
    get neighbouring blocks; a request the pool cannot hold raises RuntimeError."""

    def __init__(self, n_blocks: int, max_slots: int, blocks_per_seq: int, seed: int = 0):
        import numpy as np

        if n_blocks < 2:
            raise ValueError("a paged pool needs at least two blocks")
        self.n_blocks, self.max_slots, self.blocks_per_seq = n_blocks, max_slots, blocks_per_seq
        self.order = np.random.default_rng(seed).permutation(np.arange(1, n_blocks, dtype=np.int32))

    def assign(self, tokens, page):
        import numpy as np

        need = [-(-int(t) // page) for t in tokens]
        if len(need) > self.max_slots or any(n > self.blocks_per_seq for n in need):
            raise ValueError("more sequences or tokens than the engine was built for")
        if sum(need) > self.n_blocks - 1:
            raise RuntimeError("KV block pool exhausted: %d blocks needed, %d available"
                               % (sum(need), self.n_blocks - 1))
        table = np.zeros((self.max_slots, self.blocks_per_seq), dtype=np.int32)
        pos = 0
        for b, n in enumerate(need):
            table[b, :n] = self.order[pos:pos + n]
            pos += n
        return table


class DecodeEngine:
    """Batch-invariant serving loop for a TinyModel on one GPU.

    KV cache: per layer [max_batch, H_kv, max_seq_len, D] in the model dtype,
    zero-initialised.  A sequence's arithmetic never depends on its batch: every
    op is per-row, prefill rows of one sequence share attention tiles that
    reproduce decode-row bits, and the decode graph has a fixed shape (rows
    beyond the live batch are computed and ignored)."""

    MAX_GRAPHS = 8   # captured decode graphs kept per engine

    def __init__(self, model: TinyModel, max_batch: int, max_seq_len: int, use_graph: bool = True,
                 page_size: Optional[int] = None, n_blocks: Optional[int] = None):
        import torch

        from detkernels_b200 import _lib

        self.model = model
        cfg = model.config
        self.cfg = cfg
        self.device = torch.device(model.device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = model.dtype
        self.B = int(max_batch)
        self.S = int(max_seq_len)
        self.H, self.Hkv, self.D = cfg.num_heads, cfg.kv_heads, cfg.head_dim
        self.h = cfg.hidden_size
        self.use_graph = use_graph
        self.layers = model.fused_layer_weights()
        dev, dt = self.device, self.dtype
        self.page_size = page_size
        self.block_table = None
        if page_size is None:
            self.k_cache = [torch.zeros(self.B, self.Hkv, self.S, self.D, device=dev, dtype=dt)
                            for _ in range(cfg.num_layers)]
        else:
            if page_size <= 0 or page_size % 64:
                raise ValueError("page_size must be a positive multiple of 64, got %r" % (page_size,))
            per_seq = -(-self.S // page_size)
            if n_blocks is None:
                n_blocks = 1 + self.B * per_seq      # block 0 + every slot at full capacity
            self.allocator = BlockAllocator(int(n_blocks), self.B, per_seq)
            self.k_cache = [torch.zeros(int(n_blocks), self.Hkv, page_size, self.D, device=dev, dtype=dt)
                            for _ in range(cfg.num_layers)]
            self.block_table = torch.zeros(self.B, per_seq, dtype=torch.int32, device=dev)
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        # decode-step state
        self.tokens = torch.zeros(self.B, dtype=torch.long, device=dev)
        self.kv_lens = torch.zeros(self.B, dtype=torch.int32, device=dev)   # cache write position
        self.q_lens = torch.ones(self.B, dtype=torch.int32, device=dev)     # kv_lens + 1
        self.argmax_keys = torch.zeros(self.B, dtype=torch.int64, device=dev)
        self._graphs = {}
        self._last_events = None
        self._gemm_events = None        # list of (label, start, end) while a GEMM-timing graph is captured
        self._last_gemm_events = None
        # explicit scratch so captured graphs never allocate
        self._lib = _lib
        lib = _lib.load()
        qkv_n = (self.H + 2 * self.Hkv) * self.D
        gemm_shapes = [(self.B, qkv_n, self.h), (self.B, self.h, self.h), (self.B, self.h, cfg.mlp_hidden),
                       (self.B, cfg.vocab_size, self.h),
                       (self.B, 2 * cfg.mlp_hidden if cfg.mlp == "swiglu" else cfg.mlp_hidden, self.h)]
        g_ws = max(lib.dk_matmul_workspace_size(m, n, k) for (m, n, k) in gemm_shapes)
        a_ws = lib.dk_attention_workspace_size(self.B, 1, self.H, self.Hkv, self.D, self.S)
        self.gemm_ws = torch.zeros(max(g_ws, 1), dtype=torch.uint8, device=dev)
        self.attn_ws = torch.zeros(max(a_ws, 1), dtype=torch.uint8, device=dev)

    # ---------------- building blocks (all per-row) ----------------
    def _mm(self, x, w, epilogue="store", label=None, **kw):
        """matmul_fused on the engine's workspace; while a GEMM-timing graph is being captured,
        the call (the GEMM and its split-K fold) is bracketed by external events under `label`."""
        ev = getattr(self, "_gemm_events", None)
        if ev is None or label is None:
            return matmul_fused(x, w, epilogue, workspace=self.gemm_ws, **kw)
        import torch
        s, e = (torch.cuda.Event(enable_timing=True, external=True),
                torch.cuda.Event(enable_timing=True, external=True))
        s.record()
        out = matmul_fused(x, w, epilogue, workspace=self.gemm_ws, **kw)
        e.record()
        ev.append((label, s, e))
        return out

    def _next_norm_w(self, li):
        """The RMSNorm weight applied to block li's output: block li+1's input norm, or the final norm."""
        return self.layers[li + 1]["norm1_w"] if li + 1 < len(self.layers) else self.model.norm_f_w

    def _layer(self, li, layer, x, xn, write_seq, write_pos, q_lens, row_tiles, max_len, attn_ws, events=None):
        """One transformer block over R rows; xn = rmsnorm(x, norm1_w).  Returns (x', xn') with
        xn' = x' under the next norm (block li+1's input norm or the final norm), computed by the
        down projection's epilogue.  The QKV matmul writes K/V of every row to (write_seq,
        write_pos) (int32; write_seq None: row r is sequence r) before attention reads them."""
        import torch

        cfg = self.cfg
        R = x.shape[0]
        H, D = self.H, self.D
        q = self._mm(xn, layer["w_qkv"], "qkv_cache", q_cols=H * D, head_dim=D, k_cache=self.k_cache[li],
                     v_cache=self.v_cache[li], row_seq=write_seq, row_pos=write_pos, block_table=self.block_table,
                     label="qkv")
        if events is not None:
            events[0].record()
        attn = attention_decode(q.view(R, H, D), self.k_cache[li], self.v_cache[li], q_lens, row_tiles=row_tiles,
                                max_kv_len=max_len, workspace=attn_ws, block_table=self.block_table)
        if events is not None:
            events[1].record()
        xn = torch.empty_like(x)
        x = self._mm(attn.reshape(R, H * D), layer["w_o"], "residual_rmsnorm", residual=x,
                     norm_weight=layer["norm2_w"], norm_out=xn, eps=cfg.eps, label="o")
        if cfg.mlp == "swiglu":
            hid = self._mm(xn, layer["w_gu"], "silu_mul", label="gate_up")
        else:
            hid = self._mm(xn, layer["w_mlp1"], "silu", label="gate_up")
        xn_next = torch.empty_like(x)
        x = self._mm(hid, layer["w_mlp2"], "residual_rmsnorm", residual=x, norm_weight=self._next_norm_w(li),
                     norm_out=xn_next, eps=cfg.eps, label="down")
        return x, xn_next

    def _logits(self, xn):
        """Logits of rows already under the final norm."""
        return self._mm(xn, self.model.w_lm_head)

    # ---------------- prefill ----------------
    def plan(self, prompts: Sequence[Sequence[int]]):
        """Device-side description of a prefill: every prompt token is a row."""
        import torch

        import numpy as np

        dev = self.device
        B = len(prompts)
        assert 0 < B <= self.B, "batch exceeds engine capacity"
        G = self.H // self.Hkv
        rows_per_tile = 16 // G
        lens = np.fromiter((len(p) for p in prompts), dtype=np.int64, count=B)
        assert (lens > 0).all() and (lens <= self.S).all(), "prompt longer than engine capacity"
        tok = np.concatenate([np.asarray(p, dtype=np.int64).reshape(-1) for p in prompts])
        starts = np.cumsum(lens) - lens                       # first row of each prompt
        rows = np.repeat(np.arange(B, dtype=np.int64), lens)  # row -> prompt
        pos = np.arange(tok.size, dtype=np.int64) - np.repeat(starts, lens)
        # tiles of up to rows_per_tile consecutive rows of one prompt: (first row, rows, prompt)
        n_t = (lens + rows_per_tile - 1) // rows_per_tile
        t_b = np.repeat(np.arange(B, dtype=np.int64), n_t)
        t_k = np.arange(int(n_t.sum()), dtype=np.int64) - np.repeat(np.cumsum(n_t) - n_t, n_t)
        tiles = np.stack([starts[t_b] + t_k * rows_per_tile,
                          np.minimum(rows_per_tile, lens[t_b] - t_k * rows_per_tile), t_b], axis=1)
        host = {
            "tok": torch.from_numpy(tok),
            "rows": torch.from_numpy(rows),
            "pos": torch.from_numpy(pos),
            "tiles": torch.from_numpy(tiles.astype(np.int32)),
            "last": torch.from_numpy(starts + lens - 1),
            "lens": torch.from_numpy(lens.astype(np.int32)),
        }
        plan = {k: v.pin_memory().to(dev, non_blocking=True) for k, v in host.items()}
        plan["q_lens"] = (plan["pos"] + 1).to(torch.int32)
        plan["rows32"] = plan["rows"].to(torch.int32)
        plan["pos32"] = plan["pos"].to(torch.int32)
        plan["B"] = B
        plan["lens_host"] = lens
        plan["max_len"] = int(lens.max())
        plan["h2d_bytes"] = sum(v.numel() * v.element_size() for v in host.values())
        lib = self._lib.load()
        R = host["tok"].numel()
        a_ws = lib.dk_attention_workspace_size(len(tiles), 2, self.H, self.Hkv, self.D, plan["max_len"])
        g_ws = max([lib.dk_matmul_workspace_size(R, n, k) for (n, k) in [
            ((self.H + 2 * self.Hkv) * self.D, self.h), (self.h, self.h), (self.h, self.cfg.mlp_hidden),
            (2 * self.cfg.mlp_hidden, self.h), (self.cfg.mlp_hidden, self.h)]] +
            [lib.dk_matmul_workspace_size(B, self._head_cols(), self.h)])   # the LM head on B last rows
        plan["attn_ws"] = torch.zeros(max(a_ws, 1), dtype=torch.uint8, device=dev)
        plan["gemm_ws"] = torch.zeros(max(g_ws, 1), dtype=torch.uint8, device=dev)
        return plan

    def _reserve_blocks(self, plan, n_steps):
        """Paged cache: blocks for every prompt plus n_steps tokens (from a fresh pool; the slots
        past the batch and unused table entries point at block 0, which the padding rows of a
        decode step may write)."""
        if self.block_table is None:
            return
        import torch

        lens = plan["lens_host"]
        table = self.allocator.assign([int(L) + n_steps for L in lens], self.page_size)
        self.block_table.copy_(torch.from_numpy(table).pin_memory(), non_blocking=True)

    def prefill(self, plan):
        """Run a planned prefill; returns logits of each prompt's last token and
        leaves the cache and kv_lens ready for decoding."""
        if self.block_table is not None and plan.get("reserved") is None:
            self._reserve_blocks(plan, 1)
        saved = self.gemm_ws
        self.gemm_ws = plan["gemm_ws"]
        try:
            x, xn = rmsnorm_gather(self.model.embed, plan["tok"], self.layers[0]["norm1_w"], self.cfg.eps)
            for li, layer in enumerate(self.layers):
                x, xn = self._layer(li, layer, x, xn, plan["rows32"], plan["pos32"], plan["q_lens"], plan["tiles"],
                                    plan["max_len"], plan["attn_ws"])
            logits = self._logits(xn[plan["last"]])
        finally:
            self.gemm_ws = saved
        self.kv_lens.zero_()
        self.kv_lens[:plan["B"]] = plan["lens"]
        self.q_lens.copy_(self.kv_lens + 1)
        return logits

    def _head_cols(self):
        """Columns of the LM head matmul this engine runs."""
        return self.cfg.vocab_size

    def _prefill_tokens(self, plan):
        """Greedy first token of each prompt (device int64 [B])."""
        return self.prefill(plan).argmax(dim=-1)

    # ---------------- decode ----------------
    def _decode_step(self, max_len, out_row=None, events=None):
        """tokens -> next tokens (also into out_row) for all rows; K/V written at kv_lens,
        then kv_lens and q_lens advance.  max_len bounds every row's length after this
        step (sizes the attention grid)."""
        import torch

        x, xn = rmsnorm_gather(self.model.embed, self.tokens, self.layers[0]["norm1_w"], self.cfg.eps)
        for li, layer in enumerate(self.layers):
            ev = None
            if events is not None:
                ev = (torch.cuda.Event(enable_timing=True, external=True),
                      torch.cuda.Event(enable_timing=True, external=True))
                events.append(ev)
            x, xn = self._layer(li, layer, x, xn, None, self.kv_lens, self.q_lens, None, max_len, self.attn_ws, ev)
        self._mm(xn, self.model.w_lm_head, "argmax", argmax_keys=self.argmax_keys, label="lm_head")
        argmax_finish(self.argmax_keys, self.tokens, out_row, self.kv_lens, self.q_lens)
        return self.tokens

    def _capture(self, n_steps, start_len, timing, gemm_timing=False):
        """Capture n_steps decode steps (one graph) starting from rows of length <= start_len.
        timing: events around every attention launch; gemm_timing: around every matmul (with
        its fold).  Both end the programmatic overlap of the launches they bracket."""
        import torch

        out = torch.empty((n_steps, self.B), dtype=torch.long, device=self.device)
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        saved = (self.tokens.clone(), self.kv_lens.clone(), self.q_lens.clone())
        with torch.cuda.stream(s):   # warm-up: lazy loads and tensor-map encoding
            self._decode_step(start_len + 1)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.tokens.copy_(saved[0])
        self.kv_lens.copy_(saved[1])
        self.q_lens.copy_(saved[2])
        events = [] if timing else None
        gemm_events = [] if gemm_timing else None
        g = torch.cuda.CUDAGraph()
        n0 = self._lib.launch_count()
        self._gemm_events = gemm_events
        try:
            with torch.cuda.graph(g):
                for t in range(n_steps):
                    self._decode_step(min(start_len + t + 1, self.S), out[t], events)
        finally:
            self._gemm_events = None
        n_graph = self._lib.launch_count() - n0
        self._lib.count_launch(-n_graph)  # recorded, not executed; counted at each replay
        return g, out, events, n_graph, gemm_events

    def decode(self, n_steps: int, start_len: Optional[int] = None, timing: bool = False, gemm_timing: bool = False):
        """Run n_steps decode steps from the current tokens/kv_lens; returns [n_steps, B]
        (device).  start_len bounds the current kv_lens (defaults to the capacity).
        With timing=True, per-launch attention durations of the run are available
        from attention_times_ms() afterwards."""
        import torch

        if n_steps <= 0:
            return torch.empty((0, self.B), dtype=torch.long, device=self.device)
        if start_len is None:
            start_len = self.S - n_steps
        # the bound only sizes the attention grid (a row's bits follow its own length), so it is
        # rounded up to the 256-token KV split: batches of similar lengths share a captured graph
        start_len = min(-(-int(start_len) // 256) * 256, self.S - n_steps)
        if not self.use_graph:
            out = torch.empty((n_steps, self.B), dtype=torch.long, device=self.device)
            for t in range(n_steps):
                self._decode_step(min(start_len + t + 1, self.S), out[t])
            return out
        key = (n_steps, start_len, timing, gemm_timing)
        if key not in self._graphs:
            while len(self._graphs) >= self.MAX_GRAPHS:     # oldest capture first
                self._graphs.pop(next(iter(self._graphs)))
            self._graphs[key] = self._capture(n_steps, start_len, timing, gemm_timing)
        g, out, events, n_graph, gemm_events = self._graphs[key]
        g.replay()
        self._lib.count_launch(n_graph)
        self._last_events = events
        self._last_gemm_events = gemm_events
        return out

    def attention_times_ms(self):
        """Durations (ms) of every attention launch of the last timed decode.
        Waits for that decode's last event only (not the whole device)."""
        evs = self._last_events or []
        if not evs:
            return []
        evs[-1][1].synchronize()
        return [a.elapsed_time(b) for a, b in evs]

    def gemm_times_ms(self):
        """{label: [ms, ...]} of every matmul launch (with its fold) of the last decode run with
        gemm_timing=True; labels qkv, o, gate_up, down, lm_head."""
        evs = self._last_gemm_events or []
        if not evs:
            return {}
        evs[-1][2].synchronize()
        out = {}
        for label, s, e in evs:
            out.setdefault(label, []).append(s.elapsed_time(e))
        return out

    def run(self, plan, n_steps: int, timing: bool = False, before_decode=None, gemm_timing: bool = False):
        """Prefill + greedy decode; returns [B, n_steps] generated ids (device).
        before_decode (optional) is called on the host after the prefill has been
        queued and before the decode graph is launched."""
        import torch

        B = plan["B"]
        if n_steps <= 0:
            return torch.empty((B, 0), dtype=torch.long, device=self.device)
        if plan["max_len"] + n_steps > self.S:
            raise ValueError("prompt + n_steps exceeds the engine's max_seq_len")
        if self.block_table is not None:
            self._reserve_blocks(plan, n_steps)
            plan["reserved"] = n_steps
        first = self._prefill_tokens(plan)
        self.tokens.zero_()
        self.tokens[:B] = first
        if before_decode is not None:
            before_decode()
        rest = self.decode(n_steps - 1, start_len=plan["max_len"], timing=timing, gemm_timing=gemm_timing)
        return torch.cat([first[:, None], rest[:, :B].t()], dim=1)

    def generate(self, prompts: Sequence[Sequence[int]], n_steps: int):
        """Greedy decode of n_steps tokens after each prompt; returns [B, n_steps] (device)."""
        return self.run(self.plan(prompts), n_steps)
