"""Tensor-parallel TinyModel decoding (TP = 1, 2, 4 or 8), bitwise equal to one GPU.

No counterpart in the reference: its ``TinyModel`` runs on one device
(kernels/tiny_model.py:99-157).  The layers it shards are the ones of
``forward_step`` (tiny_model.py:114-139), split the Megatron way over the
batch-invariant matmul's fixed K slices:

* QKV (column-parallel): rank r owns query heads [r*H/tp, (r+1)*H/tp) and kv
  heads [r*Hkv/tp, (r+1)*Hkv/tp); its fused QKV matmul writes K/V of its heads
  into its own KV cache shard and attention runs on its heads only.
* Attention output projection (row-parallel): rank r's attention columns are
  exactly the K range of its aligned slice group of ``w_o``
  (``shard_k_range``); it computes that group's f32 subtree sum, the sums are
  gathered in rank order and every rank folds them along the upper levels of
  the slice tree with the residual + RMSNorm epilogue (``matmul_fold_fused``):
  the one-GPU fused layer's bits.
* Gate/up (column-parallel) and down projection (row-parallel): the hidden
  columns a rank's SiLU*up produces are the K range of its slice group of
  ``w_mlp2``; same gather and fold as above.
* LM head (column-parallel over the vocabulary): each rank folds its columns'
  greedy argmax into 64-bit keys; the keys are gathered and
  ``argmax_finish_parts`` picks the global argmax with the one-GPU tie rule.

Two ways to run the ranks: one process per rank over a ``torch.distributed``
group (NCCL all-gathers between the steps above), or every rank in this process
on one GPU, one after another between the exchanges (the exchange is then a
stack of the ranks' tensors) -- the form the bitwise tests use when fewer GPUs
than ranks are present.  The replicated state (residual stream, next tokens,
cache lengths) is shared by the ranks a process holds.
"""
from __future__ import annotations

from typing import List

from .attention import attention_decode
from .matmul import argmax_finish_parts, matmul_fold_fused, matmul_fused
from .rmsnorm import rmsnorm_gather
from .tiny_model import DecodeEngine
from .tp import K_SLICES, all_gather_ranks, check_agreement, shard_k_range, shard_n_range, shard_partial


class TPLayout:
    """Which heads, hidden columns and vocabulary columns each rank of a ``tp``-way split owns.

    Raises ValueError when the model's sizes do not line up with the matmul's fixed K slices
    (a rank's attention columns / MLP hidden columns must be its slice group's K range)."""

    def __init__(self, config, tp: int):
        if tp not in (1, 2, 4, 8):
            raise ValueError("tensor-parallel size must be 1, 2, 4 or 8, got %d" % tp)
        H, Hkv, D = config.num_heads, config.kv_heads, config.head_dim
        if H % tp or Hkv % tp:
            raise ValueError("TP=%d needs num_heads (%d) and num_kv_heads (%d) divisible by it" % (tp, H, Hkv))
        self.tp, self.H, self.Hkv, self.D = tp, H, Hkv, D
        self.h = config.hidden_size
        self.F = config.mlp_hidden
        self.V = config.vocab_size
        self.Hl, self.Hkvl = H // tp, Hkv // tp
        for r in range(tp):
            if shard_k_range(self.h, tp, r) != (r * self.Hl * D, (r + 1) * self.Hl * D):
                raise ValueError("TP=%d: the attention heads of rank %d do not match the output projection's "
                                 "K slice group %s" % (tp, r, shard_k_range(self.h, tp, r)))
            f0, f1 = shard_k_range(self.F, tp, r)
            if (f1 - f0) % 8 or f1 <= f0:
                raise ValueError("TP=%d: rank %d's MLP hidden range %s is empty or not a multiple of 8"
                                 % (tp, r, (f0, f1)))
        self.vocab_offsets = [shard_n_range(self.V, tp, r)[0] for r in range(tp)]

    def heads(self, r):
        return r * self.Hl, (r + 1) * self.Hl

    def kv_heads(self, r):
        return r * self.Hkvl, (r + 1) * self.Hkvl

    def hidden(self, r):
        return shard_k_range(self.F, self.tp, r)

    def vocab(self, r):
        return shard_n_range(self.V, self.tp, r)


def shard_weights(model, layout: TPLayout, rank: int):
    """Rank ``rank``'s weights: the columns / rows listed by ``layout``, contiguous."""
    import torch

    cfg = model.config
    D = cfg.head_dim
    q0, q1 = layout.heads(rank)
    k0, k1 = layout.kv_heads(rank)
    f0, f1 = layout.hidden(rank)
    n0, n1 = layout.vocab(rank)
    layers = []
    for L in model.layers:
        w = {"w_qkv": torch.cat([L["w_q"][:, q0 * D:q1 * D], L["w_k"][:, k0 * D:k1 * D],
                                 L["w_v"][:, k0 * D:k1 * D]], dim=1).contiguous(),
             "w_o": L["w_o"][q0 * D:q1 * D].contiguous(),
             "w_mlp2": L["w_mlp2"][f0:f1].contiguous()}
        if cfg.mlp == "swiglu":
            w["w_gu"] = torch.stack([L["w_gate"][:, f0:f1], L["w_up"][:, f0:f1]], dim=2).reshape(
                L["w_gate"].shape[0], -1).contiguous()
        else:
            w["w_mlp1"] = L["w_mlp1"][:, f0:f1].contiguous()
        layers.append(w)
    return {"layers": layers, "w_lm_head": model.w_lm_head[:, n0:n1].contiguous()}


class _Shard:
    """One rank's weights, KV cache and argmax keys."""

    def __init__(self, model, layout, rank, B, S, device):
        import torch

        self.rank = rank
        w = shard_weights(model, layout, rank)
        self.layers = w["layers"]
        self.w_lm_head = w["w_lm_head"]
        n_layers = model.config.num_layers
        self.k_cache = [torch.zeros(B, layout.Hkvl, S, layout.D, device=device, dtype=model.dtype)
                        for _ in range(n_layers)]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        self.keys = torch.zeros(B, dtype=torch.int64, device=device)


class TPDecodeEngine(DecodeEngine):
    """``DecodeEngine`` with every layer split over ``tp`` ranks (see the module docstring).

    group: a torch.distributed group of ``tp`` processes (this process is one rank), or None to
    hold all ``tp`` ranks in this process on the model's GPU."""

    def __init__(self, model, tp: int, max_batch: int, max_seq_len: int, group=None, use_graph: bool = True):
        import torch

        from detkernels_b200 import _lib

        self.layout = TPLayout(model.config, tp)
        self.tp = tp
        self.group = group
        if group is not None:
            import torch.distributed as dist
            if dist.get_world_size(group) != tp:
                raise ValueError("the process group has %d ranks, TP=%d" % (dist.get_world_size(group), tp))
            from dataclasses import asdict
            check_agreement(group, tp=tp, max_batch=int(max_batch), max_seq_len=int(max_seq_len),
                            config=asdict(model.config))
            local = [dist.get_rank(group)]
        else:
            local = list(range(tp))
        self.model = model
        cfg = model.config
        self.cfg = cfg
        self.device = torch.device(model.device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.dtype = model.dtype
        self.B, self.S = int(max_batch), int(max_seq_len)
        lay = self.layout
        # local head counts: attention planning and workspaces follow one rank's heads
        self.H, self.Hkv, self.D = lay.Hl, lay.Hkvl, lay.D
        self.h = cfg.hidden_size
        self.use_graph = use_graph
        self.page_size, self.block_table = None, None   # the shards keep contiguous caches
        self.shards: List[_Shard] = [_Shard(model, lay, r, self.B, self.S, self.device) for r in local]
        self.norms = [{"norm1_w": L["norm1_w"], "norm2_w": L["norm2_w"]} for L in model.layers]
        self.layers = self.norms   # the base class reads layers[li]["norm1_w"]
        dev = self.device
        self.tokens = torch.zeros(self.B, dtype=torch.long, device=dev)
        self.kv_lens = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.q_lens = torch.ones(self.B, dtype=torch.int32, device=dev)
        self._graphs = {}
        self._last_events = None
        self._lib = _lib
        lib = _lib.load()
        qkv_n = (lay.Hl + 2 * lay.Hkvl) * lay.D
        f_max = max(f1 - f0 for f0, f1 in (lay.hidden(r) for r in range(tp)))
        n_max = max(n1 - n0 for n0, n1 in (lay.vocab(r) for r in range(tp)))
        gemm_shapes = [(self.B, qkv_n, self.h), (self.B, 2 * f_max, self.h), (self.B, n_max, self.h)]
        g_ws = max(lib.dk_matmul_workspace_size(m, n, k) for (m, n, k) in gemm_shapes)
        a_ws = lib.dk_attention_workspace_size(self.B, 1, lay.Hl, lay.Hkvl, lay.D, self.S)
        self.gemm_ws = torch.zeros(max(g_ws, 1), dtype=torch.uint8, device=dev)
        self.attn_ws = torch.zeros(max(a_ws, 1), dtype=torch.uint8, device=dev)
        # the base class's single-GPU caches are not used; expose rank 0's for inspection
        self.k_cache = self.shards[0].k_cache
        self.v_cache = self.shards[0].v_cache

    # ---------------- exchange ----------------
    def _exchange(self, parts):
        """[tp, ...] stack of every rank's tensor, in rank order."""
        import torch

        if self.group is None:
            return torch.stack(parts)
        return all_gather_ranks(parts[0], self.group)

    # ---------------- layers ----------------
    def _layer(self, li, layer, x, xn, write_seq, write_pos, q_lens, row_tiles, max_len, attn_ws, events=None):
        import torch

        cfg, lay = self.cfg, self.layout
        R, D = x.shape[0], lay.D
        parts = []
        for sh in self.shards:
            w = sh.layers[li]
            q = self._mm(xn, w["w_qkv"], "qkv_cache", q_cols=lay.Hl * D, head_dim=D, k_cache=sh.k_cache[li],
                         v_cache=sh.v_cache[li], row_seq=write_seq, row_pos=write_pos)
            attn = attention_decode(q.view(R, lay.Hl, D), sh.k_cache[li], sh.v_cache[li], q_lens,
                                    row_tiles=row_tiles, max_kv_len=max_len, workspace=attn_ws)
            parts.append(shard_partial(attn.reshape(R, lay.Hl * D), w["w_o"], lay.h, lay.tp, sh.rank))
        xn = torch.empty_like(x)
        x = matmul_fold_fused(self._exchange(parts), x.dtype, "residual_rmsnorm", residual=x,
                              norm_weight=self.norms[li]["norm2_w"], norm_out=xn, eps=cfg.eps)
        parts = []
        for sh in self.shards:
            w = sh.layers[li]
            if cfg.mlp == "swiglu":
                hid = self._mm(xn, w["w_gu"], "silu_mul")
            else:
                hid = self._mm(xn, w["w_mlp1"], "silu")
            parts.append(shard_partial(hid, w["w_mlp2"], lay.F, lay.tp, sh.rank))
        xn_next = torch.empty_like(x)
        x = matmul_fold_fused(self._exchange(parts), x.dtype, "residual_rmsnorm", residual=x,
                              norm_weight=self._next_norm_w(li), norm_out=xn_next, eps=cfg.eps)
        return x, xn_next

    def _next_norm_w(self, li):
        return self.norms[li + 1]["norm1_w"] if li + 1 < len(self.norms) else self.model.norm_f_w

    def _argmax_step(self, xn, tokens, tokens_copy=None, lens_a=None, lens_b=None):
        """Greedy next token of every row of xn (rows under the final norm) into tokens."""
        n = xn.shape[0]   # the rows of this step; the key buffers are sized for the engine's capacity
        for sh in self.shards:
            self._mm(xn, sh.w_lm_head, "argmax", argmax_keys=sh.keys)
        gathered = self._exchange([sh.keys[:n] for sh in self.shards])
        argmax_finish_parts(gathered, self.layout.vocab_offsets, tokens, tokens_copy, lens_a, lens_b,
                            reset_keys=self.shards[0].keys)
        for sh in self.shards[1:]:
            sh.keys.zero_()
        return tokens

    def _head_cols(self):
        return max(n1 - n0 for n0, n1 in (self.layout.vocab(r) for r in range(self.tp)))

    # ---------------- prefill / decode ----------------
    def prefill(self, plan):
        raise NotImplementedError("a tensor-parallel engine returns next tokens, not full logits; use run()")

    def _prefill_tokens(self, plan):
        import torch

        saved = self.gemm_ws
        self.gemm_ws = plan["gemm_ws"]
        try:
            x, xn = rmsnorm_gather(self.model.embed, plan["tok"], self.norms[0]["norm1_w"], self.cfg.eps)
            for li in range(len(self.norms)):
                x, xn = self._layer(li, None, x, xn, plan["rows32"], plan["pos32"], plan["q_lens"], plan["tiles"],
                                    plan["max_len"], plan["attn_ws"])
            first = torch.empty(plan["B"], dtype=torch.long, device=self.device)
            self._argmax_step(xn[plan["last"]].contiguous(), first)
        finally:
            self.gemm_ws = saved
        self.kv_lens.zero_()
        self.kv_lens[:plan["B"]] = plan["lens"]
        self.q_lens.copy_(self.kv_lens + 1)
        return first

    def _decode_step(self, max_len, out_row=None, events=None):
        import torch

        x, xn = rmsnorm_gather(self.model.embed, self.tokens, self.norms[0]["norm1_w"], self.cfg.eps)
        for li in range(len(self.norms)):
            ev = None
            if events is not None:
                ev = (torch.cuda.Event(enable_timing=True, external=True),
                      torch.cuda.Event(enable_timing=True, external=True))
                events.append(ev)
            x, xn = self._layer(li, None, x, xn, None, self.kv_lens, self.q_lens, None, max_len, self.attn_ws, ev)
        self._argmax_step(xn, self.tokens, out_row, self.kv_lens, self.q_lens)
        return self.tokens


def slice_count() -> int:
    return K_SLICES
