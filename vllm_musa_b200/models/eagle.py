"""EAGLE draft head for the dense decoders (speculative decoding).

The head is one decoder layer that reads the target's own features: for a position p whose
next token t_{p+1} is known,

    x      = fc([embed(t_{p+1}) ; h_p])             h_p = the target's final hidden state at p
    x      = x + attn(x)                             (no input norm: the fc output goes in)
    x      = x + mlp(rmsnorm(x, post_attention_ln))
    logits = lm_head(x)  (or lm_head(rmsnorm(x, norm)) when the checkpoint has ``norm.weight``)
                                                     -> the draft of t_{p+2}

It shares the target's embedding, rotary tables, LM head and paged-KV block tables; its own
K/V live in one extra layer of the target's cache (the same pages and slots, so rejected
positions are simply overwritten later).  Under tensor parallelism it is sharded exactly like a
target layer (heads / intermediate / vocab) and its two reductions are the fused NVSwitch
all-reduce + residual + RMSNorm of the target, so every rank drafts the same token.

h_p is the target's final (normalised) hidden state, the feature vLLM's EAGLE proposer feeds
its heads.  Checkpoint layout (EAGLE-1, HuggingFace names): ``fc.weight`` [H, 2H] (optional
``fc.bias``), ``layers.0.self_attn.{q,k,v,o}_proj.weight``,
``layers.0.mlp.{gate,up,down}_proj.weight``, ``layers.0.post_attention_layernorm.weight``,
optional ``norm.weight``.  Extra tensors (a copy of the embedding, an input norm the head does
not use) are ignored.

With prefix caching, a reused block keeps the draft-layer K/V its first owner wrote; the entry
of a block's last position depends on the following token, so a later request may read a
slightly different feature there.  That only changes draft quality: verification is exact.
Reference counterparts: the reference drives vLLM's EAGLE proposers and prepares their inputs
with vllm_musa/v1/spec_decode/utils.py:4-124 and patches/vllm__v1__spec_decode__eagle.patch.py.
"""
from __future__ import annotations

from typing import Iterable, Tuple

import torch

from .. import ops
from .llama import _Layer, shard_cols, shard_rows


def eagle_param_shapes(cfg) -> list:
    """(name, shape, kind) of an EAGLE head for a target with config ``cfg``."""
    H, D = cfg.hidden_size, cfg.head_dim
    Hq, Hkv, I = cfg.num_heads, cfg.num_kv_heads, cfg.intermediate_size
    a, m = "layers.0.self_attn.", "layers.0.mlp."
    return [("fc.weight", (H, 2 * H), "w"),
            (a + "q_proj.weight", (Hq * D, H), "w"), (a + "k_proj.weight", (Hkv * D, H), "w"),
            (a + "v_proj.weight", (Hkv * D, H), "w"), (a + "o_proj.weight", (H, Hq * D), "w"),
            (m + "gate_proj.weight", (I, H), "w"), (m + "up_proj.weight", (I, H), "w"),
            (m + "down_proj.weight", (H, I), "w"),
            ("layers.0.post_attention_layernorm.weight", (H,), "norm")]


class EagleHead:
    """``replicated=True`` (draft tensor-parallel size 1 under a TP>1 target): every rank holds
    the whole head (all heads, the whole MLP) and its own K/V cache with all KV heads (same
    block ids and slots as the target's, allocated by the runner as ``own_kv``), so the draft
    layer runs without collectives; every rank computes the same drafts from the same
    (replicated) target hidden states.  The logits still go through the target's vocab-parallel
    LM head and sampler.  Reference: the per-rank TP=1 draft group of
    patches/vllm__distributed__parallel_state.patch.py:77-209."""

    def __init__(self, target, replicated: bool = False):
        if getattr(target, "tq", None) is not None:
            raise ValueError("EAGLE drafts need a bf16 KV cache (not TurboQuant)")
        self.t = target
        self.cfg = target.cfg
        self.layer = _Layer()
        self.fc = None
        self.fc_bias = None
        self.norm = None
        self.replicated = replicated and target.tp > 1
        self.cache_index = target.l1 - target.l0  # the extra cache layer after the target's
        self.own_kv = None
        if self.replicated:
            from ..attention import PagedAttention
            from ..parallel.communicator import LocalCommunicator
            cfg = self.cfg
            self.hq, self.hkv = cfg.num_heads, cfg.num_kv_heads
            self.attn = PagedAttention(self.hq, self.hkv, target.D)
            self.comm = LocalCommunicator(target.device)
        else:
            self.hq, self.hkv = target.hq, target.hkv
            self.attn, self.comm = target.attn, target.comm

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        t, L = self.t, self.layer
        st = {n: w for n, w in weights}
        miss = [n for n, _, k in eagle_param_shapes(self.cfg) if k == "w" and n not in st]
        if miss:
            raise RuntimeError(f"EAGLE checkpoint is missing {miss}")
        D, r, tp = t.D, t.rank, t.tp
        a, m = "layers.0.self_attn.", "layers.0.mlp."
        if self.replicated:
            L.qkv_w = t._to(torch.cat([st[a + "q_proj.weight"], st[a + "k_proj.weight"],
                                       st[a + "v_proj.weight"]], 0))
            L.o_w = t._to(st[a + "o_proj.weight"])
            gate, up, down = (st[m + n + "_proj.weight"] for n in ("gate", "up", "down"))
            pad = (-gate.shape[0]) % 8
            L.gu_w = t._to(ops.interleave_gate_up(gate, up))
            if pad:
                down = torch.cat([down, torch.zeros(down.shape[0], pad, dtype=down.dtype,
                                                    device=down.device)], 1)
            L.down_w = t._to(down)
        else:
            q = shard_rows(st[a + "q_proj.weight"], r, tp)
            k = st[a + "k_proj.weight"][t.kv0 * D:(t.kv0 + t.hkv) * D]
            v = st[a + "v_proj.weight"][t.kv0 * D:(t.kv0 + t.hkv) * D]
            L.qkv_w = t._to(torch.cat([q, k, v], 0))
            L.o_w = t._to(shard_cols(st[a + "o_proj.weight"], r, tp))
            L.gu_w, L.down_w = t._dense_mlp_weights(st[m + "gate_proj.weight"],
                                                    st[m + "up_proj.weight"],
                                                    st[m + "down_proj.weight"])
        H = self.cfg.hidden_size
        L.ln2 = t._to(st.get("layers.0.post_attention_layernorm.weight", torch.ones(H)))
        self.norm = t._to(st["norm.weight"]) if "norm.weight" in st else None
        self.fc = t._to(st["fc.weight"])
        self.fc_bias = t._to(st["fc.bias"]) if "fc.bias" in st else None

    @torch.no_grad()
    def forward_draft(self, next_ids: torch.Tensor, prev_hidden: torch.Tensor, meta,
                      kv_caches: list) -> torch.Tensor:
        """Hidden states whose logits draft token p+2 for each row (position p)."""
        t, L, cfg, eps = self.t, self.layer, self.cfg, self.cfg.rms_norm_eps
        comm = self.comm
        comm.begin_forward()
        e = ops.embedding(next_ids, t.embed)
        x = ops.linear(torch.cat([e, prev_hidden.to(e.dtype)], -1).contiguous(), self.fc)
        if self.fc_bias is not None:
            x = x + self.fc_bias
        residual = x
        kc, vc = self.own_kv if self.replicated else kv_caches[self.cache_index]
        qkv = ops.linear(x, L.qkv_w)
        ops.rope_kv(qkv, meta.positions, t.cos_sin, kc, vc, meta.slot_mapping, self.hq,
                    self.hkv, cfg.rot_dim, cfg.rope_neox, None, None, eps)
        a = self.attn.forward(qkv, kc, vc, meta)
        x, residual = comm.linear_allreduce_add_rmsnorm(a, L.o_w, residual, L.ln2, eps)
        act = ops.linear_silu_mul(x, L.gu_w)
        if self.norm is not None:  # (normalised for the logits, pre-norm for a chained step)
            return comm.linear_allreduce_add_rmsnorm(act, L.down_w, residual, self.norm, eps)
        return comm.all_reduce(ops.linear(act, L.down_w)) + residual

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.t.compute_logits(hidden)


def eagle3_param_shapes(cfg, draft_vocab: int | None = None) -> list:
    """(name, shape, kind) of an EAGLE-3 head (HuggingFace EAGLE-3 names) for a target with
    config ``cfg``; ``draft_vocab`` defaults to the target's vocabulary."""
    H, D = cfg.hidden_size, cfg.head_dim
    Hq, Hkv, I = cfg.num_heads, cfg.num_kv_heads, cfg.intermediate_size
    Vd = draft_vocab or cfg.vocab_size
    a, m = "midlayer.self_attn.", "midlayer.mlp."
    return [("fc.weight", (H, 3 * H), "w"),
            ("midlayer.input_layernorm.weight", (H,), "norm"),
            ("midlayer.hidden_norm.weight", (H,), "norm"),
            (a + "q_proj.weight", (Hq * D, 2 * H), "w"),
            (a + "k_proj.weight", (Hkv * D, 2 * H), "w"),
            (a + "v_proj.weight", (Hkv * D, 2 * H), "w"),
            (a + "o_proj.weight", (H, Hq * D), "w"),
            ("midlayer.post_attention_layernorm.weight", (H,), "norm"),
            (m + "gate_proj.weight", (I, H), "w"), (m + "up_proj.weight", (I, H), "w"),
            (m + "down_proj.weight", (H, I), "w"),
            ("norm.weight", (H,), "norm"), ("lm_head.weight", (Vd, H), "w")]


def eagle3_aux_layers(num_layers: int) -> tuple:
    """Target layers whose incoming residual stream feeds the head (low / middle / high),
    clamped into the model for very shallow targets."""
    return tuple(min(max(l, 0), num_layers - 1) for l in (2, num_layers // 2, num_layers - 3))


class Eagle3Head:
    """EAGLE-3 draft head over a dense decoder (``speculative_config={"method": "eagle3"}``).

    Its feature for a position p is three of the target's residual streams at p -- the ones
    entering layers ``eagle3_aux_layers`` (low, middle and high level) -- concatenated and
    projected by ``fc`` [H, 3H] to g.  With e = embed(t_{p+1}) from the target's table:

        x      = [rmsnorm(e, input_ln) ; rmsnorm(g, hidden_norm)]      2H wide
        g'     = g + o_proj(attn(x))                                   (q / k / v read 2H)
        out    = rmsnorm(g' + mlp(rmsnorm(g', post_attention_ln)), norm)
        logits = lm_head(out)                                          the draft vocabulary

    A draft token d maps to target token d + d2t[d] (identity without a ``d2t`` tensor).  The
    head runs whole on every rank with its own K/V cache (all KV heads, the target's block ids
    and slots), so it needs no collective; its logits are argmax-ed (or top-k for sibling
    trees) locally.  Reference counterparts: the EAGLE-3 proposer the reference's vLLM drives
    (patches/vllm__v1__spec_decode__eagle.patch.py) and the EAGLE-3 paper (Li et al., 2025)."""

    replicated = True

    def __init__(self, target):
        if getattr(target, "tq", None) is not None:
            raise ValueError("EAGLE-3 drafts need a bf16 KV cache")
        from ..attention import PagedAttention
        from ..parallel.communicator import LocalCommunicator
        self.t = target
        self.cfg = target.cfg
        self.layer = _Layer()
        self.hq, self.hkv = self.cfg.num_heads, self.cfg.num_kv_heads
        self.attn = PagedAttention(self.hq, self.hkv, target.D)
        self.comm = LocalCommunicator(target.device)
        self.own_kv = None
        self.aux_layers = eagle3_aux_layers(self.cfg.num_layers)

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        t, L = self.t, self.layer
        st = {n: w for n, w in weights}
        Vd = st["lm_head.weight"].shape[0] if "lm_head.weight" in st else None
        miss = [n for n, _, k in eagle3_param_shapes(self.cfg, Vd) if k == "w" and n not in st]
        if miss:
            raise RuntimeError(f"EAGLE-3 checkpoint is missing {miss}")
        H = self.cfg.hidden_size
        a, m = "midlayer.self_attn.", "midlayer.mlp."
        ones = torch.ones(H)
        L.qkv_w = t._to(torch.cat([st[a + "q_proj.weight"], st[a + "k_proj.weight"],
                                   st[a + "v_proj.weight"]], 0))
        L.o_w = t._to(st[a + "o_proj.weight"])
        gate, up, down = (st[m + n + "_proj.weight"] for n in ("gate", "up", "down"))
        pad = (-gate.shape[0]) % 8
        L.gu_w = t._to(ops.interleave_gate_up(gate, up))
        if pad:
            down = torch.cat([down, torch.zeros(down.shape[0], pad, dtype=down.dtype,
                                                device=down.device)], 1)
        L.down_w = t._to(down)
        L.ln2 = t._to(st.get("midlayer.post_attention_layernorm.weight", ones))
        self.in_ln = t._to(st.get("midlayer.input_layernorm.weight", ones))
        self.hidden_norm = t._to(st.get("midlayer.hidden_norm.weight", ones))
        self.norm = t._to(st.get("norm.weight", ones))
        self.fc = t._to(st["fc.weight"])
        self.lm_head = t._to(st["lm_head.weight"])
        d2t = st.get("d2t")
        self.d2t = None if d2t is None else d2t.to(device=t.device, dtype=torch.int64)

    @torch.no_grad()
    def forward_draft(self, next_ids: torch.Tensor, aux: torch.Tensor, meta,
                      kv_caches: list) -> torch.Tensor:
        """next_ids [T], aux [T, 3H] (the three residual streams of each position) -> the
        normalised hidden states whose logits draft token p+2."""
        t, L, cfg, eps = self.t, self.layer, self.cfg, self.cfg.rms_norm_eps
        comm = self.comm
        comm.begin_forward()
        e = ops.embedding(next_ids, t.embed)
        H = cfg.hidden_size
        # the target's three streams (first draft) or the head's own pre-norm output (chained)
        g = aux.to(e.dtype) if aux.shape[1] == H else \
            ops.linear(aux.to(e.dtype).contiguous(), self.fc)
        x = torch.cat([ops.rms_norm(e, self.in_ln, eps), ops.rms_norm(g, self.hidden_norm, eps)],
                      -1).contiguous()
        kc, vc = self.own_kv
        qkv = ops.linear(x, L.qkv_w)
        ops.rope_kv(qkv, meta.positions, t.cos_sin, kc, vc, meta.slot_mapping, self.hq,
                    self.hkv, cfg.rot_dim, cfg.rope_neox, None, None, eps)
        a = self.attn.forward(qkv, kc, vc, meta)
        x, residual = comm.linear_allreduce_add_rmsnorm(a, L.o_w, g, L.ln2, eps)
        act = ops.linear_silu_mul(x, L.gu_w)
        # (normalised for the logits, pre-norm for a chained step)
        return comm.linear_allreduce_add_rmsnorm(act, L.down_w, residual, self.norm, eps)

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """[S, H] -> fp32 logits over the draft vocabulary [S, Vd]."""
        return ops.linear(hidden, self.lm_head, out_dtype=torch.float32)

    def pick(self, logits: torch.Tensor, k: int) -> torch.Tensor:
        """Top-k draft tokens of each row, as target token ids [S, k] (most likely first)."""
        d = torch.topk(logits, k, dim=-1).indices
        return d if self.d2t is None else d + self.d2t[d]
