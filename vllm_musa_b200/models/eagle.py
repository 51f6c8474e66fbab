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
    def __init__(self, target):
        if getattr(target, "tq", None) is not None:
            raise ValueError("EAGLE drafts need a bf16 KV cache (not TurboQuant)")
        self.t = target
        self.cfg = target.cfg
        self.layer = _Layer()
        self.fc = None
        self.fc_bias = None
        self.norm = None
        self.cache_index = target.l1 - target.l0  # the extra cache layer after the target's

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        t, L = self.t, self.layer
        st = {n: w for n, w in weights}
        miss = [n for n, _, k in eagle_param_shapes(self.cfg) if k == "w" and n not in st]
        if miss:
            raise RuntimeError(f"EAGLE checkpoint is missing {miss}")
        D, r, tp = t.D, t.rank, t.tp
        a, m = "layers.0.self_attn.", "layers.0.mlp."
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
        T = next_ids.shape[0]
        t.comm.begin_forward()
        e = ops.embedding(next_ids, t.embed)
        x = ops.linear(torch.cat([e, prev_hidden.to(e.dtype)], -1).contiguous(), self.fc)
        if self.fc_bias is not None:
            x = x + self.fc_bias
        residual = x
        kc, vc = kv_caches[self.cache_index]
        qkv = ops.linear(x, L.qkv_w)
        ops.rope_kv(qkv, meta.positions, t.cos_sin, kc, vc, meta.slot_mapping, t.hq, t.hkv,
                    cfg.rot_dim, cfg.rope_neox, None, None, eps)
        a = t.attn.forward(qkv, kc, vc, meta)
        x, residual = t.comm.linear_allreduce_add_rmsnorm(a, L.o_w, residual, L.ln2, eps)
        if self.norm is not None:
            x, residual = t._mlp_allreduce(cfg.num_layers, L, x, T, residual, self.norm, eps)
            return x
        d = ops.linear(ops.linear_silu_mul(x, L.gu_w), L.down_w)
        return t.comm.all_reduce(d) + residual

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.t.compute_logits(hidden)
