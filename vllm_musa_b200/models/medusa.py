"""Medusa draft heads over a decoder (``speculative_config={"method": "medusa"}``).

Head i (of k) reads the target's final hidden state h_p at the position p whose next token is
the request's pending token and predicts the token i + 1 places after it:

    r_i      = h_p + silu(W_i h_p + b_i)          (one residual block per head)
    logits_i = lm_head_i(r_i)                      (the head's own LM head, full vocabulary)

so a step's k drafts cost k small GEMM pairs and no attention or KV cache.  Chained drafts
take each head's argmax; with ``tree_width`` w > 1 the drafts form a token tree filled level by
level (level i = head i's top-w tokens under each node of level i - 1, most likely parents
first) up to ``num_speculative_tokens`` nodes, verified in one step under ancestor masks.

Checkpoint layout (Medusa-1, the names vLLM's Medusa loader reads): ``blocks.{i}.layers.0.
{weight,bias}`` [H, H] / [H] and ``lm_heads.{i}.weight`` [V, H]; a checkpoint without LM heads
shares the target's LM head (at tensor-parallel size 1, where it is whole).  Every rank holds the heads whole
(the target's final hidden states are replicated), so drafting needs no collective.
Reference counterpart: Cai et al., "Medusa", 2024, as served by the vLLM the reference
patches.
"""
from __future__ import annotations

from typing import Iterable, List, Tuple

import torch

from .. import ops


def medusa_param_shapes(cfg, num_heads: int) -> list:
    H, V = cfg.hidden_size, cfg.vocab_size
    out = []
    for i in range(num_heads):
        out += [(f"blocks.{i}.layers.0.weight", (H, H), "w"),
                (f"blocks.{i}.layers.0.bias", (H,), "bias"),
                (f"lm_heads.{i}.weight", (V, H), "w")]
    return out


class MedusaHeads:
    def __init__(self, target, num_heads: int):
        if num_heads < 1:
            raise ValueError("Medusa needs at least one head")
        self.t = target
        self.cfg = target.cfg
        self.k = num_heads
        self.w: List[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = []

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        t = self.t
        st = {n: w for n, w in weights}
        shared = st.get("lm_head.weight")
        if shared is None and t.tp == 1:
            shared = getattr(t, "lm_head", None)  # the target's LM head (whole at TP = 1)
        for i in range(self.k):
            p = f"blocks.{i}.layers.0."
            if p + "weight" not in st:
                raise RuntimeError(f"Medusa checkpoint is missing {p}weight")
            lm = st.get(f"lm_heads.{i}.weight", shared)
            if lm is None:
                raise RuntimeError(f"Medusa checkpoint is missing lm_heads.{i}.weight")
            b = st.get(p + "bias", torch.zeros(self.cfg.hidden_size))
            self.w.append((t._to(st[p + "weight"]), t._to(b), t._to(lm)))

    @torch.no_grad()
    def logits(self, h: torch.Tensor) -> List[torch.Tensor]:
        """h [R, H] -> per head fp32 logits [R, V]."""
        out = []
        for W, b, lm in self.w:
            z = ops.linear(h.contiguous(), W) + b
            r = h + torch.nn.functional.silu(z.float()).to(h.dtype)
            out.append(ops.linear(r.contiguous(), lm, out_dtype=torch.float32))
        return out
