"""Pure-PyTorch reference decoder (no paging, no fusion) used as the numerics oracle.

Implements the textbook Llama/Qwen3 forward over a whole sequence from HF-named weights:
embedding -> [RMSNorm -> causal GQA attention with RoPE (NeoX) -> residual -> RMSNorm ->
SwiGLU MLP -> residual] x L -> RMSNorm -> LM head.  Computation in fp32.
"""
from __future__ import annotations

from typing import Dict, List

import torch
import torch.nn.functional as F

from ..config import ModelConfig


class ReferenceDecoder:
    def __init__(self, cfg: ModelConfig, weights: Dict[str, torch.Tensor]):
        self.cfg = cfg
        self.w = {k: v.float() for k, v in weights.items()}
        D = cfg.head_dim
        rot = cfg.rot_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
        t = torch.arange(cfg.max_position, dtype=torch.float64)
        f = torch.outer(t, inv)
        self.cos, self.sin = f.cos().float(), f.sin().float()
        self.D = D

    def _rms(self, x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps) * w

    def _rope(self, x, pos):  # x [S, H, D]
        rot = self.cfg.rot_dim
        half = rot // 2
        c, s = self.cos[pos][:, None, :], self.sin[pos][:, None, :]
        x1, x2 = x[..., :half], x[..., half:rot]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s, x[..., rot:]], -1)

    @torch.no_grad()
    def logits(self, tokens: List[int]) -> torch.Tensor:
        """Logits [S, V] for every position of ``tokens``."""
        cfg, w, D = self.cfg, self.w, self.D
        S = len(tokens)
        ids = torch.tensor(tokens)
        pos = torch.arange(S)
        h = w["model.embed_tokens.weight"][ids]
        G = cfg.num_heads // cfg.num_kv_heads
        mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            x = self._rms(h, w[p + "input_layernorm.weight"])
            q = (x @ w[p + "self_attn.q_proj.weight"].t()).view(S, cfg.num_heads, D)
            k = (x @ w[p + "self_attn.k_proj.weight"].t()).view(S, cfg.num_kv_heads, D)
            v = (x @ w[p + "self_attn.v_proj.weight"].t()).view(S, cfg.num_kv_heads, D)
            if cfg.qk_norm:
                q = self._rms(q, w[p + "self_attn.q_norm.weight"])
                k = self._rms(k, w[p + "self_attn.k_norm.weight"])
            q, k = self._rope(q, pos), self._rope(k, pos)
            k = k.repeat_interleave(G, 1)
            v = v.repeat_interleave(G, 1)
            s = torch.einsum("qhd,khd->hqk", q, k) / D ** 0.5
            s = s.masked_fill(mask[None], float("-inf"))
            a = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(S, -1)
            h = h + a @ w[p + "self_attn.o_proj.weight"].t()
            x = self._rms(h, w[p + "post_attention_layernorm.weight"])
            g = x @ w[p + "mlp.gate_proj.weight"].t()
            u = x @ w[p + "mlp.up_proj.weight"].t()
            h = h + (F.silu(g) * u) @ w[p + "mlp.down_proj.weight"].t()
        h = self._rms(h, w["model.norm.weight"])
        head = w.get("lm_head.weight", w["model.embed_tokens.weight"])
        return h @ head.t()

    def greedy(self, prompt: List[int], n: int):
        """Greedy continuation of ``n`` tokens; returns (tokens, per-step logits list)."""
        toks = list(prompt)
        step_logits = []
        for _ in range(n):
            lg = self.logits(toks)[-1]
            step_logits.append(lg)
            toks.append(int(lg.argmax()))
        return toks[len(prompt):], step_logits
