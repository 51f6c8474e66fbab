"""Pure-PyTorch reference decoder (no paging, no fusion) used as the numerics oracle.

Implements the textbook Llama/Qwen3 forward over a whole sequence from HF-named weights:
embedding -> [RMSNorm -> causal GQA attention with RoPE (NeoX) -> residual -> RMSNorm ->
SwiGLU MLP -> residual] x L -> RMSNorm -> LM head.  Computation in fp32.
"""
from __future__ import annotations

from typing import Dict, List, Optional

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
        w = self.w
        head = w.get("lm_head.weight", w["model.embed_tokens.weight"])
        return self.hidden(tokens) @ head.t()

    @torch.no_grad()
    def hidden(self, tokens: List[int], streams: Optional[dict] = None) -> torch.Tensor:
        """Final normalised hidden states [S, H] for every position of ``tokens``; ``streams``
        (a dict) receives the residual stream entering each layer, by layer index."""
        cfg, w, D = self.cfg, self.w, self.D
        S = len(tokens)
        ids = torch.tensor(tokens)
        pos = torch.arange(S)
        h = w["model.embed_tokens.weight"][ids]
        G = cfg.num_heads // cfg.num_kv_heads
        mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
        for i in range(cfg.num_layers):
            if streams is not None:
                streams[i] = h.clone()
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
        return self._rms(h, w["model.norm.weight"])

    def greedy(self, prompt: List[int], n: int):
        """Greedy continuation of ``n`` tokens; returns (tokens, per-step logits list)."""
        toks = list(prompt)
        step_logits = []
        for _ in range(n):
            lg = self.logits(toks)[-1]
            step_logits.append(lg)
            toks.append(int(lg.argmax()))
        return toks[len(prompt):], step_logits


class HybridReferenceDecoder(ReferenceDecoder):
    """Whole-sequence fp32 reference of the Qwen3-Next hybrid decoder from HF-named weights.

    Layer i is full attention when (i + 1) % full_attention_interval == 0, else a Gated
    DeltaNet layer; every layer ends in a routed MoE with a sigmoid-gated shared expert.  All
    RMSNorm weights except the gated output norm are stored zero-centred, y = norm(x) * (1 + w).
    Weight layouts follow the HF checkpoint: ``in_proj_qkvz`` rows grouped per key head as
    [q | k | v (rep heads) | z (rep heads)], ``in_proj_ba`` per key head as [b (rep) | a (rep)],
    ``q_proj`` per attention head as [q | gate].  The delta rule runs token by token.
    """

    def _rms1(self, x, w):
        return self._rms(x, 1.0 + w)

    def _moe(self, p, x):
        cfg, w = self.cfg, self.w
        probs = torch.softmax(x @ w[p + "mlp.gate.weight"].t(), -1)
        top_w, top_i = probs.topk(cfg.num_experts_per_tok, -1)
        if cfg.norm_topk_prob:
            top_w = top_w / top_w.sum(-1, keepdim=True)
        out = torch.zeros_like(x)
        for t in range(x.shape[0]):
            for j in range(top_i.shape[1]):
                q = f"{p}mlp.experts.{int(top_i[t, j])}."
                h = F.silu(x[t] @ w[q + "gate_proj.weight"].t()) * (x[t] @ w[q + "up_proj.weight"].t())
                out[t] += top_w[t, j] * (h @ w[q + "down_proj.weight"].t())
        if cfg.shared_expert_intermediate_size:
            q = p + "mlp.shared_expert."
            s = (F.silu(x @ w[q + "gate_proj.weight"].t()) * (x @ w[q + "up_proj.weight"].t())) @ \
                w[q + "down_proj.weight"].t()
            out = out + torch.sigmoid(x @ w[p + "mlp.shared_expert_gate.weight"].t()) * s
        return out

    def _gated_attention(self, p, x, pos, mask):
        cfg, w, D = self.cfg, self.w, self.D
        S = x.shape[0]
        qg = (x @ w[p + "self_attn.q_proj.weight"].t()).view(S, cfg.num_heads, 2 * D)
        q, gate = qg[..., :D], qg[..., D:].reshape(S, -1)
        k = (x @ w[p + "self_attn.k_proj.weight"].t()).view(S, cfg.num_kv_heads, D)
        v = (x @ w[p + "self_attn.v_proj.weight"].t()).view(S, cfg.num_kv_heads, D)
        q = self._rope(self._rms1(q, w[p + "self_attn.q_norm.weight"]), pos)
        k = self._rope(self._rms1(k, w[p + "self_attn.k_norm.weight"]), pos)
        G = cfg.num_heads // cfg.num_kv_heads
        k, v = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) / D ** 0.5
        s = s.masked_fill(mask[None], float("-inf"))
        a = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(S, -1)
        return (a * torch.sigmoid(gate)) @ w[p + "self_attn.o_proj.weight"].t()

    def _gated_deltanet(self, p, x):
        cfg, w = self.cfg, self.w
        S = x.shape[0]
        Hk, Hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        dk, dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        rep = Hv // Hk
        qkvz = (x @ w[p + "linear_attn.in_proj_qkvz.weight"].t()).view(S, Hk, 2 * dk + 2 * rep * dv)
        q = qkvz[..., :dk].reshape(S, Hk * dk)
        k = qkvz[..., dk:2 * dk].reshape(S, Hk * dk)
        v = qkvz[..., 2 * dk:2 * dk + rep * dv].reshape(S, Hv * dv)
        z = qkvz[..., 2 * dk + rep * dv:].reshape(S, Hv, dv)
        ba = (x @ w[p + "linear_attn.in_proj_ba.weight"].t()).view(S, Hk, 2 * rep)
        b, a = ba[..., :rep].reshape(S, Hv), ba[..., rep:].reshape(S, Hv)
        mixed = torch.cat([q, k, v], -1)  # [S, C]
        cw = w[p + "linear_attn.conv1d.weight"]  # [C, 1, K]
        Kc = cw.shape[-1]
        y = F.conv1d(F.pad(mixed.t().unsqueeze(0), (Kc - 1, 0)), cw, groups=cw.shape[0])[0]
        mixed = F.silu(y).t()
        q = mixed[:, :Hk * dk].view(S, Hk, dk).repeat_interleave(rep, 1)
        k = mixed[:, Hk * dk:2 * Hk * dk].view(S, Hk, dk).repeat_interleave(rep, 1)
        v = mixed[:, 2 * Hk * dk:].view(S, Hv, dv)
        q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
        k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
        beta = torch.sigmoid(b)
        g = -torch.exp(w[p + "linear_attn.A_log"]) * F.softplus(a + w[p + "linear_attn.dt_bias"])
        state = torch.zeros(Hv, dk, dv)
        o = torch.empty(S, Hv, dv)
        for t in range(S):
            state = state * torch.exp(g[t]).view(Hv, 1, 1)
            mem = (state * k[t].unsqueeze(-1)).sum(-2)
            delta = (v[t] - mem) * beta[t].unsqueeze(-1)
            state = state + k[t].unsqueeze(-1) * delta.unsqueeze(-2)
            o[t] = (state * q[t].unsqueeze(-1)).sum(-2)
        o = self._rms(o, w[p + "linear_attn.norm.weight"]) * F.silu(z)
        return o.reshape(S, -1) @ w[p + "linear_attn.out_proj.weight"].t()

    @torch.no_grad()
    def logits(self, tokens: List[int]) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        S = len(tokens)
        pos = torch.arange(S)
        mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
        h = w["model.embed_tokens.weight"][torch.tensor(tokens)]
        interval = cfg.full_attention_interval or 4
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            x = self._rms1(h, w[p + "input_layernorm.weight"])
            if (i + 1) % interval == 0:
                h = h + self._gated_attention(p, x, pos, mask)
            else:
                h = h + self._gated_deltanet(p, x)
            h = h + self._moe(p, self._rms1(h, w[p + "post_attention_layernorm.weight"]))
        h = self._rms1(h, w["model.norm.weight"])
        head = w.get("lm_head.weight", w["model.embed_tokens.weight"])
        return h @ head.t()


class DeepseekReferenceDecoder(ReferenceDecoder):
    """Whole-sequence fp32 reference of the DeepSeek-V3 / V3.2 decoder from HF-named weights:
    MLA in its expanded form (per-head keys and values from kv_b_proj, no absorption), the
    V3.2 lightning indexer as an explicit causal top-k mask, sigmoid grouped-top-k MoE with
    the score-correction bias and shared experts.  Latent RoPE is the interleaved form."""

    def __init__(self, cfg, weights):
        super().__init__(cfg, weights)
        rot = cfg.qk_rope_head_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, rot, 2, dtype=torch.float64) / rot))
        f = torch.outer(torch.arange(cfg.max_position, dtype=torch.float64), inv)
        self.cos, self.sin = f.cos().float(), f.sin().float()

    def _rope_il(self, x, pos):
        c, s = self.cos[pos], self.sin[pos]
        while c.dim() < x.dim():
            c, s = c.unsqueeze(-2), s.unsqueeze(-2)
        out = torch.empty_like(x)
        out[..., 0::2] = x[..., 0::2] * c - x[..., 1::2] * s
        out[..., 1::2] = x[..., 1::2] * c + x[..., 0::2] * s
        return out

    def _rope_nx(self, x, pos):
        c, s = self.cos[pos], self.sin[pos]
        while c.dim() < x.dim():
            c, s = c.unsqueeze(-2), s.unsqueeze(-2)
        h = x.shape[-1] // 2
        return torch.cat([x[..., :h] * c - x[..., h:] * s, x[..., h:] * c + x[..., :h] * s], -1)

    def _attention(self, p, x, pos):
        cfg, w = self.cfg, self.w
        S, Hq = x.shape[0], cfg.num_heads
        nope, rope, vd = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim
        a = p + "self_attn."
        if cfg.q_lora_rank:
            q_a = self._rms(x @ w[a + "q_a_proj.weight"].t(), w[a + "q_a_layernorm.weight"])
            q = (q_a @ w[a + "q_b_proj.weight"].t()).view(S, Hq, nope + rope)
        else:
            q = (x @ w[a + "q_proj.weight"].t()).view(S, Hq, nope + rope)
        kv = x @ w[a + "kv_a_proj_with_mqa.weight"].t()
        c = self._rms(kv[:, :cfg.kv_lora_rank], w[a + "kv_a_layernorm.weight"])
        k_pe = self._rope_il(kv[:, cfg.kv_lora_rank:], pos)                   # [S, 64]
        q = torch.cat([q[..., :nope], self._rope_il(q[..., nope:], pos)], -1)
        kvb = (c @ w[a + "kv_b_proj.weight"].t()).view(S, Hq, nope + vd)
        k = torch.cat([kvb[..., :nope], k_pe.unsqueeze(1).expand(S, Hq, rope)], -1)
        v = kvb[..., nope:]
        scale = (nope + rope) ** -0.5
        s = torch.einsum("qhd,khd->hqk", q, k) * scale
        allow = torch.tril(torch.ones(S, S, dtype=torch.bool))
        if cfg.index_topk:
            allow = allow & self._indexer_mask(a, x, q_a, pos, allow)
        s = s.masked_fill(~allow[None], float("-inf"))
        o = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(S, -1)
        return o @ w[a + "o_proj.weight"].t()

    def _indexer_mask(self, a, x, q_a, pos, causal):
        cfg, w = self.cfg, self.w
        S, nh, dh = x.shape[0], cfg.index_n_heads, cfg.index_head_dim
        i = a + "indexer."
        q = (q_a @ w[i + "wq_b.weight"].t()).view(S, nh, dh)
        q = torch.cat([self._rope_nx(q[..., :64], pos), q[..., 64:]], -1)
        k = F.layer_norm(x @ w[i + "wk.weight"].t(), (dh,), w[i + "k_norm.weight"],
                         w[i + "k_norm.bias"], 1e-6)
        k = torch.cat([self._rope_nx(k[..., :64], pos), k[..., 64:]], -1)
        hw = (x @ w[i + "weights_proj.weight"].t()) * (nh ** -0.5 * dh ** -0.5)
        sc = (hw.unsqueeze(-1) * torch.relu(torch.einsum("thd,sd->ths", q, k))).sum(1)
        sc = sc.masked_fill(~causal, float("-inf"))
        mask = torch.zeros(S, S, dtype=torch.bool)
        for t in range(S):
            n = min(cfg.index_topk, t + 1)
            mask[t, sc[t, :t + 1].topk(n).indices] = True
        return mask

    def _moe(self, p, x):
        cfg, w = self.cfg, self.w
        T = x.shape[0]
        logits = x @ w[p + "mlp.gate.weight"].t()
        scores = torch.sigmoid(logits) if cfg.scoring_func == "sigmoid" else torch.softmax(logits, -1)
        choice = scores + w.get(p + "mlp.gate.e_score_correction_bias", torch.zeros(cfg.num_experts))
        g = choice.view(T, cfg.n_group, -1).topk(2, -1).values.sum(-1)
        keep = torch.zeros_like(g).scatter_(1, g.topk(cfg.topk_group, -1).indices, 1.0)
        keep = keep.repeat_interleave(cfg.num_experts // cfg.n_group, 1)
        ids = choice.masked_fill(keep == 0, float("-inf")).topk(cfg.num_experts_per_tok, -1).indices
        wts = scores.gather(1, ids)
        if cfg.norm_topk_prob:
            wts = wts / wts.sum(-1, keepdim=True)
        wts = wts * cfg.routed_scaling_factor
        out = torch.zeros_like(x)
        for t in range(T):
            for j in range(ids.shape[1]):
                q = f"{p}mlp.experts.{int(ids[t, j])}."
                h = F.silu(x[t] @ w[q + "gate_proj.weight"].t()) * (x[t] @ w[q + "up_proj.weight"].t())
                out[t] += wts[t, j] * (h @ w[q + "down_proj.weight"].t())
        if cfg.shared_expert_intermediate_size:
            q = p + "mlp.shared_experts."
            out += (F.silu(x @ w[q + "gate_proj.weight"].t()) * (x @ w[q + "up_proj.weight"].t())) @ \
                w[q + "down_proj.weight"].t()
        return out

    @torch.no_grad()
    def logits(self, tokens: List[int]) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        S = len(tokens)
        pos = torch.arange(S)
        h = w["model.embed_tokens.weight"][torch.tensor(tokens)]
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            h = h + self._attention(p, self._rms(h, w[p + "input_layernorm.weight"]), pos)
            x = self._rms(h, w[p + "post_attention_layernorm.weight"])
            if cfg.num_experts and i >= cfg.first_k_dense:
                h = h + self._moe(p, x)
            else:
                h = h + (F.silu(x @ w[p + "mlp.gate_proj.weight"].t()) *
                         (x @ w[p + "mlp.up_proj.weight"].t())) @ w[p + "mlp.down_proj.weight"].t()
        h = self._rms(h, w["model.norm.weight"])
        head = w.get("lm_head.weight", w["model.embed_tokens.weight"])
        return h @ head.t()
