"""Qwen3-Next (hybrid) family: Gated-DeltaNet linear-attention layers interleaved 3:1 with
gated full-attention layers, every layer followed by a sparse MoE (+ gated shared expert).

Linear-attention layer (per rank, heads sharded by key-head groups):
    qkvz = x W_qkvz   (rows reordered at load to [q | k | v | z], q/k per key head, v/z per
                       value head), ba = x W_ba ([b | a])
    conv = silu(causal_conv1d_k4([q | k | v]))       per-request conv state slot
    o    = gated_delta_rule(conv, b, a)               per-request 128x128 fp32 state slots
    out  = (RMSNorm_128(o) * w * silu(z)) W_out       -> fused all-reduce + residual + norm
Full-attention layer: one GEMM produces [q | k | v | gate]; QK-norm + partial RoPE (64 of 256
dims) + KV insert; paged attention; out *= sigmoid(gate); o_proj.
Norm weights use the (1 + w) convention; the 1 is folded into the weights at load so the
plain RMSNorm kernels apply.  Reference: vllm_musa/model_executor/layers/mamba/gdn/
qwen_gdn_linear_attn.py:121-754 (GDN layer), vllm_musa/kernels/gated_qkv.py:28-257 (gated
attention QK norm + RoPE); layer math as in HF transformers' Qwen3-Next implementation.
"""
from __future__ import annotations

import torch

from .. import ops
from ..ops import gdn as gdn_ops
from .llama import _LAYER_RE, shard_cols, shard_rows
from .qwen3_moe import Qwen3MoeForCausalLM


class Qwen3NextForCausalLM(Qwen3MoeForCausalLM):
    def __init__(self, cfg, pstate=None, comm=None, device="cuda"):
        super().__init__(cfg, pstate, comm, device)
        t, r = self.tp, self.rank
        interval = cfg.full_attention_interval or 4
        self.full = [(i + 1) % interval == 0 for i in range(cfg.num_layers)]
        self.attn_index = {}
        self.gdn_index = {}
        for i, f in enumerate(self.full):
            (self.attn_index if f else self.gdn_index)[i] = len(
                self.attn_index if f else self.gdn_index)
        self.Hk_g = cfg.linear_num_key_heads // t
        self.Hv_g = cfg.linear_num_value_heads // t
        if cfg.linear_num_key_heads % t or cfg.linear_num_value_heads % t:
            raise ValueError("linear-attention heads must be divisible by tensor_parallel_size")
        self.dk = cfg.linear_key_head_dim
        self.dv = cfg.linear_value_head_dim
        self.conv_dim = 2 * self.Hk_g * self.dk + self.Hv_g * self.dv
        self.conv_state = None
        self.ssm_state = None

    # ------------------------------------------------------------------ state
    def allocate_state(self, slots: int) -> None:
        n = len(self.gdn_index)
        self.conv_state = torch.zeros(n, slots, self.conv_dim, 3, dtype=self.dtype,
                                      device=self.device)
        self.ssm_state = torch.zeros(n, slots, self.Hv_g, self.dv, self.dk, dtype=torch.float32,
                                     device=self.device)

    def kv_cache_spec(self) -> dict:
        spec = super().kv_cache_spec()
        spec["num_layers"] = len(self.attn_index)
        return spec

    # ------------------------------------------------------------------ weights
    def _attn_keys(self, i):
        if self.full[i]:
            return ["self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                    "self_attn.o_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight"]
        return ["linear_attn.in_proj_qkvz.weight", "linear_attn.in_proj_ba.weight",
                "linear_attn.conv1d.weight", "linear_attn.dt_bias", "linear_attn.A_log",
                "linear_attn.norm.weight", "linear_attn.out_proj.weight"]

    def _try_finalize(self, i):
        st = self._staging[i]
        need = ["input_layernorm.weight", "post_attention_layernorm.weight"] + \
            self._attn_keys(i) + self._mlp_keys(i)
        if not all(k in st for k in need):
            return
        L = self.layers[i]
        one = lambda w: self._to(w.float() + 1.0)  # noqa: E731  ((1 + w) norms)
        if self.full[i]:
            self._finalize_gated_attention(L, st)
        else:
            self._finalize_gdn(L, st)
        self._finalize_mlp(i, L, st)
        L.ln1 = one(st["input_layernorm.weight"])
        L.ln2 = one(st["post_attention_layernorm.weight"])
        del self._staging[i]

    def _finalize_gated_attention(self, L, st):
        D, r, t = self.D, self.rank, self.tp
        Hq = self.cfg.num_heads
        qg = st["self_attn.q_proj.weight"].view(Hq, 2, D, -1)  # per head: [q, gate]
        q = shard_rows(qg[:, 0].reshape(Hq * D, -1), r, t)
        gate = shard_rows(qg[:, 1].reshape(Hq * D, -1), r, t)
        k = st["self_attn.k_proj.weight"][self.kv0 * D:(self.kv0 + self.hkv) * D]
        v = st["self_attn.v_proj.weight"][self.kv0 * D:(self.kv0 + self.hkv) * D]
        L.qkv_w = self._to(torch.cat([q, k, v, gate], 0))
        L.o_w = self._to(shard_cols(st["self_attn.o_proj.weight"], r, t))
        L.q_norm = self._to(st["self_attn.q_norm.weight"].float() + 1.0)
        L.k_norm = self._to(st["self_attn.k_norm.weight"].float() + 1.0)

    def _finalize_gdn(self, L, st):
        c, r, t = self.cfg, self.rank, self.tp
        Hk, Hv, dk, dv = c.linear_num_key_heads, c.linear_num_value_heads, self.dk, self.dv
        rep = Hv // Hk
        w = st["linear_attn.in_proj_qkvz.weight"]
        H = w.shape[1]
        g = w.view(Hk, 2 * dk + 2 * rep * dv, H)  # grouped per key head
        q = g[:, :dk].reshape(Hk * dk, H)
        k = g[:, dk:2 * dk].reshape(Hk * dk, H)
        v = g[:, 2 * dk:2 * dk + rep * dv].reshape(Hv * dv, H)
        z = g[:, 2 * dk + rep * dv:].reshape(Hv * dv, H)
        qkvz = torch.cat([shard_rows(q, r, t), shard_rows(k, r, t), shard_rows(v, r, t),
                          shard_rows(z, r, t)], 0)
        ba = st["linear_attn.in_proj_ba.weight"].view(Hk, 2 * rep, H)
        b = ba[:, :rep].reshape(Hv, H)
        a = ba[:, rep:].reshape(Hv, H)
        conv = st["linear_attn.conv1d.weight"].reshape(-1, 4)
        cq, ck, cv = conv[:Hk * dk], conv[Hk * dk:2 * Hk * dk], conv[2 * Hk * dk:]
        L.extra = {
            "qkvz_w": self._to(qkvz),
            "ba_w": self._to(torch.cat([shard_rows(b, r, t), shard_rows(a, r, t)], 0)),
            "conv_w": self._to(torch.cat([shard_rows(cq, r, t), shard_rows(ck, r, t),
                                          shard_rows(cv, r, t)], 0)),
            "dt_bias": shard_rows(st["linear_attn.dt_bias"], r, t).float().to(self.device).contiguous(),
            "A_log": shard_rows(st["linear_attn.A_log"], r, t).float().to(self.device).contiguous(),
            "norm_w": self._to(st["linear_attn.norm.weight"]),
        }
        L.o_w = self._to(shard_cols(st["linear_attn.out_proj.weight"], r, t))

    def load_weights(self, weights):
        cfg = self.cfg
        for name, w in weights:
            if name == "model.embed_tokens.weight":
                self.embed = self._to(w)
                if cfg.tie_word_embeddings:
                    self.lm_head = self._to(shard_rows(w, self.rank, self.tp))
            elif name == "lm_head.weight":
                self.lm_head = self._to(shard_rows(w, self.rank, self.tp))
            elif name == "model.norm.weight":
                self.final_norm = self._to(w.float() + 1.0)
            else:
                m = _LAYER_RE.match(name)
                if not m or int(m.group(1)) >= cfg.num_layers or \
                        not self._wanted(int(m.group(1)), m.group(2)):
                    continue
                self._staging[int(m.group(1))][m.group(2)] = w
                self._try_finalize(int(m.group(1)))
        missing = [i for i in range(cfg.num_layers) if self.layers[i].ln1 is None]
        if missing or self.embed is None or self.final_norm is None or self.lm_head is None:
            raise RuntimeError(f"incomplete checkpoint: layers {missing[:8]}")
        self._staging.clear()

    def linear_shapes(self):
        out = {tuple(self.lm_head.shape)}
        for L in self.layers:
            for w in (L.qkv_w, L.o_w, L.gu_w, L.down_w, L.router_w, L.shared_gu, L.shared_down):
                if w is not None:
                    out.add(tuple(w.shape))
            if L.extra:
                out.add(tuple(L.extra["qkvz_w"].shape))
                out.add(tuple(L.extra["ba_w"].shape))
        return sorted(out)

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids, meta, kv_caches):
        cfg, eps = self.cfg, self.cfg.rms_norm_eps
        T = input_ids.shape[0]
        self.comm.begin_forward()
        h = ops.embedding(input_ids, self.embed)
        residual = h
        x = ops.rms_norm(h, self.layers[0].ln1, eps)
        n = len(self.layers)
        D = self.D
        for i, L in enumerate(self.layers):
            if self.full[i]:
                kc, vc = kv_caches[self.attn_index[i]]
                qkvg = ops.linear(x, L.qkv_w)
                ops.rope_kv(qkvg, meta.positions, self.cos_sin, kc, vc, meta.slot_mapping,
                            self.hq, self.hkv, cfg.rot_dim, cfg.rope_neox, L.q_norm, L.k_norm,
                            eps)
                a = self.attn.forward(qkvg, kc, vc, meta)
                gate = qkvg[:, (self.hq + 2 * self.hkv) * D:]
                gdn_ops.sigmoid_gate(a, gate)
            else:
                a = self._gdn(self.gdn_index[i], L, x, meta)
            o = ops.linear(a, L.o_w, out=self.comm.out_buffer(T))
            x, residual = self.comm.allreduce_add_rmsnorm(o, residual, L.ln2, eps)
            d = self._mlp(i, L, x, T)
            nxt = self.layers[i + 1].ln1 if i + 1 < n else self.final_norm
            x, residual = self.comm.allreduce_add_rmsnorm(d, residual, nxt, eps)
        return x

    def _delta_rule(self, conv, ba, e, state, meta):
        """Gated delta rule over this step's tokens: decode rows (first in the batch) with the
        token-recurrent kernel, prefill rows with the chunked kernels once they fill a chunk."""
        nd, npf = meta.num_decodes, meta.num_prefills
        T = conv.shape[0]
        if npf == 0 or not conv.is_cuda:
            return gdn_ops.gdn_recurrent(conv, ba, e["A_log"], e["dt_bias"], state, meta.cu_q,
                                         meta.seq_lens, meta.state_slots, self.Hk_g, self.Hv_g,
                                         single_token=npf == 0)
        out = torch.empty(T, self.Hv_g * 128, dtype=conv.dtype, device=conv.device)
        sl, slots = meta.seq_lens, meta.state_slots
        if nd > 0:
            gdn_ops.gdn_recurrent(conv, ba, e["A_log"], e["dt_bias"], state, meta.cu_q[:nd + 1],
                                  sl[:nd], slots[:nd], self.Hk_g, self.Hv_g, out=out,
                                  single_token=True)
        cu_p = meta.cu_q[nd:nd + npf + 1]
        fn = gdn_ops.gdn_chunked if T - nd >= gdn_ops.CHUNK_MIN_TOKENS else \
            gdn_ops.gdn_recurrent
        fn(conv, ba, e["A_log"], e["dt_bias"], state, cu_p, sl[nd:nd + npf],
           slots[nd:nd + npf], self.Hk_g, self.Hv_g, out=out)
        return out

    def _gdn(self, j, L, x, meta):
        e = L.extra
        qkvz = ops.linear(x, e["qkvz_w"])
        ba = ops.linear(x, e["ba_w"])
        conv = gdn_ops.causal_conv1d(qkvz, e["conv_w"], self.conv_state[j], meta.cu_q,
                                     meta.seq_lens, meta.state_slots)
        o = self._delta_rule(conv, ba, e, self.ssm_state[j], meta)
        z = qkvz[:, self.conv_dim:]
        return ops.rms_norm_gated(o, z, e["norm_w"], self.dv, self.cfg.rms_norm_eps)
