"""Qwen3-MoE family (Qwen3-30B-A3B and relatives): Qwen3 attention (QK-RMSNorm, GQA) with a
softmax top-k routed expert MLP in every layer, optional shared expert.

Experts are tensor-parallel sharded on their intermediate dimension (every rank holds all
experts, 1/tp of each), so the MoE output is a partial sum that rides on the same fused
all-reduce + residual + RMSNorm as the dense layers.  The expert computation is the fused MoE
path of ops/moe.py (device-side routing and expert-sorted layout, grouped tcgen05 GEMMs with
SwiGLU epilogue, weighted combine written straight into the all-reduce staging buffer).
Reference counterparts: vllm_musa/model_executor/layers/fused_moe/* (dispatcher, router),
upstream vLLM's qwen3_moe model it patches.
"""
from __future__ import annotations

import torch

from .. import ops
from ..ops import moe as moe_ops
from ..utils import moe_inventory
from .llama import DenseDecoderForCausalLM, shard_cols, shard_rows


class Qwen3MoeForCausalLM(DenseDecoderForCausalLM):
    def __init__(self, cfg, pstate=None, comm=None, device="cuda"):
        super().__init__(cfg, pstate, comm, device)
        if cfg.moe_intermediate_size % self.tp:
            raise ValueError("moe_intermediate_size must be divisible by tensor_parallel_size")
        self.E = cfg.num_experts
        self.topk = cfg.num_experts_per_tok
        # Expert parallelism (attention stays tensor-parallel): rank r owns a contiguous slice
        # of whole experts; the routed partial sums join the shared expert's TP partial sum in
        # the fused all-reduce + residual + RMSNorm that follows the MoE block.
        self.ep = self.pstate.ep_size > 1
        if self.ep:
            if cfg.num_experts % self.pstate.ep_size:
                raise ValueError("num_experts must be divisible by the expert-parallel size")
            self.E_local = cfg.num_experts // self.pstate.ep_size
            self.e0 = self.pstate.ep_rank * self.E_local
            self.I_e = cfg.moe_intermediate_size
        else:
            self.E_local, self.e0 = self.E, 0
            self.I_e = cfg.moe_intermediate_size // self.tp

    def _is_moe(self, i: int) -> bool:
        return self.cfg.num_experts > 0 and i >= self.cfg.first_k_dense

    def _mlp_keys(self, i):
        if not self._is_moe(i):
            return super()._mlp_keys(i)
        keys = ["mlp.gate.weight"]
        for e in range(self.e0, self.e0 + self.E_local):
            keys += [f"mlp.experts.{e}.gate_proj.weight", f"mlp.experts.{e}.up_proj.weight",
                     f"mlp.experts.{e}.down_proj.weight"]
        if self.cfg.shared_expert_intermediate_size:
            keys += ["mlp.shared_expert.gate_proj.weight", "mlp.shared_expert.up_proj.weight",
                     "mlp.shared_expert.down_proj.weight", "mlp.shared_expert_gate.weight"]
        return keys

    def _wanted(self, i, key):
        if key.startswith("mlp.experts.") and self._is_moe(i):
            e = int(key.split(".")[2])
            return self.e0 <= e < self.e0 + self.E_local
        return True

    def _finalize_mlp(self, i, L, st):
        if not self._is_moe(i):
            return super()._finalize_mlp(i, L, st)
        r, t = self.rank, self.tp
        router = st["mlp.gate.weight"]
        if "mlp.shared_expert_gate.weight" in st:
            # the shared expert's gate logit rides in the router GEMM as row E (padded to a
            # multiple of 8 rows); the combine kernel applies its sigmoid
            sg = st["mlp.shared_expert_gate.weight"].reshape(1, -1)
            router = torch.cat([router, sg, sg.new_zeros(7, sg.shape[1])], 0)
            L.shared_gate = True
        L.router_w = self._to(router)
        gus, downs = [], []
        er, et = (0, 1) if self.ep else (r, t)  # EP keeps whole experts
        for e in range(self.e0, self.e0 + self.E_local):
            g = shard_rows(st[f"mlp.experts.{e}.gate_proj.weight"], er, et)
            u = shard_rows(st[f"mlp.experts.{e}.up_proj.weight"], er, et)
            gus.append(ops.interleave_gate_up(g, u))
            downs.append(shard_cols(st[f"mlp.experts.{e}.down_proj.weight"], er, et))
        L.experts_gu = self._to(torch.cat(gus, 0))      # [E * 2I, H]
        L.experts_down = self._to(torch.cat(downs, 0))  # [E * H, I]
        if self.cfg.shared_expert_intermediate_size:
            L.shared_gu, L.shared_down = self._dense_mlp_weights(
                st["mlp.shared_expert.gate_proj.weight"], st["mlp.shared_expert.up_proj.weight"],
                st["mlp.shared_expert.down_proj.weight"])

    def _mlp_allreduce(self, i, L, x, T, residual, nxt, eps):
        """MoE layers under expert parallelism with the NVSwitch all-to-all: route this rank's
        token shard, dispatch / experts / return into the owners' staging blocks, then the
        local-source two-shot reduce (+ residual, norm, all-gather).  Layers with a
        (tensor-sharded) shared expert keep the replicated-token path."""
        a2a = getattr(self.comm, "ep_a2a", None)
        if not (self._is_moe(i) and self.ep and a2a is not None and x.is_cuda and
                L.shared_gu is None and a2a.can_run(T)):
            return super()._mlp_allreduce(i, L, x, T, residual, nxt, eps)
        per = (T + self.tp - 1) // self.tp
        r0 = min(T, self.rank * per)
        xs = x[r0:min(T, r0 + per)]
        logits = ops.linear(xs, L.router_w, out_dtype=torch.float32)
        ids, w = moe_ops.topk_softmax(logits[:, :self.E], self.topk, self.cfg.norm_topk_prob)

        def experts(rx, rids):
            moe_inventory.note("ep_grouped", rx, rids, self.E_local,
                               L.experts_gu.shape[0] // self.E_local // 2, L.experts_gu.dtype)
            return moe_ops.moe_experts(rx, L.experts_gu, L.experts_down, rids, self.E_local)

        return a2a.moe_allreduce_add_rmsnorm(x, ids, w, experts, None, residual, nxt, eps)

    def _mlp(self, i, L, x, T):
        if not self._is_moe(i):
            return super()._mlp(i, L, x, T)
        logits = ops.linear(x, L.router_w, out_dtype=torch.float32)
        E = self.E
        ids, w = moe_ops.topk_softmax(logits[:, :E], self.topk, self.cfg.norm_topk_prob)
        shared = gate = None
        if L.shared_gu is not None:
            shared = ops.linear(ops.linear_silu_mul(x, L.shared_gu), L.shared_down)
            if L.shared_gate:
                gate = logits[:, E:E + 1]
        return moe_ops.fused_moe(x, L.experts_gu, L.experts_down, ids, w, self.E_local, shared,
                                 out=self.comm.out_buffer(T), expert_offset=self.e0,
                                 shared_gate=gate)

    def linear_shapes(self):
        return [s for s in super().linear_shapes()]
