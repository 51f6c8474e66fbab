"""Tensor-parallel communicator: the collectives the model layers call.

``allreduce_add_rmsnorm`` is the hot one: every row-parallel projection (o_proj, down_proj)
ends in it.  With TP == 1 it is the fused residual-add + RMSNorm kernel; with TP > 1 the
NVSwitch peer-memory kernel (parallel/custom_ar.py) performs all-reduce + residual-add +
RMSNorm in one launch when available, otherwise NCCL all-reduce followed by the fused norm.
Reference: MusaJitCustomAllreduce (vllm_musa/distributed/device_communicators/
musa_jit_custom_all_reduce.py:1762-1938) and the fused ops in
vllm_musa/fused_allreduce_rmsnorm_ops.py:25-214.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .. import ops
from .state import ParallelState


class TPCommunicator:
    def __init__(self, st: ParallelState, device: torch.device, custom: Optional[object] = None):
        self.st = st
        self.device = device
        self.world = st.tp_size
        self.rank = st.tp_rank
        self.group = st.tp_group
        self.custom = custom  # CustomAllReduce (NVSwitch P2P) or None
        self.ep_a2a = None    # EPAllToAll (expert-parallel dispatch/combine) or None

    # -- plain collectives ----------------------------------------------------------------
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return x
        if self.custom is not None and self.custom.can_run(x):
            return self.custom.all_reduce(x)
        dist.all_reduce(x, group=self.group)
        return x

    def all_gather(self, x: torch.Tensor, dim: int = 0) -> torch.Tensor:
        if self.world == 1:
            return x
        if x.is_cuda:
            out = torch.empty((self.world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
            dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        else:
            parts = [torch.empty_like(x) for _ in range(self.world)]
            dist.all_gather(parts, x.contiguous(), group=self.group)
            out = torch.stack(parts)
        if dim == 0:
            return out.reshape((-1,) + tuple(x.shape[1:]))
        return torch.cat(list(out.unbind(0)), dim=dim)

    def reduce_scatter(self, x: torch.Tensor, dim: int = 0) -> torch.Tensor:
        """Sum over ranks, then rank r keeps the r-th of ``world`` equal slices along ``dim``."""
        if self.world == 1:
            return x
        xt = x.movedim(dim, 0).contiguous()
        n = xt.shape[0] // self.world
        if x.is_cuda:
            out = torch.empty((n,) + tuple(xt.shape[1:]), dtype=x.dtype, device=x.device)
            dist.reduce_scatter_tensor(out, xt, group=self.group)
        else:  # gloo has no reduce-scatter: all-reduce and keep this rank's slice
            dist.all_reduce(xt, group=self.group)
            r = dist.get_rank(self.group)
            out = xt[r * n:(r + 1) * n].contiguous()
        return out.movedim(0, dim)

    # -- buffers ----------------------------------------------------------------------------
    def begin_forward(self) -> None:
        """Called once at the start of every forward pass (resets the slot parity)."""
        if self.custom is not None:
            self.custom.begin_forward()

    def out_buffer(self, T: int) -> Optional[torch.Tensor]:
        """Where a row-parallel GEMM should write its [T, hidden] partial sums (None: anywhere)."""
        if self.custom is not None and T <= self.custom.max_tokens:
            return self.custom.staging_view(T)
        return None

    # -- fused ------------------------------------------------------------------------------
    def allreduce_add_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                              eps: float) -> tuple[torch.Tensor, torch.Tensor]:
        """residual <- AR(x) + residual; x <- RMSNorm(residual) * weight (x, residual in place)."""
        if self.world > 1:
            if self.custom is not None and self.custom.can_run(x):
                return self.custom.allreduce_add_rmsnorm(x, residual, weight, eps)
            dist.all_reduce(x, group=self.group)
        return ops.fused_add_rms_norm(x, residual, weight, eps)

    def allreduce_add_rmsnorm_quant(self, x: torch.Tensor, residual: torch.Tensor,
                                    weight: torch.Tensor, eps: float):
        """Like ``allreduce_add_rmsnorm`` for a normalised output consumed by an fp8 GEMM:
        returns (x, residual, (q, scales)) with x's rows quantised per token (1x128 e4m3).  One
        GPU: residual add, RMSNorm and quantisation in one kernel (x is left unnormalised);
        TP over NVLS: all-reduce, residual add, RMSNorm and quantisation in one kernel (x is
        returned as None: the caller consumes only the quantised rows); otherwise the fused
        all-reduce + norm, then the group quantisation."""
        if self.world > 1:
            if self.custom is not None and self.custom.can_quant(x):
                q, sc = self.custom.allreduce_add_rmsnorm_quant(x, residual, weight, eps)
                return None, residual, (q, sc)
            x, residual = self.allreduce_add_rmsnorm(x, residual, weight, eps)
            return x, residual, ops.activation.group_quant_fp8(x)
        q, sc, _ = ops.rms_norm_quant_fp8(x, weight, eps, residual=residual)
        return x, residual, (q, sc)

    def linear_allreduce_add_rmsnorm(self, x: torch.Tensor, w: torch.Tensor,
                                     residual: torch.Tensor, weight: torch.Tensor, eps: float,
                                     delta=None) -> tuple[torch.Tensor, torch.Tensor]:
        """Row-parallel projection followed by all-reduce + residual + RMSNorm.  On the
        NVSwitch communicator the reduce-scatter is fused into the GEMM epilogue; otherwise
        GEMM into the staging buffer, then ``allreduce_add_rmsnorm``.  ``delta(x, o)`` adds to
        the projection's partial sum ``o`` in place before the reduction (LoRA)."""
        T = x.shape[0]
        if delta is None and self.world > 1 and self.custom is not None and x.is_cuda and \
                self.custom.can_fuse_gemm(T):
            return self.custom.linear_allreduce_add_rmsnorm(x, w, residual, weight, eps)
        o = ops.linear(x, w, out=self.out_buffer(T))
        if delta is not None:
            delta(x, o)
        return self.allreduce_add_rmsnorm(o, residual, weight, eps)

    def close(self) -> None:
        if self.ep_a2a is not None:
            self.ep_a2a.close()
            self.ep_a2a = None
        if self.custom is not None:
            self.custom.close()
            self.custom = None


class LocalCommunicator(TPCommunicator):
    """Single-GPU / CPU stand-in with the same interface."""

    def __init__(self, device: torch.device):
        super().__init__(ParallelState(), device)
