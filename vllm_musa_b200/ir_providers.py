"""``b200`` implementations of vLLM's IR ops (rms_norm, fused_add_rms_norm).

Kept free of ``from __future__ import annotations``: vLLM infers the op schema from the
runtime annotations.  Reference counterpart: vllm_musa/kernels/musa_ops.py:66-241.
"""
from typing import Optional, Tuple

import torch
from torch import Tensor

PROVIDER = "b200"


def _rms_supported(x: Tensor, weight: Optional[Tensor], epsilon: float,
                   variance_size: Optional[int] = None) -> bool:
    return (variance_size is None and x.dtype == torch.bfloat16 and x.is_cuda and
            x.shape[-1] % 8 == 0 and x.stride(-1) == 1 and
            (weight is None or weight.dtype == x.dtype))


def _rms_add_supported(x: Tensor, x_residual: Tensor, weight: Optional[Tensor], epsilon: float,
                       variance_size: Optional[int] = None) -> bool:
    return (_rms_supported(x, weight, epsilon, variance_size) and x.is_contiguous() and
            x_residual.is_contiguous())


def register(ir) -> None:
    from . import ops

    def rms_norm(x: Tensor, weight: Optional[Tensor], epsilon: float,
                 variance_size: Optional[int] = None) -> Tensor:
        if weight is None:
            weight = torch.ones(x.shape[-1], device=x.device, dtype=x.dtype)
        x2 = x.reshape(-1, x.shape[-1])
        return ops.rms_norm(x2, weight, epsilon).reshape(x.shape)

    def fused_add_rms_norm(x: Tensor, x_residual: Tensor, weight: Optional[Tensor],
                           epsilon: float, variance_size: Optional[int] = None
                           ) -> Tuple[Tensor, Tensor]:
        if weight is None:
            weight = torch.ones(x.shape[-1], device=x.device, dtype=x.dtype)
        x2, r2 = x.view(-1, x.shape[-1]), x_residual.view(-1, x.shape[-1])
        ops.fused_add_rms_norm(x2, r2, weight, epsilon)
        return x, x_residual

    ir.ops.rms_norm.register_impl(PROVIDER, supports_args=_rms_supported)(rms_norm)
    ir.ops.fused_add_rms_norm.register_impl(PROVIDER, supports_args=_rms_add_supported,
                                            inplace=True)(fused_add_rms_norm)
