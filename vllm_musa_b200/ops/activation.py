"""Gated activations (reference: vllm_musa/model_executor/layers/activation.py:11-53)."""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _ext

SILU, GELU_TANH = 0, 1


def act_and_mul(x: torch.Tensor, kind: int = SILU, limit: float = 0.0) -> torch.Tensor:
    """[rows, 2I] -> act(x[:, :I]) * x[:, I:]; ``limit`` > 0 clamps (SwiGLU-with-clamp)."""
    I = x.shape[-1] // 2
    if x.is_cuda:
        out = torch.empty(x.shape[0], I, dtype=x.dtype, device=x.device)
        _ext.ops().act_and_mul(out, x, kind, limit)
        return out
    g, u = x[..., :I].float(), x[..., I:].float()
    if limit > 0:
        g = g.clamp(max=limit)
        u = u.clamp(-limit, limit)
    a = F.silu(g) if kind == SILU else F.gelu(g, approximate="tanh")
    return (a * u).to(x.dtype)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    return act_and_mul(x, SILU)


def silu_mul_fp8_quant(x: torch.Tensor, limit: float = 0.0) -> tuple[torch.Tensor, torch.Tensor]:
    """SwiGLU (clamped when ``limit`` > 0: gate <= limit, |up| <= limit) followed by per-token
    1x128 FP8 (e4m3) group quantisation -> (q, scales).  Reference:
    csrc/musa/quantization/silu_and_mul_per_token_group_fp8_quant.cu:37 (+clamp variant)."""
    I = x.shape[-1] // 2
    if x.is_cuda:
        q = torch.empty(x.shape[0], I, dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.empty(x.shape[0], I // 128, dtype=torch.float32, device=x.device)
        _ext.ops().silu_mul_fp8_quant(q, s, x, limit)
        return q, s
    return group_quant_fp8(act_and_mul(x, SILU, limit) if limit > 0 else silu_and_mul(x))


def group_quant_fp8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token 1x128 group FP8 quantisation: scale = amax / 448."""
    if x.is_cuda:
        q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.empty(x.shape[0], x.shape[1] // 128, dtype=torch.float32, device=x.device)
        _ext.ops().group_quant_fp8(q, s, x)
        return q, s
    xf = x.float().reshape(x.shape[0], -1, 128)
    s = xf.abs().amax(-1).clamp(min=1e-10) / 448.0
    q = (xf / s.unsqueeze(-1)).reshape(x.shape).to(torch.float8_e4m3fn)
    return q, s
