"""RMSNorm family (reference: csrc/musa/fused_add_rmsnorm.mu:54,
vllm_musa/model_executor/layers/layernorm.py:37-179)."""
from __future__ import annotations

import torch

from . import _ext


def _rms_ref(x: torch.Tensor, w: torch.Tensor, eps: float, gemma: bool) -> torch.Tensor:
    xf = x.float()
    var = xf.pow(2).mean(-1, keepdim=True)
    wf = w.float() + 1.0 if gemma else w.float()
    return (xf * torch.rsqrt(var + eps) * wf).to(x.dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, gemma: bool = False,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x / rms(x) * w  (Gemma: * (1 + w)).  x: [rows, H]."""
    if x.is_cuda:
        out = torch.empty_like(x) if out is None else out
        _ext.ops().rms_norm(out, x, weight, eps, gemma)
        return out
    y = _rms_ref(x, weight, eps, gemma)
    if out is not None:
        out.copy_(y)
        return out
    return y


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                       gemma: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """In place: residual <- x + residual; x <- RMSNorm(residual).  Returns (x, residual)."""
    if x.is_cuda:
        _ext.ops().fused_add_rms_norm(x, residual, weight, eps, gemma)
        return x, residual
    s = (x.float() + residual.float()).to(x.dtype)
    residual.copy_(s)
    x.copy_(_rms_ref(s, weight, eps, gemma))
    return x, residual


def rms_norm_quant_fp8(x: torch.Tensor, weight: torch.Tensor, eps: float,
                       residual: torch.Tensor | None = None, want_bf16: bool = False):
    """(residual <- x + residual;) y = RMSNorm(residual or x) * w, quantised per token in 1x128
    e4m3 groups in the same pass.  Returns (q [rows, H] e4m3, scales [rows, H/128] fp32, y bf16
    or None).  Reference: csrc/musa/quantization/fused_add_rms_norm_per_token_group_fp8_quant.cu:59."""
    rows, H = x.shape
    if x.is_cuda:
        q = torch.empty(rows, H, dtype=torch.float8_e4m3fn, device=x.device)
        sc = torch.empty(rows, H // 128, dtype=torch.float32, device=x.device)
        y = torch.empty_like(x) if want_bf16 else None
        _ext.ops().rms_norm_quant_fp8(q, sc, y, x, residual, weight, eps)
        return q, sc, y
    if residual is not None:
        s = (x.float() + residual.float()).to(x.dtype)
        residual.copy_(s)
        y = _rms_ref(s, weight, eps, False)
    else:
        y = _rms_ref(x, weight, eps, False)
    g = y.float().view(rows, H // 128, 128)
    sc = g.abs().amax(-1).clamp_min(1e-10) / 448.0
    q = (g / sc.unsqueeze(-1)).view(rows, H).to(torch.float8_e4m3fn)
    return q, sc, (y if want_bf16 else None)


def rms_norm_gated(x: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, group: int,
                   eps: float) -> torch.Tensor:
    """RMSNorm over groups of ``group`` channels, times weight, times silu(z) (GDN output)."""
    if x.is_cuda:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        _ext.ops().rms_norm_gated(out, x, z, weight, group, eps)
        return out
    shp = x.shape
    xf = x.float().reshape(-1, group)
    var = xf.pow(2).mean(-1, keepdim=True)
    y = (xf * torch.rsqrt(var + eps)).reshape(shp) * weight.float().repeat(shp[-1] // group)
    return (y * torch.nn.functional.silu(z.float())).to(x.dtype)
