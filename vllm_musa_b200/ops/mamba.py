"""Mamba2 mixer ops: the selective state-space scan with per-request state slots and the
gate-then-normalise RMSNorm.

CUDA: csrc/scan/mamba2.cu (conv1d with bias: csrc/scan/gdn.cu).  CPU: the same recurrence in
PyTorch (token loop), which is also the numerics oracle of the GPU tests.  State layout
[slots, H, P, N] fp32; a request whose ``seq_len`` equals its step token count starts from a
zero state.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _ext


def mamba2_scan(xbc: torch.Tensor, b_off: int, c_off: int, dt: torch.Tensor,
                dt_bias: torch.Tensor, A_log: torch.Tensor, D: torch.Tensor,
                state: torch.Tensor, cu_q: torch.Tensor, seq_lens: torch.Tensor,
                slots: torch.Tensor, H: int, G: int, P: int, N: int,
                dt_min: float = 0.0, dt_max: float = math.inf,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """xbc [T, >= c_off + G*N]: x (H*P) at column 0, B (G*N) at ``b_off``, C at ``c_off``;
    dt [T, >= H] raw (before softplus).  Returns y [T, H*P] = S C + D x, updating ``state``."""
    T = xbc.shape[0]
    if out is None:
        out = torch.empty(T, H * P, dtype=xbc.dtype, device=xbc.device)
    if T == 0:
        return out
    if xbc.is_cuda:
        _ext.ops().mamba2_scan(xbc, b_off, c_off, dt, dt_bias, A_log, D, state, cu_q, seq_lens,
                               slots, out, H, G, P, N, dt_min, dt_max)
        return out
    A = -torch.exp(A_log.float())
    rep = H // G
    cu = cu_q.tolist()
    for r in range(len(cu) - 1):
        a, b = cu[r], cu[r + 1]
        if b == a:
            continue
        slot = int(slots[r])
        S = state[slot].float() if int(seq_lens[r]) - (b - a) > 0 else \
            torch.zeros(H, P, N, dtype=torch.float32)
        for t in range(a, b):
            x = xbc[t, :H * P].float().view(H, P)
            Bt = xbc[t, b_off:b_off + G * N].float().view(G, N).repeat_interleave(rep, 0)
            Ct = xbc[t, c_off:c_off + G * N].float().view(G, N).repeat_interleave(rep, 0)
            d = F.softplus(dt[t, :H].float() + dt_bias.float()).clamp(dt_min, dt_max)
            S = S * torch.exp(d * A).view(H, 1, 1) + (d.view(H, 1) * x).unsqueeze(-1) * \
                Bt.unsqueeze(1)
            y = (S * Ct.unsqueeze(1)).sum(-1) + D.float().view(H, 1) * x
            out[t] = y.reshape(H * P).to(out.dtype)
        state[slot] = S.to(state.dtype)
    return out


def gated_rmsnorm(y: torch.Tensor, z: torch.Tensor, w: torch.Tensor, group: int, eps: float,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over groups of ``group`` channels of y * silu(z), times w (gate, then norm)."""
    C = w.numel()
    T = y.shape[0]
    if out is None:
        out = torch.empty(T, C, dtype=y.dtype, device=y.device)
    if T == 0:
        return out
    if y.is_cuda:
        _ext.ops().gated_rmsnorm(out, y, z, w, group, eps)
        return out
    v = (y[:, :C].float() * F.silu(z[:, :C].float())).view(T, C // group, group)
    v = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps)
    out.copy_((v.view(T, C) * w.float()).to(out.dtype))
    return out
