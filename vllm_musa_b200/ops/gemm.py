"""Linear layers on the tcgen05 BF16 GEMM (csrc/gemm/gemm_bf16.cu).

``linear(x, w)`` = x @ w.T with w in nn.Linear layout [N, K].  ``linear_silu_mul`` applies
SwiGLU in the GEMM epilogue; its weight must be laid out by :func:`interleave_gate_up`
(groups of 8 gate rows followed by the matching 8 up rows).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _ext
from .. import tuning

_WS: dict = {}
_COUNTERS: dict = {}
MAX_TILES = 1 << 16


def _workspace(device: torch.device, numel: int) -> torch.Tensor:
    """Split-K fp32 workspace, grown on demand and reused (never freed while in use)."""
    key = (device.type, device.index)
    ws = _WS.get(key)
    if ws is None or ws.numel() < numel:
        if device.type == "cuda" and torch.cuda.is_current_stream_capturing():
            raise RuntimeError("split-K workspace must be reserved before CUDA-graph capture")
        ws = torch.empty(max(numel, 1 << 20), dtype=torch.float32, device=device)
        _WS[key] = ws
    return ws


def _counters(device: torch.device) -> torch.Tensor:
    """Per-tile split-K arrival counters: zeroed once, reset by the kernel after every use."""
    key = (device.type, device.index)
    c = _COUNTERS.get(key)
    if c is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("split-K counters must be allocated before CUDA-graph capture")
        c = torch.zeros(MAX_TILES, dtype=torch.int32, device=device)
        _COUNTERS[key] = c
    return c


def reserve_workspace(device: torch.device, numel: int) -> None:
    """Pre-size the split-K workspace and counters (call before CUDA-graph capture)."""
    _workspace(device, numel)
    _counters(device)


def plan_for(M: int, N: int, K: int, bn: int = 0, splits: int = 0, mt: int = 0) -> tuple:
    """(bn, splits, mt, workspace_floats): forced plan, else the measured table, else the
    kernel's cost model (zeros let the launcher decide)."""
    if bn <= 0 and splits <= 0 and mt <= 0:
        hit = tuning.gemm_table().lookup(M, N, K)
        if hit is not None:
            bn, splits, mt = hit
    if bn > 0 or splits > 0 or mt > 0:
        if splits <= 0:
            splits = 1
        return bn, splits, mt, (splits if splits > 1 else 0) * M * N
    pl = _ext.require().gemm_plan(M, N, K)
    return 0, 0, 0, pl[2]


def _run(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, mode: int, bn: int = 0,
         splits: int = 0, mt: int = 0, swap: bool = False) -> torch.Tensor:
    """mode 0 store / 1 SwiGLU / 2 fp32.  ``swap`` (or a measured swapped plan for a decode-
    sized M) runs C^T = W X^T with the tokens in the MMA's N dimension (modes 0 and 1)."""
    _ext.require()  # registers torch.ops.b200
    M, N, K = x.shape[0], w.shape[0], x.shape[1]
    if mode in (0, 1) and M % 8 == 0 and (mode == 0 or N % 16 == 0):
        sp = None
        if swap:
            sp = (bn, splits, mt)
        elif bn <= 0 and splits <= 0 and mt <= 0 and M <= 256:
            sp = tuning.gemm_table().swap_plan(M, N, K)
        if sp is not None:
            sbn, ss, smt = sp
            need = ss * M * N if ss > 1 else 0
            ws = _workspace(x.device, need) if need > 0 else None
            cnt = _counters(x.device) if need > 0 else None
            torch.ops.b200.gemm_bf16(w, x, out, mode + 4, sbn, ss, ws, smt, cnt)
            return out
    bn, splits, mt, need = plan_for(M, N, K, bn, splits, mt)
    ws = _workspace(x.device, need) if need > 0 else None
    cnt = _counters(x.device) if need > 0 else None
    torch.ops.b200.gemm_bf16(x, w, out, mode, bn, splits, ws, mt, cnt)
    return out


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
           out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """x [M, K] @ w[N, K]^T -> [M, N]; ``out_dtype=torch.float32`` keeps fp32 (logits)."""
    if x.is_cuda:
        f32 = out_dtype == torch.float32
        if out is None:
            out = torch.empty(x.shape[0], w.shape[0], device=x.device,
                              dtype=torch.float32 if f32 else torch.bfloat16)
        if x.shape[0] == 0:
            return out
        return _run(x, w, out, 2 if f32 else 0)
    y = x.float() @ w.float().t()
    y = y if out_dtype == torch.float32 else y.to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, group: int = 8) -> torch.Tensor:
    """[I, K] gate and up -> [2I, K] with rows (gate[8g:8g+8], up[8g:8g+8]) per group.

    I is zero-padded to a multiple of ``group``; padded channels contribute silu(0)*0 = 0.
    """
    I, K = gate.shape
    pad = (-I) % group
    if pad:
        z = torch.zeros(pad, K, dtype=gate.dtype, device=gate.device)
        gate, up = torch.cat([gate, z]), torch.cat([up, z])
    G = gate.shape[0] // group
    return torch.stack([gate.reshape(G, group, K), up.reshape(G, group, K)], 1).reshape(-1, K)


def deinterleave_gate_up(w: torch.Tensor, group: int = 8) -> tuple[torch.Tensor, torch.Tensor]:
    K = w.shape[1]
    v = w.reshape(-1, 2, group, K)
    return v[:, 0].reshape(-1, K), v[:, 1].reshape(-1, K)


def linear_silu_mul(x: torch.Tensor, w_interleaved: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(x @ gate^T) * (x @ up^T) from an interleaved [2I, K] weight -> [M, I]."""
    if x.is_cuda:
        if out is None:
            out = torch.empty(x.shape[0], w_interleaved.shape[0] // 2, device=x.device,
                              dtype=torch.bfloat16)
        if x.shape[0] == 0:
            return out
        return _run(x, w_interleaved, out, 1)
    g, u = deinterleave_gate_up(w_interleaved)
    y = (F.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())).to(x.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y
