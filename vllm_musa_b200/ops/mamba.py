"""Mamba2 mixer ops: the selective state-space scan with per-request state slots (token
recurrence for decode, chunked matrix form for prefill) and the gate-then-normalise RMSNorm.

CUDA: csrc/scan/mamba2.cu, csrc/scan/mamba2_chunked.cu (conv1d with bias: csrc/scan/gdn.cu).  CPU: the same recurrence in
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


CHUNK = 64               # tokens per chunk of the chunked SSD kernels
CHUNK_MIN_TOKENS = 64    # prefill parts with at least this many tokens take the chunked path


def mamba2_chunked_supported(P: int, N: int) -> bool:
    return P in (32, 64) and N in (64, 128)


def mamba2_chunk_step(S: torch.Tensor, x, Bm, Cm, dt, A, D):
    """One chunk of the SSD in matrix form, for all heads (the algorithm of the chunked CUDA
    kernels, fp32): S [H, P, N] at the chunk start; x [n, H, P], Bm / Cm [n, H, N] (per-head
    groups expanded), dt [n, H] after softplus / clamp, A [H] (< 0), D [H].
    Returns (y [n, H, P], S at the chunk end)."""
    a = torch.cumsum(dt * A, 0)                                   # [n, H]
    n = x.shape[0]
    seg = a[:, None, :] - a[None, :, :]                           # [i, j, H] a_i - a_j
    causal = torch.tril(torch.ones(n, n, dtype=torch.bool))[:, :, None]
    L = torch.where(causal, torch.exp(seg.clamp(max=0.0)), torch.zeros(()))
    G = torch.einsum("ihn,jhn->ijh", Cm, Bm) * L * dt[None, :, :]  # [i, j, H]
    y = torch.einsum("ijh,jhp->ihp", G, x)
    y = y + torch.exp(a)[:, :, None] * torch.einsum("ihn,hpn->ihp", Cm, S)
    y = y + D[None, :, None] * x
    w = torch.exp(a[-1][None, :] - a) * dt                        # [j, H]
    S = torch.exp(a[-1])[:, None, None] * S + torch.einsum("jh,jhp,jhn->hpn", w, x, Bm)
    return y, S


def mamba2_chunked_ref(xbc, b_off, c_off, dt_raw, dt_bias, A_log, D, state, cu_q, seq_lens,
                       slots, H, G, P, N, dt_min=0.0, dt_max=math.inf, chunk=CHUNK):
    """The SSD evaluated chunk by chunk in PyTorch (same results as the token recurrence of
    ``mamba2_scan``, up to fp32 rounding); updates ``state``, returns y [T, H*P] fp32."""
    A = -torch.exp(A_log.float())
    rep = H // G
    T = xbc.shape[0]
    out = torch.zeros(T, H * P)
    cu = cu_q.tolist()
    for r in range(len(cu) - 1):
        a0, b0 = cu[r], cu[r + 1]
        if b0 == a0:
            continue
        slot = int(slots[r])
        S = state[slot].float().clone() if int(seq_lens[r]) - (b0 - a0) > 0 else \
            torch.zeros(H, P, N)
        for c0 in range(a0, b0, chunk):
            c1 = min(b0, c0 + chunk)
            x = xbc[c0:c1, :H * P].float().view(-1, H, P)
            Bm = xbc[c0:c1, b_off:b_off + G * N].float().view(-1, G, N).repeat_interleave(rep, 1)
            Cm = xbc[c0:c1, c_off:c_off + G * N].float().view(-1, G, N).repeat_interleave(rep, 1)
            d = F.softplus(dt_raw[c0:c1, :H].float() + dt_bias.float()).clamp(dt_min, dt_max)
            y, S = mamba2_chunk_step(S, x, Bm, Cm, d, A, D.float())
            out[c0:c1] = y.reshape(c1 - c0, H * P)
        state[slot] = S.to(state.dtype)
    return out


def mamba2_chunked(xbc: torch.Tensor, b_off: int, c_off: int, dt: torch.Tensor,
                   dt_bias: torch.Tensor, A_log: torch.Tensor, D: torch.Tensor,
                   state: torch.Tensor, cu_q: torch.Tensor, seq_lens: torch.Tensor,
                   slots: torch.Tensor, H: int, G: int, P: int, N: int,
                   dt_min: float = 0.0, dt_max: float = math.inf,
                   out: torch.Tensor | None = None, num_tokens: int | None = None) -> torch.Tensor:
    """Same contract as ``mamba2_scan``, evaluated 64 tokens at a time: chunk states and chunk
    outputs as tensor-core products over all chunks in parallel, with a short sequential pass
    carrying the state between a request's chunks (csrc/scan/mamba2_chunked.cu).
    ``num_tokens`` = rows covered by ``cu_q`` (default: all of xbc).  CPU: ``mamba2_chunked_ref``."""
    T = xbc.shape[0]
    if out is None:
        out = torch.empty(T, H * P, dtype=xbc.dtype, device=xbc.device)
    if T == 0:
        return out
    if not xbc.is_cuda:
        y = mamba2_chunked_ref(xbc, b_off, c_off, dt, dt_bias, A_log, D, state, cu_q, seq_lens,
                               slots, H, G, P, N, dt_min, dt_max)
        cu = cu_q.tolist()
        out[cu[0]:cu[-1]] = y[cu[0]:cu[-1]].to(out.dtype)
        return out
    R = seq_lens.shape[0]
    nt = T if num_tokens is None else num_tokens
    mc = (nt + CHUNK - 1) // CHUNK + R
    dev = xbc.device
    offs = torch.empty(R + 1, dtype=torch.int32, device=dev)
    ws = torch.empty(mc * H * P * N, dtype=torch.float32, device=dev)
    start = torch.empty(mc * H * P * N, dtype=torch.bfloat16, device=dev)
    decay = torch.empty(mc * H, dtype=torch.float32, device=dev)
    _ext.ops().mamba2_chunked(xbc, b_off, c_off, dt, dt_bias, A_log, D, state, cu_q, seq_lens,
                              slots, out, H, G, P, N, dt_min, dt_max, offs, ws, start, decay, nt)
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
