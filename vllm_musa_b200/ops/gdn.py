"""Gated DeltaNet ops (Qwen3-Next linear attention): causal conv1d with per-request state,
the gated delta-rule recurrence with per-request state, and the sigmoid output gate.

CUDA: csrc/scan/gdn.cu.  CPU: the same math in PyTorch (token loop), which is also the
numerics oracle of the GPU tests.  States: conv [slots, C, 3] (last three inputs), recurrent
[slots, Hv, dv, dk] fp32 (value-major).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _ext


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, state: torch.Tensor, cu_q: torch.Tensor,
                  seq_lens: torch.Tensor, slots: torch.Tensor,
                  out: torch.Tensor | None = None,
                  bias: torch.Tensor | None = None) -> torch.Tensor:
    """x [T, >= C] (first C channels used); w [C, 4]; optional bias [C]; updates ``state`` in
    place.  out = silu(conv(x) + bias)."""
    C = w.shape[0]
    T = x.shape[0]
    if out is None:
        out = torch.empty(T, C, dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    if x.is_cuda:
        _ext.ops().causal_conv1d(x, w, state, cu_q, seq_lens, slots, out, bias)
        return out
    cu = cu_q.tolist()
    for r in range(len(cu) - 1):
        a, b = cu[r], cu[r + 1]
        L = b - a
        slot = int(slots[r])
        hist = state[slot].float() if int(seq_lens[r]) - L > 0 else torch.zeros(C, 3)
        xs = torch.cat([hist, x[a:b, :C].float().t()], dim=1)  # [C, 3 + L]
        y = F.conv1d(xs.unsqueeze(0), w.float().unsqueeze(1), groups=C)[0]  # [C, L]
        if bias is not None:
            y = y + bias.float().unsqueeze(1)
        out[a:b] = F.silu(y).t().to(out.dtype)
        state[slot] = xs[:, -3:].to(state.dtype)
    return out


def gdn_recurrent(qkv: torch.Tensor, ba: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
                  state: torch.Tensor, cu_q: torch.Tensor, seq_lens: torch.Tensor,
                  slots: torch.Tensor, Hk: int, Hv: int,
                  out: torch.Tensor | None = None, single_token: bool = False) -> torch.Tensor:
    """Gated delta rule over each request's new tokens.  qkv [T, 2*Hk*128 + Hv*128] (conv
    output: q | k | v), ba [T, 2*Hv] (b | a); state [slots, Hv, 128, 128] updated in place.
    ``single_token``: the caller guarantees one new token per request (decode rows), which
    runs the decode kernel (every value row of a head's state loaded at once)."""
    T = qkv.shape[0]
    D = 128
    if out is None:
        out = torch.empty(T, Hv * D, dtype=qkv.dtype, device=qkv.device)
    if T == 0:
        return out
    if qkv.is_cuda:
        _ext.ops().gdn_recurrent(qkv, ba, A_log, dt_bias, state, cu_q, seq_lens, slots, Hk, Hv,
                                 out, single_token)
        return out
    rep = Hv // Hk
    cu = cu_q.tolist()
    for r in range(len(cu) - 1):
        a, b = cu[r], cu[r + 1]
        L = b - a
        slot = int(slots[r])
        S = state[slot].float().clone() if int(seq_lens[r]) - L > 0 else torch.zeros(Hv, D, D)
        q = qkv[a:b, :Hk * D].float().view(L, Hk, D).repeat_interleave(rep, 1)
        k = qkv[a:b, Hk * D:2 * Hk * D].float().view(L, Hk, D).repeat_interleave(rep, 1)
        v = qkv[a:b, 2 * Hk * D:2 * Hk * D + Hv * D].float().view(L, Hv, D)
        q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) / D ** 0.5
        k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
        bb = torch.sigmoid(ba[a:b, :Hv].float())
        g = -torch.exp(A_log.float()) * F.softplus(ba[a:b, Hv:2 * Hv].float() + dt_bias.float())
        for t in range(L):
            S = S * torch.exp(g[t]).view(Hv, 1, 1)               # S[h, v, k]
            kv = torch.einsum("hvk,hk->hv", S, k[t])
            u = (v[t] - kv) * bb[t].view(Hv, 1)
            S = S + u.unsqueeze(-1) * k[t].unsqueeze(1)
            out[a + t] = torch.einsum("hvk,hk->hv", S, q[t]).reshape(-1).to(out.dtype)
        state[slot] = S.to(state.dtype)
    return out


def _gdn_inputs(qkv, ba, A_log, dt_bias, a, b, Hk, Hv):
    """Normalised q (scaled by 1/sqrt(dk)), k, v, beta, log-decay g for tokens [a, b)."""
    D = 128
    L = b - a
    rep = Hv // Hk
    q = qkv[a:b, :Hk * D].float().view(L, Hk, D).repeat_interleave(rep, 1)
    k = qkv[a:b, Hk * D:2 * Hk * D].float().view(L, Hk, D).repeat_interleave(rep, 1)
    v = qkv[a:b, 2 * Hk * D:2 * Hk * D + Hv * D].float().view(L, Hv, D)
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) / D ** 0.5
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    beta = torch.sigmoid(ba[a:b, :Hv].float())
    g = -torch.exp(A_log.float()) * F.softplus(ba[a:b, Hv:2 * Hv].float() + dt_bias.float())
    return q, k, v, beta, g


def gdn_chunk_step(S: torch.Tensor, q, k, v, beta, g):
    """One chunk of the gated delta rule in matrix form (the algorithm of the chunked CUDA
    kernels), for all heads: S [H, dv, dk] fp32 at the chunk start; q, k [C, H, dk], v [C, H,
    dv], beta, g [C, H].  With G = cumsum(g), Gam = exp(G), u_t the delta-rule updates:
        (I + diag(beta) L) U = diag(beta) (V - diag(Gam) K S^T),  L[t,i] = e^{G_t-G_i} k_t.k_i (i<t)
        O = diag(Gam) Q S^T + tril(e^{G_t-G_i} q_t.k_i) U
        S' = e^{G_C} S + U^T diag(e^{G_C - G}) K
    Returns (O [C, H, dv], S')."""
    C = q.shape[0]
    G = torch.cumsum(g, 0)                                    # [C, H]
    qh, kh, vh = q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1)   # [H, C, d]
    Gh = G.t()                                                # [H, C]
    causal = torch.tril(torch.ones(C, C))
    strict = torch.tril(torch.ones(C, C), -1)
    diff = (Gh.unsqueeze(2) - Gh.unsqueeze(1)).masked_fill(causal == 0, float("-inf"))
    decay = torch.exp(diff)                                   # [H, t, i] = e^{G_t - G_i}, i <= t
    Lm = (kh @ kh.transpose(1, 2)) * decay * strict           # [H, C, C]
    bh = beta.t().unsqueeze(2)                                # [H, C, 1]
    T = torch.eye(C).expand_as(Lm) + bh * Lm
    gam = torch.exp(Gh).unsqueeze(2)                          # [H, C, 1]
    rhs = bh * (vh - gam * (kh @ S.transpose(1, 2)))          # [H, C, dv]
    U = torch.linalg.solve_triangular(T, rhs, upper=False, unitriangular=True)
    Mq = (qh @ kh.transpose(1, 2)) * decay * causal
    O = gam * (qh @ S.transpose(1, 2)) + Mq @ U               # [H, C, dv]
    tail = torch.exp(Gh[:, -1:] - Gh).unsqueeze(2)            # [H, C, 1]
    S2 = torch.exp(Gh[:, -1]).view(-1, 1, 1) * S + U.transpose(1, 2) @ (tail * kh)
    return O.transpose(0, 1), S2


def gdn_chunked_ref(qkv: torch.Tensor, ba: torch.Tensor, A_log: torch.Tensor,
                    dt_bias: torch.Tensor, state: torch.Tensor, cu_q: torch.Tensor,
                    seq_lens: torch.Tensor, slots: torch.Tensor, Hk: int, Hv: int,
                    chunk: int = 64) -> torch.Tensor:
    """The gated delta rule evaluated chunk by chunk (same results as ``gdn_recurrent``)."""
    T = qkv.shape[0]
    D = 128
    out = torch.empty(T, Hv * D, dtype=qkv.dtype)
    cu = cu_q.tolist()
    for r in range(len(cu) - 1):
        a, b = cu[r], cu[r + 1]
        slot = int(slots[r])
        S = state[slot].float().clone() if int(seq_lens[r]) - (b - a) > 0 else \
            torch.zeros(Hv, D, D)
        q, k, v, beta, g = _gdn_inputs(qkv, ba, A_log, dt_bias, a, b, Hk, Hv)
        for c0 in range(0, b - a, chunk):
            c1 = min(b - a, c0 + chunk)
            O, S = gdn_chunk_step(S, q[c0:c1], k[c0:c1], v[c0:c1], beta[c0:c1], g[c0:c1])
            out[a + c0:a + c1] = O.reshape(c1 - c0, Hv * D).to(out.dtype)
        state[slot] = S.to(state.dtype)
    return out


CHUNK_MIN_TOKENS = 64   # requests with at least this many new tokens use the chunked kernels
_BLOCK_BYTES = 3 * 64 * 128 * 2 + 64 * 64 * 2 + 64 * 128 * 4


def gdn_chunked(qkv: torch.Tensor, ba: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
                state: torch.Tensor, cu_q: torch.Tensor, seq_lens: torch.Tensor,
                slots: torch.Tensor, Hk: int, Hv: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Same contract as ``gdn_recurrent``, evaluated 64 tokens at a time: a parallel per-chunk
    kernel (triangular solve, decayed Q K^T / K K^T) and a tensor-core chunk scan carrying the
    state (csrc/scan/gdn_chunked.cu).  CPU: ``gdn_chunked_ref``."""
    T = qkv.shape[0]
    if out is None:
        out = torch.empty(T, Hv * 128, dtype=qkv.dtype, device=qkv.device)
    if T == 0:
        return out
    if not qkv.is_cuda:
        out.copy_(gdn_chunked_ref(qkv, ba, A_log, dt_bias, state, cu_q, seq_lens, slots, Hk, Hv))
        return out
    R = seq_lens.shape[0]
    max_chunks = (T + 63) // 64 + R
    ws = torch.empty(max_chunks * Hv * _BLOCK_BYTES, dtype=torch.uint8, device=qkv.device)
    offs = torch.empty(R + 1, dtype=torch.int32, device=qkv.device)
    gam = torch.empty(max_chunks * Hv, dtype=torch.float32, device=qkv.device)
    _ext.ops().gdn_chunked(qkv, ba, A_log, dt_bias, state, cu_q, seq_lens, slots, Hk, Hv, out,
                           ws, offs, gam)
    return out


def sigmoid_gate(out: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """out *= sigmoid(gate) in place (both [T, W], rows may be strided)."""
    if out.is_cuda:
        if out.shape[0]:
            _ext.ops().sigmoid_gate(out, gate)
        return out
    out.copy_((out.float() * torch.sigmoid(gate.float())).to(out.dtype))
    return out
