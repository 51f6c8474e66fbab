"""Mixture-of-experts ops: routing, expert-sorted layout, grouped GEMMs, weighted combine.

CUDA path (csrc/moe/moe.cu + the grouped mode of csrc/gemm/gemm_bf16.cu):
    ids, w   = topk_softmax(router_logits)            (or grouped_topk)
    sorted   = moe_align(ids)     every expert's rows padded to 128, counts stay on device
    xs       = moe_gather(x)      [max_rows, H] expert-contiguous activations
    h        = grouped GEMM(xs, W_gate_up, SwiGLU epilogue)   [max_rows, I]
    y        = grouped GEMM(h, W_down)                         [max_rows, H]
    out      = moe_combine(y, w)  (+ shared-expert output)
No host synchronisation anywhere, so decode MoE layers run inside CUDA graphs.
CPU path: a per-expert loop in PyTorch (reference semantics).  Reference counterpart:
vllm_musa/model_executor/layers/fused_moe/fused_moe.py:2214-2765 (dispatcher and backends).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import _ext
from ..utils import moe_inventory
from .gemm import deinterleave_gate_up


def topk_softmax(logits: torch.Tensor, k: int, renorm: bool = True):
    T, E = logits.shape
    if logits.is_cuda:
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        if T:
            lg = logits if logits.dtype == torch.float32 and logits.stride(1) == 1 else \
                logits.float().contiguous()
            _ext.ops().topk_softmax(lg, ids, w, renorm)
        return ids, w
    p = torch.softmax(logits.float(), -1)
    w, ids = torch.topk(p, k, dim=-1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return ids.to(torch.int32), w


def grouped_topk(logits: torch.Tensor, k: int, n_group: int, topk_group: int,
                 bias: Optional[torch.Tensor] = None, sigmoid: bool = True, renorm: bool = True,
                 scale: float = 1.0):
    T, E = logits.shape
    if logits.is_cuda:
        ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
        if T:
            _ext.ops().grouped_topk(logits.float().contiguous(),
                                    bias.float().contiguous() if bias is not None else None,
                                    ids, w, n_group, topk_group, sigmoid, renorm, scale)
        return ids, w
    s = torch.sigmoid(logits.float()) if sigmoid else torch.softmax(logits.float(), -1)
    b = s + (bias.float() if bias is not None else 0.0)
    g = b.view(T, n_group, E // n_group)
    gscore = g.topk(min(2, E // n_group), dim=-1).values.sum(-1)
    keep = torch.zeros(T, n_group, dtype=torch.bool)
    keep.scatter_(1, gscore.topk(topk_group, dim=-1).indices, True)
    b = b.masked_fill(~keep.repeat_interleave(E // n_group, dim=1), float("-inf"))
    ids = b.topk(k, dim=-1).indices
    w = s.gather(1, ids)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return ids.to(torch.int32), w * scale


def _fused_moe_ref(x, w_gu, w_down, ids, w, num_experts, shared, expert_offset=0,
                   shared_gate=None):
    T, H = x.shape
    I2 = w_gu.shape[0] // num_experts
    out = torch.zeros(T, H, dtype=torch.float32)
    xf = x.float()
    for e in range(num_experts):
        tok, slot = torch.nonzero(ids == e + expert_offset, as_tuple=True)
        if tok.numel() == 0:
            continue
        g, u = deinterleave_gate_up(w_gu[e * I2:(e + 1) * I2])
        h = F.silu(xf[tok] @ g.float().t()) * (xf[tok] @ u.float().t())
        h = h.to(x.dtype).float()
        d = w_down[e * H:(e + 1) * H].float()
        y = (h @ d.t()).to(x.dtype).float()
        out.index_add_(0, tok, y * w[tok, slot].unsqueeze(1).float())
    if shared is not None:
        s = shared.float()
        if shared_gate is not None:
            s = s * torch.sigmoid(shared_gate.float().reshape(T, 1))
        out += s
    return out.to(x.dtype)


def fused_moe(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor, ids: torch.Tensor,
              w: torch.Tensor, num_experts: int, shared: Optional[torch.Tensor] = None,
              out: Optional[torch.Tensor] = None, expert_offset: int = 0,
              shared_gate: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [T, H]; w_gu [E * 2I, H] (gate/up interleaved per expert); w_down [E * H, I];
    ids/w [T, k] -> [T, H] = sum_j w[:, j] * expert_{ids[:, j]}(x) (+ shared).

    With expert parallelism this rank holds experts [expert_offset, expert_offset + E); routed
    slots naming other experts contribute nothing here (their owners add them).
    ``shared_gate`` [T, 1] fp32 logits (any row stride) scale ``shared`` by their sigmoid."""
    T, H = x.shape
    k = ids.shape[1]
    if out is None:
        out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    I = w_gu.shape[0] // num_experts // 2
    gemv = x.is_cuda and use_gemv(T, k, H, I)
    moe_inventory.note("cpu" if not x.is_cuda else "gemv" if gemv else "grouped", x, ids,
                       num_experts, I, w_gu.dtype, expert_offset)
    if not x.is_cuda:
        out.copy_(_fused_moe_ref(x, w_gu, w_down, ids, w, num_experts, shared, expert_offset,
                                 shared_gate))
        return out
    if gemv:
        y, pos = moe_experts_gemv(x, w_gu, w_down, ids, num_experts, expert_offset)
    else:
        y, pos = moe_experts(x, w_gu, w_down, ids, num_experts, expert_offset)
    torch.ops.b200.moe_combine(y, pos, w.contiguous(), shared, out, shared_gate)
    return out


def use_gemv(T: int, k: int, H: int, I: int) -> bool:
    """Dispatch policy: per-pair GEMVs for at most ``B200_MOE_GEMV_MAX_PAIRS`` routed (token,
    slot) pairs, the grouped GEMMs above (decided on host shapes only: graph-capture safe)."""
    from .. import envs
    return T * k <= envs.get("B200_MOE_GEMV_MAX_PAIRS") and H % 32 == 0 and I % 32 == 0


def moe_experts_gemv(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor,
                     ids: torch.Tensor, num_experts: int,
                     expert_offset: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Routed experts of a few tokens as per-(token, slot) GEMVs (CUDA): same outputs as
    ``moe_experts`` (y rows addressed through pos)."""
    T, H = x.shape
    k = ids.shape[1]
    E = num_experts
    I = w_gu.shape[0] // E // 2
    dev = x.device
    h = torch.empty(T * k, I, dtype=x.dtype, device=dev)
    y = torch.empty(T * k, H, dtype=x.dtype, device=dev)
    pos = torch.empty(T, k, dtype=torch.int32, device=dev)
    _ext.require()
    torch.ops.b200.moe_gemv(x, ids.contiguous(), E, expert_offset, w_gu, w_down, h, y, pos)
    return y, pos


def moe_experts(x: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor, ids: torch.Tensor,
                num_experts: int, expert_offset: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Routed experts without the combine (CUDA): align -> gather -> grouped GEMM (SwiGLU) ->
    grouped GEMM.  Returns (y [max_rows, H] expert outputs in expert-sorted order, pos [T, k]:
    the row of y holding (token t, slot j), -1 when that expert is not served here)."""
    T, H = x.shape
    k = ids.shape[1]
    mod = _ext.require()
    E = num_experts
    max_rows = int(mod.moe_max_rows(T * k, E))
    dev = x.device
    sorted_ids = torch.empty(max_rows, dtype=torch.int32, device=dev)
    tile_expert = torch.empty(max_rows // 128, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    pos = torch.empty(T, k, dtype=torch.int32, device=dev)
    num_tiles = torch.empty(1, dtype=torch.int32, device=dev)
    ops = torch.ops.b200
    ops.moe_align(ids.contiguous(), E, sorted_ids, tile_expert, offsets, pos, num_tiles,
                  expert_offset)
    xs = torch.empty(max_rows, H, dtype=x.dtype, device=dev)
    ops.moe_gather(x, sorted_ids, num_tiles, k, xs)
    I = w_gu.shape[0] // E // 2
    h = torch.empty(max_rows, I, dtype=x.dtype, device=dev)
    ops.gemm_grouped_bf16(xs, w_gu, h, tile_expert, num_tiles, E, 1, 0)
    y = torch.empty(max_rows, H, dtype=x.dtype, device=dev)
    ops.gemm_grouped_bf16(h, w_down, y, tile_expert, num_tiles, E, 0, 0)
    return y, pos


def _fq(x: torch.Tensor) -> torch.Tensor:
    """x rounded through per-token 1x128 e4m3 quantisation (what the GPU path feeds its GEMMs)."""
    from .activation import group_quant_fp8
    q, s = group_quant_fp8(x)
    return q.float() * s.repeat_interleave(128, 1)


def _fused_moe_fp8_ref(x, w_gu, s_gu, w_down, s_down, ids, w, E, shared, expert_offset,
                       limit=0.0):
    from .fp8 import dequantize_weight_block
    T, H = x.shape
    I2 = w_gu.shape[0] // E
    out = torch.zeros(T, H, dtype=torch.float32)
    xf = _fq(x.to(torch.bfloat16))
    for e in range(E):
        tok, slot = torch.nonzero(ids == e + expert_offset, as_tuple=True)
        if tok.numel() == 0:
            continue
        gu = dequantize_weight_block(w_gu[e * I2:(e + 1) * I2], s_gu[e * I2 // 128:(e + 1) * I2 // 128])
        dn = dequantize_weight_block(w_down[e * H:(e + 1) * H],
                                     s_down[e * (H // 128):(e + 1) * (H // 128)])
        hg = (xf[tok] @ gu.t()).to(torch.bfloat16).float()
        g, u = hg[:, :I2 // 2], hg[:, I2 // 2:]
        if limit > 0:
            g, u = g.clamp(max=limit), u.clamp(-limit, limit)
        h = _fq((F.silu(g) * u).to(torch.bfloat16))
        y = (h @ dn.t()).to(torch.bfloat16).float()
        out.index_add_(0, tok, y * w[tok, slot].unsqueeze(1).float())
    if shared is not None:
        out += shared.float()
    return out.to(x.dtype)


def fused_moe_fp8(x: torch.Tensor, w_gu: torch.Tensor, s_gu: torch.Tensor, w_down: torch.Tensor,
                  s_down: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, num_experts: int,
                  shared: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                  expert_offset: int = 0, swiglu_limit: float = 0.0) -> torch.Tensor:
    """Block-FP8 routed experts (DeepSeek): w_gu e4m3 [E * 2I, H] with rows [gate (I) ; up (I)]
    per expert and 128x128 scales s_gu [E * 2I/128, H/128]; w_down e4m3 [E * H, I], s_down
    [E * H/128, I/128].

        align -> gather -> 1x128 quant -> grouped FP8 GEMM (gate|up) -> SwiGLU + 1x128 quant
        -> grouped FP8 GEMM (down) -> weighted combine (+ shared)
    Every step is a device kernel with device-side counts (graph-capturable)."""
    T, H = x.shape
    k = ids.shape[1]
    if out is None:
        out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    moe_inventory.note("fp8_grouped" if x.is_cuda else "cpu", x, ids, num_experts,
                       w_gu.shape[0] // num_experts // 2, w_gu.dtype, expert_offset)
    if not x.is_cuda:
        out.copy_(_fused_moe_fp8_ref(x, w_gu, s_gu, w_down, s_down, ids, w, num_experts, shared,
                                     expert_offset, swiglu_limit))
        return out
    from .activation import group_quant_fp8, silu_mul_fp8_quant
    mod = _ext.require()
    E = num_experts
    max_rows = int(mod.moe_max_rows(T * k, E))
    dev = x.device
    sorted_ids = torch.empty(max_rows, dtype=torch.int32, device=dev)
    tile_expert = torch.empty(max_rows // 128, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    pos = torch.empty(T, k, dtype=torch.int32, device=dev)
    num_tiles = torch.empty(1, dtype=torch.int32, device=dev)
    ops = torch.ops.b200
    ops.moe_align(ids.contiguous(), E, sorted_ids, tile_expert, offsets, pos, num_tiles,
                  expert_offset)
    xs = torch.empty(max_rows, H, dtype=x.dtype, device=dev)
    ops.moe_gather(x, sorted_ids, num_tiles, k, xs)
    xq, xsc = group_quant_fp8(xs)
    I2 = w_gu.shape[0] // E
    hg = torch.empty(max_rows, I2, dtype=x.dtype, device=dev)
    ops.gemm_fp8(xq, xsc, w_gu, s_gu, hg, 1, None, None, tile_expert, num_tiles, E)
    hq, hsc = silu_mul_fp8_quant(hg, swiglu_limit)
    y = torch.empty(max_rows, H, dtype=x.dtype, device=dev)
    ops.gemm_fp8(hq, hsc, w_down, s_down, y, 1, None, None, tile_expert, num_tiles, E)
    ops.moe_combine(y, pos, w.contiguous(), shared, out, None)
    return out
