"""W4AFP8 routed experts: packed signed INT4 expert weights with bf16 group-128 scales and
dynamic per-token e4m3 activations.

Checkpoint layout (the interface the format fixes): ``w13`` int8 [E, 2I, H/2] with rows
[gate (I) ; up (I)] per expert, ``w2`` int8 [E, H, I/2], element 2j of a row in the low nibble
of byte j and element 2j+1 in the high nibble; scales bf16 [E, 2I, H/128] and [E, H, I/128],
one per (output row, 128 input columns).  Activations are quantised per token with one scale,
max(|x|, 1e-4) / 448, before each expert GEMM; the SwiGLU may be clamped (``swiglu_limit``).

CUDA path, every step a device kernel with device-side counts (graph-capturable):
    per-token e4m3 round trip of x -> moe_align (expert_map applied) -> gather rows ->
    expand the live experts' int4 gate/up weights to bf16 -> tcgen05 grouped GEMM ->
    SwiGLU(+clamp) + per-row e4m3 round trip -> expand down weights -> grouped GEMM ->
    weighted combine.

Reference: vllm_musa/kernels/w4afp8_moe.py:163-337 (w4afp8_moe),
vllm_musa/model_executor/layers/quantization/w4afp8.py:26-170 (config + expert weights).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import _ext


def pack_int4(w: torch.Tensor) -> torch.Tensor:
    """int values in [-8, 7], last dim even -> int8 with two values per byte (low nibble first)."""
    lo = w[..., ::2].to(torch.int16) & 15
    hi = (w[..., 1::2].to(torch.int16) & 15) << 4
    return (lo | hi).to(torch.int8)


def unpack_int4(p: torch.Tensor) -> torch.Tensor:
    b = p.to(torch.int16) & 255
    lo = ((b & 15) ^ 8) - 8
    hi = ((b >> 4) ^ 8) - 8
    return torch.stack((lo, hi), dim=-1).flatten(-2).to(torch.int8)


def dequant_w4(p: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """[E, N, K/2] packed + [E, N, K/128] scales -> fp32 [E, N, K]."""
    return unpack_int4(p).float() * scales.float().repeat_interleave(128, dim=-1)


def quantize_w4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """float [..., N, K] -> (packed int4 [..., N, K/2], bf16 scales [..., N, K/128]): symmetric
    per (row, 128 columns), scale = amax / 7 (random-init models and tests)."""
    g = w.float().unflatten(-1, (w.shape[-1] // 128, 128))
    s = (g.abs().amax(-1).clamp_min(1e-8) / 7.0).to(torch.bfloat16)
    q = torch.round(g / s.float().unsqueeze(-1)).clamp(-8, 7).to(torch.int8).flatten(-2)
    return pack_int4(q), s


def _fp8_round_trip(v: torch.Tensor) -> torch.Tensor:
    s = v.float().abs().amax(-1, keepdim=True).clamp_min(1e-4) / 448.0
    return (v.float() / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s


def _local_ids(ids: torch.Tensor, expert_map: Optional[torch.Tensor], E: int,
               expert_offset: int = 0) -> torch.Tensor:
    """Routed ids -> this rank's expert index, or E for a slot served elsewhere."""
    ids = ids.to(torch.int64) - expert_offset
    if expert_map is not None:
        ok = (ids >= 0) & (ids < expert_map.numel())
        ids = torch.where(ok, expert_map.to(torch.int64)[ids.clamp(0, expert_map.numel() - 1)], -1)
    return torch.where((ids >= 0) & (ids < E), ids, E).to(torch.int32)


def w4afp8_moe_ref(x, w13, w2, s13, s2, topk_w, topk_ids, expert_map=None, swiglu_limit=None,
                   expert_offset=0, shared=None):
    """fp32 restatement of the op (CPU)."""
    T, H = x.shape
    E = w13.shape[0]
    gu, dn = dequant_w4(w13, s13), dequant_w4(w2, s2)
    ids = _local_ids(topk_ids, expert_map, E, expert_offset)
    xq = _fp8_round_trip(x)
    out = torch.zeros(T, H, dtype=torch.float32)
    for e in range(E):
        tok, slot = torch.nonzero(ids == e, as_tuple=True)
        if tok.numel() == 0:
            continue
        p = (xq[tok] @ gu[e].t()).to(torch.bfloat16).float()
        g, u = p.chunk(2, dim=-1)
        if swiglu_limit is not None:
            g, u = g.clamp(max=swiglu_limit), u.clamp(-swiglu_limit, swiglu_limit)
        h = (F.silu(g) * u).to(torch.bfloat16)
        y = (_fp8_round_trip(h) @ dn[e].t()).to(torch.bfloat16).float()
        out.index_add_(0, tok, y * topk_w[tok, slot].float().unsqueeze(1))
    if shared is not None:
        out += shared.float()
    return out.to(x.dtype)


def w4afp8_moe(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, s13: torch.Tensor,
               s2: torch.Tensor, topk_w: torch.Tensor, topk_ids: torch.Tensor,
               expert_map: Optional[torch.Tensor] = None, swiglu_limit: Optional[float] = None,
               out: Optional[torch.Tensor] = None, expert_offset: int = 0,
               shared: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x bf16 [T, H] -> [T, H] = sum_j topk_w[:, j] * expert_{topk_ids[:, j]}(x) (+ shared).
    ``expert_map`` maps a global expert id to this rank's index (-1: another rank's expert);
    without one, this rank holds experts [expert_offset, expert_offset + E)."""
    T, H = x.shape
    E, I2, Hp = w13.shape
    I = I2 // 2
    if Hp * 2 != H or H % 128 or I % 128:
        raise ValueError("W4AFP8 needs packed int4 [E, 2I, H/2] with H and I multiples of 128")
    if w2.shape != (E, H, I // 2):
        raise ValueError("W4AFP8 down weight shape does not match gate/up")
    if s13.shape != (E, I2, H // 128) or s2.shape != (E, H, I // 128):
        raise ValueError("W4AFP8 scales must be [E, N, K/128]")
    if out is None:
        out = torch.empty(T, H, dtype=x.dtype, device=x.device)
    if T == 0:
        return out
    if not x.is_cuda:
        out.copy_(w4afp8_moe_ref(x, w13, w2, s13, s2, topk_w, topk_ids, expert_map, swiglu_limit,
                                 expert_offset, shared))
        return out
    mod = _ext.require()
    ops = torch.ops.b200
    dev = x.device
    k = topk_ids.shape[1]
    limit = float(swiglu_limit) if swiglu_limit is not None else 0.0
    ids = _local_ids(topk_ids, expert_map, E, expert_offset).contiguous()
    max_rows = int(mod.moe_max_rows(T * k, E))
    sorted_ids = torch.empty(max_rows, dtype=torch.int32, device=dev)
    tile_expert = torch.empty(max_rows // 128, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    pos = torch.empty(T, k, dtype=torch.int32, device=dev)
    num_tiles = torch.empty(1, dtype=torch.int32, device=dev)
    ops.moe_align(ids, E, sorted_ids, tile_expert, offsets, pos, num_tiles, 0)
    xq = torch.empty_like(x)
    ops.row_fp8_qdq(xq, x.contiguous(), False, 0.0, None)
    xs = torch.empty(max_rows, H, dtype=x.dtype, device=dev)
    ops.moe_gather(xq, sorted_ids, num_tiles, k, xs)
    wgu = torch.empty(E * I2, H, dtype=torch.bfloat16, device=dev)
    ops.w4_dequant(wgu, w13.contiguous(), s13.contiguous(), offsets)
    hg = torch.empty(max_rows, I2, dtype=torch.bfloat16, device=dev)
    ops.gemm_grouped_bf16(xs, wgu, hg, tile_expert, num_tiles, E, 0, 0)
    del wgu
    h = torch.empty(max_rows, I, dtype=torch.bfloat16, device=dev)
    ops.row_fp8_qdq(h, hg, True, limit, num_tiles)
    wd = torch.empty(E * H, I, dtype=torch.bfloat16, device=dev)
    ops.w4_dequant(wd, w2.contiguous(), s2.contiguous(), offsets)
    y = torch.empty(max_rows, H, dtype=torch.bfloat16, device=dev)
    ops.gemm_grouped_bf16(h, wd, y, tile_expert, num_tiles, E, 0, 0)
    ops.moe_combine(y, pos, topk_w.float().contiguous(), shared, out, None)
    return out
