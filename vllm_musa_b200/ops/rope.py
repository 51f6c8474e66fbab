"""Fused QK-RMSNorm + RoPE + paged KV insert (reference: vllm_musa/jit_kernel/csrc/norm/
qk_mrope.mu:168-1311, vllm_musa/model_executor/layers/rotary_embedding/base.py:8-35,
csrc/musa/cache_kernels.mu:16)."""
from __future__ import annotations

import math

import torch

from . import _bounds, _ext


def build_cos_sin_cache(rot_dim: int, max_pos: int, theta: float, device=None,
                        scaling: dict | None = None) -> torch.Tensor:
    """[max_pos, rot_dim] fp32 = [cos(f) | sin(f)] for f in rot_dim/2 frequencies.

    ``scaling`` supports the Llama-3 long-context frequency scaling
    (``{"rope_type": "llama3", "factor", "low_freq_factor", "high_freq_factor",
    "original_max_position_embeddings"}``) and linear scaling (``{"rope_type": "linear"}``).
    """
    inv = 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim))
    if scaling:
        kind = scaling.get("rope_type", scaling.get("type"))
        if kind == "llama3":
            factor = scaling["factor"]
            lo, hi = scaling.get("low_freq_factor", 1.0), scaling.get("high_freq_factor", 4.0)
            old = scaling.get("original_max_position_embeddings", 8192)
            wl = 2 * math.pi / inv
            lo_wl, hi_wl = old / lo, old / hi
            smooth = (old / wl - lo) / (hi - lo)
            scaled = torch.where(wl > lo_wl, inv / factor, inv)
            mid = (wl <= lo_wl) & (wl >= hi_wl)
            inv = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
        elif kind == "linear":
            inv = inv / scaling["factor"]
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    cs = torch.cat([f.cos(), f.sin()], dim=-1).float()
    return cs.to(device) if device is not None else cs


def _mrope_cos_sin(cos_sin: torch.Tensor, positions: torch.Tensor, rot_dim: int,
                   section: list, interleaved: bool) -> torch.Tensor:
    """[T, rot_dim] cos | sin where frequency f uses position row comp(f) of [3, T]."""
    half = rot_dim // 2
    f = torch.arange(half)
    if interleaved:
        comp = torch.zeros(half, dtype=torch.long)
        comp[(f % 3 == 1) & (f < 3 * section[1])] = 1
        comp[(f % 3 == 2) & (f < 3 * section[2])] = 2
    else:
        assert sum(section) == half, "M-RoPE sections must cover rot_dim / 2 frequencies"
        comp = torch.repeat_interleave(torch.arange(3), torch.tensor(section))
    cs = cos_sin[positions.long()]                       # [3, T, rot_dim]
    idx = torch.cat([comp, comp])                         # cos half then sin half
    cols = torch.arange(rot_dim)
    return cs[idx.to(cs.device), :, cols.to(cs.device)].transpose(0, 1).contiguous()


def _rotate_ref(x: torch.Tensor, cs: torch.Tensor, rot_dim: int, neox: bool) -> torch.Tensor:
    # x [T, H, D] fp32; cs [T, rot_dim]
    half = rot_dim // 2
    cos, sin = cs[:, None, :half], cs[:, None, half:]
    xr, xp = x[..., :rot_dim], x[..., rot_dim:]
    if neox:
        x1, x2 = xr[..., :half], xr[..., half:]
        out = torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)
    else:
        x1, x2 = xr[..., 0::2], xr[..., 1::2]
        out = torch.stack([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).flatten(-2)
    return torch.cat([out, xp], -1)


def rope_kv(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
            k_cache: torch.Tensor | None, v_cache: torch.Tensor | None,
            slot_mapping: torch.Tensor, num_q_heads: int, num_kv_heads: int, rot_dim: int,
            neox: bool = True, q_norm_w: torch.Tensor | None = None,
            k_norm_w: torch.Tensor | None = None, eps: float = 1e-6,
            write_k: bool = False, head_dim: int | None = None,
            mrope_section: list | None = None, mrope_interleaved: bool = False) -> None:
    """In place on ``qkv`` [T, (Hq+2Hkv)*D]: q <- rope(norm(q)); cache[slot] <- rope(norm(k)), v.

    Caches are [num_blocks, Hkv, block_size, D]; slot = block * block_size + offset; slot < 0
    skips the write.  Without caches (``write_k``) q and k are only rotated in place.
    M-RoPE (``mrope_section`` = [temporal, height, width] frequency counts): positions are
    [3, >= T] and each rotary frequency takes its position from the row its section names
    (``mrope_interleaved``: frequencies assigned round-robin, Qwen3-VL layout).
    Reference: vllm_musa/jit_kernel/csrc/norm/qk_mrope.mu:168-1311.
    """
    T = qkv.shape[0]
    if T == 0:
        return
    if head_dim is None:
        head_dim = k_cache.shape[-1] if k_cache is not None else qkv.shape[1] // (
            num_q_heads + 2 * num_kv_heads)
    if _bounds.enabled():
        if k_cache is not None:
            _bounds.check("rope_kv", "slot_mapping", slot_mapping,
                          k_cache.shape[0] * k_cache.shape[2], skip_negative=True)
        _bounds.check("rope_kv", "positions", positions, cos_sin.shape[0])
    if qkv.is_cuda:
        _ext.ops().rope_kv(qkv, positions, cos_sin, q_norm_w, k_norm_w, k_cache, v_cache,
                           slot_mapping, num_q_heads, num_kv_heads, rot_dim, neox, eps, head_dim,
                           list(mrope_section) if mrope_section is not None else None,
                           mrope_interleaved)
        return
    D = head_dim
    Hq, Hkv = num_q_heads, num_kv_heads
    q = qkv[:, :Hq * D].view(T, Hq, D).float()
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D).float()
    v = qkv[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D].view(T, Hkv, D)
    if q_norm_w is not None:
        q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + eps) * q_norm_w.float()
    if k_norm_w is not None:
        k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + eps) * k_norm_w.float()
    if rot_dim > 0:
        if mrope_section is not None:
            cs = _mrope_cos_sin(cos_sin, positions[:, :T], rot_dim, mrope_section,
                                mrope_interleaved)
        else:
            cs = cos_sin[positions.long()]
        q = _rotate_ref(q, cs, rot_dim, neox)
        k = _rotate_ref(k, cs, rot_dim, neox)
    qkv[:, :Hq * D] = q.reshape(T, Hq * D).to(qkv.dtype)
    if k_cache is None:
        qkv[:, Hq * D:(Hq + Hkv) * D] = k.reshape(T, Hkv * D).to(qkv.dtype)
        return
    bs = k_cache.shape[2]
    sl = slot_mapping.long()
    ok = sl >= 0
    blk, off = sl[ok] // bs, sl[ok] % bs
    k_cache[blk, :, off] = k[ok].to(k_cache.dtype)
    v_cache[blk, :, off] = v[ok].to(v_cache.dtype)
