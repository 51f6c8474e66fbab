"""Paged attention over the [num_blocks, Hkv, block_size, D] KV cache.

CUDA: csrc/attention/paged_attention.cu (TMA page loads, split-KV decode, chunked-prefill
kernel).  CPU: a direct PyTorch restatement used by the tiny CPU configuration and as the
numerics oracle (reference: the MATE FA3 varlen path behind
vllm_musa/v1/attention/backends/flash_attn.py:1186-1537).
"""
from __future__ import annotations

import torch

from . import _bounds, _ext

_WS: dict = {}


def decode_workspace(device: torch.device, B: int, Hq: int, D: int, splits: int):
    """Split-KV partial buffers (fp32 O and log-sum-exp), reused across calls."""
    need_o, need_l = B * Hq * splits * D, B * Hq * splits
    key = (device.type, device.index)
    ws = _WS.get(key)
    if ws is None or ws[0].numel() < need_o or ws[1].numel() < need_l:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("decode workspace must be reserved before CUDA-graph capture")
        ws = (torch.empty(max(need_o, 1 << 16), dtype=torch.float32, device=device),
              torch.empty(max(need_l, 1 << 12), dtype=torch.float32, device=device))
        _WS[key] = ws
    return ws


def num_decode_splits(B: int, Hkv: int, max_seq_len: int) -> int:
    return int(_ext.require().decode_num_splits(B, Hkv, max_seq_len))


def _gather_kv(cache: torch.Tensor, table: torch.Tensor, n: int) -> torch.Tensor:
    # -> [n, Hkv, D]
    bs = cache.shape[2]
    nb = (n + bs - 1) // bs
    blocks = cache[table[:nb].long()]            # [nb, Hkv, bs, D]
    return blocks.permute(0, 2, 1, 3).reshape(nb * bs, cache.shape[1], cache.shape[3])[:n]


def _attend_ref(q, k, v, q_pos, scale, window, sinks=None, causal=True, allowed=None):
    # q [Tq, Hq, D], k/v [S, Hkv, D]; causal by absolute position.  A sink is an extra softmax
    # column per head (logit sinks[h]) that carries no value.
    Hq, Hkv = q.shape[1], k.shape[1]
    G = Hq // Hkv
    k = k.float().repeat_interleave(G, dim=1)
    v = v.float().repeat_interleave(G, dim=1)
    s = torch.einsum("thd,shd->hts", q.float(), k) * scale
    if allowed is not None:  # [Tq, S] visibility (tree attention)
        s = s.masked_fill(~allowed[None], float("-inf"))
    elif causal:
        kv_pos = torch.arange(k.shape[0])
        mask = kv_pos[None, :] > q_pos[:, None]
        if window > 0:
            mask |= kv_pos[None, :] <= q_pos[:, None] - window
        s = s.masked_fill(mask[None], float("-inf"))
    if sinks is not None:
        col = sinks.float().cpu().view(Hq, 1, 1).expand(Hq, s.shape[1], 1)
        p = torch.softmax(torch.cat([s, col], dim=-1), dim=-1)[..., :-1]
    else:
        p = torch.softmax(s, dim=-1)
    return torch.einsum("hts,shd->thd", p, v)


def _check_tables(op, k_cache, block_tables, seq_lens) -> None:
    """Debug bounds: the pages a request's length reaches are cache blocks; the length fits the
    table's width."""
    bs = k_cache.shape[2]
    W = block_tables.shape[1]
    _bounds.check(op, "seq_lens", seq_lens, W * bs + 1)
    if seq_lens.numel():
        used = (torch.arange(W, device=block_tables.device)[None, :] * bs <
                seq_lens.to(block_tables.device).long()[:, None])
        _bounds.check(op, "block_tables", block_tables[used], k_cache.shape[0])


def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 block_tables: torch.Tensor, seq_lens: torch.Tensor, num_q_heads: int,
                 num_kv_heads: int, scale: float, max_seq_len: int,
                 out: torch.Tensor | None = None, num_splits: int | None = None,
                 sinks: torch.Tensor | None = None) -> torch.Tensor:
    """One query token per sequence.  q: [B, >= Hq*D] (row stride may exceed Hq*D).
    ``sinks`` fp32 [Hq]: per-head attention-sink logits (a softmax column without a value)."""
    B = q.shape[0]
    D = k_cache.shape[-1]
    Hq = num_q_heads
    if out is None:
        out = torch.empty(B, Hq * D, dtype=q.dtype, device=q.device)
    if B == 0:
        return out
    if _bounds.enabled():
        _check_tables("paged_decode", k_cache, block_tables[:B], seq_lens[:B])
    if q.is_cuda:
        if num_splits is None:
            num_splits = num_decode_splits(B, num_kv_heads, max_seq_len)
        ws_o = ws_l = None
        if num_splits > 1:
            ws_o, ws_l = decode_workspace(q.device, B, Hq, D, num_splits)
        _ext.ops().paged_decode(q, out, k_cache, v_cache, block_tables, seq_lens, Hq,
                                num_kv_heads, max_seq_len, scale, num_splits, ws_o, ws_l, sinks)
        return out
    for b in range(B):
        n = int(seq_lens[b])
        if n == 0:
            out[b].zero_()
            continue
        k = _gather_kv(k_cache, block_tables[b], n)
        v = _gather_kv(v_cache, block_tables[b], n)
        qb = q[b, :Hq * D].view(1, Hq, D)
        o = _attend_ref(qb, k, v, torch.tensor([n - 1]), scale, 0, sinks)
        out[b] = o.reshape(Hq * D).to(out.dtype)
    return out


def paged_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  cu_q: torch.Tensor, seq_lens: torch.Tensor, block_tables: torch.Tensor,
                  num_q_heads: int, num_kv_heads: int, scale: float, window: int = 0,
                  out: torch.Tensor | None = None,
                  tile_scratch: torch.Tensor | None = None,
                  sinks: torch.Tensor | None = None, causal: bool = True,
                  tree_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of each request's new tokens over its whole cached sequence
    (``causal=False``: every query sees the whole sequence, as encoders need).

    ``tree_mask`` int64 [T] (speculative token trees): bit j of row t lets query t see draft j
    of its request (its last q_len <= 64 tokens); the cached context stays visible.  A zero row
    is an ordinary causal row (prefill chunks and chains batched with a tree).

    q: [T, >= Hq*D] for the prefill tokens (request r owns rows cu_q[r]:cu_q[r+1]); the K/V
    of those tokens must already be in the cache.  ``sinks`` as in ``paged_decode``.
    """
    T = q.shape[0]
    D = k_cache.shape[-1]
    Hq = num_q_heads
    R = seq_lens.shape[0]
    if out is None:
        out = torch.empty(T, Hq * D, dtype=q.dtype, device=q.device)
    if T == 0 or R == 0:
        return out
    if _bounds.enabled():
        _check_tables("paged_prefill", k_cache, block_tables[:R], seq_lens[:R])
        _bounds.check("paged_prefill", "cu_q", cu_q[:R + 1], T + 1)
    if q.is_cuda:
        if tile_scratch is None:
            tile_scratch = torch.empty(R + 1, dtype=torch.int32, device=q.device)
        _ext.ops().paged_prefill(q, out, k_cache, v_cache, cu_q, seq_lens, block_tables,
                                 tile_scratch, Hq, num_kv_heads, scale, window, sinks, causal,
                                 tree_mask)
        return out
    cu = cu_q.tolist()
    for r in range(R):
        a, b = cu[r], cu[r + 1]
        if b == a:
            continue
        n = int(seq_lens[r])
        k = _gather_kv(k_cache, block_tables[r], n)
        v = _gather_kv(v_cache, block_tables[r], n)
        qr = q[a:b, :Hq * D].reshape(b - a, Hq, D)
        pos = torch.arange(n - (b - a), n)
        allowed = None
        if tree_mask is not None:
            ctx = n - (b - a)
            bits = tree_mask[a:b].cpu().view(-1, 1)
            j = torch.arange(n) - ctx
            allowed = (j[None, :] < 0) | ((j[None, :] < 64) & (j[None, :] >= 0) &
                                          (((bits >> j.clamp(0, 63)[None, :]) & 1) == 1))
            causal_rows = torch.arange(n)[None, :] <= pos[:, None]
            if window > 0:
                causal_rows &= torch.arange(n)[None, :] > pos[:, None] - window
            allowed = torch.where(bits == 0, causal_rows, allowed)
        o = _attend_ref(qr, k, v, pos, scale, window, sinks, causal, allowed)
        out[a:b] = o.reshape(b - a, Hq * D).to(out.dtype)
    return out


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor,
                     scale: float, causal: bool = False,
                     sinks: torch.Tensor | None = None) -> torch.Tensor:
    """Attention over packed variable-length sequences without a KV cache (vision / audio
    encoders): q [T, Hq, D], k/v [T, Hkv, D], sequence r owns rows cu_seqlens[r]:cu_seqlens[r+1].
    Returns [T, Hq, D].

    CUDA: K/V are laid into 64-token pages (each sequence starting on a page) and the paged
    prefill kernel runs with ``causal=False``; the page copy is one gather per tensor.
    Reference: vllm_musa/model_executor/layers/attention/mm_encoder_attention.py:14-170."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    cu = cu_seqlens.to(torch.int32)
    if T == 0:
        return torch.empty_like(q)
    if not q.is_cuda:
        out = torch.empty(T, Hq, D, dtype=q.dtype)
        c = cu.tolist()
        for r in range(len(c) - 1):
            a, b = c[r], c[r + 1]
            if b > a:
                pos = torch.arange(b - a)
                out[a:b] = _attend_ref(q[a:b], k[a:b], v[a:b], pos, scale, 0, sinks,
                                       causal).to(q.dtype)
        return out
    dev = q.device
    lens = (cu[1:] - cu[:-1]).long()
    R = lens.numel()
    pages = (lens + 63) // 64
    first = torch.cumsum(pages, 0) - pages                       # first page of each sequence
    n_pages = int(pages.sum())
    max_pages = int(pages.max())
    seq_of = torch.repeat_interleave(torch.arange(R, device=dev), lens, output_size=T)
    idx = torch.arange(T, device=dev) - cu[:-1].long()[seq_of]   # token index within its sequence
    page = first[seq_of] + idx // 64
    off = idx % 64
    kc = torch.zeros(n_pages, Hkv, 64, D, dtype=k.dtype, device=dev)
    vc = torch.zeros_like(kc)
    kc[page, :, off] = k
    vc[page, :, off] = v
    table = first[:, None] + torch.arange(max_pages, device=dev)[None, :]
    table = torch.minimum(table, torch.full_like(table, n_pages - 1)).to(torch.int32)
    out = paged_prefill(q.reshape(T, Hq * D), kc, vc, cu, lens.to(torch.int32), table, Hq, Hkv,
                        scale, sinks=sinks, causal=causal)
    return out.view(T, Hq, D)


def tree_ancestor_masks(parents: list) -> torch.Tensor:
    """Draft-token tree given as parent indices (-1: child of the last accepted token) -> int64
    [n] masks: bit j of row i is set when draft j is i or one of its ancestors."""
    n = len(parents)
    if n > 64:
        raise ValueError("tree attention supports at most 64 draft tokens per request")
    masks = [0] * n
    for i, par in enumerate(parents):
        if par >= i:
            raise ValueError("parents must precede their children")
        masks[i] = (1 << i) | (masks[par] if par >= 0 else 0)
    # int64 storage of the unsigned bit pattern
    return torch.tensor([m - (1 << 64) if m >= 1 << 63 else m for m in masks], dtype=torch.int64)


def kv_insert(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
              v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Write key / value rows [T, Hkv, D] into the paged caches [num_blocks, Hkv, block_size,
    D] at ``slot_mapping`` (int64, slot = block * block_size + offset; < 0 skipped; only the
    first len(slot_mapping) rows are written)."""
    n = min(int(slot_mapping.numel()), key.shape[0])
    if n == 0:
        return
    _bounds.check("kv_insert", "slot_mapping", slot_mapping[:n],
                  k_cache.shape[0] * k_cache.shape[2], skip_negative=True)
    if key.is_cuda:
        _ext.ops().kv_insert(key, value, k_cache, v_cache, slot_mapping.to(torch.int64))
        return
    bs = k_cache.shape[2]
    s = slot_mapping[:n].long()
    keep = s >= 0
    s = s[keep]
    blk, off = s // bs, s % bs
    k_cache[blk, :, off, :] = key[:n][keep].to(k_cache.dtype)
    v_cache[blk, :, off, :] = value[:n][keep].to(v_cache.dtype)
