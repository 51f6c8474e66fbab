"""Multi-head latent attention (DeepSeek-V2/V3/V3.2) and the V3.2 lightning indexer.

CUDA: csrc/attention/mla.cu.  CPU: the same math in PyTorch (per-token loops), which is also
the numerics oracle of the kernel tests.

Latent cache: [num_blocks, block_size, 576] = RMSNorm(c_kv) (512) | RoPE(k_pe) (64).
Index cache:  [num_blocks, block_size, 128] = RoPE(LayerNorm(k_idx)).
RoPE of the latent path is the interleaved (GPT-J) form; the indexer uses NeoX halves.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from . import _bounds, _ext

LAT, PE = 512, 64


def choose_splits(groups: int, max_keys: int, sms: int = 148) -> int:
    """KV splits for `groups` (query token x 16-head group) CTAs: one CTA per SM, so minimise
    whole waves per unit of work (ceil(groups * s / sms) / s) plus a small per-split merge cost,
    keeping at least 256 keys per split."""
    best, best_cost = 1, None
    for s in range(1, 17):
        if s > 1 and max_keys // s < 256:
            break
        cost = -(-groups * s // sms) / s + 0.005 * s
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = s, cost
    return best


def _rope_gptj(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., 64] rotated in interleaved pairs (2i, 2i+1) with frequency i."""
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * cos - x1 * sin
    out[..., 1::2] = x1 * cos + x0 * sin
    return out


def _rope_neox(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    x0, x1 = x[..., :h], x[..., h:]
    return torch.cat([x0 * cos - x1 * sin, x1 * cos + x0 * sin], -1)


def mla_prep(q: torch.Tensor, kv: torch.Tensor, kv_norm_w: torch.Tensor, eps: float,
             positions: torch.Tensor, cos_sin: torch.Tensor, cache: torch.Tensor,
             slot_mapping: torch.Tensor, num_heads: int) -> None:
    """In place: RoPE on q's 64 rope dims of every head (q [T, H*192] = per head nope 128 |
    rope 64); cache[slot] = RMSNorm(kv[:, :512]) * w | RoPE(kv[:, 512:576])."""
    T = q.shape[0]
    if T == 0:
        return
    if q.is_cuda:
        _ext.ops().mla_prep(q, kv, kv_norm_w, eps, positions, cos_sin, cache, slot_mapping,
                            num_heads)
        return
    cs = cos_sin[positions.long()]
    cos, sin = cs[:, :PE // 2], cs[:, PE // 2:]
    qv = q.view(T, num_heads, 192)
    qv[..., 128:] = _rope_gptj(qv[..., 128:].float(), cos[:, None], sin[:, None]).to(q.dtype)
    c = kv[:, :LAT].float()
    c = c * torch.rsqrt(c.pow(2).mean(-1, keepdim=True) + eps) * kv_norm_w.float()
    pe = _rope_gptj(kv[:, LAT:LAT + PE].float(), cos, sin)
    rows = torch.cat([c, pe], -1).to(cache.dtype)
    flat = cache.view(-1, LAT + PE)
    ok = slot_mapping >= 0
    flat[slot_mapping[ok].long()] = rows[ok]


def _req_of_tokens(cu_q: torch.Tensor, seq_lens: torch.Tensor):
    """Per query token: (request, causal prefix length)."""
    cu = cu_q.tolist()
    out = []
    for r in range(len(cu) - 1):
        L = cu[r + 1] - cu[r]
        base = int(seq_lens[r]) - L
        for i in range(L):
            out.append((r, base + i + 1))
    return out


def _gather_rows(cache: torch.Tensor, bt_row: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    bs = cache.shape[1]
    slots = bt_row[(pos // bs).long()].long() * bs + (pos % bs).long()
    return cache.reshape(-1, cache.shape[-1])[slots]


def dcp_local_count(count: int, dcp: tuple) -> int:
    """Tokens p < count with p % size == rank (those this decode-context-parallel rank holds)."""
    size, rank = dcp
    return (count - rank + size - 1) // size if count > rank else 0


def mla_attention(q_lat: torch.Tensor, q_pe: torch.Tensor, cache: torch.Tensor,
                  block_tables: torch.Tensor, cu_q: torch.Tensor, seq_lens: torch.Tensor,
                  indices: Optional[torch.Tensor], out: torch.Tensor, scale: float,
                  splits: int = 1, ws: Optional[tuple] = None, dcp: tuple = (1, 0),
                  lse_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Absorbed MLA: q_lat [T, H, 512], q_pe [T, H, 64] (views with any token / head stride)
    -> out [T, H, 512] = softmax(q . [c_kv | k_pe]^T * scale) . c_kv over the causal prefix
    (indices None) or the listed token positions (indices [T, topk], -1 = unused).

    ``dcp`` = (size, rank): decode context parallelism, dense mode only -- this rank's cache
    holds the tokens p with p % size == rank at local index p // size, and the attention runs
    over those.  ``lse_out`` [T, H] fp32 receives log2(sum exp2(score * scale * log2 e)) of the
    keys attended (the weight of this partial in a cross-rank combine)."""
    T = q_lat.shape[0]
    if T == 0:
        return out
    if _bounds.enabled():
        bs = cache.shape[1] if cache.dim() == 3 else cache.shape[-2]
        R = seq_lens.shape[0]
        W = block_tables.shape[1]
        _bounds.check("mla_attention", "seq_lens", seq_lens, W * bs * max(1, dcp[0]) + 1)
        _bounds.check("mla_attention", "block_tables", block_tables[:R], cache.shape[0])
        if indices is not None:
            _bounds.check("mla_attention", "indices", indices, int(seq_lens.max()) + 1,
                          skip_negative=True)
    if q_lat.is_cuda:
        wo, wl = ws if ws is not None else (None, None)
        _ext.ops().mla_attention(q_lat, q_pe, cache, block_tables, cu_q, seq_lens, indices, out,
                                 scale, splits, wo, wl, dcp[0], dcp[1], lse_out)
        return out
    assert dcp[0] == 1 or indices is None, "decode context parallelism: dense mode only"
    for t, (r, count) in enumerate(_req_of_tokens(cu_q, seq_lens)):
        if dcp[0] > 1:
            count = dcp_local_count(count, dcp)
        if indices is None:
            pos = torch.arange(count)
        else:
            pos = indices[t][:min(indices.shape[1], count)]
            pos = pos[(pos >= 0) & (pos < count)]
        if pos.numel() == 0:
            out[t] = 0
            if lse_out is not None:
                lse_out[t] = float("-inf")
            continue
        kv = _gather_rows(cache, block_tables[r], pos).float()  # [n, 576]
        q = torch.cat([q_lat[t].float(), q_pe[t].float()], -1)  # [H, 576]
        sc = q @ kv.t() * scale
        p = torch.softmax(sc, -1)
        out[t] = (p @ kv[:, :LAT]).to(out.dtype)
        if lse_out is not None:
            lse_out[t] = torch.logsumexp(sc, -1) / math.log(2.0)
    return out


def dcp_combine(out: torch.Tensor, lse: torch.Tensor, comm) -> torch.Tensor:
    """Cross-rank combine of decode-context-parallel partials: every rank holds out [T, H, C]
    and lse [T, H] (log2 domain) for ALL heads over its token shard.  The log-sum-exp values
    are all-gathered, each rank scales its partial by its softmax weight, and a reduce-scatter
    over heads sums the weighted partials and leaves rank r its H / world heads.
    Reference: vllm_musa/v1/attention/backends/flash_attn.py:179-237 (LSE-corrected
    reduce-scatter), :1593-1726 (DCP attention)."""
    world = comm.world
    T, H, C = out.shape
    lses = comm.all_gather(lse.unsqueeze(0), dim=0)            # [world, T, H]
    m = lses.max(0).values
    m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    wts = torch.exp2(lses - m)                                 # [world, T, H]
    wsum = wts.sum(0)
    mine = torch.where(wsum > 0, wts[comm.rank] / wsum.clamp_min(1e-30), torch.zeros_like(wsum))
    part = (out.float() * mine.unsqueeze(-1))                  # [T, H, C]
    return comm.reduce_scatter(part, dim=1).to(out.dtype)      # [T, H / world, C]


def indexer_k_prep(k: torch.Tensor, ln_w: torch.Tensor, ln_b: torch.Tensor, eps: float,
                   positions: torch.Tensor, cos_sin: torch.Tensor, cache: torch.Tensor,
                   slot_mapping: torch.Tensor) -> None:
    T = k.shape[0]
    if T == 0:
        return
    if k.is_cuda:
        _ext.ops().indexer_k_prep(k, ln_w, ln_b, eps, positions, cos_sin, cache, slot_mapping)
        return
    x = F.layer_norm(k[:, :128].float(), (128,), ln_w.float(), ln_b.float(), eps)
    cs = cos_sin[positions.long()]
    x = torch.cat([_rope_neox(x[:, :PE], cs[:, :PE // 2], cs[:, PE // 2:]), x[:, PE:]], -1)
    flat = cache.view(-1, 128)
    ok = slot_mapping >= 0
    flat[slot_mapping[ok].long()] = x[ok].to(cache.dtype)


def indexer_scores(q: torch.Tensor, w: torch.Tensor, cache: torch.Tensor,
                   block_tables: torch.Tensor, cu_q: torch.Tensor, seq_lens: torch.Tensor,
                   scores: torch.Tensor) -> torch.Tensor:
    """scores[t, j] = sum_h w[t, h] * relu(q[t, h] . k[j]) for j < prefix length, else -inf.
    q [T, 64*128], w [T, 64] fp32, scores [T, L] fp32."""
    T = q.shape[0]
    if T == 0:
        return scores
    if q.is_cuda:
        _ext.ops().indexer_scores(q, w, cache, block_tables, cu_q, seq_lens, scores)
        return scores
    scores.fill_(float("-inf"))
    for t, (r, count) in enumerate(_req_of_tokens(cu_q, seq_lens)):
        n = min(count, scores.shape[1])
        k = _gather_rows(cache, block_tables[r], torch.arange(n)).float()  # [n, 128]
        s = torch.relu(q[t].float().view(64, 128) @ k.t())  # [64, n]
        scores[t, :n] = (w[t, :64].float().unsqueeze(1) * s).sum(0)
    return scores


def topk_indices(scores: torch.Tensor, cu_q: torch.Tensor, seq_lens: torch.Tensor,
                 k: int) -> torch.Tensor:
    """[T, k] int32 positions of each row's k largest scores among its prefix (all of them,
    in order, then -1, when the prefix is not longer than k).  Order within a row is free."""
    T = scores.shape[0]
    out = torch.empty(T, k, dtype=torch.int32, device=scores.device)
    if T == 0:
        return out
    if scores.is_cuda:
        _ext.ops().mla_topk(scores, cu_q, seq_lens, out)
        return out
    out.fill_(-1)
    for t, (r, count) in enumerate(_req_of_tokens(cu_q, seq_lens)):
        if count <= k:
            out[t, :count] = torch.arange(count, dtype=torch.int32)
        else:
            out[t] = scores[t, :count].topk(k).indices.to(torch.int32)
    return out
