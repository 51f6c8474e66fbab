"""Embedding lookup and row gather."""
from __future__ import annotations

import torch

from . import _bounds, _ext


def embedding(ids: torch.Tensor, table: torch.Tensor, vocab_start: int = 0,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Rows of ``table`` for ``ids`` (int32); ids outside this shard's range give zeros."""
    T, H = ids.shape[0], table.shape[1]
    if out is None:
        out = torch.empty(T, H, dtype=table.dtype, device=table.device)
    _bounds.check("embedding", "ids", ids, 1 << 31)  # token ids are never negative
    if table.is_cuda:
        if T:
            _ext.ops().embedding(out, table, ids, vocab_start)
        return out
    local = ids.long() - vocab_start
    ok = (local >= 0) & (local < table.shape[0])
    out.zero_()
    out[ok] = table[local[ok]]
    return out


def gather_rows(x: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(idx.shape[0], x.shape[1], dtype=x.dtype, device=x.device)
    _bounds.check("gather_rows", "idx", idx, x.shape[0])
    if x.is_cuda:
        if idx.shape[0]:
            _ext.ops().gather_rows(out, x, idx)
        return out
    out.copy_(x[idx.long()])
    return out
