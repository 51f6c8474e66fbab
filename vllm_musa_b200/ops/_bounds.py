"""Debug bounds checks at the kernel boundary (``B200_DEBUG_BOUNDS=1``).

The kernels index caches and tables through device-resident index tensors (KV slots, block
tables, token ids, row indices).  With the flag on, every op wrapper that passes such a tensor
first checks it against the bound the kernel assumes and raises ``IndexError`` naming the op,
the tensor and the first offending value -- before any kernel touches memory, so a bad index is
a Python error instead of a device fault.  The checks synchronise with the device (they read a
reduction back), which is why they are off unless asked for; off, every call is one branch.
TMA-fed lookups (the paged-attention page tables) are bounds-checked by the TMA unit itself
(out-of-range boxes read zeros) and are checked here as well.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

_ON = os.environ.get("B200_DEBUG_BOUNDS", "0") == "1"


def enabled() -> bool:
    return _ON


def set_enabled(on: bool) -> None:
    """Turn the checks on or off for this process (tests, debugging sessions)."""
    global _ON
    _ON = bool(on)


def check(op: str, name: str, idx: Optional[torch.Tensor], upper: int, lower: int = 0,
          skip_negative: bool = False) -> None:
    """Every element of ``idx`` must lie in [lower, upper) (``skip_negative``: values < 0 are
    "no entry" markers and pass)."""
    if not _ON or idx is None or idx.numel() == 0:
        return
    v = idx.reshape(-1).long()
    if skip_negative:
        v = v[v >= 0]
        if v.numel() == 0:
            return
    lo, hi = int(v.min()), int(v.max())
    if lo < lower or hi >= upper:
        bad = lo if lo < lower else hi
        raise IndexError(f"{op}: {name} holds {bad}, outside [{lower}, {upper})")
