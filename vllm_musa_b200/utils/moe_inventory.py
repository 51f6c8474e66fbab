"""MoE shape inventory and dispatch counters.

Two observability aids for the routed-expert layers:

* ``dispatch_counts()`` — how many MoE layer calls took each path since the process started
  (``gemv``: per (token, slot) GEMVs; ``grouped``: align + gather + tcgen05 grouped GEMMs;
  ``fp8_grouped``: the block-FP8 grouped path; ``cpu``: the PyTorch reference).  Counted when
  the host issues the call, so a CUDA graph counts once, at capture, not per replay.  A served
  A/B that claims a path's win should see that path's count move.
* A JSON-lines inventory of the shapes MoE layers actually receive, written when
  ``B200_MOE_SHAPE_INVENTORY`` names a file: one record per eager call with at least
  ``B200_MOE_SHAPE_INVENTORY_MIN_TOKENS`` tokens, up to ``B200_MOE_SHAPE_INVENTORY_MAX_RECORDS``
  records per process, never during graph capture.  A record holds the token count, top-k,
  local / global expert counts, hidden and intermediate sizes, dtypes, the dispatch path taken
  and the routed-token histogram (per expert and per top-k slot).  The histogram is read back
  to the host, so the inventory synchronises the stream: it is for collecting tuning shapes,
  not for timed runs.

Reference counterpart: the DeepSeek-V4 MoE shape inventory and routed-token histogram
(vllm_musa/model_executor/layers/fused_moe/fused_moe.py:180-310) and the router activation
counter (vllm_musa/model_executor/layers/fused_moe/musa_router_gemm.py:112-135); the record
keys that describe a shape keep the reference's names so inventories from both can be merged.
"""
from __future__ import annotations

import json
import logging
import os
import threading
import time
from collections import Counter
from typing import Dict, Optional

import torch

from .. import envs

log = logging.getLogger("vllm_musa_b200")

_lock = threading.Lock()
_counts: Counter = Counter()
_records = 0
_warned = False


def dispatch_counts() -> Dict[str, int]:
    """Calls per MoE dispatch path since start (or the last ``reset()``)."""
    with _lock:
        return dict(_counts)


def reset() -> None:
    global _records, _warned
    with _lock:
        _counts.clear()
        _records = 0
        _warned = False


def routed_histogram(ids: torch.Tensor, num_experts: int, expert_offset: int = 0) -> dict:
    """Histogram of routed (token, slot) pairs over this rank's experts
    [expert_offset, expert_offset + num_experts): overall and per top-k slot; ids outside the
    range (other ranks' experts, or -1 padding) are counted as ``outside``."""
    local = ids.detach().to("cpu", torch.int64) - expert_offset
    inside = (local >= 0) & (local < num_experts)
    hist = torch.bincount(local[inside], minlength=num_experts).tolist()
    per_slot = [torch.bincount(local[:, j][inside[:, j]], minlength=num_experts).tolist()
                for j in range(local.shape[1])]
    used = [c for c in hist if c]
    return {"histogram": hist, "slot_histograms": per_slot,
            "outside_count": int((~inside).sum()), "nonzero_experts": len(used),
            "max_routes_per_expert": max(used) if used else 0,
            "min_routes_per_nonzero_expert": min(used) if used else 0}


def _capturing(x: torch.Tensor) -> bool:
    return x.is_cuda and torch.cuda.is_current_stream_capturing()


def note(path: str, x: torch.Tensor, ids: torch.Tensor, num_experts: int, intermediate: int,
         weight_dtype: torch.dtype, expert_offset: int = 0,
         global_num_experts: Optional[int] = None) -> None:
    """Count one MoE call on ``path`` and, when the inventory is on, append its record."""
    global _records, _warned
    with _lock:
        _counts[path] += 1
    dest = envs.get("B200_MOE_SHAPE_INVENTORY")
    if not dest or _capturing(x):
        return
    T = x.shape[0]
    if T < envs.get("B200_MOE_SHAPE_INVENTORY_MIN_TOKENS"):
        return
    with _lock:
        cap = envs.get("B200_MOE_SHAPE_INVENTORY_MAX_RECORDS")
        if 0 <= cap <= _records:
            return
        index = _records
        _records += 1
    try:
        rec = {"event": "moe_shape_inventory", "time": time.time(), "pid": os.getpid(),
               "record_index": index, "path": path, "num_tokens": T, "top_k": ids.shape[1],
               "num_local_experts": num_experts, "expert_offset": expert_offset,
               "global_num_experts": global_num_experts or num_experts,
               "hidden_size": x.shape[1], "w1_intermediate_size": 2 * intermediate,
               "w2_output_size": x.shape[1], "activation_dtype": str(x.dtype),
               "weight_dtype": str(weight_dtype),
               "routed_token_stats": routed_histogram(ids, num_experts, expert_offset)}
        d = os.path.dirname(dest)
        if d:
            os.makedirs(d, exist_ok=True)
        with _lock, open(dest, "a", encoding="utf-8") as f:
            f.write(json.dumps(rec, sort_keys=True) + "\n")
    except Exception as e:  # the inventory never fails a forward pass
        if not _warned:
            _warned = True
            log.warning("MoE shape inventory not written: %s", e)
