"""Measured tuning tables (JSON, validated on load).

Reference counterpart: vllm_musa/tuning/__init__.py:24-59 (``tuning.load`` with schema checks)
and its offline-measured fp8_block_splitk.json.  Here the tables are measured on B200 by the
sweep scripts under benchmarks/ and consulted at run time by the kernel wrappers.

Table ``gemm_bf16``: {"device": str, "entries": [{"n": N, "k": K, "m": M, "bn": BN,
"splits": S, "mt": MT, "us": t}, ...]}: the fastest plan measured for each (N, K) at each M
bucket (BN a multiple of 16 up to 256; MT = 128-row tiles per CTA (1 or 2), 3 = one 128-row tile
per CTA with the K splits reduced inside a thread-block cluster through distributed shared
memory, or 4 = a 2-CTA cluster on a 256-row tile with cta_group::2 MMAs).
"""
from __future__ import annotations

import bisect
import json
import os
from functools import lru_cache
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))

_SCHEMAS = {
    "gemm_bf16": {"entry_keys": {"n", "k", "m", "bn", "splits"},
                  "bn": set(range(16, 257, 16))},
}


class TuningTableError(ValueError):
    pass


def path_of(name: str) -> str:
    return os.environ.get(f"B200_TUNING_{name.upper()}", os.path.join(HERE, f"{name}.json"))


def validate(name: str, table: dict) -> dict:
    sch = _SCHEMAS.get(name)
    if sch is None:
        raise TuningTableError(f"unknown tuning table {name!r}")
    if not isinstance(table, dict) or not isinstance(table.get("entries"), list):
        raise TuningTableError(f"{name}: expected an object with an 'entries' list")
    for e in table["entries"]:
        missing = sch["entry_keys"] - set(e)
        if missing:
            raise TuningTableError(f"{name}: entry {e} lacks {sorted(missing)}")
        if e["bn"] not in sch["bn"] or int(e["splits"]) < 1:
            raise TuningTableError(f"{name}: bad plan in entry {e}")
    return table


@lru_cache(maxsize=None)
def load(name: str) -> Optional[dict]:
    p = path_of(name)
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return validate(name, json.load(f))


class GemmPlanTable:
    """(N, K, M) -> plan: exact (N, K) match, smallest measured M bucket >= M.  Entries with
    ``"swap": 1`` are plans of the swapped problem (C^T = W X^T, tokens in the MMA's N)."""

    def __init__(self, table: Optional[dict]):
        self.by_nk = {}
        for e in (table or {}).get("entries", []):
            key = (int(e["n"]), int(e["k"]), int(e.get("swap", 0)))
            self.by_nk.setdefault(key, []).append(
                (int(e["m"]), int(e["bn"]), int(e["splits"]), int(e.get("mt", 1)),
                 float(e.get("us", 0.0))))
        for v in self.by_nk.values():
            v.sort()

    def entry(self, M: int, N: int, K: int, swap: bool = False):
        rows = self.by_nk.get((N, K, int(swap)))
        if not rows:
            return None
        i = bisect.bisect_left([r[0] for r in rows], M)
        if i == len(rows):
            return None  # larger than anything measured: cost model decides
        return rows[i]

    def lookup(self, M: int, N: int, K: int):
        e = self.entry(M, N, K)
        return None if e is None else e[1:4]

    def swap_plan(self, M: int, N: int, K: int):
        """(bn, splits, mt) of the swapped problem when it was measured faster, else None."""
        s, d = self.entry(M, N, K, True), self.entry(M, N, K, False)
        if s is None or (d is not None and d[0] == s[0] and d[4] <= s[4]):
            return None
        return s[1:4]


@lru_cache(maxsize=None)
def gemm_table() -> GemmPlanTable:
    if os.environ.get("B200_DISABLE_TUNING", "0") == "1":
        return GemmPlanTable(None)
    return GemmPlanTable(load("gemm_bf16"))
