"""Multi-LoRA serving for the dense decoders (vLLM's ``LoRARequest`` surface).

Adapters (PEFT format: ``adapter_config.json`` with ``r`` / ``lora_alpha`` / target modules, and
``adapter_model.safetensors`` with ``...layers.{i}.{self_attn,mlp}.{q,k,v,o,gate,up,down}_proj.
lora_{A,B}.weight``) are loaded into a fixed number of device slots; the requests of one batch
may use different adapters or none.  For every target module of every layer the slots hold

    A [slots, r_max, K_local]   B [slots, N_local, r_max]   (B scaled by lora_alpha / r)

sharded like the base weight under tensor parallelism: column-parallel modules (q, k, v,
gate, up) keep A whole and shard B's rows exactly as the base weight's rows; row-parallel
modules (o, down) shard A's columns and keep B whole, so each rank's B (A_shard x_shard) is a
partial sum that rides the layer's existing all-reduce.  Per step the tokens are grouped by
adapter slot and each group's delta  B (A x)  runs as two of this package's GEMMs (gathered
rows, then added back into the base GEMM's output before any epilogue or collective).  Steps
with adapters run eagerly (no decode graph) and the KV cache is not shared across adapters
(prefix caching is off with LoRA enabled).

Reference counterpart: upstream vLLM's LoRA layers and punica kernels, which the reference
serves unchanged; this is this package's own, for its engine.
"""
from __future__ import annotations

import json
import os
import re
from collections import OrderedDict
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from . import ops

_KEY = re.compile(r"layers\.(\d+)\.(self_attn|mlp)\.(q|k|v|o|gate|up|down)_proj\."
                  r"lora_(A|B)\.weight$")
MODULES = ("q", "k", "v", "o", "gate", "up", "down")


@dataclass(frozen=True)
class LoRARequest:
    """Which adapter a request runs with (vLLM's LoRARequest): a name, a positive integer id
    unique per adapter, and the adapter directory."""
    lora_name: str
    lora_int_id: int
    lora_path: str


@dataclass
class LoRABatch:
    """Token groups of one step: (slot, token indices on the device) per adapter in use."""
    groups: List[Tuple[int, torch.Tensor]]


def read_adapter(path: str) -> Tuple[dict, Dict[str, torch.Tensor]]:
    from safetensors.torch import load_file
    with open(os.path.join(path, "adapter_config.json")) as f:
        cfg = json.load(f)
    files = [n for n in os.listdir(path) if n.endswith(".safetensors")]
    if not files:
        raise FileNotFoundError(f"no adapter safetensors under {path}")
    tensors = {}
    for n in sorted(files):
        tensors.update(load_file(os.path.join(path, n)))
    return cfg, tensors


class LoRAManager:
    def __init__(self, model, max_loras: int = 4, max_lora_rank: int = 64):
        self.m = model
        self.slots = max_loras
        self.r_max = max_lora_rank
        self.by_id: "OrderedDict[int, int]" = OrderedDict()  # lora_int_id -> slot (LRU order)
        self.refs: Dict[int, int] = {}  # lora_int_id -> unfinished requests using it
        self.w: Dict[Tuple[int, str], Tuple[torch.Tensor, torch.Tensor]] = {}
        self._alloc()

    # ------------------------------------------------------------------ slots
    def _shapes(self, mod: str) -> Tuple[int, int, bool]:
        """(N_local, K_local, row_parallel) of a module on this rank."""
        m, cfg = self.m, self.m.cfg
        H, D = cfg.hidden_size, m.D
        if mod == "q":
            return m.hq * D, H, False
        if mod in ("k", "v"):
            return m.hkv * D, H, False
        if mod == "o":
            return H, m.hq * D, True
        if mod in ("gate", "up"):
            return m.I, H, False
        return H, m.I_pad, True  # down

    def _alloc(self) -> None:
        m = self.m
        for i in range(m.l0, m.l1):
            L = m.layers[i]
            for mod in MODULES:
                if mod in ("gate", "up", "down") and (L.gu_w is None or L.down_w is None):
                    continue  # MoE layers: adapters on attention only
                N, K, _ = self._shapes(mod)
                A = torch.zeros(self.slots, self.r_max, K, dtype=m.dtype, device=m.device)
                B = torch.zeros(self.slots, N, self.r_max, dtype=m.dtype, device=m.device)
                self.w[(i, mod)] = (A, B)

    def acquire(self, req: LoRARequest) -> int:
        """The slot holding ``req``'s adapter (one more request uses it), loading it into a
        free slot or over the least recently used adapter no unfinished request uses."""
        if req.lora_int_id <= 0:
            raise ValueError("lora_int_id must be a positive integer")
        s = self.by_id.get(req.lora_int_id)
        if s is None:
            used = set(self.by_id.values())
            free = [k for k in range(self.slots) if k not in used]
            if free:
                s = free[0]
            else:
                idle = [i for i in self.by_id if self.refs.get(i, 0) == 0]
                if not idle:
                    raise ValueError(f"more than max_loras={self.slots} adapters in use at once")
                s = self.by_id.pop(idle[0])
            self._load(s, req.lora_path)
            self.by_id[req.lora_int_id] = s
        self.by_id.move_to_end(req.lora_int_id)
        self.refs[req.lora_int_id] = self.refs.get(req.lora_int_id, 0) + 1
        return s

    def release(self, lora_int_id: int) -> None:
        """One request using the adapter finished (the adapter stays loaded until evicted)."""
        if self.refs.get(lora_int_id, 0) > 0:
            self.refs[lora_int_id] -= 1

    def _load(self, slot: int, path: str) -> None:
        cfg, tensors = read_adapter(path)
        r = int(cfg["r"])
        if r > self.r_max:
            raise ValueError(f"adapter rank {r} exceeds max_lora_rank {self.r_max}")
        scale = float(cfg.get("lora_alpha", r)) / r
        m = self.m
        for A, B in self.w.values():
            A[slot].zero_()
            B[slot].zero_()
        per = {}
        for name, t in tensors.items():
            mt = _KEY.search(name)
            if mt:
                per[(int(mt.group(1)), mt.group(3), mt.group(4))] = t
        D, rank, tp = m.D, m.rank, m.tp
        for (i, mod, ab), t in per.items():
            if ab != "A" or (i, mod) not in self.w:
                continue
            a, b = t.float(), per[(i, mod, "B")].float() * scale   # a [r, K], b [N, r]
            N, K, row_par = self._shapes(mod)
            if mod == "q":
                b = b[rank * N:(rank + 1) * N]
            elif mod in ("k", "v"):
                b = b[m.kv0 * D:(m.kv0 + m.hkv) * D]
            elif mod in ("gate", "up"):
                b = b[rank * N:(rank + 1) * N]
            elif mod == "o":
                a = a[:, rank * K:(rank + 1) * K]
            else:  # down: K_local = I_pad (zero columns past I)
                I = m.I
                a = a[:, rank * I:(rank + 1) * I]
                if K != I:
                    a = torch.cat([a, torch.zeros(a.shape[0], K - I)], 1)
            A, B = self.w[(i, mod)]
            A[slot, :r].copy_(a.to(A.dtype))
            B[slot, :, :r].copy_(b.to(B.dtype))

    # ------------------------------------------------------------------ forward
    def has(self, layer: int, mod: str) -> bool:
        return (layer, mod) in self.w

    def add_delta(self, layer: int, mod: str, x: torch.Tensor, out: torch.Tensor,
                  batch: LoRABatch) -> None:
        """out[t] += B[slot(t)] (A[slot(t)] x[t]) for every token with an adapter."""
        A, B = self.w[(layer, mod)]
        for slot, idx in batch.groups:
            xs = x.index_select(0, idx)
            h = ops.linear(xs.contiguous(), A[slot])
            d = ops.linear(h, B[slot])
            out.index_add_(0, idx, d.to(out.dtype))


def silu_mul_interleaved(gu: torch.Tensor, group: int = 8) -> torch.Tensor:
    """silu(gate) * up of a [T, 2 * I_pad] gate/up output interleaved in groups of ``group``
    rows (the layout of the fused gate/up weight) -> [T, I_pad]."""
    T = gu.shape[0]
    v = gu.view(T, -1, 2, group)
    return (torch.nn.functional.silu(v[:, :, 0].float()) * v[:, :, 1].float()) \
        .to(gu.dtype).reshape(T, -1)


def add_interleaved(gu: torch.Tensor, gate_d: torch.Tensor, up_d: torch.Tensor,
                    group: int = 8) -> None:
    """gu [T, 2 * I_pad] (gate/up interleaved in groups of ``group`` rows) += the [T, I_pad]
    gate and up deltas, in place."""
    T = gu.shape[0]
    v = gu.view(T, -1, 2, group)
    v[:, :, 0] += gate_d.view(T, -1, group)
    v[:, :, 1] += up_d.view(T, -1, group)
