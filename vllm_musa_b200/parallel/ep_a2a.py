"""Expert-parallel all-to-all MoE over NVSwitch peer memory (csrc/comm/ep_a2a.cu).

With tensor-parallel attention every rank holds all T tokens after the attention all-reduce.
Rank r routes only its token shard (rows [r*P, r*P+P), P = ceil(T / N) -- the same chunk the
two-shot all-reduce gives it), dispatches each token ONCE to every rank owning one of its
experts, runs its local experts on what it received, and returns each token's weighted expert
sum straight into block r of the token owner's all-reduce staging slot.  The owner's two-shot
all-reduce kernel (local-source mode) then sums the N blocks with the residual, normalises and
all-gathers the rows for the next attention layer.  Compared with the replicated-token expert
parallelism, the router and the dispatch touch T/N tokens per rank and the reduce-scatter half
of the all-reduce is replaced by the return stores.

One IPC buffer per rank:  [x: N*cap*H bf16][ids: N*cap*k i32][w: N*cap*k f32][tok: N*cap i32]
[cnt: N i32][flags: 8 u32], peers' addresses exchanged once over the CPU group (fail-closed).
"""
from __future__ import annotations

import logging
import os
from typing import Optional

import torch
import torch.distributed as dist

from ..ops import _ext

log = logging.getLogger("vllm_musa_b200")


def _align(n: int) -> int:
    return (n + 255) // 256 * 256


class EPAllToAll:
    def __init__(self, st, device: torch.device, ar, max_tokens: int, hidden: int, k: int,
                 e_local: int):
        self.mod = mod = _ext.require()
        self.world, self.rank = st.tp_size, st.tp_rank
        self.ar, self.H, self.k, self.E_local = ar, hidden, k, e_local
        self.cap = (max_tokens + self.world - 1) // self.world
        rows = self.world * self.cap
        self.off = {}
        o = 0
        for name, nbytes in (("x", rows * hidden * 2), ("ids", rows * k * 4), ("w", rows * k * 4),
                             ("tok", rows * 4), ("cnt", self.world * 4), ("flags", 8 * 4)):
            self.off[name] = o
            o += _align(nbytes)
        self.base = mod.ipc_malloc(o)
        handles = [None] * self.world
        dist.all_gather_object(handles, mod.ipc_handle(self.base), group=st.tp_cpu_group)
        self.opened, peers = [], []
        for p in range(self.world):
            if p == self.rank:
                peers.append(self.base)
            else:
                a = mod.ipc_open(handles[p])
                self.opened.append(a)
                peers.append(a)
        self.peers = peers
        self.send_cnt = torch.zeros(self.world, dtype=torch.int32, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        dev = device.index
        self.recv_x = mod.tensor_from_ptr(self.base + self.off["x"], [rows, hidden],
                                          torch.bfloat16, dev)
        self.recv_ids = mod.tensor_from_ptr(self.base + self.off["ids"], [rows, k], torch.int32, dev)
        self.recv_w = mod.tensor_from_ptr(self.base + self.off["w"], [rows, k], torch.float32, dev)

    def _ptrs(self) -> list:
        per = lambda name: [b + self.off[name] for b in self.peers]  # noqa: E731
        staging = self.ar._bufs[self.ar.parity][:self.world]
        return ([self.send_cnt.data_ptr(), self.epoch.data_ptr()] + per("x") + per("ids") +
                per("w") + per("tok") + per("cnt") + per("flags") + list(staging))

    def can_run(self, T: int) -> bool:
        return T >= self.world and (T + self.world - 1) // self.world <= self.cap and \
            self.ar.local_source_ok(T)

    def moe_allreduce_add_rmsnorm(self, x, router_ids, router_w, experts, shared_fn, residual,
                                  weight, eps):
        """x [T, H] replicated; router_ids / router_w [Tc, k] routing of this rank's shard;
        experts(recv_x, recv_ids) -> (y, pos); shared_fn(x_shard) -> [Tc, H] or None.
        Returns (RMSNorm(residual + moe) * weight, residual) like the all-reduce path."""
        T = x.shape[0]
        per = (T + self.world - 1) // self.world
        r0 = min(T, self.rank * per)
        Tc = max(0, min(T, r0 + per) - r0)
        ints = [self.rank, self.world, Tc, r0, self.H, self.k, self.E_local, per, per]
        ptrs = self._ptrs()
        # blocks of ranks that serve none of a token's experts must read as zero
        self.ar.staging_blocks(per).zero_()
        self.mod.ep_dispatch(x, router_ids, router_w, ints, ptrs)
        rows = self.world * per
        y, pos = experts(self.recv_x[:rows], self.recv_ids[:rows])
        self.mod.ep_return(y, pos, ints, ptrs)
        if shared_fn is not None and Tc > 0:
            residual[r0:r0 + Tc] += shared_fn(x[r0:r0 + Tc])
        return self.ar.reduce_blocks_add_rmsnorm(T, residual, weight, eps, x)

    def close(self) -> None:
        for a in self.opened:
            try:
                self.mod.ipc_close(a)
            except Exception:  # pragma: no cover
                pass
        self.opened = []
        if self.base:
            try:
                torch.cuda.synchronize()
                self.mod.ipc_free(self.base)
            except Exception:  # pragma: no cover
                pass
            self.base = 0


def maybe_create_ep_a2a(st, device, ar, max_tokens: int, hidden: int, k: int,
                        e_local: int) -> Optional[EPAllToAll]:
    """Build on every rank or on none (MIN consensus), like the all-reduce communicator."""
    if ar is None or st.tp_size < 2 or os.environ.get("B200_EP_A2A", "1") != "1":
        return None
    obj, ok = None, 1
    try:
        obj = EPAllToAll(st, device, ar, max_tokens, hidden, k, e_local)
    except Exception as e:  # fail closed
        log.warning("EP all-to-all unavailable on rank %d: %s", st.rank, e)
        ok = 0
    t = torch.tensor([ok], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=st.tp_cpu_group)
    if int(t) == 0:
        if obj is not None:
            obj.close()
        return None
    return obj
