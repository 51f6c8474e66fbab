"""Multi-process executor for tensor parallelism without an external launcher.

``LLM(..., tensor_parallel_size=N)`` outside ``torchrun`` spawns N-1 follower processes (one
per GPU).  The driver (rank 0) owns the user-facing API; at the start of every engine step it
broadcasts the requests added / aborted since the previous step over the Gloo group, so each
follower's C++ scheduler sees the same inputs at the same step boundary and the ranks stay in
lock-step (they draw identical tokens; see sample/sampler.py).

Shutdown mirrors the reference's worker-termination escalation
(vllm_musa/v1/executor/multiproc_executor.py:15-74): ask followers to exit, wait up to
``B200_WORKER_TERMINATION_TIMEOUT_S`` (default 10 s), then SIGTERM, then SIGKILL.
"""
from __future__ import annotations

import atexit
import logging
import os
import pickle
import socket
import time
from typing import List, Optional

import torch
import torch.distributed as dist

log = logging.getLogger("vllm_musa_b200")

OP_ADD, OP_ABORT, OP_SHUTDOWN = 0, 1, 2


class StepSync:
    """Broadcast of per-step request operations from the driver to the followers."""

    def __init__(self, group, rank: int):
        self.group = group
        self.rank = rank
        self.src = dist.get_global_rank(group, 0) if group is not None else 0
        self.pending: List[tuple] = []

    def record(self, op: tuple) -> None:
        if self.rank == 0:
            self.pending.append(op)

    def exchange(self) -> List[tuple]:
        """Driver: send pending ops.  Follower: receive them.  Called on every rank per step."""
        hdr = torch.zeros(1, dtype=torch.int64)
        payload = None
        if self.rank == 0:
            payload = pickle.dumps(self.pending) if self.pending else b""
            hdr[0] = len(payload)
        dist.broadcast(hdr, src=self.src, group=self.group)
        n = int(hdr[0])
        if n == 0:
            self.pending = []
            return []
        buf = torch.empty(n, dtype=torch.uint8)
        if self.rank == 0:
            buf.copy_(torch.frombuffer(bytearray(payload), dtype=torch.uint8))
        dist.broadcast(buf, src=self.src, group=self.group)
        ops = self.pending if self.rank == 0 else pickle.loads(buf.numpy().tobytes())
        self.pending = []
        return ops


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _follower_main(config, rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), B200_SPMD_ROLE="follower")
    from .llm_engine import LLMEngine
    eng = LLMEngine(config)
    try:
        eng.follow()
    finally:
        eng.shutdown()
        from ..parallel.state import destroy_distributed
        destroy_distributed()


class MultiprocExecutor:
    """Spawns and supervises the follower ranks of a driver engine."""

    def __init__(self, config, world: int):
        import multiprocessing as mp
        self.world = world
        self.port = _free_port()
        ctx = mp.get_context("spawn")
        self.procs = []
        for r in range(1, world):
            p = ctx.Process(target=_follower_main, args=(config, r, world, self.port), daemon=False)
            p.start()
            self.procs.append(p)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(self.port), RANK="0",
                          WORLD_SIZE=str(world), LOCAL_RANK="0", B200_SPMD_ROLE="driver")
        atexit.register(self.shutdown)

    def shutdown(self, timeout: Optional[float] = None) -> None:
        timeout = float(os.environ.get("B200_WORKER_TERMINATION_TIMEOUT_S", "10")) \
            if timeout is None else timeout
        deadline = time.time() + timeout
        for p in self.procs:
            p.join(timeout=max(0.0, deadline - time.time()))
        for p in self.procs:
            if p.is_alive():
                log.warning("follower pid %d did not exit in %.0fs: SIGTERM", p.pid, timeout)
                p.terminate()
        for p in self.procs:
            p.join(timeout=5)
            if p.is_alive():
                log.warning("follower pid %d ignored SIGTERM: SIGKILL", p.pid)
                p.kill()
                p.join(timeout=5)
        self.procs = []
