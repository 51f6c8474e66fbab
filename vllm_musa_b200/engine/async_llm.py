"""Asynchronous front end of the engine for the HTTP server.

A background thread owns the ``LLMEngine`` and steps it while requests are in flight; API
handlers submit requests through a thread-safe queue and consume per-request asyncio
queues of incremental ``RequestOutput``s.  Text is detokenised incrementally; ``stop``
strings end a request early (the request is aborted in the scheduler and its text cut at the
match).  With follower ranks (multi-process TP) the loop also steps while idle, at most every
``B200_IDLE_SYNC_S`` seconds, so followers keep receiving the (empty) per-step broadcast.
"""
from __future__ import annotations

import asyncio
import logging
import os
import queue
import threading
import time
import uuid
from dataclasses import dataclass, field
from typing import AsyncIterator, Dict, List, Optional

from ..outputs import CompletionOutput, RequestOutput
from ..sample.sampling_params import SamplingParams
from .llm_engine import LLMEngine

log = logging.getLogger("vllm_musa_b200")


@dataclass
class _Stream:
    loop: asyncio.AbstractEventLoop
    q: asyncio.Queue
    params: SamplingParams
    prompt_len: int
    text: str = ""
    done: bool = False
    token_ids: List[int] = field(default_factory=list)


class EngineDeadError(RuntimeError):
    """The engine loop stopped after a step raised (vLLM's EngineDeadError)."""


class AsyncLLM:
    def __init__(self, engine: LLMEngine):
        self.engine = engine
        self.engine.stream_outputs = True
        self.tokenizer = engine.tokenizer
        self._in: "queue.Queue" = queue.Queue()
        self._streams: Dict[str, _Stream] = {}
        self._lock = threading.Lock()
        self._wake = threading.Event()
        self._stop = False
        self.dead: Optional[BaseException] = None  # the error that stopped the engine loop
        self.idle_sync_s = float(os.environ.get("B200_IDLE_SYNC_S", "1.0"))
        self.stats = {"finished": 0, "ttft": [], "tpot": [], "prompt_tokens": 0,
                      "generation_tokens": 0}
        self._thread = threading.Thread(target=self._loop, name="b200-engine", daemon=True)
        self._thread.start()

    # ------------------------------------------------------------------ API side
    async def generate(self, prompt_ids: List[int], params: SamplingParams,
                       request_id: Optional[str] = None, prompt: Optional[str] = None,
                       lora_request=None, priority: int = 0) -> AsyncIterator[RequestOutput]:
        if self.dead is not None:
            raise EngineDeadError(f"the engine stopped after an error: {self.dead!r}")
        rid = request_id or uuid.uuid4().hex
        loop = asyncio.get_running_loop()
        st = _Stream(loop, asyncio.Queue(), params, len(prompt_ids))
        with self._lock:
            self._streams[rid] = st
        self._in.put(("add", rid, list(prompt_ids), params, prompt, lora_request, priority))
        self._wake.set()
        try:
            while True:
                out = await st.q.get()
                if isinstance(out, BaseException):
                    raise out
                yield out
                if out.finished:
                    break
        finally:
            if not st.done:
                self.abort(rid)

    def abort(self, request_id: str) -> None:
        self._in.put(("abort", request_id))
        self._wake.set()

    def shutdown(self) -> None:
        self._stop = True
        self._wake.set()
        self._thread.join(timeout=30)
        self.engine.shutdown()

    # ------------------------------------------------------------------ engine thread
    def _drain_inputs(self) -> None:
        while True:
            try:
                op = self._in.get_nowait()
            except queue.Empty:
                return
            try:
                if op[0] == "add":
                    _, rid, ids, params, prompt, lora, prio = op
                    self.engine.add_request(rid, ids, params, prompt=prompt, lora_request=lora,
                                            priority=prio)
                    self.stats["prompt_tokens"] += len(ids)
                else:
                    self._finish(op[1], None, "abort", abort_engine=True)
            except Exception as e:  # bad request: report to its stream
                if op[0] == "add":
                    self._push(op[1], e)

    def _push(self, rid: str, item) -> None:
        with self._lock:
            st = self._streams.get(rid)
        if st is not None:
            st.loop.call_soon_threadsafe(st.q.put_nowait, item)

    def _decode(self, ids: List[int]) -> str:
        if self.tokenizer is None:
            return ""
        try:
            return self.tokenizer.decode(ids, skip_special_tokens=True)
        except Exception:  # pragma: no cover
            return ""

    def _finish(self, rid: str, out: Optional[RequestOutput], reason: str,
                abort_engine: bool = False) -> None:
        with self._lock:
            st = self._streams.pop(rid, None)
        if abort_engine:
            self.engine.abort_request(rid)
        if st is None or st.done:
            return
        st.done = True
        if out is None:
            out = RequestOutput(rid, [], [CompletionOutput(0, st.token_ids, st.text, reason)], True)
        st.loop.call_soon_threadsafe(st.q.put_nowait, out)

    def _handle(self, out: RequestOutput) -> None:
        rid = out.request_id
        with self._lock:
            st = self._streams.get(rid)
        if st is None:
            return
        comp = out.outputs[0]
        st.token_ids = list(comp.token_ids)
        # embedding requests (PoolingParams) carry no text options
        if getattr(st.params, "detokenize", False) and self.tokenizer is not None:
            st.text = self._decode(st.token_ids)
            comp.text = st.text
            for s in st.params.stop:
                k = st.text.find(s)
                if k >= 0:
                    comp.text = st.text = st.text[:k]
                    comp.finish_reason = "stop"
                    out.finished = True
                    self._record(out)
                    self._finish(rid, out, "stop", abort_engine=True)
                    return
        if out.finished:
            self._record(out)
            self._finish(rid, out, comp.finish_reason or "stop")
        else:
            st.loop.call_soon_threadsafe(st.q.put_nowait, out)

    def _record(self, out: RequestOutput) -> None:
        self.stats["finished"] += 1
        self.stats["generation_tokens"] += len(out.outputs[0].token_ids)
        if out.metrics.ttft is not None:
            self.stats["ttft"].append(out.metrics.ttft)
        t = out.tpot()
        if t is not None:
            self.stats["tpot"].append(t)

    def _loop(self) -> None:
        last = time.time()
        following = self.engine.sync is not None
        while not self._stop:
            self._drain_inputs()
            busy = self.engine.has_unfinished_requests()
            if busy or (following and time.time() - last > self.idle_sync_s):
                try:
                    outs = self.engine.step()
                except Exception as e:  # engine failure: fail every open request
                    log.exception("engine step failed")
                    self.dead = e  # later requests fail at once; /health reports 503
                    with self._lock:
                        rids = list(self._streams)
                    for rid in rids:
                        self._push(rid, e)
                    return
                last = time.time()
                for o in outs:
                    self._handle(o)
            else:
                self._wake.wait(timeout=self.idle_sync_s if following else 0.05)
                self._wake.clear()
