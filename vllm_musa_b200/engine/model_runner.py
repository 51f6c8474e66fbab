"""GPU model runner: step buffers, KV cache, CUDA graphs, forward + sampling.

Per engine step:
  1. the C++ scheduler has written the step's inputs into pinned host buffers;
  2. the used prefix of each buffer is copied host->device (async, on the compute stream);
  3. decode-only steps replay a captured CUDA graph of the padded batch size (forward +
     LM head + sampler in one replay); prefill / mixed steps run eagerly;
  4. the sampled token ids come back device->host into a pinned buffer.
Under pipeline parallelism the step runs as micro-batches of whole requests: each stage
receives a micro-batch's residual stream from the previous stage (NCCL send / recv on the
stage pair), runs its layers and sends it on while the next micro-batch arrives, so the stages
overlap; the last stage samples the whole step and broadcasts the token ids to the other
stages of its pipeline (every rank's scheduler stays in lock-step).  Pipeline steps run eagerly.
The reference uses vLLM's GPUModelRunner with its static graph wrapper and graph-capture
hooks (vllm_musa/platform.py:908-910, v1/worker/*); this runner is written for this engine.
"""
from __future__ import annotations

import logging
import os
import time
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops
from ..attention import AttnMetadata
from ..config import EngineConfig

log = logging.getLogger("vllm_musa_b200")

_I32, _F32, _I64 = torch.int32, torch.float32, torch.int64


class StepBuffers:
    """Fixed-capacity step inputs: pinned host side + device side (same tensors on CPU)."""

    FIELDS = [("input_ids", "tok", _I32), ("positions", "tok", _I32),
              ("slot_mapping", "tok", _I32), ("cu_q", "req1", _I32), ("seq_lens", "req", _I32),
              ("block_tables", "bt", _I32), ("logits_idx", "smp", _I32),
              ("temperature", "smp", _F32), ("top_k", "smp", _I32), ("top_p", "smp", _F32),
              ("min_p", "smp", _F32), ("seeds", "smp", _I64), ("steps", "smp", _I32),
              ("state_slots", "req", _I32), ("tree_mask", "tok", _I64)]
    # sampling rows: one per request, or 1 + drafts under speculative verification; never
    # more than the step's tokens

    def __init__(self, max_tokens: int, max_reqs: int, max_blocks: int, device: torch.device):
        self.max_tokens, self.max_reqs, self.max_blocks = max_tokens, max_reqs, max_blocks
        self.device = device
        pin = device.type == "cuda"
        sizes = {"tok": max_tokens, "req": max_reqs, "req1": max_reqs + 1,
                 "bt": max_reqs * max_blocks, "smp": max(max_tokens, max_reqs)}
        self.h, self.d = {}, {}
        for name, kind, dt in self.FIELDS:
            self.h[name] = torch.zeros(sizes[kind], dtype=dt, pin_memory=pin)
            self.d[name] = self.h[name] if not pin else torch.zeros(sizes[kind], dtype=dt,
                                                                    device=device)
        self.sampled_h = torch.zeros(max(max_tokens, max_reqs), dtype=_I64, pin_memory=pin)

    def pointers(self) -> dict:
        p = {name: self.h[name].data_ptr() for name, _, _ in self.FIELDS}
        p["max_tokens"], p["max_reqs"] = self.max_tokens, self.max_reqs
        return p

    def bt2d(self, which: str = "d") -> torch.Tensor:
        return getattr(self, which)["block_tables"].view(self.max_reqs, self.max_blocks)

    def upload(self, n_tok: int, n_req: int, n_sample: int, sampling: bool,
               tree: bool = False) -> int:
        """Copy the used prefixes host->device.  Returns the number of bytes copied."""
        if self.device.type != "cuda":
            return 0
        nbytes = 0

        def cp(name, n):
            nonlocal nbytes
            if n > 0:
                self.d[name][:n].copy_(self.h[name][:n], non_blocking=True)
                nbytes += n * self.h[name].element_size()

        for name in ("input_ids", "positions", "slot_mapping"):
            cp(name, n_tok)
        cp("cu_q", n_req + 1)
        cp("seq_lens", n_req)
        cp("state_slots", n_req)
        cp("block_tables", n_req * self.max_blocks)
        cp("logits_idx", n_sample)
        if tree:
            cp("tree_mask", n_tok)
        if sampling:
            for name in ("temperature", "top_k", "top_p", "min_p", "seeds", "steps"):
                cp(name, n_sample)
        return nbytes


class StepExtras:
    """Per-step logits processing beyond sampling, for the rows whose requests ask for it:
    penalty entries (ops.sampling.penalty_entries) with per-row penalties, the rows whose
    raw-logit log-probabilities are returned (top ``lp_k`` per row), and the constrained rows
    with their next-token bitmasks (int32 [len(mask_rows), words], structured outputs)."""

    def __init__(self, entries=None, rep=None, pres=None, freq=None, lp_rows=None, lp_k=0,
                 bitmask=None, mask_rows=None):
        self.entries, self.rep, self.pres, self.freq = entries, rep, pres, freq
        self.lp_rows = lp_rows or []
        self.lp_k = lp_k
        self.bitmask = bitmask
        self.mask_rows = mask_rows or []
        self.lora = None  # LoRABatch of the step (adapters in use)
        self.row_req = {}  # sampling row -> request id of the rows above
        self.bias = None   # (rows, token ids, values) added to the raw logits (logit_bias,
        #                    bad words as -inf)
        self.plp = None    # prompt log-probabilities: (rows, target tokens, top-k, owners)
        self.prompt_logprobs = None  # filled by the runner: (top ids, top logprobs, logprob, rank)
        self.pool = []       # embedding requests: (request id, first row, end row) to sum
        self.pooled = None   # filled by the runner: fp32 host vectors, one per pool entry
        self.logprobs = None  # filled by the runner: (top ids, top logprobs, logprob, rank)


class ModelRunner:
    def __init__(self, cfg: EngineConfig, model, sampler, device: torch.device):
        self.cfg = cfg
        self.model = model
        self.sampler = sampler
        self.device = device
        sc = cfg.scheduler
        self.block_size = cfg.cache.block_size  # per-rank cache block
        # block-table width in scheduler blocks (dcp ranks' cache blocks each)
        span = self.block_size * cfg.parallel.decode_context_parallel_size
        self.max_blocks = (sc.max_model_len + span - 1) // span
        self.buf = StepBuffers(sc.max_num_batched_tokens, sc.max_num_seqs, self.max_blocks, device)
        self.kv_caches: list = []
        self.kv_tensor: Optional[torch.Tensor] = None
        self.num_blocks = 0
        self.tile_scratch = torch.zeros(sc.max_num_seqs + 1, dtype=_I32, device=device)
        self.graphs: dict = {}
        self.graph_hidden: dict = {}       # hidden-state output of each decode graph
        self.last_hidden: Optional[torch.Tensor] = None
        self.graph_launches: dict = {}     # our kernels recorded in each decode graph
        self.graph_launches_replayed = 0   # ... summed over replays
        self.graph_pool = None
        self.use_graphs = device.type == "cuda" and not cfg.enforce_eager
        self.timing = False
        self.step_times: list = []  # (kind, start_event, end_event)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.gen = torch.Generator(device="cpu").manual_seed(cfg.seed) if device.type == "cpu" else None
        # recurrent-state slot written by padded CUDA-graph rows (one spare slot past the
        # scheduler's range, so padding never touches a live request's state)
        self.dummy_state_slot = sc.max_num_seqs
        if hasattr(model, "allocate_state"):
            model.allocate_state(sc.max_num_seqs + 1)
        self.record_logits = False  # debugging / tests: keep every step's logits (eager only)
        self.logits_log: list = []
        self._extras: Optional[StepExtras] = None
        st = getattr(model, "pstate", None)
        self.pp = st if st is not None and st.pp_size > 1 else None
        if self.pp is not None:
            self.use_graphs = False
            self.pp_micro_batches = int(os.environ.get("B200_PP_MICRO_BATCHES", "0")) or \
                self.pp.pp_size

    # ------------------------------------------------------------------ memory / KV cache
    def kv_bytes_per_block(self) -> int:
        if hasattr(self.model, "kv_bytes_per_block"):  # model-defined caches (e.g. MLA)
            return self.model.kv_bytes_per_block(self.block_size)
        spec = self.model.kv_cache_spec()
        elt = torch.tensor([], dtype=spec["dtype"]).element_size()
        heads = spec["num_layers"] * spec["num_kv_heads"] + spec.get("draft_kv_heads", 0)
        return heads * 2 * self.block_size * spec["head_dim"] * elt

    def profile_and_allocate_kv(self) -> int:
        """Measure the activation peak of a full-budget prefill, then size the KV cache."""
        cc = self.cfg.cache
        if cc.num_gpu_blocks is not None or self.device.type != "cuda":
            n = cc.num_gpu_blocks or max(64, 4 * self.cfg.scheduler.max_num_seqs)
            self.allocate_kv(n)
            return n
        spec = self.model.kv_cache_spec()
        if hasattr(self.model, "allocate_kv_cache"):
            tmp = self.model.allocate_kv_cache(1, self.block_size)
        else:
            tmp = [(torch.zeros(1, spec["num_kv_heads"], self.block_size, spec["head_dim"],
                                dtype=spec["dtype"], device=self.device),) * 2
                   for _ in range(spec["num_layers"])]
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        T = self.cfg.scheduler.max_num_batched_tokens
        R = min(self.cfg.scheduler.max_num_seqs, max(1, T // 1024))
        b = self.buf
        per = T // R
        b.d["input_ids"][:T].zero_()
        b.d["positions"][:T].copy_(torch.arange(T, device=self.device) % per)
        b.d["slot_mapping"][:T].fill_(-1)
        b.d["cu_q"][:R + 1].copy_(torch.arange(R + 1, device=self.device) * per)
        b.d["cu_q"][R] = T
        b.d["seq_lens"][:R].fill_(per)
        b.d["seq_lens"][R - 1] = T - per * (R - 1)
        b.bt2d()[:R].zero_()
        b.d["logits_idx"][:R].copy_(b.d["cu_q"][1:R + 1] - 1)
        b.d["state_slots"][:R].copy_(torch.arange(R, dtype=_I32, device=self.device))
        meta = AttnMetadata(T, 0, R, b.d["positions"][:T], b.d["slot_mapping"][:T],
                            b.d["seq_lens"][:R], b.bt2d()[:R], b.d["cu_q"][:R + 1],
                            max_seq_len=T, tile_scratch=self.tile_scratch,
                            state_slots=b.d["state_slots"][:R])
        self.kv_caches = tmp
        self._forward_sample(T, R, R, meta, sampling=False, any_filter=False)
        torch.cuda.synchronize()
        peak = torch.cuda.max_memory_allocated() - base
        self.kv_caches = []
        del tmp
        torch.cuda.empty_cache()
        free, total = torch.cuda.mem_get_info()
        graph_reserve = (1 << 30) if self.use_graphs else 0
        budget = free - (1.0 - cc.gpu_memory_utilization) * total - peak - graph_reserve
        n = int(budget // self.kv_bytes_per_block())
        if n < 16:
            raise RuntimeError(f"not enough GPU memory for the KV cache (budget {budget/2**30:.1f} GiB)")
        log.info("KV cache: %d blocks of %d tokens (%.1f GiB); activation peak %.2f GiB",
                 n, self.block_size, n * self.kv_bytes_per_block() / 2**30, peak / 2**30)
        self.allocate_kv(n)
        return n

    def allocate_kv(self, num_blocks: int) -> None:
        spec = self.model.kv_cache_spec()
        self.num_blocks = num_blocks
        if hasattr(self.model, "allocate_kv_cache"):
            self.kv_tensor = None
            self.kv_caches = self.model.allocate_kv_cache(num_blocks, self.block_size)
            return
        self.kv_tensor = torch.zeros(spec["num_layers"], 2, num_blocks, spec["num_kv_heads"],
                                     self.block_size, spec["head_dim"], dtype=spec["dtype"],
                                     device=self.device)
        self.kv_caches = [(self.kv_tensor[i, 0], self.kv_tensor[i, 1])
                          for i in range(spec["num_layers"])]
        if spec.get("draft_kv_heads"):  # replicated draft layer: all KV heads, same pages
            shape = (num_blocks, spec["draft_kv_heads"], self.block_size, spec["head_dim"])
            self.model.draft_head.own_kv = tuple(
                torch.zeros(shape, dtype=spec["dtype"], device=self.device) for _ in range(2))

    def apply_kv_moves(self, moves) -> None:
        """Copy KV rows between cache slots (slot = block * block_size + offset) in every layer:
        the accepted path of a verified draft tree moved to consecutive positions.  All rows
        are gathered before any is written (a destination may be another move's source)."""
        if not moves:
            return
        bs = self.block_size
        src = torch.tensor([m[0] for m in moves], dtype=torch.long)
        dst = torch.tensor([m[1] for m in moves], dtype=torch.long)
        sb, so = (src // bs).to(self.device), (src % bs).to(self.device)
        db, do = (dst // bs).to(self.device), (dst % bs).to(self.device)
        if self.kv_tensor is not None:  # [L, 2, blocks, Hkv, bs, D]: one gather + one scatter
            rows = self.kv_tensor[:, :, sb, :, so]
            self.kv_tensor[:, :, db, :, do] = rows
            return
        for kc, vc in self.kv_caches:  # per-layer [blocks, Hkv, bs, D] pairs
            for c in (kc, vc):
                rows = c[sb, :, so]
                c[db, :, do] = rows

    # ------------------------------------------------------------------ forward
    def _forward_sample(self, T: int, R: int, S: int, meta: AttnMetadata, sampling: bool,
                        any_filter: bool, decode_only: bool = False) -> torch.Tensor:
        b = self.buf
        if self.pp is not None:
            return self._forward_sample_pp(T, R, S, meta, sampling, any_filter, decode_only)
        hidden = self.model.forward(b.d["input_ids"][:T], meta, self.kv_caches)
        self.last_hidden = hidden  # final hidden states of the step (the MTP drafter reads them)
        return self._sample_hidden(hidden, S, sampling, any_filter, decode_only)

    def _sample_hidden(self, hidden: torch.Tensor, S: int, sampling: bool, any_filter: bool,
                       decode_only: bool) -> torch.Tensor:
        b = self.buf
        rows = hidden if decode_only else ops.gather_rows(hidden, b.d["logits_idx"][:S])
        logits = self.model.compute_logits(rows)
        if self.record_logits:
            self.logits_log.append(logits.detach().float().cpu())
        ex = self._extras
        raw = None
        mode = self.cfg.logprobs_mode
        if ex is not None and ex.plp is not None:
            ex.prompt_logprobs = self._prompt_logprobs(hidden, ex.plp, mode)
        if ex is not None and ex.pool:
            ex.pooled = list(torch.stack([hidden[a:b].float().sum(0) for _, a, b in ex.pool])
                             .cpu().unbind(0))
        if ex is not None:
            if ex.lp_rows:
                idx = torch.tensor(ex.lp_rows, dtype=torch.int64, device=logits.device)
                if mode.startswith("raw"):
                    raw = logits.index_select(0, idx)
            if ex.entries is not None and ex.entries.numel():
                dev = logits.device
                ops.apply_penalties(logits, ex.entries.to(dev), ex.rep.to(dev), ex.pres.to(dev),
                                    ex.freq.to(dev), getattr(self.model, "vocab_start", 0))
            if ex.bias is not None:
                r, c, v = ex.bias
                vs, Vl = getattr(self.model, "vocab_start", 0), logits.shape[1]
                keep = (c >= vs) & (c < vs + Vl)  # this rank's vocab shard
                if bool(keep.any()):
                    dev = logits.device
                    logits.index_put_((r[keep].to(dev), (c[keep] - vs).to(dev)),
                                      v[keep].to(dev), accumulate=True)
            if ex.mask_rows:
                dev = logits.device
                ops.sampling.apply_token_bitmask(
                    logits, ex.bitmask.to(dev),
                    torch.tensor(ex.mask_rows, dtype=_I32, device=dev),
                    getattr(self.model, "vocab_start", 0))
        if ex is not None and ex.lp_rows and not mode.startswith("raw"):
            raw = logits.index_select(0, idx)  # processed: after penalties / bias / masks
            if sampling:
                t = b.d["temperature"][:S].index_select(0, idx).float()
                raw = raw / torch.where(t > 0, t, torch.ones_like(t)).unsqueeze(1)
        if sampling:
            ids = self.sampler(logits, b.d["temperature"][:S], b.d["top_k"][:S],
                               b.d["top_p"][:S], b.d["min_p"][:S], b.d["seeds"][:S],
                               b.d["steps"][:S], any_filter=any_filter, generator=self.gen)
        else:
            ids = self.sampler(logits, None, None, None, None, None, None)
        if raw is not None:
            if self.sampler.tp > 1:  # vocab-sharded rows: the full distribution
                raw = self.sampler.comm.all_gather(raw, dim=1)
            sel = ids.index_select(0, idx)
            ex.logprobs = [t.cpu() for t in ops.sampling.token_logprobs(
                raw, sel, ex.lp_k, as_logits=mode.endswith("logits"))]
        return ids

    def _prompt_logprobs(self, hidden: torch.Tensor, plp, mode: str) -> list:
        """Log-probabilities of prompt tokens from the step's hidden rows, 256 rows at a time
        (each block's logits are [256, V] fp32): (top ids, top values, token value, rank), on
        the host.  Prompt positions see raw logits (no sampling parameters apply to them)."""
        rows, targets, k, _ = plp
        dev = hidden.device
        parts = []
        for a in range(0, rows.numel(), 256):
            r = rows[a:a + 256].to(dev)
            lg = self.model.compute_logits(hidden.index_select(0, r).contiguous())
            if self.sampler.tp > 1:
                lg = self.sampler.comm.all_gather(lg, dim=1)
            lg = lg[:, :self.model.cfg.vocab_size]
            parts.append([t.cpu() for t in ops.sampling.token_logprobs(
                lg, targets[a:a + 256].to(dev), k, as_logits=mode.endswith("logits"))])
        return [torch.cat([p[i] for p in parts]) for i in range(4)]

    # ------------------------------------------------------------------ pipeline parallelism
    def _pp_chunks(self, meta: AttnMetadata, T: int, R: int) -> list:
        """Micro-batches of whole requests with about equal token counts: (r0, r1, t0, t1)."""
        cu = meta.cu_q[:R + 1].tolist()
        m = max(1, min(self.pp_micro_batches, R))
        out, r0 = [], 0
        for k in range(m):
            if r0 >= R:
                break
            goal = T * (k + 1) / m
            r1 = r0 + 1
            while r1 < R and cu[r1] < goal and R - r1 > m - k - 1:
                r1 += 1
            if k == m - 1:
                r1 = R
            out.append((r0, r1, cu[r0], cu[r1]))
            r0 = r1
        return out

    @staticmethod
    def _meta_slice(meta: AttnMetadata, r0: int, r1: int, t0: int, t1: int) -> AttnMetadata:
        nd = max(0, min(r1, meta.num_decodes) - r0)
        m = AttnMetadata(t1 - t0, nd, (r1 - r0) - nd, meta.positions[t0:t1],
                         meta.slot_mapping[t0:t1], meta.seq_lens[r0:r1],
                         meta.block_tables[r0:r1], meta.cu_q[r0:r1 + 1] - t0,
                         max_seq_len=meta.max_seq_len, tile_scratch=meta.tile_scratch,
                         sliding_window=meta.sliding_window,
                         state_slots=None if meta.state_slots is None
                         else meta.state_slots[r0:r1])
        if meta.tree_mask is not None:
            m.tree_mask = meta.tree_mask[t0:t1]
        if meta.lora is not None:  # adapter token groups re-based to the micro-batch
            from ..lora import LoRABatch
            groups = []
            for slot, idx in meta.lora.groups:
                sel = idx[(idx >= t0) & (idx < t1)] - t0
                if sel.numel():
                    groups.append((slot, sel))
            m.lora = LoRABatch(groups) if groups else None
        return m

    def _forward_sample_pp(self, T: int, R: int, S: int, meta: AttnMetadata, sampling: bool,
                           any_filter: bool, decode_only: bool) -> torch.Tensor:
        st, b, dev = self.pp, self.buf, self.device
        first, last = st.is_first_stage, st.is_last_stage
        H, dt = self.model.cfg.hidden_size, self.model.dtype
        chunks = self._pp_chunks(meta, T, R)
        recvs = []
        if not first:  # post every micro-batch's receive up front
            src = st.pp_ranks[st.pp_rank - 1]
            for (_, _, t0, t1) in chunks:
                buf = torch.empty(t1 - t0, H, dtype=dt, device=dev)
                recvs.append((buf, dist.irecv(buf, src=src, group=st.pp_group)))
        hidden = torch.empty(T, H, dtype=dt, device=dev) if last else None
        sends = []
        ids_all = b.d["input_ids"][:T]
        for k, (r0, r1, t0, t1) in enumerate(chunks):
            m = self._meta_slice(meta, r0, r1, t0, t1)
            hin = None
            if recvs:
                hin, work = recvs[k]
                work.wait()
            out = self.model.forward(ids_all[t0:t1], m, self.kv_caches, hidden_in=hin)
            if last:
                hidden[t0:t1].copy_(out)
            else:
                out = out.contiguous()
                sends.append((out, dist.isend(out, dst=st.pp_ranks[st.pp_rank + 1],
                                              group=st.pp_group)))
        for _, work in sends:
            work.wait()
        if last:
            self.last_hidden = hidden
            ids = self._sample_hidden(hidden, S, sampling, any_filter, decode_only).to(torch.int64)
        else:
            ids = torch.empty(S, dtype=torch.int64, device=dev)
        dist.broadcast(ids, src=st.pp_ranks[-1], group=st.pp_group)
        ex = self._extras
        if ex is not None and (ex.lp_rows or ex.plp is not None or ex.pool):
            obj = [ex.logprobs, ex.prompt_logprobs, ex.pooled]
            dist.broadcast_object_list(obj, src=st.pp_ranks[-1], group=st.pp_cpu_group)
            ex.logprobs, ex.prompt_logprobs, ex.pooled = obj
        return ids

    def _meta(self, T: int, R: int, nd: int, npf: int, max_seq_len: int,
              decode_splits: Optional[int] = None) -> AttnMetadata:
        b = self.buf
        return AttnMetadata(T, nd, npf, b.d["positions"][:T], b.d["slot_mapping"][:T],
                            b.d["seq_lens"][:R], b.bt2d()[:R], b.d["cu_q"][:R + 1],
                            max_seq_len=max_seq_len, decode_splits=decode_splits,
                            tile_scratch=self.tile_scratch, state_slots=b.d["state_slots"][:R])

    # ------------------------------------------------------------------ CUDA graphs
    def graph_sizes(self) -> list:
        if self.cfg.cuda_graph_sizes:
            sizes = sorted(set(int(s) for s in self.cfg.cuda_graph_sizes))
        else:
            mx = self.cfg.scheduler.max_num_seqs
            sizes = [1, 2, 4, 8] + list(range(16, 257, 16)) + list(range(288, 1025, 32))
            sizes = [s for s in sizes if s <= mx]
            if mx not in sizes:
                sizes.append(mx)
        return [s for s in sizes if s <= self.buf.max_reqs]

    def _pad_decode_inputs(self, B: int) -> None:
        b = self.buf
        b.d["seq_lens"][:B].zero_()
        b.d["slot_mapping"][:B].fill_(-1)
        b.d["input_ids"][:B].zero_()
        b.d["positions"][:B].zero_()
        b.d["cu_q"][:B + 1].copy_(torch.arange(B + 1, dtype=_I32, device=self.device))
        b.d["logits_idx"][:B].copy_(torch.arange(B, dtype=_I32, device=self.device))
        b.d["temperature"][:B].zero_()
        b.d["top_k"][:B].zero_()
        b.d["top_p"][:B].fill_(1.0)
        b.d["min_p"][:B].zero_()
        b.d["state_slots"][:B].fill_(self.dummy_state_slot)

    def reserve_workspaces(self) -> None:
        """Size the split-K GEMM and split-KV workspaces for every shape the runner can see."""
        if self.device.type != "cuda":
            return
        mod = ops._ext.require()
        Ms = sorted(set(self.graph_sizes() + [self.cfg.scheduler.max_num_batched_tokens,
                                                self.cfg.scheduler.max_num_seqs]))
        need = 0
        for (N, K) in self.model.linear_shapes():
            for M in Ms + [1, 2, 4, 8, 16, 32, 64, 128]:
                need = max(need, ops.gemm.plan_for(M, N, K)[3], mod.gemm_plan(M, N, K)[2])
        ops.gemm.reserve_workspace(self.device, need)
        if hasattr(self.model, "reserve_workspaces"):
            self.model.reserve_workspaces(max(self.graph_sizes() + [1]))
        spec = self.model.kv_cache_spec()
        hq = getattr(self.model, "hq", spec["num_kv_heads"])
        worst = 0
        for B in range(1, self.cfg.scheduler.max_num_seqs + 1):
            s = ops.attention.num_decode_splits(B, spec["num_kv_heads"], self.cfg.scheduler.max_model_len)
            worst = max(worst, B * s)
        if worst:
            ops.attention.decode_workspace(self.device, worst, hq, spec["head_dim"], 1)

    def capture_graphs(self) -> None:
        if not self.use_graphs:
            return
        t0 = time.time()
        mod = ops._ext.require()
        self.reserve_workspaces()
        self.graph_pool = torch.cuda.graph_pool_handle()
        max_len = self.cfg.scheduler.max_model_len
        hkv = self.model.kv_cache_spec()["num_kv_heads"]
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for B in sorted(self.graph_sizes(), reverse=True):
                self._pad_decode_inputs(B)
                splits = ops.attention.num_decode_splits(B, hkv, max_len)
                meta = self._meta(B, B, B, 0, max_len, splits)
                for _ in range(2):
                    self._forward_sample(B, B, B, meta, sampling=True, any_filter=False,
                                         decode_only=True)
                g = torch.cuda.CUDAGraph()
                c0 = mod.launch_count()
                with torch.cuda.graph(g, pool=self.graph_pool, stream=stream):
                    out = self._forward_sample(B, B, B, meta, sampling=True, any_filter=False,
                                               decode_only=True)
                self.graph_launches[B] = mod.launch_count() - c0
                self.graphs[B] = (g, out)
                self.graph_hidden[B] = self.last_hidden
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()
        log.info("captured %d decode CUDA graphs in %.1fs", len(self.graphs), time.time() - t0)

    def release_graphs(self) -> None:
        self.graphs.clear()
        self.graph_hidden.clear()
        self.graph_pool = None

    # ------------------------------------------------------------------ step
    def execute(self, plan, extras: Optional[StepExtras] = None) -> torch.Tensor:
        """Run one scheduled step; returns the sampled ids (host int64 tensor, [num_samples]).
        ``extras`` (penalties / log-probabilities for some rows) runs the step eagerly."""
        T, R, S = plan.num_tokens, plan.num_reqs, plan.num_samples
        nd, npf = plan.num_decodes, plan.num_prefills
        b = self.buf
        cuda = self.device.type == "cuda"
        decode_only = npf == 0 and nd == R and S == R
        self._extras = extras
        B = None
        if decode_only and self.graphs and not self.record_logits and extras is None and \
                not (plan.any_filter and self.sampler.tp > 1):
            for s in sorted(self.graphs):
                if s >= R:
                    B = s
                    break
        ev = None
        if self.timing and cuda:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        if B is not None:
            h = b.h
            if B > R:
                h["slot_mapping"][T:B] = -1
                h["seq_lens"][R:B] = 0
                h["input_ids"][T:B] = 0
                h["positions"][T:B] = 0
                h["logits_idx"][S:B] = 0
                h["temperature"][S:B] = 0
                h["top_k"][S:B] = 0
                h["top_p"][S:B] = 1.0
                h["min_p"][S:B] = 0
                h["cu_q"][R + 1:B + 1] = torch.arange(R + 1, B + 1, dtype=_I32)
                h["state_slots"][R:B] = self.dummy_state_slot
            self.h2d_bytes += b.upload(B, B, B, True)
            g, out = self.graphs[B]
            g.replay()
            self.last_hidden = self.graph_hidden[B][:T]
            self.graph_launches_replayed += self.graph_launches[B]
            ids = out[:S]
        else:
            sampling = not plan.all_greedy
            self.h2d_bytes += b.upload(T, R, S, sampling, plan.tree)
            meta = self._meta(T, R, nd, npf, plan.max_seq_len)
            meta.lora = extras.lora if extras is not None else None
            if plan.tree:
                meta.tree_mask = b.d["tree_mask"][:T]
            ids = self._forward_sample(T, R, S, meta, sampling=sampling,
                                       any_filter=plan.any_filter, decode_only=decode_only)
        self._extras = None
        out_h = b.sampled_h[:S]
        if cuda:
            out_h.copy_(ids, non_blocking=True)
            self.d2h_bytes += S * 8
            if ev is not None:
                ev[1].record()
                self.step_times.append(("decode" if decode_only else "mixed", ev[0], ev[1]))
            torch.cuda.current_stream().synchronize()
        else:
            out_h.copy_(ids)
        return out_h
