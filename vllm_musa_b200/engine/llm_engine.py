"""The serving engine: requests in, tokens out.

    add_request() -> C++ Scheduler (admission, KV blocks, chunked prefill, preemption)
    step()        -> Scheduler.schedule() fills the pinned step buffers
                  -> ModelRunner.execute() (H2D, forward / CUDA-graph replay, sample, D2H)
                  -> Scheduler.update() appends tokens, applies stop conditions
Tensor parallelism is SPMD: every rank (one process per GPU, launched by torchrun) runs
its own engine on the same requests; the schedulers stay in lock-step because every rank
draws the same tokens (vocab-parallel sampler, parallel/sampler).  The reference gets this
layer from upstream vLLM's V1 EngineCore.
"""
from __future__ import annotations

import itertools
import logging
import os
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .. import ops, plan
from ..config import EngineConfig
from ..models.registry import get_model_class
from ..models.weights import dummy_weights, safetensors_weights
from ..outputs import CompletionOutput, RequestMetrics, RequestOutput
from ..parallel.communicator import LocalCommunicator, TPCommunicator
from ..parallel.state import get_parallel_state, init_distributed
from ..sample.sampler import Sampler
from ..sample.sampling_params import SamplingParams
from .model_runner import ModelRunner
from ..ops._ext import require as _native  # C++ scheduler + KV block pool (csrc/runtime)

log = logging.getLogger("vllm_musa_b200")

_REASONS = {1: "length", 2: "stop", 3: "abort"}


@dataclass
class _Req:
    request_id: str
    int_id: int
    prompt_token_ids: List[int]
    params: SamplingParams
    arrival: float
    prompt: Optional[str] = None
    parent: Optional[str] = None
    index: int = 0
    tokens: List[int] = field(default_factory=list)
    first_token_time: Optional[float] = None
    logprobs: Optional[list] = None       # per generated token {id: Logprob} (if requested)
    cum_logprob: float = 0.0
    matcher: Optional[object] = None      # structured outputs: the request's grammar matcher
    stop_hit: Optional[tuple] = None      # (stop string, text up to it) once one matched
    lora: Optional[object] = None         # LoRARequest of the request (None: base model)
    lora_slot: int = -1
    bad_words_ids: Optional[list] = None  # token-id sequences of the request's bad words
    prompt_logprobs: Optional[list] = None  # per prompt position (None first), if requested
    pooling: Optional[object] = None        # PoolingParams of an embedding request
    pool_sum: Optional[object] = None       # running sum of the pooled hidden rows
    pool_n: int = 0


def _mix_seed(a: int, b: int) -> int:
    x = (a * 0x9E3779B97F4A7C15 + b * 0xBF58476D1CE4E5B9 + 0x94D049BB133111EB) & (2**64 - 1)
    x ^= x >> 31
    return x & 0x7FFFFFFFFFFFFFFF


class LLMEngine:
    def __init__(self, config: EngineConfig, tokenizer=None):
        self.config = config
        self.tokenizer = tokenizer
        # which optimised paths this configuration uses (fails closed on unserved combinations)
        self.contract = plan.resolve(config)
        plan.validate(self.contract)
        log.info("optimisation contract %s", self.contract.describe())
        mcfg = config.model
        tp = config.parallel.tensor_parallel_size
        pp = config.parallel.pipeline_parallel_size
        device = torch.device(config.device)
        if device.type == "cuda":
            ops._ext.require()
        st = get_parallel_state()
        if (tp > 1 or pp > 1) and (st.tp_size != tp or st.pp_size != pp):
            st = init_distributed(tp_size=tp, ep=config.parallel.enable_expert_parallel,
                                  backend="nccl" if device.type == "cuda" else "gloo",
                                  pp_size=pp)
        if device.type == "cuda":
            device = torch.device("cuda", st.local_rank if st.world_size > 1 else
                                  (device.index or 0))
            torch.cuda.set_device(device)
        self.device = device
        self.pstate = st
        if st.tp_size > 1:
            custom = None
            if device.type == "cuda" and config.parallel.use_custom_allreduce:
                from ..parallel.custom_ar import maybe_create_custom_allreduce
                custom = maybe_create_custom_allreduce(
                    st, device, max_tokens=config.scheduler.max_num_batched_tokens,
                    hidden=mcfg.hidden_size)
            self.comm = TPCommunicator(st, device, custom)
            if custom is not None and st.ep_size > 1 and mcfg.num_experts and \
                    mcfg.num_experts % st.ep_size == 0:
                from ..parallel.ep_a2a import maybe_create_ep_a2a
                self.comm.ep_a2a = maybe_create_ep_a2a(
                    st, device, custom, config.scheduler.max_num_batched_tokens,
                    mcfg.hidden_size, mcfg.num_experts_per_tok, mcfg.num_experts // st.ep_size)
            st.comm = self.comm
        else:
            self.comm = LocalCommunicator(device)
        cls = get_model_class(mcfg)
        self.model = cls(mcfg, st, self.comm, device)
        t0 = time.time()
        self._load_weights()
        if config.speculative.method == "eagle":
            self._load_eagle()
        elif config.speculative.method == "eagle3":
            self._load_eagle3()
        elif config.speculative.method == "medusa":
            self._load_medusa()
        if config.lora.enable_lora:
            from ..lora import LoRAManager
            if not hasattr(self.model, "lora") or not hasattr(self.model, "I_pad"):
                raise ValueError("LoRA adapters are served for the Llama / Qwen decoders")
            self.model.lora = LoRAManager(self.model, config.lora.max_loras,
                                          config.lora.max_lora_rank)
        log.info("weights ready in %.1fs", time.time() - t0)
        self.sampler = Sampler(self.comm, getattr(self.model, "vocab_start", 0), st.tp_size)
        dcp = config.parallel.decode_context_parallel_size
        if dcp > 1:
            if not hasattr(self.model, "enable_dcp"):
                raise ValueError("decode context parallelism needs an MLA model (DeepSeek-V2/V3)")
            self.model.enable_dcp(dcp, config.cache.block_size)
        self.runner = ModelRunner(config, self.model, self.sampler, device)
        self.drafter = None  # model-based speculative proposer (MTP / EAGLE)
        num_blocks = self.runner.profile_and_allocate_kv()
        if st.mp_size > 1:
            # every rank of the replica must run with the same block count (lock-step
            # schedulers; pipeline stages hold different layer counts)
            t = torch.tensor([num_blocks], dtype=torch.int64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN, group=st.mp_cpu_group)
            if int(t) != num_blocks:
                num_blocks = int(t)
                self.runner.allocate_kv(num_blocks)
        self.num_blocks = num_blocks
        cap = num_blocks * config.cache.block_size * dcp
        if cap < config.scheduler.max_model_len:
            # a request of max_model_len tokens could never hold its blocks: it would be
            # preempted and re-admitted forever
            raise ValueError(f"the KV cache holds {cap} tokens ({num_blocks} blocks), fewer than "
                             f"max_model_len={config.scheduler.max_model_len}: lower "
                             f"max_model_len or give the cache more memory / blocks")
        sc = _native().SchedulerConfig()
        # with decode context parallelism a scheduler block spans dcp ranks' cache blocks
        sc.block_size = config.cache.block_size * dcp
        sc.max_num_seqs = config.scheduler.max_num_seqs
        sc.max_num_batched_tokens = config.scheduler.max_num_batched_tokens
        sc.max_model_len = config.scheduler.max_model_len
        sc.max_blocks_per_seq = self.runner.max_blocks
        sc.chunked_prefill = config.scheduler.enable_chunked_prefill
        # recurrent-state (hybrid) models cannot resume from cached KV blocks alone
        # (adapters change the KV of a prompt: no cross-request cache reuse with LoRA on)
        sc.prefix_caching = (config.cache.enable_prefix_caching
                             and self.contract.prefers(plan.Feature.PREFIX_CACHING)
                             and not hasattr(self.model, "allocate_state")
                             and not config.lora.enable_lora)
        sc.long_prefill_threshold = config.scheduler.long_prefill_token_threshold
        sc.priority_policy = config.scheduler.scheduling_policy == "priority"
        self._sched_cfg = sc
        self.scheduler = _native().Scheduler(sc, num_blocks, self.runner.buf.pointers())
        self.sleep_level = 0
        self._offloaded: list = []
        self._profiler = None
        if config.speculative.method == "mtp":
            from .spec_decode import MTPDrafter
            self.drafter = MTPDrafter(self, config.speculative.num_speculative_tokens or 1,
                                      config.speculative.tree_width)
        elif config.speculative.method == "eagle":
            from .spec_decode import EagleDrafter
            self.drafter = EagleDrafter(self, config.speculative.num_speculative_tokens or 1,
                                        config.speculative.tree_width)
        elif config.speculative.method == "medusa":
            from .spec_decode import MedusaDrafter
            self.drafter = MedusaDrafter(self, config.speculative.num_speculative_tokens or 1,
                                         config.speculative.tree_width)
        elif config.speculative.method == "eagle3":
            from .spec_decode import Eagle3Drafter
            self.drafter = Eagle3Drafter(self, config.speculative.num_speculative_tokens or 1,
                                         config.speculative.tree_width)
        self.runner.capture_graphs()
        self._ids = itertools.count()
        self._reqs: Dict[int, _Req] = {}
        self._by_name: Dict[str, int] = {}
        self._parents: Dict[str, dict] = {}
        self._special: Dict[int, _Req] = {}  # requests with penalties or logprobs
        self.step_end_times: List[float] = []
        self.stream_outputs = False
        self.num_steps = 0
        # multi-process TP without torchrun: the driver broadcasts request ops every step
        self.role = os.environ.get("B200_SPMD_ROLE", "replicated") if st.mp_size > 1 else "single"
        self.sync = None
        if self.role in ("driver", "follower"):
            from .executor import StepSync
            self.sync = StepSync(st.mp_cpu_group, st.mp_rank)

    # ------------------------------------------------------------------ requests
    def add_request(self, request_id: str, prompt_token_ids: List[int],
                    params: Optional[SamplingParams] = None, arrival_time: Optional[float] = None,
                    prompt: Optional[str] = None, lora_request=None, priority: int = 0) -> None:
        params = params or SamplingParams()
        k = getattr(params, "truncate_prompt_tokens", None)
        if k is not None and len(prompt_token_ids) > k:
            prompt_token_ids = list(prompt_token_ids)[-k:]
            prompt = None  # the text no longer matches the ids
        arrival = time.time() if arrival_time is None else arrival_time
        if self.sync is not None and self.role == "follower":
            raise RuntimeError("requests are added on the driver rank only")
        if lora_request is not None and getattr(self.model, "lora", None) is None:
            raise ValueError("lora_request needs LLM(..., enable_lora=True)")
        self._add_local(request_id, prompt_token_ids, params, arrival, prompt, lora_request,
                        priority)
        if self.sync is not None:  # followers replay only requests the driver accepted
            self.sync.record(("add", request_id, list(prompt_token_ids), params, arrival, prompt,
                              lora_request, priority))

    def _add_local(self, request_id, prompt_token_ids, params, arrival, prompt, lora_request,
                   priority) -> None:
        from ..sample.sampling_params import PoolingParams
        if isinstance(params, PoolingParams):
            self._add_one(request_id, prompt_token_ids,
                          SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True),
                          arrival, prompt, lora=lora_request, pooling=params, priority=priority)
            return
        if params.n > 1:
            self._parents[request_id] = {"n": params.n, "done": {}, "prompt_ids": prompt_token_ids,
                                         "prompt": prompt, "arrival": arrival}
            for k in range(params.n):
                child = SamplingParams(**{**params.__dict__, "n": 1})
                if params.seed is not None:
                    child.seed = params.seed + k
                self._add_one(f"{request_id}#{k}", prompt_token_ids, child, arrival, prompt,
                              parent=request_id, index=k, lora=lora_request, priority=priority)
            return
        self._add_one(request_id, prompt_token_ids, params, arrival, prompt, lora=lora_request,
                      priority=priority)

    def _add_one(self, name, prompt_ids, params, arrival, prompt, parent=None, index=0,
                 lora=None, pooling=None, priority=0):
        if name in self._by_name:
            raise ValueError(f"duplicate request id {name!r}")
        # every check that can reject the request comes before its internal id is taken: the
        # ranks of a tensor-parallel group draw ids in lock-step and only see accepted requests
        so = params.structured_outputs
        if (params.stop or params.bad_words) and self.tokenizer is None:
            raise ValueError("stop strings and bad words need the model's tokenizer")
        V = self.config.model.vocab_size
        for t in list(params.logit_bias or {}) + list(params.allowed_token_ids or []):
            if not 0 <= t < V:
                raise ValueError(f"token id {t} is outside the vocabulary (size {V})")
        if not prompt_ids:
            raise ValueError("empty prompt")
        if len(prompt_ids) >= self.config.scheduler.max_model_len:
            raise ValueError(f"prompt has {len(prompt_ids)} tokens; max_model_len is "
                             f"{self.config.scheduler.max_model_len}")
        matcher = self._grammar_backend().matcher(so) if so is not None else None
        bad_words_ids = self._bad_words_ids(params.bad_words) if params.bad_words else None
        lora_slot = self.model.lora.acquire(lora) if lora is not None else -1
        iid = next(self._ids)
        sp = _native().SamplingCfg()
        sp.max_tokens = params.max_tokens
        sp.min_tokens = params.min_tokens
        sp.ignore_eos = params.ignore_eos
        eos = self.config.model.eos_token_id
        sp.eos_id = -1 if eos is None else int(eos)
        sp.stop_ids = list(params.stop_token_ids)
        sp.temperature = params.temperature
        sp.top_k = params.top_k
        sp.top_p = params.top_p
        sp.min_p = params.min_p
        sp.seed = _mix_seed(self.config.seed, iid) if params.seed is None else int(params.seed)
        sp.priority = int(priority)
        special = params.has_penalties or params.logprobs is not None or so is not None or \
            bool(params.stop) or lora is not None or params.has_logits_processors or \
            params.prompt_logprobs is not None or pooling is not None
        # prompt log-probabilities and mean / cls pooling read every prompt row
        sp.no_prefix_cache = params.prompt_logprobs is not None or \
            (pooling is not None and pooling.pooling_type != "last")
        # with speculative decoding configured, these requests simply decode without drafts
        # (their penalties, log-probabilities, grammars, stop strings and adapters apply per
        # drawn token); the other requests of the batch keep theirs
        self.scheduler.add_request(iid, list(map(int, prompt_ids)), sp)
        r = _Req(name, iid, list(prompt_ids), params, arrival, prompt, parent, index)
        if params.logprobs is not None:
            r.logprobs = []
        if params.prompt_logprobs is not None:
            r.prompt_logprobs = [None]
        r.pooling = pooling
        r.matcher = matcher
        r.lora, r.lora_slot = lora, lora_slot
        r.bad_words_ids = bad_words_ids
        self._reqs[iid] = r
        self._by_name[name] = iid
        if special:
            self._special[iid] = r

    def _bad_words_ids(self, words) -> list:
        """Token sequences of each bad word: the word as written (leading spaces dropped) and,
        when it tokenizes to as many tokens with a different first token, with one leading
        space (the form it takes inside a sentence)."""
        def enc(text):
            try:
                return self.tokenizer.encode(text, add_special_tokens=False)
            except TypeError:  # tokenizers without the keyword add no special tokens
                return self.tokenizer.encode(text)

        out = []
        for w in words:
            base = enc(w.lstrip())
            if base:
                out.append(list(base))
            spaced = enc(" " + w.lstrip())
            if spaced and base and len(spaced) == len(base) and spaced[0] != base[0]:
                out.append(list(spaced))
        return out

    def _grammar_backend(self):
        """Structured-output grammar compiler over the model's vocabulary (created on the first
        constrained request; needs the tokenizer)."""
        if getattr(self, "_grammar", None) is None:
            from ..sample.structured import GrammarBackend
            tok = self.tokenizer
            if tok is None and self.config.model_path:
                from ..entrypoints.llm import _load_tokenizer
                tok = self.tokenizer = _load_tokenizer(self.config.model_path)
            self._grammar = GrammarBackend(tok, self.config.model.vocab_size,
                                           self.config.model.eos_token_id)
        return self._grammar

    def abort_request(self, request_id: str) -> None:
        if self.sync is not None and self.role == "driver":
            self.sync.record(("abort", request_id))
        names = [request_id] + [n for n in self._by_name if n.startswith(request_id + "#")]
        for n in names:
            iid = self._by_name.get(n)
            if iid is not None:
                self.scheduler.abort_request(iid)
                self._by_name.pop(n, None)
                r = self._reqs.pop(iid, None)
                if r is not None and r.lora is not None:
                    self.model.lora.release(r.lora.lora_int_id)
                self._special.pop(iid, None)
                self.scheduler.forget(iid)
        self._parents.pop(request_id, None)

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished()

    # ------------------------------------------------------------------ stepping
    def step(self) -> List[RequestOutput]:
        if self.sync is not None:
            ops_ = self.sync.exchange()
            if self.role == "follower":
                for op in ops_:
                    if op[0] == "add":
                        self._follower_add(*op[1:])
                    elif op[0] == "abort":
                        self.abort_request(op[1])
                    elif op[0] == "shutdown":
                        self._stop = True
                    elif op[0] == "sleep":
                        self._sleep_local(op[1])
                    elif op[0] == "wake":
                        self._wake_local()
            if not self.scheduler.has_unfinished():
                return []
        spec = self.config.speculative
        if spec.method == "ngram" and spec.num_speculative_tokens > 0:
            if spec.tree:
                self.scheduler.propose_ngram_tree(spec.num_speculative_tokens,
                                                  spec.prompt_lookup_min, spec.prompt_lookup_max,
                                                  spec.tree_width)
            else:
                self.scheduler.propose_ngram(spec.num_speculative_tokens,
                                             spec.prompt_lookup_min, spec.prompt_lookup_max)
        elif spec.method in ("mtp", "eagle", "eagle3", "medusa") and self.drafter is not None:
            self.drafter.propose(self.scheduler)
        if self._special and spec.method is not None:
            # penalties, log-probabilities and grammars are applied per drawn token: requests
            # that use them decode without drafts
            for iid in self._special:
                self.scheduler.set_draft(iid, [])
        plan = self.scheduler.schedule()
        if plan.num_reqs == 0:
            return []
        extras = self._step_extras(plan) if self._special else None
        sampled = self.runner.execute(plan, extras)
        if extras is not None and extras.logprobs is not None:
            self._record_logprobs(plan, extras, sampled)
        if extras is not None and extras.prompt_logprobs is not None:
            self._record_prompt_logprobs(extras)
        if extras is not None and extras.pooled is not None:
            self._record_pooled(extras)
        if extras is not None and extras.mask_rows:
            self._advance_grammars(plan, extras, sampled)
        finished = self.scheduler.update(sampled.data_ptr(), plan.num_samples)
        if plan.tree:  # accepted tree paths: KV rows to consecutive slots before the next step
            self.runner.apply_kv_moves(self.scheduler.take_kv_moves())
        if self._special:
            finished = self._match_stop_strings(plan, finished)
        now = time.time()
        self.step_end_times.append(now)
        self.num_steps += 1
        outs: List[RequestOutput] = []
        if self.drafter is not None:
            self.drafter.after_step(plan, sampled)
        if self.stream_outputs:
            for iid in plan.sample_req_ids:
                r = self._reqs.get(iid)
                if r is not None:
                    r.tokens = list(self.scheduler.output_tokens(iid))
                    if r.first_token_time is None:
                        r.first_token_time = now
            done = {iid for iid, _ in finished}
            for iid in plan.sample_req_ids:
                if iid not in done and iid in self._reqs:
                    outs.append(self._make_output(self._reqs[iid], None, False))
        for iid, reason in finished:
            self._special.pop(iid, None)
            r = self._reqs.pop(iid, None)
            if r is None:
                continue
            if r.lora is not None:
                self.model.lora.release(r.lora.lora_int_id)
            self._by_name.pop(r.request_id, None)
            o = self._finish(r, _REASONS.get(reason, "stop"))
            if o is not None:
                outs.append(o)
        return outs

    def _step_extras(self, plan):
        """Penalty entries and log-probability rows for this step's special requests (every
        rank builds the same ones: they depend only on the lock-step scheduler state)."""
        from ..ops.sampling import penalty_entries
        from .model_runner import StepExtras
        rows_tok, lp_rows, k = [], [], 0
        mask_rows, matchers = [], []
        S = plan.num_samples
        rep = torch.ones(S)
        pres = torch.zeros(S)
        freq = torch.zeros(S)
        row_req, nxt = {}, 0
        bias = []       # (row, token, value) added to the raw logits
        allowed = {}    # row -> allowed token ids
        for iid, cnt in zip(plan.sample_req_ids, plan.sample_counts):
            row, nxt = nxt, nxt + cnt  # the request's first sampling row
            r = self._special.get(iid)
            if r is None:
                continue
            row_req[row] = iid
            p = r.params
            if r.matcher is not None or p.allowed_token_ids:
                mask_rows.append(row)
                matchers.append(r.matcher)
                if p.allowed_token_ids:
                    allowed[len(mask_rows) - 1] = p.allowed_token_ids
            if p.logit_bias:
                bias.extend((row, t, v) for t, v in p.logit_bias.items())
            if r.bad_words_ids:
                out = self.scheduler.output_tokens(iid)
                for seq in r.bad_words_ids:
                    pre = seq[:-1]
                    if not pre or (len(out) >= len(pre) and list(out[len(out) - len(pre):]) == pre):
                        bias.append((row, seq[-1], float("-inf")))
            if p.has_penalties:
                n = self.scheduler.num_tokens(iid)
                toks = self.scheduler.tokens_range(iid, 0, n)
                np_ = len(r.prompt_token_ids)
                rows_tok.append((row, toks[:np_], toks[np_:]))
                rep[row], pres[row], freq[row] = (p.repetition_penalty, p.presence_penalty,
                                                  p.frequency_penalty)
            if p.logprobs is not None:
                lp_rows.append(row)
                k = max(k, p.logprobs)
        plp = self._prompt_logprob_rows(plan)
        pool = self._pool_rows(plan)
        lora = self._lora_batch(plan)
        if not rows_tok and not lp_rows and not mask_rows and lora is None and not bias and \
                plp is None and not pool:
            return None
        entries = penalty_entries(rows_tok) if rows_tok else None
        bitmask = self._token_masks(matchers, allowed) if matchers else None
        ex = StepExtras(entries, rep, pres, freq, lp_rows, k, bitmask, mask_rows)
        ex.lora = lora
        ex.row_req = row_req
        ex.plp = plp
        ex.pool = pool
        if bias:
            ex.bias = (torch.tensor([b[0] for b in bias], dtype=torch.int64),
                       torch.tensor([b[1] for b in bias], dtype=torch.int64),
                       torch.tensor([b[2] for b in bias], dtype=torch.float32))
        return ex

    def _prompt_logprob_rows(self, plan):
        """Step rows whose next token is a prompt token of a request asking for prompt
        log-probabilities: (rows, target tokens, top-k, [(request id, row count)]) or None."""
        if not any(r.prompt_logprobs is not None for r in self._special.values()):
            return None
        h = self.runner.buf.h
        cu = h["cu_q"][:plan.num_reqs + 1].tolist()
        pos = h["positions"]
        rows, targets, owners, k = [], [], [], 0
        for i, iid in enumerate(plan.req_ids):
            r = self._special.get(iid)
            if r is None or r.prompt_logprobs is None:
                continue
            P = len(r.prompt_token_ids)
            have = len(r.prompt_logprobs)  # positions already recorded (a recompute repeats)
            start = int(pos[cu[i]])
            n = 0
            for j in range(cu[i + 1] - cu[i]):
                p = start + j  # this row predicts token p + 1
                if p + 1 >= P:
                    break
                if p + 1 < have:
                    continue
                rows.append(cu[i] + j)
                targets.append(r.prompt_token_ids[p + 1])
                n += 1
            if n:
                owners.append((iid, n))
                k = max(k, r.params.prompt_logprobs)
        if not rows:
            return None
        return (torch.tensor(rows, dtype=torch.int64), torch.tensor(targets, dtype=torch.int64),
                k, owners)

    def _pool_rows(self, plan) -> list:
        """Step rows each embedding request pools: [(request id, first row, end row)] --
        the last prompt row (last), the prompt rows of the step (mean), the first (cls)."""
        if not any(r.pooling is not None for r in self._special.values()):
            return []
        h = self.runner.buf.h
        cu = h["cu_q"][:plan.num_reqs + 1].tolist()
        pos = h["positions"]
        out = []
        for i, iid in enumerate(plan.req_ids):
            r = self._special.get(iid)
            if r is None or r.pooling is None:
                continue
            P = len(r.prompt_token_ids)
            start = int(pos[cu[i]])
            q = cu[i + 1] - cu[i]
            kind = r.pooling.pooling_type
            if kind == "last" and start <= P - 1 < start + q:
                a = cu[i] + (P - 1 - start)
                out.append((iid, a, a + 1))
            elif kind == "mean" and start < P:
                out.append((iid, cu[i], cu[i] + min(q, P - start)))
            elif kind == "cls" and start == 0:
                out.append((iid, cu[i], cu[i] + 1))
        return out

    def _record_pooled(self, extras) -> None:
        for (iid, a, b), v in zip(extras.pool, extras.pooled):
            r = self._reqs.get(iid)
            if r is None:
                continue
            r.pool_sum = v if r.pool_sum is None else r.pool_sum + v
            r.pool_n += b - a

    def _embedding(self, r) -> list:
        pp = r.pooling
        v = r.pool_sum / max(1, r.pool_n) if pp.pooling_type == "mean" else r.pool_sum
        if pp.dimensions is not None:
            v = v[:pp.dimensions]
        if pp.normalize:
            v = v / v.norm().clamp_min(1e-12)
        return v.tolist()

    def _record_prompt_logprobs(self, extras) -> None:
        from ..outputs import Logprob
        ids, vals, tok_lp, rank = (t.tolist() for t in extras.prompt_logprobs)
        at = 0
        for iid, n in extras.plp[3]:
            r = self._reqs.get(iid)
            for j in range(at, at + n):
                if r is None:
                    continue
                tok = extras.plp[1][j].item()
                d = {tok: Logprob(tok_lp[j], int(rank[j]))}
                for m in range(r.params.prompt_logprobs):
                    if ids[j][m] not in d:
                        d[ids[j][m]] = Logprob(vals[j][m], m + 1)
                r.prompt_logprobs.append(d)
            at += n

    def _token_masks(self, matchers, allowed) -> torch.Tensor:
        """int32 [len(matchers), words] next-token bitmasks: a grammar's mask where the row has
        a matcher (all tokens otherwise), ANDed with the row's allowed_token_ids."""
        words = (self.config.model.vocab_size + 31) // 32
        if any(m is not None for m in matchers):
            gb = self._grammar_backend()
            words = gb.words
            bm = torch.full((len(matchers), words), -1, dtype=torch.int32)
            for i, m in enumerate(matchers):
                if m is not None:
                    m.fill_next_token_bitmask(bm, i)
        else:
            bm = torch.full((len(matchers), words), -1, dtype=torch.int32)
        for i, ids in allowed.items():
            row = torch.zeros(words * 32, dtype=torch.bool)
            row[torch.tensor(ids, dtype=torch.long)] = True
            bits = row.view(words, 32).to(torch.int64) << torch.arange(32, dtype=torch.int64)
            packed = bits.sum(1)
            packed = torch.where(packed >= 2 ** 31, packed - 2 ** 32, packed).to(torch.int32)
            bm[i] &= packed
        return bm

    def _lora_batch(self, plan):
        """Token indices of this step grouped by adapter slot (None: no adapter in the step)."""
        if getattr(self.model, "lora", None) is None:
            return None
        from ..lora import LoRABatch
        cu = self.runner.buf.h["cu_q"][:plan.num_reqs + 1].tolist()
        by_slot = {}
        for i, iid in enumerate(plan.req_ids):
            r = self._reqs.get(iid)
            if r is not None and r.lora_slot >= 0:
                by_slot.setdefault(r.lora_slot, []).extend(range(cu[i], cu[i + 1]))
        if not by_slot:
            return None
        dev = self.runner.device
        return LoRABatch([(s, torch.tensor(t, dtype=torch.long, device=dev))
                          for s, t in sorted(by_slot.items())])

    def _match_stop_strings(self, plan, finished):
        """Finish (reason "stop") every request whose output text now contains one of its stop
        strings; its text is cut before the string (kept with include_stop_str_in_output).
        Every rank decides the same: the tokens are lock-step."""
        done = {iid for iid, _ in finished}
        extra = []
        for iid in plan.sample_req_ids:
            r = self._special.get(iid)
            if r is None or not r.params.stop or iid in done:
                continue
            text = self.tokenizer.decode(list(self.scheduler.output_tokens(iid)),
                                         skip_special_tokens=True)
            # the newest token can complete a stop string that starts up to len - 1 chars back
            hits = [(text.find(s), s) for s in r.params.stop if s in text]
            if not hits:
                continue
            at, s = min(hits)
            keep = at + len(s) if r.params.include_stop_str_in_output else at
            r.stop_hit = (s, text[:keep])
            self.scheduler.abort_request(iid)
            extra.append((iid, 2))  # reason code 2 = "stop"
        return list(finished) + extra

    def _advance_grammars(self, plan, extras, sampled) -> None:
        """Feed each constrained request's sampled token to its matcher."""
        for row in extras.mask_rows:
            r = self._reqs.get(extras.row_req[row])
            if r is None or r.matcher is None:
                continue
            tok = int(sampled[row])
            if not r.matcher.is_terminated() and not r.matcher.accept_token(tok):
                log.warning("request %s: token %d rejected by its grammar", r.request_id, tok)

    def _record_logprobs(self, plan, extras, sampled) -> None:
        from ..outputs import Logprob
        ids, vals, tok_lp, rank = (t.tolist() for t in extras.logprobs)
        for j, row in enumerate(extras.lp_rows):
            r = self._reqs.get(extras.row_req[row])
            if r is None or r.logprobs is None:
                continue
            tok = int(sampled[row])
            d = {tok: Logprob(tok_lp[j], int(rank[j]))}
            for m in range(r.params.logprobs):
                if ids[j][m] not in d:
                    d[ids[j][m]] = Logprob(vals[j][m], m + 1)
            r.logprobs.append(d)
            r.cum_logprob += tok_lp[j]

    def _step_time(self, step: int) -> Optional[float]:
        # scheduler steps are 1-based and one engine step == one scheduler step
        if step is None or step < 1 or step > len(self.step_end_times):
            return None
        return self.step_end_times[step - 1]

    def _finish(self, r: _Req, reason: str) -> Optional[RequestOutput]:
        info = self.scheduler.request_info(r.int_id)
        toks = self.scheduler.output_tokens(r.int_id)
        self.scheduler.forget(r.int_id)
        r.tokens = list(toks)
        first = self._step_time(info["first_token_step"]) if info else None
        last = self._step_time(info["finish_step"]) if info else None
        out = self._make_output(r, reason, True, first, last)
        if r.parent is None:
            return out
        par = self._parents.get(r.parent)
        if par is None:
            return None
        par["done"][r.index] = out
        if len(par["done"]) < par["n"]:
            return None
        del self._parents[r.parent]
        comps = [par["done"][k].outputs[0] for k in range(par["n"])]
        ftimes = [par["done"][k].metrics.first_token_time for k in range(par["n"])]
        ltimes = [par["done"][k].metrics.finished_time for k in range(par["n"])]
        m = RequestMetrics(par["arrival"], min([t for t in ftimes if t] or [None]) if any(ftimes) else None,
                           max([t for t in ltimes if t] or [None]) if any(ltimes) else None)
        out = RequestOutput(r.parent, par["prompt_ids"], comps, True, par["prompt"], m)
        out.prompt_logprobs = par["done"][0].prompt_logprobs
        return out

    def _decode(self, ids, params) -> str:
        kw = {"skip_special_tokens": params.skip_special_tokens}
        if not params.spaces_between_special_tokens:
            kw["spaces_between_special_tokens"] = False
        try:
            return self.tokenizer.decode(ids, **kw)
        except TypeError:  # tokenizers without the spacing option
            return self.tokenizer.decode(ids, skip_special_tokens=params.skip_special_tokens)

    def _make_output(self, r: _Req, reason, finished, first=None, last=None) -> RequestOutput:
        text = ""
        if self.tokenizer is not None and r.params.detokenize:
            try:
                text = self._decode(r.tokens, r.params)
            except Exception:  # pragma: no cover - tokenizer specific
                text = ""
        stop_reason = None
        if r.stop_hit is not None:
            stop_reason, text = r.stop_hit
        comp = CompletionOutput(r.index, list(r.tokens), text, reason,
                                cumulative_logprob=r.cum_logprob if r.logprobs is not None else None,
                                logprobs=list(r.logprobs) if r.logprobs is not None else None,
                                stop_reason=stop_reason)
        m = RequestMetrics(r.arrival, first if first is not None else r.first_token_time, last)
        out = RequestOutput(r.request_id, r.prompt_token_ids, [comp], finished, r.prompt, m)
        if r.prompt_logprobs is not None:
            out.prompt_logprobs = list(r.prompt_logprobs)
        if r.pooling is not None and finished and r.pool_sum is not None:
            out.embedding = self._embedding(r)
        return out

    def _follower_add(self, request_id, prompt_ids, params, arrival, prompt, lora_request=None,
                      priority=0):
        sync, self.sync = self.sync, None  # apply locally without re-recording
        try:
            self.add_request(request_id, prompt_ids, params, arrival, prompt, lora_request,
                             priority)
        finally:
            self.sync = sync

    def follow(self) -> None:
        """Follower rank main loop: mirror the driver's steps until it shuts down."""
        self._stop = False
        while not self._stop:
            self.step()

    def stop_followers(self) -> None:
        if self.sync is not None and self.role == "driver":
            self.sync.record(("shutdown",))
            self.sync.exchange()
            self.sync = None

    def _load_weights(self) -> None:
        cfg, mcfg, device = self.config, self.config.model, self.device
        if cfg.load_format == "dummy":
            dev = str(device) if device.type == "cuda" else "cpu"
            self.model.load_weights(dummy_weights(mcfg, cfg.seed, cfg.init_std, device=dev))
        else:
            self.model.load_weights(safetensors_weights(cfg.model_path))

    def _load_medusa(self) -> None:
        """Attach Medusa heads: as many as the checkpoint has, or (random init) one per chained
        draft / four for a tree."""
        import re as _re
        from ..models.medusa import MedusaHeads, medusa_param_shapes
        cfg, mcfg, device = self.config, self.config.model, self.device
        spec = cfg.speculative
        path = spec.model
        if path:
            st = list(safetensors_weights(path))
            n = 1 + max(int(m.group(1)) for m in
                        (_re.match(r"blocks\.(\d+)\.", name) for name, _ in st) if m)
        else:
            n = spec.num_speculative_tokens if spec.tree_width == 1 else \
                min(4, spec.num_speculative_tokens)
            dev = str(device) if device.type == "cuda" else "cpu"
            st = dummy_weights(mcfg, cfg.seed + 1, cfg.init_std, device=dev,
                               shapes=medusa_param_shapes(mcfg, n))
        heads = MedusaHeads(self.model, n)
        heads.load_weights(st)
        self.model.medusa = heads

    def _load_eagle3(self) -> None:
        """Attach an EAGLE-3 head (whole on this rank, its own KV cache) and make the model
        record the residual streams the head reads."""
        from ..models.eagle import Eagle3Head, eagle3_param_shapes
        cfg, mcfg, device = self.config, self.config.model, self.device
        if not hasattr(self.model, "enable_aux"):
            raise ValueError("EAGLE-3 heads are served over the dense decoders (Llama / Qwen)")
        head = Eagle3Head(self.model)
        path = cfg.speculative.model
        if path:
            head.load_weights(safetensors_weights(path))
        else:
            dev = str(device) if device.type == "cuda" else "cpu"
            head.load_weights(dummy_weights(mcfg, cfg.seed + 1, cfg.init_std, device=dev,
                                            shapes=eagle3_param_shapes(mcfg)))
        self.model.enable_aux(head.aux_layers, cfg.scheduler.max_num_batched_tokens)
        self.model.draft_head = head

    def _load_eagle(self) -> None:
        """Attach an EAGLE head to the dense decoder (its KV is one extra cache layer)."""
        from ..models.eagle import EagleHead, eagle_param_shapes
        cfg, mcfg, device = self.config, self.config.model, self.device
        dtp = cfg.speculative.draft_tensor_parallel_size
        tp = cfg.parallel.tensor_parallel_size
        if dtp not in (None, 1, tp):
            raise ValueError(f"draft_tensor_parallel_size must be 1 or {tp} (the target's)")
        head = EagleHead(self.model, replicated=dtp == 1)
        path = cfg.speculative.model
        if path:
            head.load_weights(safetensors_weights(path))
        else:
            dev = str(device) if device.type == "cuda" else "cpu"
            head.load_weights(dummy_weights(mcfg, cfg.seed + 1, cfg.init_std, device=dev,
                                            shapes=eagle_param_shapes(mcfg)))
        self.model.draft_head = head

    # ------------------------------------------------------------------ sleep mode
    def _weight_tensors(self) -> list:
        """Every tensor the model object graph holds on the engine's device (weights, rotary
        tables), unique by identity.  Communicator / parallel-state objects are not walked:
        their peer-mapped buffers must stay where the other ranks mapped them."""
        out, seen, stack = [], set(), [self.model]
        while stack:
            o = stack.pop()
            if id(o) in seen:
                continue
            seen.add(id(o))
            if isinstance(o, torch.Tensor):
                if o.device == self.device and o.numel():
                    out.append(o)
            elif isinstance(o, (list, tuple)):
                stack.extend(o)
            elif isinstance(o, dict):
                stack.extend(o.values())
            elif type(o).__module__.startswith(("vllm_musa_b200.models", "vllm_musa_b200.attention")):
                if hasattr(o, "__dict__"):
                    stack.extend(vars(o).values())
                for slot in getattr(type(o), "__slots__", ()):
                    stack.append(getattr(o, slot, None))
        return out

    def sleep(self, level: int = 1) -> None:
        """Give the GPU memory back while the engine idles: level 1 copies the weights to
        host memory, level 2 discards them (``wake_up`` loads them again); both release the
        KV cache and the CUDA graphs (their contents are discarded, the prefix cache starts
        empty after waking).  Reference: the platform declares vLLM's sleep mode available
        (vllm_musa/platform.py:274-276).  Only between requests; recurrent-state models
        (Qwen3-Next, Mamba2) keep their state buffers and are refused.  With spawned follower
        ranks the driver forwards the call, so every rank releases (and later restores) its
        shards in the same step."""
        if level not in (1, 2):
            raise ValueError("sleep level must be 1 or 2")
        if self.sleep_level:
            return
        if self.has_unfinished_requests():
            raise RuntimeError("sleep() needs an idle engine (requests still running)")
        if hasattr(self.model, "allocate_state"):
            raise NotImplementedError("sleep mode does not cover recurrent-state models")
        if self.sync is not None and self.role == "driver":
            self.sync.record(("sleep", level))
            self.sync.exchange()
        self._sleep_local(level)

    def _sleep_local(self, level: int) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self.runner.release_graphs()
        # one entry per storage: views that share a storage (a fused weight and slices of it
        # kept as separate attributes) are offloaded once and re-seated on the same restored
        # storage, so waking neither grows memory nor splits the aliasing
        groups: dict = {}
        for t in self._weight_tensors():
            st = t.untyped_storage()
            g = groups.setdefault(st.data_ptr(), {"storage": st, "views": []})
            g["views"].append((t, t.storage_offset(), tuple(t.shape), tuple(t.stride())))
        self._offloaded, self._discarded = [], []
        for g in groups.values():
            st = g["storage"]
            nbytes = st.nbytes()
            # level 2 discards the large storages (the checkpoint weights, which the loader
            # re-creates); small ones (norms, rotary tables) are kept on the host either way
            if level == 1 or nbytes < (16 << 20):
                whole = torch.empty(0, dtype=torch.uint8, device=self.device).set_(st)
                host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=self.device.type == "cuda")
                host.copy_(whole)
                self._offloaded.append((host, g["views"]))
                del whole
            else:
                self._discarded.extend(t for t, _, _, _ in g["views"])
            for t, _, _, _ in g["views"]:
                t.data = torch.empty(0, dtype=t.dtype, device=t.device)
        groups.clear()
        self.runner.kv_caches = []
        self.runner.kv_tensor = None
        self.sleep_level = level
        if self.device.type == "cuda":
            torch.cuda.empty_cache()
        log.info("engine asleep (level %d)", level)

    def wake_up(self) -> None:
        """Undo ``sleep``: weights back (host copy or a fresh load), a new KV cache of the same
        block count, a fresh scheduler (empty prefix cache) and re-captured CUDA graphs (every
        rank at once: graph capture runs the tensor-parallel collectives)."""
        if not self.sleep_level:
            return
        if self.sync is not None and self.role == "driver":
            self.sync.record(("wake",))
            self.sync.exchange()
        self._wake_local()

    def _wake_local(self) -> None:
        for host, views in self._offloaded:
            dev = host.to(self.device, non_blocking=False)
            st = dev.untyped_storage()
            for t, off, shape, stride in views:
                t.data = torch.empty(0, dtype=t.dtype, device=self.device).set_(
                    st, off, shape, stride)
        self._offloaded = []
        if self.sleep_level == 2:
            self._load_weights()
            live = {id(t) for t in self._weight_tensors()}
            # a discarded tensor the loader did not replace is still reachable (and empty)
            lost = [t for t in self._discarded if id(t) in live]
            self._discarded = []
            if lost:
                raise RuntimeError(f"wake_up: {len(lost)} discarded tensors were not re-created "
                                   "by the weight loader; use sleep(level=1) for this model")
        self.runner.allocate_kv(self.num_blocks)
        self.scheduler = _native().Scheduler(self._sched_cfg, self.num_blocks,
                                              self.runner.buf.pointers())
        self.sleep_level = 0
        self.runner.capture_graphs()
        log.info("engine awake")

    # ------------------------------------------------------------------ profiling
    def start_profile(self) -> None:
        """torch.profiler over the following steps (CPU ops + CUDA kernels); ``stop_profile``
        writes a Chrome trace per rank under ``B200_TORCH_PROFILER_DIR``.  Reference: the
        reference extends vLLM's torch profiler with its device activity."""
        import torch.profiler as tp
        acts = [tp.ProfilerActivity.CPU]
        if self.device.type == "cuda":
            acts.append(tp.ProfilerActivity.CUDA)
        self._profiler = tp.profile(activities=acts)
        self._profiler.__enter__()

    def stop_profile(self) -> Optional[str]:
        if self._profiler is None:
            return None
        from .. import envs
        prof, self._profiler = self._profiler, None
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        prof.__exit__(None, None, None)
        d = envs.FLAGS["B200_TORCH_PROFILER_DIR"].get()
        os.makedirs(d, exist_ok=True)
        rank = torch.distributed.get_rank() if torch.distributed.is_initialized() else 0
        path = os.path.join(d, f"trace_rank{rank}_{int(time.time() * 1000)}.json")
        prof.export_chrome_trace(path)
        return path

    # ------------------------------------------------------------------ lifecycle
    def shutdown(self) -> None:
        self.stop_followers()
        self.runner.release_graphs()
        if self.comm is not None and hasattr(self.comm, "close"):
            self.comm.close()
