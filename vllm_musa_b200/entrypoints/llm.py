"""Offline inference API: ``LLM(...).generate(prompts, sampling_params)``.

Same call shape as vLLM's ``LLM`` (the surface the reference's users drive through
``vllm serve`` / ``LLM()``): prompts may be strings (tokenised with the model's tokenizer),
token-id lists, or ``{"prompt_token_ids": [...]}`` / ``{"prompt": "..."}`` dicts.
With ``tensor_parallel_size > 1`` run one process per GPU under ``torchrun``; every rank
calls ``generate`` with the same prompts and receives the same outputs.
"""
from __future__ import annotations

import os
from typing import List, Optional, Sequence, Union

from ..config import (CacheConfig, EngineConfig, LoRAConfig, ModelConfig, ParallelConfig,
                      SchedulerConfig, SpeculativeConfig)
from ..engine.llm_engine import LLMEngine
from ..models.presets import PRESETS, get_preset
from ..outputs import RequestOutput
from ..sample.sampling_params import SamplingParams

PromptType = Union[str, List[int], dict]


def _load_tokenizer(path: Optional[str]):
    if not path or not os.path.isdir(path):
        return None
    try:
        from transformers import AutoTokenizer
        return AutoTokenizer.from_pretrained(path)
    except Exception:  # pragma: no cover - optional
        return None


class LLM:
    def __init__(self, model: Union[str, ModelConfig, None] = None, *,
                 tensor_parallel_size: int = 1, pipeline_parallel_size: int = 1,
                 enable_expert_parallel: bool = False,
                 decode_context_parallel_size: int = 1, data_parallel_size: int = 1,
                 max_model_len: Optional[int] = None, max_num_seqs: int = 256,
                 max_num_batched_tokens: int = 8192, block_size: int = 64,
                 gpu_memory_utilization: float = 0.90, num_gpu_blocks: Optional[int] = None,
                 enable_prefix_caching: bool = True, enable_chunked_prefill: bool = True,
                 enforce_eager: bool = False, seed: int = 0, load_format: Optional[str] = None,
                 device: str = "cuda", dtype=None, tokenizer=None,
                 cuda_graph_sizes: Optional[list] = None, num_layers: Optional[int] = None,
                 speculative_config: Optional[dict] = None,
                 enable_lora: bool = False, max_loras: int = 4, max_lora_rank: int = 64,
                 kv_cache_dtype: Optional[str] = None, logprobs_mode: str = "raw_logprobs",
                 scheduling_policy: str = "fcfs", **unused):
        path = None
        if isinstance(model, ModelConfig):
            mcfg = model
        elif isinstance(model, str) and model.lower() in PRESETS:
            mcfg = get_preset(model)
        elif isinstance(model, str):
            path = model
            mcfg = ModelConfig.from_hf(model)
        else:
            raise ValueError("model must be a preset name, a checkpoint directory or a ModelConfig")
        if dtype is not None:
            mcfg.dtype = dtype
        if num_layers is not None:
            mcfg.num_layers = num_layers
        if kv_cache_dtype is not None:
            mcfg.kv_cache_dtype = kv_cache_dtype
        if load_format is None:
            load_format = "safetensors" if path else "dummy"
        mlen = max_model_len or min(mcfg.max_position, 8192)
        cfg = EngineConfig(
            model=mcfg,
            cache=CacheConfig(block_size=block_size, gpu_memory_utilization=gpu_memory_utilization,
                              num_gpu_blocks=num_gpu_blocks,
                              enable_prefix_caching=enable_prefix_caching),
            scheduler=SchedulerConfig(max_num_seqs=max_num_seqs,
                                      max_num_batched_tokens=max(max_num_batched_tokens, max_num_seqs),
                                      max_model_len=mlen,
                                      enable_chunked_prefill=enable_chunked_prefill,
                                      scheduling_policy=scheduling_policy),
            parallel=ParallelConfig(tensor_parallel_size=tensor_parallel_size,
                                    pipeline_parallel_size=pipeline_parallel_size,
                                    enable_expert_parallel=enable_expert_parallel,
                                    decode_context_parallel_size=decode_context_parallel_size,
                                    data_parallel_size=data_parallel_size),
            device=device, seed=seed, load_format=load_format, model_path=path,
            enforce_eager=enforce_eager, cuda_graph_sizes=cuda_graph_sizes,
            speculative=SpeculativeConfig.from_dict(speculative_config),
            lora=LoRAConfig(enable_lora=enable_lora, max_loras=max_loras,
                            max_lora_rank=max_lora_rank),
            logprobs_mode=logprobs_mode)
        tok = tokenizer if tokenizer is not None else _load_tokenizer(path)
        self.executor = None
        self.dp_size, self.dp_rank = 1, 0
        if data_parallel_size > 1:
            # data parallelism: WORLD_SIZE = dp x tp ranks under one launcher; ranks
            # [k*tp, (k+1)*tp) run engine replica k (its own TP group, KV cache and scheduler)
            # and generate() splits the prompts over the replicas
            world = int(os.environ.get("WORLD_SIZE", "1"))
            mp = tensor_parallel_size * pipeline_parallel_size
            if world != data_parallel_size * mp:
                raise ValueError("data_parallel_size > 1 needs WORLD_SIZE == data_parallel_size"
                                 " * tensor_parallel_size * pipeline_parallel_size (torchrun)")
            from ..parallel.state import init_distributed
            st = init_distributed(tp_size=tensor_parallel_size,
                                  ep=enable_expert_parallel,
                                  backend="nccl" if device == "cuda" else "gloo",
                                  pp_size=pipeline_parallel_size)
            self.dp_size, self.dp_rank = st.dp_size, st.dp_rank
        mp = tensor_parallel_size * pipeline_parallel_size
        if mp > 1 and "WORLD_SIZE" not in os.environ:
            # no launcher: spawn follower ranks and drive them from this process
            from ..engine.executor import MultiprocExecutor
            self.executor = MultiprocExecutor(cfg, mp)
        self.engine = LLMEngine(cfg, tok)
        self._counter = 0

    def get_tokenizer(self):
        return self.engine.tokenizer

    def _prompt_ids(self, p: PromptType):
        if isinstance(p, dict):
            if "prompt_token_ids" in p:
                return list(p["prompt_token_ids"]), p.get("prompt")
            p = p["prompt"]
        if isinstance(p, str):
            tok = self.engine.tokenizer
            if tok is None:
                raise ValueError("string prompts need a tokenizer (checkpoint directory); "
                                 "pass token ids for preset / random-weight models")
            return tok.encode(p), p
        return list(p), None

    def generate(self, prompts: Union[PromptType, Sequence[PromptType]],
                 sampling_params: Union[SamplingParams, Sequence[SamplingParams], None] = None,
                 use_tqdm: bool = False, lora_request=None,
                 priority: Optional[List[int]] = None) -> List[RequestOutput]:
        """``lora_request``: one LoRARequest for every prompt, or a list with one (or None)
        per prompt.  ``priority``: one int per prompt (lower first) under
        ``scheduling_policy="priority"``."""
        if isinstance(prompts, (str, dict)) or (isinstance(prompts, list) and prompts and
                                                isinstance(prompts[0], int)):
            prompts = [prompts]
        if sampling_params is None:
            sampling_params = SamplingParams()
        if isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params] * len(prompts)
        loras = lora_request if isinstance(lora_request, (list, tuple)) else \
            [lora_request] * len(prompts)
        if self.dp_size > 1:
            if any(x is not None for x in loras):
                raise ValueError("LoRA with data parallelism is not served")
            return self._generate_dp(prompts, sampling_params)
        prios = list(priority) if priority is not None else [0] * len(prompts)
        if len(prios) != len(prompts):
            raise ValueError("priority needs one value per prompt")
        order = []
        for p, sp, lr, pr in zip(prompts, sampling_params, loras, prios):
            ids, text = self._prompt_ids(p)
            rid = str(self._counter)
            self._counter += 1
            self.engine.add_request(rid, ids, sp, prompt=text, lora_request=lr, priority=pr)
            order.append(rid)
        done = {}
        while self.engine.has_unfinished_requests():
            for o in self.engine.step():
                if o.finished:
                    done[o.request_id] = o
        return [done[r] for r in order]

    def chat(self, messages, sampling_params: Union[SamplingParams, Sequence[SamplingParams],
                                                    None] = None,
             lora_request=None, add_generation_prompt: bool = True) -> List[RequestOutput]:
        """Chat completion offline: ``messages`` is one conversation ([{"role", "content"}, ...])
        or a list of conversations; each is rendered with the tokenizer's chat template (a
        ``role: content`` transcript without one) and generated like ``generate``."""
        from .chat_utils import chat_prompt_ids
        convs = [messages] if messages and isinstance(messages[0], dict) else list(messages)
        tok = self.engine.tokenizer
        prompts = [{"prompt_token_ids": chat_prompt_ids(tok, c, add_generation_prompt)}
                   for c in convs]
        return self.generate(prompts, sampling_params, lora_request=lora_request)

    def embed(self, prompts, pooling_params=None, use_tqdm: bool = False) -> list:
        """Embeddings of the prompts (vLLM's ``LLM.embed``): each prompt runs once and its final
        hidden states are pooled per ``pooling_params`` (PoolingParams: last token by default,
        L2-normalised).  Returns EmbeddingRequestOutput objects (``.outputs.embedding``)."""
        from ..outputs import EmbeddingOutput, EmbeddingRequestOutput
        from ..sample.sampling_params import PoolingParams
        if isinstance(prompts, (str, dict)) or (isinstance(prompts, list) and prompts and
                                                isinstance(prompts[0], int)):
            prompts = [prompts]
        pp = pooling_params or PoolingParams()
        pps = pp if isinstance(pp, (list, tuple)) else [pp] * len(prompts)
        order = []
        for p, q in zip(prompts, pps):
            ids, text = self._prompt_ids(p)
            rid = str(self._counter)
            self._counter += 1
            self.engine.add_request(rid, ids, q, prompt=text)
            order.append((rid, ids))
        done = {}
        while self.engine.has_unfinished_requests():
            for o in self.engine.step():
                if o.finished:
                    done[o.request_id] = o
        return [EmbeddingRequestOutput(rid, ids, EmbeddingOutput(done[rid].embedding))
                for rid, ids in order]

    encode = embed

    def beam_search(self, prompts, params) -> list:
        """Beam search over the engine (vLLM's ``LLM.beam_search``): each step runs every live
        beam of every prompt as a one-token request with the top 2 x beam_width
        log-probabilities (prefix caching serves the shared prefixes), keeps the best
        beam_width continuations per prompt and sets aside the finished ones.  Returns one
        BeamSearchOutput per prompt with its best beam_width sequences, best first."""
        from ..outputs import BeamSearchOutput, BeamSearchSequence
        if isinstance(prompts, (str, dict)) or (isinstance(prompts, list) and prompts and
                                                isinstance(prompts[0], int)):
            prompts = [prompts]
        w = params.beam_width
        eos = self.engine.config.model.eos_token_id
        base = [self._prompt_ids(p)[0] for p in prompts]
        live = [[([], [], 0.0)] for _ in base]      # per prompt: (generated, logprobs, cum)
        done = [[] for _ in base]
        step_sp = SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True, logprobs=2 * w)

        def score(prompt_len, gen, cum):
            n = prompt_len + len(gen) - (1 if gen and eos is not None and gen[-1] == eos else 0)
            return cum / (max(n, 1) ** params.length_penalty)

        for _ in range(params.max_tokens):
            jobs = [(i, b) for i, beams in enumerate(live) for b in beams]
            if not jobs:
                break
            outs = self.generate([{"prompt_token_ids": base[i] + b[0]} for i, b in jobs],
                                 step_sp)
            cands = [[] for _ in base]
            for (i, (gen, lps, cum)), o in zip(jobs, outs):
                for tok, lp in o.outputs[0].logprobs[0].items():
                    cands[i].append((gen + [tok], lps + [lp.logprob], cum + lp.logprob))
            for i, cs in enumerate(cands):
                cs.sort(key=lambda c: c[2], reverse=True)
                keep = []
                for c in cs:
                    if not params.ignore_eos and eos is not None and c[0][-1] == eos:
                        done[i].append(c)
                    else:
                        keep.append(c)
                    if len(keep) == w:
                        break
                live[i] = keep
        tok = self.engine.tokenizer
        res = []
        for i, p in enumerate(base):
            allb = done[i] + live[i]
            allb.sort(key=lambda c: score(len(p), c[0], c[2]), reverse=True)
            seqs = []
            for gen, lps, cum in allb[:w]:
                text = tok.decode(gen, skip_special_tokens=True) if tok is not None else None
                fin = "stop" if (eos is not None and gen and gen[-1] == eos and
                                 not params.ignore_eos) else "length"
                seqs.append(BeamSearchSequence(list(p) + gen, lps, cum, text, fin))
            res.append(BeamSearchOutput(seqs))
        return res

    def _generate_dp(self, prompts, sampling_params) -> List[RequestOutput]:
        """Replica k serves prompts k, k + dp, ...; the outputs are exchanged over the world
        group so every rank returns the full list in prompt order."""
        import torch.distributed as dist
        k, n = self.dp_rank, self.dp_size
        mine = list(range(k, len(prompts), n))
        saved, self.dp_size = self.dp_size, 1
        try:
            outs = self.generate([prompts[i] for i in mine], [sampling_params[i] for i in mine])
        finally:
            self.dp_size = saved
        parts = [None] * dist.get_world_size()
        dist.all_gather_object(parts, (k, mine, outs))
        res: List[Optional[RequestOutput]] = [None] * len(prompts)
        seen = set()
        for rep, idx, o in parts:
            if rep in seen:  # every TP rank of a replica returns the same outputs
                continue
            seen.add(rep)
            for i, out in zip(idx, o):
                res[i] = out
        return res

    def sleep(self, level: int = 1) -> None:
        """Release GPU memory while idle (level 1: weights to host memory; level 2: weights
        discarded and reloaded by ``wake_up``); the KV cache is released in both."""
        self.engine.sleep(level)

    def wake_up(self) -> None:
        self.engine.wake_up()

    def start_profile(self) -> None:
        self.engine.start_profile()

    def stop_profile(self):
        """Stop the profiler; returns the path of this rank's Chrome trace."""
        return self.engine.stop_profile()

    def shutdown(self):
        self.engine.shutdown()
        if self.executor is not None:
            from ..parallel.state import destroy_distributed
            destroy_distributed()
            self.executor.shutdown()
            self.executor = None
