"""OpenAI-compatible HTTP server (``/v1/completions``, ``/v1/chat/completions``,
``/v1/embeddings``, ``/v1/models``, ``/tokenize``, ``/detokenize``, ``/health``, ``/metrics``),
the role ``vllm serve`` plays for the reference
(usage: docs/usage.md of the reference).

    python -m vllm_musa_b200.entrypoints.openai.api_server --model /path/or/preset --port 8000
    b200-vllm serve llama3-8b --tensor-parallel-size 8

Tensor parallelism: without a launcher the server process spawns its follower ranks; under
``torchrun`` rank 0 serves HTTP and the other ranks follow it.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import logging
import os
import time
import uuid
from typing import List, Optional

from .protocol import (ChatChoice, ChatCompletionRequest, ChatCompletionResponse, ChatMessage,
                       CompletionChoice, CompletionRequest, CompletionResponse, ErrorResponse,
                       DetokenizeRequest, EmbeddingRequest, ModelCard, ModelList,
                       TokenizeRequest, Usage, chat_logprobs, completion_logprobs,
                       prompt_logprobs_json)

log = logging.getLogger("vllm_musa_b200")


def _chat_prompt(tokenizer, messages: List[ChatMessage]) -> List[int]:
    from ..chat_utils import chat_prompt_ids
    return chat_prompt_ids(tokenizer, [m.model_dump() for m in messages])


def build_app(llm, model_name: str, max_model_len: int, lora_modules: Optional[dict] = None):
    """FastAPI app over an ``AsyncLLM``.  ``lora_modules``: served adapter name -> LoRARequest
    (a request whose ``model`` names an adapter runs with it)."""
    from fastapi import FastAPI, Request
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    from ...sample.sampling_params import SamplingParams
    from ...engine.async_llm import AsyncLLM  # noqa: F401  (type)

    app = FastAPI(title="vllm_musa_b200 OpenAI-compatible server")
    tok = llm.tokenizer
    default_max = 16

    def err(msg: str, code: int = 400):
        return JSONResponse(ErrorResponse(message=msg, code=code).model_dump(), status_code=code)

    def encode_prompts(prompt) -> List[tuple]:
        if isinstance(prompt, str):
            if tok is None:
                raise ValueError("text prompts need a tokenizer; send token ids instead")
            return [(tok.encode(prompt), prompt)]
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], int):
            return [(list(prompt), None)]
        out = []
        for p in prompt:
            out += encode_prompts(p)
        return out

    def check_len(ids, params: SamplingParams):
        n = len(ids)
        if params.truncate_prompt_tokens is not None:
            n = min(n, params.truncate_prompt_tokens)  # the engine keeps the last tokens
        if n + 1 > max_model_len:
            raise ValueError(f"prompt has {n} tokens; max_model_len is {max_model_len}")
        params.max_tokens = min(params.max_tokens, max_model_len - n)

    @app.get("/health")
    async def health():
        if getattr(llm, "dead", None) is not None:
            return PlainTextResponse(f"engine dead: {llm.dead!r}", status_code=503)
        return PlainTextResponse("ok")

    @app.get("/version")
    async def version():
        from ... import __version__
        return {"version": __version__}

    loras = dict(lora_modules or {})

    def lora_of(req):
        if req.model is None or req.model == model_name:
            return None
        if req.model in loras:
            return loras[req.model]
        raise ValueError(f"model {req.model!r} is not served")

    @app.get("/v1/models")
    async def models():
        cards = [ModelCard(id=model_name, max_model_len=max_model_len)]
        cards += [ModelCard(id=n, max_model_len=max_model_len) for n in loras]
        return ModelList(data=cards).model_dump()

    @app.get("/metrics")
    async def metrics():
        s = llm.stats
        eng = llm.engine
        lines = [
            "# TYPE b200_request_success_total counter",
            f"b200_request_success_total {s['finished']}",
            "# TYPE b200_prompt_tokens_total counter",
            f"b200_prompt_tokens_total {s['prompt_tokens']}",
            "# TYPE b200_generation_tokens_total counter",
            f"b200_generation_tokens_total {s['generation_tokens']}",
            "# TYPE b200_num_requests_running gauge",
            f"b200_num_requests_running {eng.scheduler.num_running()}",
            "# TYPE b200_num_requests_waiting gauge",
            f"b200_num_requests_waiting {eng.scheduler.num_waiting()}",
            "# TYPE b200_kv_cache_free_blocks gauge",
            f"b200_kv_cache_free_blocks {eng.scheduler.num_free_blocks()}",
        ]
        total = max(1, getattr(eng, "num_blocks", 0))
        sch = eng.scheduler
        q, h = sch.prefix_cache_queries(), sch.prefix_cache_hits()
        lines += [
            "# TYPE b200_kv_cache_usage_perc gauge",
            f"b200_kv_cache_usage_perc {1.0 - sch.num_free_blocks() / total:.6f}",
            "# TYPE b200_prefix_cache_queries_total counter",
            f"b200_prefix_cache_queries_total {q}",
            "# TYPE b200_prefix_cache_hits_total counter",
            f"b200_prefix_cache_hits_total {h}",
            "# TYPE b200_spec_decode_num_draft_tokens_total counter",
            f"b200_spec_decode_num_draft_tokens_total {sch.spec_proposed()}",
            "# TYPE b200_spec_decode_num_accepted_tokens_total counter",
            f"b200_spec_decode_num_accepted_tokens_total {sch.spec_accepted()}",
            "# TYPE b200_engine_steps_total counter",
            f"b200_engine_steps_total {eng.num_steps}",
        ]
        for name, vals in (("time_to_first_token_seconds", s["ttft"]),
                           ("time_per_output_token_seconds", s["tpot"])):
            lines.append(f"# TYPE b200_{name} summary")
            lines.append(f"b200_{name}_count {len(vals)}")
            lines.append(f"b200_{name}_sum {sum(vals):.6f}")
        return PlainTextResponse("\n".join(lines) + "\n")

    async def run_one(ids, params, rid, lora=None, priority=0):
        final = None
        async for o in llm.generate(ids, params, rid, lora_request=lora, priority=priority):
            final = o
        return final

    @app.post("/v1/embeddings")
    async def embeddings(req: EmbeddingRequest):
        from ...sample.sampling_params import PoolingParams
        try:
            lora_of(req)
            prompts = encode_prompts(req.input)
            pp = PoolingParams(pooling_type=req.pooling_type, normalize=req.normalize,
                               dimensions=req.dimensions)
            for ids, _ in prompts:
                if len(ids) + 1 > max_model_len:
                    raise ValueError(f"input has {len(ids)} tokens; max_model_len is "
                                     f"{max_model_len}")
            rid = f"embd-{uuid.uuid4().hex}"
            outs = await asyncio.gather(*[run_one(ids, pp, f"{rid}-{i}")
                                          for i, (ids, _) in enumerate(prompts)])
        except ValueError as e:
            return err(str(e))
        n = sum(len(ids) for ids, _ in prompts)
        data = [{"object": "embedding", "index": i, "embedding": o.embedding}
                for i, o in enumerate(outs)]
        return {"object": "list", "data": data, "model": model_name,
                "usage": {"prompt_tokens": n, "total_tokens": n}}

    @app.post("/tokenize")
    async def tokenize(req: TokenizeRequest):
        if tok is None:
            return err("tokenize needs a tokenizer")
        ids = list(tok.encode(req.prompt))
        return {"tokens": ids, "count": len(ids), "max_model_len": max_model_len}

    @app.post("/detokenize")
    async def detokenize(req: DetokenizeRequest):
        if tok is None:
            return err("detokenize needs a tokenizer")
        return {"prompt": tok.decode(list(req.tokens))}

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest):
        try:
            lora = lora_of(req)
            prompts = encode_prompts(req.prompt)
            base = req.sampling_params(default_max)
            jobs = []
            for pi, (ids, text) in enumerate(prompts):
                for k in range(base.n):
                    p = SamplingParams(**{**base.__dict__, "n": 1})
                    if base.seed is not None:
                        p.seed = base.seed + k
                    check_len(ids, p)
                    jobs.append((pi * base.n + k, ids, text, p))
        except ValueError as e:
            return err(str(e))
        rid = f"cmpl-{uuid.uuid4().hex}"
        if req.stream:
            async def gen():
                qs = []
                for idx, ids, text, p in jobs:
                    qs.append((idx, llm.generate(ids, p, f"{rid}-{idx}", lora_request=lora,
                                                 priority=req.priority)))
                n_prompt = n_gen = 0
                for (idx, ids, _, _), (_, it) in zip(jobs, qs):
                    sent, n_ids = "", 0
                    async for o in it:
                        c = o.outputs[0]
                        delta = c.text[len(sent):]
                        sent = c.text
                        # every token since the last chunk (a speculative step adds several)
                        new_ids = list(c.token_ids[n_ids:])
                        n_ids = len(c.token_ids)
                        chunk = {"id": rid, "object": "text_completion", "created": int(time.time()),
                                 "model": model_name,
                                 "choices": [{"index": idx, "text": delta, "token_ids": new_ids,
                                              "finish_reason": c.finish_reason if o.finished else None}]}
                        yield f"data: {json.dumps(chunk)}\n\n"
                    n_prompt += len(ids)
                    n_gen += n_ids
                if (req.stream_options or {}).get("include_usage"):
                    usage = {"prompt_tokens": n_prompt, "completion_tokens": n_gen,
                             "total_tokens": n_prompt + n_gen}
                    yield f"data: {json.dumps({'id': rid, 'object': 'text_completion', 'created': int(time.time()), 'model': model_name, 'choices': [], 'usage': usage})}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        try:
            outs = await asyncio.gather(*[run_one(ids, p, f"{rid}-{idx}", lora, req.priority)
                                          for idx, ids, _, p in jobs])
        except ValueError as e:  # rejected by the engine (e.g. a token id off the vocabulary)
            return err(str(e))
        choices, n_prompt, n_gen = [], 0, 0
        for (idx, ids, text, _), o in zip(jobs, outs):
            c = o.outputs[0]
            body = (text or "") + c.text if req.echo else c.text
            choices.append(CompletionChoice(index=idx, text=body, token_ids=c.token_ids,
                                            finish_reason=c.finish_reason,
                                            logprobs=completion_logprobs(c, tok),
                                            prompt_logprobs=prompt_logprobs_json(o, tok)))
            n_prompt += len(ids)
            n_gen += len(c.token_ids)
        return CompletionResponse(id=rid, model=model_name, choices=choices,
                                  usage=Usage(prompt_tokens=n_prompt, completion_tokens=n_gen,
                                              total_tokens=n_prompt + n_gen)).model_dump()

    @app.post("/v1/chat/completions")
    async def chat(req: ChatCompletionRequest):
        try:
            lora = lora_of(req)
            ids = _chat_prompt(tok, req.messages)
            p = req.sampling_params(req.max_completion_tokens or default_max)
            if req.max_completion_tokens:
                p.max_tokens = req.max_completion_tokens
            check_len(ids, p)
        except ValueError as e:
            return err(str(e))
        rid = f"chatcmpl-{uuid.uuid4().hex}"
        if req.stream:
            async def gen():
                sent = ""
                n_gen = 0
                async for o in llm.generate(ids, SamplingParams(**{**p.__dict__, "n": 1}), rid,
                                            lora_request=lora, priority=req.priority):
                    c = o.outputs[0]
                    delta = c.text[len(sent):]
                    sent = c.text
                    n_gen = len(c.token_ids)
                    chunk = {"id": rid, "object": "chat.completion.chunk", "created": int(time.time()),
                             "model": model_name,
                             "choices": [{"index": 0, "delta": {"role": "assistant", "content": delta},
                                          "finish_reason": c.finish_reason if o.finished else None}]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                if (req.stream_options or {}).get("include_usage"):
                    usage = {"prompt_tokens": len(ids), "completion_tokens": n_gen,
                             "total_tokens": len(ids) + n_gen}
                    yield f"data: {json.dumps({'id': rid, 'object': 'chat.completion.chunk', 'created': int(time.time()), 'model': model_name, 'choices': [], 'usage': usage})}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(gen(), media_type="text/event-stream")
        try:
            outs = await asyncio.gather(*[
                run_one(ids, SamplingParams(**{**p.__dict__, "n": 1,
                                               "seed": (p.seed + k) if p.seed is not None else None}),
                        f"{rid}-{k}", lora) for k in range(p.n)])
        except ValueError as e:
            return err(str(e))
        choices = [ChatChoice(index=k, message=ChatMessage(role="assistant", content=o.outputs[0].text),
                              finish_reason=o.outputs[0].finish_reason,
                              logprobs=chat_logprobs(o.outputs[0], tok, req.top_logprobs or 0))
                   for k, o in enumerate(outs)]
        n_gen = sum(len(o.outputs[0].token_ids) for o in outs)
        return ChatCompletionResponse(id=rid, model=model_name, choices=choices,
                                      usage=Usage(prompt_tokens=len(ids), completion_tokens=n_gen,
                                                  total_tokens=len(ids) + n_gen)).model_dump()

    return app


def make_arg_parser(p: Optional[argparse.ArgumentParser] = None) -> argparse.ArgumentParser:
    p = p or argparse.ArgumentParser(description="vllm_musa_b200 OpenAI-compatible server")
    p.add_argument("--model", default="llama3-8b", help="checkpoint directory or preset name")
    p.add_argument("--served-model-name", default=None)
    p.add_argument("--host", default="0.0.0.0")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--tensor-parallel-size", "-tp", type=int, default=1)
    p.add_argument("--pipeline-parallel-size", "-pp", type=int, default=1)
    p.add_argument("--enable-expert-parallel", action="store_true")
    p.add_argument("--enable-lora", action="store_true")
    p.add_argument("--max-loras", type=int, default=4)
    p.add_argument("--max-lora-rank", type=int, default=64)
    p.add_argument("--lora-modules", nargs="*", default=[],
                   help="name=path adapters served under their own model names")
    p.add_argument("--speculative-config", type=json.loads, default=None,
                   help='JSON, e.g. {"method": "eagle", "num_speculative_tokens": 1, '
                        '"model": "/path/to/eagle"}')
    p.add_argument("--max-model-len", type=int, default=None)
    p.add_argument("--max-num-seqs", type=int, default=256)
    p.add_argument("--max-num-batched-tokens", type=int, default=8192)
    p.add_argument("--block-size", type=int, default=64)
    p.add_argument("--gpu-memory-utilization", type=float, default=0.90)
    p.add_argument("--enforce-eager", action="store_true")
    p.add_argument("--no-enable-prefix-caching", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default="cuda")
    p.add_argument("--num-gpu-blocks", type=int, default=None)
    p.add_argument("--kv-cache-dtype", default=None,
                   help="auto | fp8 | turboquant_k8v4 | turboquant_4bit_nc | ...")
    p.add_argument("--scheduling-policy", default="fcfs", choices=["fcfs", "priority"])
    p.add_argument("--logprobs-mode", default="raw_logprobs",
                   choices=["raw_logprobs", "raw_logits", "processed_logprobs",
                            "processed_logits"])
    return p


def build_llm(args):
    from ..llm import LLM
    return LLM(args.model, tensor_parallel_size=args.tensor_parallel_size,
               pipeline_parallel_size=getattr(args, "pipeline_parallel_size", 1),
               speculative_config=getattr(args, "speculative_config", None),
               enable_lora=(getattr(args, "enable_lora", False) or
                            bool(getattr(args, "lora_modules", []))),
               max_loras=getattr(args, "max_loras", 4),
               max_lora_rank=getattr(args, "max_lora_rank", 64),
               enable_expert_parallel=args.enable_expert_parallel,
               max_model_len=args.max_model_len, max_num_seqs=args.max_num_seqs,
               max_num_batched_tokens=args.max_num_batched_tokens, block_size=args.block_size,
               gpu_memory_utilization=args.gpu_memory_utilization,
               enforce_eager=args.enforce_eager,
               enable_prefix_caching=not args.no_enable_prefix_caching, seed=args.seed,
               device=args.device, num_gpu_blocks=args.num_gpu_blocks,
               kv_cache_dtype=getattr(args, "kv_cache_dtype", None),
               logprobs_mode=getattr(args, "logprobs_mode", "raw_logprobs"),
               scheduling_policy=getattr(args, "scheduling_policy", "fcfs"))


def parse_lora_modules(specs) -> dict:
    """["name=path", ...] -> {name: LoRARequest} (ids 1, 2, ... in order)."""
    from ...lora import LoRARequest
    out = {}
    for k, spec in enumerate(specs or []):
        name, _, path = spec.partition("=")
        if not name or not path:
            raise ValueError(f"--lora-modules entries are name=path, got {spec!r}")
        out[name] = LoRARequest(name, k + 1, path)
    return out


def run_server(args) -> None:
    import uvicorn

    from ...engine.async_llm import AsyncLLM
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        os.environ["B200_SPMD_ROLE"] = "driver" if rank == 0 else "follower"
    llm = build_llm(args)
    if world > 1 and rank != 0:
        llm.engine.follow()
        llm.shutdown()
        return
    alm = AsyncLLM(llm.engine)
    name = args.served_model_name or args.model
    app = build_app(alm, name, llm.engine.config.scheduler.max_model_len,
                    parse_lora_modules(getattr(args, "lora_modules", [])))
    try:
        uvicorn.run(app, host=args.host, port=args.port, log_level="info")
    finally:
        alm.shutdown()
        llm.shutdown()


def main(argv=None):
    logging.basicConfig(level=logging.INFO)
    run_server(make_arg_parser().parse_args(argv))


if __name__ == "__main__":
    main()
