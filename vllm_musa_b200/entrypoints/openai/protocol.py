"""OpenAI-compatible request / response schemas (the subset vLLM's server exposes)."""
from __future__ import annotations

import time
import uuid
from typing import Dict, List, Optional, Union

from pydantic import BaseModel, Field

from ...sample.sampling_params import SamplingParams


class _Sampling(BaseModel):
    model: Optional[str] = None
    max_tokens: Optional[int] = None
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    min_p: float = 0.0
    n: int = 1
    seed: Optional[int] = None
    stop: Optional[Union[str, List[str]]] = None
    stop_token_ids: Optional[List[int]] = None
    ignore_eos: bool = False
    min_tokens: int = 0
    stream: bool = False
    # OpenAI: {"include_usage": true} adds a final chunk with the token counts
    stream_options: Optional[Dict] = None
    user: Optional[str] = None
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0
    # OpenAI logit_bias (token id as a string -> bias in [-100, 100]); vLLM's allowed_token_ids
    # and bad_words
    logit_bias: Optional[Dict[str, float]] = None
    allowed_token_ids: Optional[List[int]] = None
    bad_words: Optional[List[str]] = None
    # vLLM extensions: prompt log-probabilities, detokenization options
    prompt_logprobs: Optional[int] = None
    priority: int = 0  # under --scheduling-policy priority: lower values are served first
    truncate_prompt_tokens: Optional[int] = None
    skip_special_tokens: bool = True
    spaces_between_special_tokens: bool = True
    # structured outputs: vLLM's extra parameters and the OpenAI response_format
    structured_outputs: Optional[Dict] = None
    guided_json: Optional[Union[Dict, str]] = None
    guided_regex: Optional[str] = None
    guided_choice: Optional[List[str]] = None
    guided_grammar: Optional[str] = None
    response_format: Optional[Dict] = None

    def num_logprobs(self) -> Optional[int]:
        return None

    def structured(self) -> Optional[Dict]:
        """The request's constraint as StructuredOutputsParams fields (None: unconstrained)."""
        if self.structured_outputs:
            return dict(self.structured_outputs)
        for key, val in (("json", self.guided_json), ("regex", self.guided_regex),
                         ("choice", self.guided_choice), ("grammar", self.guided_grammar)):
            if val is not None:
                return {key: val}
        rf = self.response_format or {}
        if rf.get("type") == "json_object":
            return {"json_object": True}
        if rf.get("type") == "json_schema":
            js = rf.get("json_schema") or {}
            return {"json": js.get("schema", js)}
        return None

    def sampling_params(self, default_max: int) -> SamplingParams:
        stop = [self.stop] if isinstance(self.stop, str) else list(self.stop or [])
        return SamplingParams(n=self.n, temperature=self.temperature, top_p=self.top_p,
                              top_k=self.top_k, min_p=self.min_p, seed=self.seed,
                              max_tokens=self.max_tokens or default_max,
                              min_tokens=self.min_tokens, stop=stop,
                              stop_token_ids=list(self.stop_token_ids or []),
                              ignore_eos=self.ignore_eos,
                              presence_penalty=self.presence_penalty,
                              frequency_penalty=self.frequency_penalty,
                              repetition_penalty=self.repetition_penalty,
                              logprobs=self.num_logprobs(),
                              structured_outputs=self.structured(),
                              logit_bias=({int(k): v for k, v in self.logit_bias.items()}
                                          if self.logit_bias else None),
                              allowed_token_ids=self.allowed_token_ids,
                              bad_words=self.bad_words,
                              prompt_logprobs=self.prompt_logprobs,
                              truncate_prompt_tokens=self.truncate_prompt_tokens,
                              skip_special_tokens=self.skip_special_tokens,
                              spaces_between_special_tokens=self.spaces_between_special_tokens)


class CompletionRequest(_Sampling):
    prompt: Union[str, List[int], List[str], List[List[int]]]
    echo: bool = False
    logprobs: Optional[int] = None  # top log-probabilities per generated token (OpenAI legacy)

    def num_logprobs(self) -> Optional[int]:
        return self.logprobs


class ChatMessage(BaseModel):
    role: str
    content: str


class ChatCompletionRequest(_Sampling):
    messages: List[ChatMessage]
    max_completion_tokens: Optional[int] = None
    logprobs: bool = False
    top_logprobs: Optional[int] = None

    def num_logprobs(self) -> Optional[int]:
        return (self.top_logprobs or 0) if self.logprobs else None


class Usage(BaseModel):
    prompt_tokens: int = 0
    completion_tokens: int = 0
    total_tokens: int = 0


class CompletionChoice(BaseModel):
    index: int
    text: str
    token_ids: Optional[List[int]] = None
    finish_reason: Optional[str] = None
    logprobs: Optional[Dict] = None
    prompt_logprobs: Optional[List[Optional[Dict]]] = None


class CompletionResponse(BaseModel):
    id: str = Field(default_factory=lambda: f"cmpl-{uuid.uuid4().hex}")
    object: str = "text_completion"
    created: int = Field(default_factory=lambda: int(time.time()))
    model: str
    choices: List[CompletionChoice]
    usage: Usage


class ChatChoice(BaseModel):
    index: int
    message: ChatMessage
    finish_reason: Optional[str] = None
    logprobs: Optional[Dict] = None


def _tok_str(tokenizer, t: int) -> str:
    if tokenizer is None:
        return str(t)
    try:
        return tokenizer.decode([t])
    except Exception:  # pragma: no cover - tokenizer specific
        return str(t)


def prompt_logprobs_json(o, tokenizer) -> Optional[List[Optional[Dict]]]:
    """vLLM's ``prompt_logprobs`` field: per prompt position None or {token id: {logprob,
    rank, decoded_token}}."""
    if o.prompt_logprobs is None:
        return None
    return [None if d is None else
            {str(t): {"logprob": v.logprob, "rank": v.rank,
                      "decoded_token": _tok_str(tokenizer, t)} for t, v in d.items()}
            for d in o.prompt_logprobs]


def completion_logprobs(c, tokenizer) -> Optional[Dict]:
    """OpenAI completions ``logprobs`` object from a CompletionOutput's per-token logprobs."""
    if c.logprobs is None:
        return None
    toks = [_tok_str(tokenizer, t) for t in c.token_ids]
    return {"tokens": toks,
            "token_logprobs": [d[t].logprob for t, d in zip(c.token_ids, c.logprobs)],
            "top_logprobs": [{_tok_str(tokenizer, k): v.logprob for k, v in d.items()}
                             for d in c.logprobs],
            "text_offset": []}


def chat_logprobs(c, tokenizer, top: int) -> Optional[Dict]:
    """OpenAI chat ``logprobs.content`` from a CompletionOutput's per-token logprobs."""
    if c.logprobs is None:
        return None
    content = []
    for t, d in zip(c.token_ids, c.logprobs):
        ranked = sorted(((k, v) for k, v in d.items() if v.rank is not None and v.rank <= top),
                        key=lambda kv: kv[1].rank)
        content.append({"token": _tok_str(tokenizer, t), "logprob": d[t].logprob,
                        "top_logprobs": [{"token": _tok_str(tokenizer, k), "logprob": v.logprob}
                                         for k, v in ranked]})
    return {"content": content}


class ChatCompletionResponse(BaseModel):
    id: str = Field(default_factory=lambda: f"chatcmpl-{uuid.uuid4().hex}")
    object: str = "chat.completion"
    created: int = Field(default_factory=lambda: int(time.time()))
    model: str
    choices: List[ChatChoice]
    usage: Usage


class ModelCard(BaseModel):
    id: str
    object: str = "model"
    created: int = Field(default_factory=lambda: int(time.time()))
    owned_by: str = "vllm_musa_b200"
    max_model_len: Optional[int] = None


class ModelList(BaseModel):
    object: str = "list"
    data: List[ModelCard]


class ErrorResponse(BaseModel):
    object: str = "error"
    message: str
    type: str = "invalid_request_error"
    code: int = 400
    extra: Optional[Dict] = None


class EmbeddingRequest(BaseModel):
    """OpenAI /v1/embeddings: ``input`` is a string, a list of strings, a list of token ids or
    a list of token-id lists; vLLM's extras choose the pooling."""
    model: Optional[str] = None
    input: Union[str, List[str], List[int], List[List[int]]]
    encoding_format: str = "float"
    dimensions: Optional[int] = None
    pooling_type: str = "last"
    normalize: bool = True


class TokenizeRequest(BaseModel):
    model: Optional[str] = None
    prompt: str = ""


class DetokenizeRequest(BaseModel):
    model: Optional[str] = None
    tokens: List[int] = Field(default_factory=list)
