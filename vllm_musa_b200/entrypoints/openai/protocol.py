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
    user: Optional[str] = None

    def sampling_params(self, default_max: int) -> SamplingParams:
        stop = [self.stop] if isinstance(self.stop, str) else list(self.stop or [])
        return SamplingParams(n=self.n, temperature=self.temperature, top_p=self.top_p,
                              top_k=self.top_k, min_p=self.min_p, seed=self.seed,
                              max_tokens=self.max_tokens or default_max,
                              min_tokens=self.min_tokens, stop=stop,
                              stop_token_ids=list(self.stop_token_ids or []),
                              ignore_eos=self.ignore_eos)


class CompletionRequest(_Sampling):
    prompt: Union[str, List[int], List[str], List[List[int]]]
    echo: bool = False


class ChatMessage(BaseModel):
    role: str
    content: str


class ChatCompletionRequest(_Sampling):
    messages: List[ChatMessage]
    max_completion_tokens: Optional[int] = None


class Usage(BaseModel):
    prompt_tokens: int = 0
    completion_tokens: int = 0
    total_tokens: int = 0


class CompletionChoice(BaseModel):
    index: int
    text: str
    token_ids: Optional[List[int]] = None
    finish_reason: Optional[str] = None


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
