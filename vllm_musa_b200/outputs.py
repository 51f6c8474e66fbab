"""Request outputs returned by the engine / ``LLM.generate`` (vLLM-compatible fields)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional


@dataclass
class Logprob:
    """Log-probability of one token at one position, with its rank among the vocabulary
    (1 = most likely), as vLLM reports them."""
    logprob: float
    rank: Optional[int] = None


@dataclass
class CompletionOutput:
    index: int
    token_ids: List[int]
    text: str = ""
    finish_reason: Optional[str] = None
    cumulative_logprob: Optional[float] = None
    # per generated token: {token id: Logprob} for the top-k tokens and the generated one
    logprobs: Optional[List[Dict[int, Logprob]]] = None
    # the stop string that ended the request (finish_reason "stop"), if one did
    stop_reason: Optional[str] = None


@dataclass
class RequestMetrics:
    arrival_time: float = 0.0
    first_token_time: Optional[float] = None
    finished_time: Optional[float] = None

    @property
    def ttft(self) -> Optional[float]:
        if self.first_token_time is None:
            return None
        return self.first_token_time - self.arrival_time


@dataclass
class RequestOutput:
    request_id: str
    prompt_token_ids: List[int]
    outputs: List[CompletionOutput]
    finished: bool
    prompt: Optional[str] = None
    metrics: RequestMetrics = field(default_factory=RequestMetrics)
    # per prompt position: {token id: Logprob} (None at position 0), when requested
    prompt_logprobs: Optional[List[Optional[Dict[int, Logprob]]]] = None
    embedding: Optional[List[float]] = None  # pooled hidden state of an embedding request

    def tpot(self) -> Optional[float]:
        m = self.metrics
        n = len(self.outputs[0].token_ids) if self.outputs else 0
        if m.first_token_time is None or m.finished_time is None or n < 2:
            return None
        return (m.finished_time - m.first_token_time) / (n - 1)


@dataclass
class BeamSearchSequence:
    """One beam: prompt + generated token ids, the generated tokens' log-probabilities and
    their sum, the decoded text of the generated part (with a tokenizer)."""
    tokens: List[int]
    logprobs: List[float]
    cum_logprob: float
    text: Optional[str] = None
    finish_reason: Optional[str] = None


@dataclass
class BeamSearchOutput:
    sequences: List[BeamSearchSequence]


@dataclass
class EmbeddingOutput:
    embedding: List[float]


@dataclass
class EmbeddingRequestOutput:
    request_id: str
    prompt_token_ids: List[int]
    outputs: EmbeddingOutput
    finished: bool = True
