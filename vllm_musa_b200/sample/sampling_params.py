"""Sampling parameters (the vLLM ``SamplingParams`` surface the reference's users rely on)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Union


@dataclass
class StructuredOutputsParams:
    """Constrained decoding (vLLM's ``StructuredOutputsParams``): exactly one of a JSON schema
    (dict or JSON text), ``json_object`` (any JSON object), a regular expression, a list of
    choices or an EBNF grammar.  Generated tokens always keep the output a prefix of a valid
    string; the request stops at the end of the structure."""
    json: Optional[Union[dict, str]] = None
    json_object: bool = False
    regex: Optional[str] = None
    choice: Optional[List[str]] = None
    grammar: Optional[str] = None
    # JSON without free whitespace between tokens (compact separators)
    disable_any_whitespace: bool = False

    def __post_init__(self):
        given = [self.json is not None, bool(self.json_object), self.regex is not None,
                 self.choice is not None, self.grammar is not None]
        if sum(given) != 1:
            raise ValueError("structured outputs: give exactly one of json, json_object, regex, "
                             "choice, grammar")
        if self.choice is not None and not self.choice:
            raise ValueError("structured outputs: choice needs at least one string")

    def key(self) -> tuple:
        import json as _json
        j = self.json if self.json is None or isinstance(self.json, str) else \
            _json.dumps(self.json, sort_keys=True)
        return (j, self.json_object, self.regex,
                None if self.choice is None else tuple(self.choice), self.grammar,
                self.disable_any_whitespace)


@dataclass
class SamplingParams:
    n: int = 1
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0          # 0 or -1: disabled
    min_p: float = 0.0
    seed: Optional[int] = None
    max_tokens: int = 16
    min_tokens: int = 0
    stop_token_ids: List[int] = field(default_factory=list)
    stop: List[str] = field(default_factory=list)
    # keep the matched stop string at the end of the returned text (vLLM: excluded)
    include_stop_str_in_output: bool = False
    ignore_eos: bool = False
    detokenize: bool = True
    # vLLM's logits processors: repetition (> 1 discourages tokens of the prompt and the
    # output so far), presence and frequency penalties (subtracted per output occurrence)
    repetition_penalty: float = 1.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    # number of most likely tokens whose log-probabilities are returned per generated token
    # (plus the generated token's own), computed from the raw logits as vLLM's default
    # logprobs mode; None = no log-probabilities
    logprobs: Optional[int] = None
    # constrained decoding (JSON schema / regex / choice / grammar); a dict is accepted too
    structured_outputs: Optional[Any] = None
    # vLLM / OpenAI logits processors: token id -> bias added to the raw logits (clamped to
    # [-100, 100]); the only tokens that may be drawn; words (strings) that are never completed
    # (the last token of a word is banned when the output ends with the rest of it)
    logit_bias: Optional[Dict[int, float]] = None
    allowed_token_ids: Optional[List[int]] = None
    bad_words: Optional[List[str]] = None
    # log-probabilities of every prompt token given the tokens before it (top ``k`` per
    # position plus the prompt token's own; the first position has none); the request's
    # prompt is computed in full (no prefix-cache reuse)
    prompt_logprobs: Optional[int] = None
    # keep only the last k prompt tokens (vLLM's truncate_prompt_tokens; None: the whole prompt)
    truncate_prompt_tokens: Optional[int] = None
    # detokenization of the returned text
    skip_special_tokens: bool = True
    spaces_between_special_tokens: bool = True

    def __post_init__(self):
        if isinstance(self.structured_outputs, dict):
            self.structured_outputs = StructuredOutputsParams(**self.structured_outputs)
        if self.top_k is None or self.top_k < 0:
            self.top_k = 0
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if not 0.0 <= self.min_p <= 1.0:
            raise ValueError("min_p must be in [0, 1]")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if self.n < 1:
            raise ValueError("n must be >= 1")
        if self.repetition_penalty <= 0:
            raise ValueError("repetition_penalty must be > 0")
        if not -2.0 <= self.presence_penalty <= 2.0 or not -2.0 <= self.frequency_penalty <= 2.0:
            raise ValueError("presence_penalty and frequency_penalty must be in [-2, 2]")
        if self.logprobs is not None and not 0 <= self.logprobs <= 20:
            raise ValueError("logprobs must be in [0, 20]")
        if self.prompt_logprobs is not None and not 0 <= self.prompt_logprobs <= 20:
            raise ValueError("prompt_logprobs must be in [0, 20]")
        if self.truncate_prompt_tokens is not None and self.truncate_prompt_tokens < 1:
            raise ValueError("truncate_prompt_tokens must be >= 1")
        if isinstance(self.stop, str):
            self.stop = [self.stop]
        self.stop = [x for x in self.stop if x]
        if self.temperature < 1e-5:
            self.temperature = 0.0  # greedy
        if self.logit_bias:
            self.logit_bias = {int(k): max(-100.0, min(100.0, float(v)))
                               for k, v in self.logit_bias.items()}
        else:
            self.logit_bias = None
        if self.allowed_token_ids is not None:
            self.allowed_token_ids = sorted({int(t) for t in self.allowed_token_ids})
            if not self.allowed_token_ids:
                raise ValueError("allowed_token_ids must not be empty")
        if isinstance(self.bad_words, str):
            self.bad_words = [self.bad_words]
        self.bad_words = [w for w in (self.bad_words or []) if w] or None

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0

    @property
    def has_logits_processors(self) -> bool:
        return bool(self.logit_bias or self.allowed_token_ids or self.bad_words)

    @property
    def has_penalties(self) -> bool:
        return (self.repetition_penalty != 1.0 or self.presence_penalty != 0.0 or
                self.frequency_penalty != 0.0)


@dataclass
class BeamSearchParams:
    """Offline beam search (``LLM.beam_search``): ``beam_width`` live sequences per prompt, each
    step expanded by its 2 x beam_width most likely next tokens; finished sequences (EOS unless
    ``ignore_eos``) are ranked with the live ones by cumulative log-probability divided by
    (sequence length ** ``length_penalty``)."""
    beam_width: int
    max_tokens: int
    ignore_eos: bool = False
    length_penalty: float = 1.0

    def __post_init__(self):
        if self.beam_width < 1 or self.max_tokens < 1:
            raise ValueError("beam_width and max_tokens must be >= 1")


@dataclass
class PoolingParams:
    """Embedding requests (``LLM.embed`` / ``/v1/embeddings``): the prompt is run once and its
    final hidden states are pooled -- ``last`` token (the decoder-embedding default), ``mean``
    over the prompt, or ``cls`` (the first token) -- then L2-normalised when ``normalize``, and
    truncated to ``dimensions`` (Matryoshka) when given."""
    pooling_type: str = "last"
    normalize: bool = True
    dimensions: Optional[int] = None

    def __post_init__(self):
        self.pooling_type = self.pooling_type.lower()
        if self.pooling_type not in ("last", "mean", "cls"):
            raise ValueError("pooling_type must be last, mean or cls")
        if self.dimensions is not None and self.dimensions < 1:
            raise ValueError("dimensions must be >= 1")
