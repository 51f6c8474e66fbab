"""Constrained decoding over xgrammar grammars.

Per request a grammar (JSON schema, any JSON object, regex, choice list or EBNF) is compiled
once per distinct spec (cached) against the model's vocabulary and driven by a matcher.  Every
step the engine asks each constrained request's matcher for its next-token bitmask (bit t of
32-bit word t // 32: token t allowed), the runner masks those logits rows to -inf outside the
bitmask on the device (ops.sampling.apply_token_bitmask, per vocab shard under tensor
parallelism) before sampling, and the sampled token is fed back to the matcher.  When a
structure is complete only the stop tokens stay allowed, so the request ends with EOS.

Reference counterpart: upstream vLLM's structured-output manager and xgrammar backend, which
the reference serves unchanged (its sampler masks through vLLM's bitmask path).
"""
from __future__ import annotations

import json
from typing import List, Optional

import torch

from .sampling_params import StructuredOutputsParams


def _tokenizer_info(tokenizer, vocab_size: int, eos_token_id: Optional[int]):
    import xgrammar as xgr
    stops = [] if eos_token_id is None else [int(eos_token_id)]
    vocab = getattr(tokenizer, "b200_vocab", None)
    if vocab is not None:  # plain string vocabulary (tests, custom tokenizers)
        return xgr.TokenizerInfo(list(vocab), vocab_type=xgr.VocabType.RAW,
                                 vocab_size=vocab_size, stop_token_ids=stops)
    return xgr.TokenizerInfo.from_huggingface(tokenizer, vocab_size=vocab_size,
                                              stop_token_ids=stops or None)


class GrammarBackend:
    def __init__(self, tokenizer, vocab_size: int, eos_token_id: Optional[int]):
        import xgrammar as xgr
        if tokenizer is None:
            raise ValueError("structured outputs need the model's tokenizer (vocabulary)")
        self.xgr = xgr
        self.vocab_size = vocab_size
        self.info = _tokenizer_info(tokenizer, vocab_size, eos_token_id)
        self.compiler = xgr.GrammarCompiler(self.info)
        self._compiled = {}
        self.words = (vocab_size + 31) // 32

    def compile(self, so: StructuredOutputsParams):
        key = so.key()
        g = self._compiled.get(key)
        if g is None:
            c = self.compiler
            ws = not so.disable_any_whitespace
            if so.json is not None:
                schema = so.json if isinstance(so.json, str) else json.dumps(so.json)
                g = c.compile_json_schema(schema, any_whitespace=ws)
            elif so.json_object:
                g = c.compile_json_schema('{"type": "object"}', any_whitespace=ws)
            elif so.regex is not None:
                g = c.compile_regex(so.regex)
            elif so.choice is not None:
                alts = " | ".join(json.dumps(ch) for ch in so.choice)
                g = c.compile_grammar(f"root ::= {alts}")
            else:
                g = c.compile_grammar(so.grammar)
            self._compiled[key] = g
        return g

    def matcher(self, so: StructuredOutputsParams):
        return self.xgr.GrammarMatcher(self.compile(so))

    def bitmask(self, matchers: List) -> torch.Tensor:
        """int32 [len(matchers), words]: row i = the next-token bitmask of matchers[i]."""
        bm = torch.full((len(matchers), self.words), -1, dtype=torch.int32)
        for i, m in enumerate(matchers):
            m.fill_next_token_bitmask(bm, i)
        return bm
