"""Chat prompts: the tokenizer's chat template (HuggingFace ``apply_chat_template`` with the
generation prompt), or a plain ``role: content`` transcript for tokenizers without one.  Shared
by ``LLM.chat`` and the OpenAI server's chat completions.  Reference: vLLM's chat utilities,
which the reference serves unchanged."""
from __future__ import annotations

from typing import List


def chat_prompt_ids(tokenizer, messages: List[dict], add_generation_prompt: bool = True) -> List[int]:
    """messages [{"role": ..., "content": ...}, ...] -> prompt token ids."""
    if tokenizer is None:
        raise ValueError("chat needs a tokenizer (serve or load a checkpoint directory)")
    if getattr(tokenizer, "chat_template", None):
        ids = tokenizer.apply_chat_template(messages, add_generation_prompt=add_generation_prompt,
                                            tokenize=True)
        return list(ids["input_ids"] if isinstance(ids, dict) else ids)
    text = "".join(f"{m['role']}: {m['content']}\n" for m in messages)
    if add_generation_prompt:
        text += "assistant:"
    return list(tokenizer.encode(text))
