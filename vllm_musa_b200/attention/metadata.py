"""Per-step attention metadata shared by every attention layer of the forward pass.

Token order is decodes first (one query token per request), then prefill chunks; the decode
kernel consumes rows [0, num_decodes), the prefill kernel the rest (its query-start offsets
are absolute token indices, so it reads q/out of the whole step buffer).  Reference
counterpart: FlashAttentionMetadata built by vllm_musa/v1/attention/backends/
flash_attn.py:478-1092.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


@dataclass
class AttnMetadata:
    num_tokens: int
    num_decodes: int
    num_prefills: int
    positions: torch.Tensor      # int32 [T]
    slot_mapping: torch.Tensor   # int32 [T]  (-1 = do not write the cache)
    seq_lens: torch.Tensor       # int32 [R]  context length after this step
    block_tables: torch.Tensor   # int32 [R, W]
    cu_q: torch.Tensor           # int32 [R+1] absolute token offsets
    max_seq_len: int
    decode_splits: Optional[int] = None
    tile_scratch: Optional[torch.Tensor] = None
    sliding_window: int = 0
    state_slots: Optional[torch.Tensor] = None  # int32 [R] recurrent-state slot per request
    lora: Optional[object] = None  # LoRABatch: token groups per adapter slot (lora.py)
    # int64 [T] draft-tree attention masks (steps verifying a token tree; 0 = causal row)
    tree_mask: Optional[torch.Tensor] = None

    @property
    def prefill_cu_q(self) -> torch.Tensor:
        return self.cu_q[self.num_decodes:self.num_decodes + self.num_prefills + 1]

    @property
    def prefill_seq_lens(self) -> torch.Tensor:
        return self.seq_lens[self.num_decodes:self.num_decodes + self.num_prefills]

    @property
    def prefill_block_tables(self) -> torch.Tensor:
        return self.block_tables[self.num_decodes:self.num_decodes + self.num_prefills]
