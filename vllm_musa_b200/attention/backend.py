"""Paged attention backend: one object per attention layer geometry.

Dispatches the step's decode rows to the split-KV decode kernel and its prefill rows to the
chunked-prefill kernel (csrc/attention/paged_attention.cu).  Capabilities mirror what the
reference's MUSA FlashAttention backend advertises (vllm_musa/v1/attention/backends/
flash_attn.py:238-400): paged KV with 16/32/64/128-token pages, GQA, causal, sliding
window, attention sinks (per-head softmax-only logits); head dims 64/128/256.  Non-causal
packed sequences without a cache (encoders) go through ``MMEncoderAttention``.
"""
from __future__ import annotations

import math

import torch

from .. import ops
from .metadata import AttnMetadata


class PagedAttention:
    SUPPORTED_HEAD_DIMS = (64, 128, 256)
    SUPPORTED_BLOCK_SIZES = (16, 32, 64, 128, 256)

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int,
                 scale: float | None = None, sliding_window: int = 0,
                 sinks: torch.Tensor | None = None):
        if head_dim not in self.SUPPORTED_HEAD_DIMS:
            raise ValueError(f"head_dim {head_dim} not supported")
        self.hq, self.hkv, self.d = num_heads, num_kv_heads, head_dim
        self.scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)
        self.window = sliding_window
        self.sinks = sinks.float().contiguous() if sinks is not None else None

    def forward(self, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                meta: AttnMetadata, out: torch.Tensor | None = None) -> torch.Tensor:
        """q: [T, >= Hq*D] (rows of the packed qkv buffer); K/V already written to the cache."""
        T = q.shape[0]
        if out is None:
            out = torch.empty(T, self.hq * self.d, dtype=q.dtype, device=q.device)
        nd, npf = meta.num_decodes, meta.num_prefills
        if nd:
            ops.paged_decode(q[:nd], k_cache, v_cache, meta.block_tables[:nd], meta.seq_lens[:nd],
                             self.hq, self.hkv, self.scale, meta.max_seq_len, out=out[:nd],
                             num_splits=meta.decode_splits, sinks=self.sinks)
        if npf:
            ops.paged_prefill(q, k_cache, v_cache, meta.prefill_cu_q, meta.prefill_seq_lens,
                              meta.prefill_block_tables, self.hq, self.hkv, self.scale,
                              self.window or meta.sliding_window, out=out,
                              tile_scratch=meta.tile_scratch, sinks=self.sinks,
                              tree_mask=meta.tree_mask)
        return out


class MMEncoderAttention:
    """Bidirectional attention over packed variable-length sequences (vision / audio encoder
    layers): no KV cache, ``cu_seqlens`` delimits the images or clips.  Reference:
    vllm_musa/model_executor/layers/attention/mm_encoder_attention.py:14-170."""

    def __init__(self, num_heads: int, head_dim: int, scale: float | None = None,
                 num_kv_heads: int | None = None):
        if head_dim not in PagedAttention.SUPPORTED_HEAD_DIMS:
            raise ValueError(f"head_dim {head_dim} not supported")
        self.hq, self.d = num_heads, head_dim
        self.hkv = num_kv_heads or num_heads
        self.scale = scale if scale is not None else 1.0 / math.sqrt(head_dim)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                cu_seqlens: torch.Tensor) -> torch.Tensor:
        """q [T, Hq*D] or [T, Hq, D]; k/v likewise with Hkv heads -> [T, Hq*D]."""
        T = q.shape[0]
        q3 = q.reshape(T, self.hq, self.d)
        k3 = k.reshape(T, self.hkv, self.d)
        v3 = v.reshape(T, self.hkv, self.d)
        return ops.varlen_attention(q3, k3, v3, cu_seqlens, self.scale).reshape(T, -1)


class TreeAttention(PagedAttention):
    """Attention of speculative token trees: each request's step tokens are a draft tree (at
    most 64 nodes) appended after its cached context; a node sees the context and its own
    ancestors only.  ``tree_mask`` (int64 per step token, from ``ops.attention.
    tree_ancestor_masks``) carries the visibility bits.  Runs the paged prefill kernel with the
    tree mask.  Reference: vllm_musa/v1/attention/backends/tree_attn.py:41-451."""

    def forward_tree(self, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     cu_q: torch.Tensor, seq_lens: torch.Tensor, block_tables: torch.Tensor,
                     tree_mask: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return ops.paged_prefill(q, k_cache, v_cache, cu_q, seq_lens, block_tables, self.hq,
                                 self.hkv, self.scale, out=out, sinks=self.sinks,
                                 tree_mask=tree_mask)


class TurboQuantAttention(PagedAttention):
    """Attention over the TurboQuant quantised KV cache (``kv_cache_dtype`` turboquant_k8v4 /
    turboquant_4bit_nc / turboquant_k3v4_nc / turboquant_3bit_nc; format in
    csrc/attention/turboquant.cu).  Decode rows run ``tq_decode_kernel`` straight on the packed
    slots (q rotated in-kernel for the Hadamard-rotated keys); prefill rows dequantise the pages
    they read into a bf16 scratch cache and run the paged prefill kernel, so a prompt attends
    to the same quantised keys and values that its later decode steps see.  Like the
    reference's backend (vllm_musa/v1/attention/backends/turboquant.py:37-114) it takes no
    attention sinks, MLA or sparse attention; sliding windows are refused too."""

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, kv_cache_dtype: str,
                 scale: float | None = None, sliding_window: int = 0,
                 sinks: torch.Tensor | None = None):
        if sinks is not None:
            raise ValueError("TurboQuant KV cache does not support attention sinks")
        if sliding_window:
            raise ValueError("TurboQuant KV cache does not support sliding-window attention")
        super().__init__(num_heads, num_kv_heads, head_dim, scale)
        from ..ops.turboquant import tq_format
        self.fmt = tq_format(kv_cache_dtype, head_dim)

    def write_kv(self, k: torch.Tensor, v: torch.Tensor, cache: torch.Tensor,
                 slot_mapping: torch.Tensor) -> None:
        from ..ops.turboquant import tq_store
        tq_store(k, v, cache, slot_mapping, self.fmt)

    def forward(self, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor | None,
                meta: AttnMetadata, out: torch.Tensor | None = None) -> torch.Tensor:
        """q: [T, >= Hq*D]; ``k_cache`` is the packed uint8 cache (``v_cache`` unused)."""
        from ..ops.turboquant import tq_decode, tq_dequant_pages
        T = q.shape[0]
        if out is None:
            out = torch.empty(T, self.hq * self.d, dtype=q.dtype, device=q.device)
        nd, npf = meta.num_decodes, meta.num_prefills
        if nd:
            tq_decode(q[:nd], k_cache, meta.block_tables[:nd], meta.seq_lens[:nd], self.hq,
                      self.scale, self.fmt, out=out[:nd], num_splits=meta.decode_splits)
        if npf:
            bs = k_cache.shape[2]
            pages = max(1, -(-int(meta.max_seq_len) // bs))
            pages = min(pages, meta.prefill_block_tables.shape[1])
            kd, vd, bt = tq_dequant_pages(k_cache, meta.prefill_block_tables,
                                          meta.prefill_seq_lens, self.fmt, pages)
            ops.paged_prefill(q, kd, vd, meta.prefill_cu_q, meta.prefill_seq_lens, bt, self.hq,
                              self.hkv, self.scale, 0, out=out, tile_scratch=meta.tile_scratch)
        return out
