"""vLLM attention backend over this package's paged attention kernels (``B200Platform``
selects it for bf16 decoder attention with head sizes 64 / 128 / 256).

* KV cache: per layer ``[2, num_blocks, num_kv_heads, block_size, head_size]`` bf16, i.e. K and
  V each ``[num_blocks, Hkv, block_size, D]``: one KV head's page is one contiguous
  ``block_size x D`` run, the 2-D TMA box the decode / prefill kernels load.
* Cache writes: ``do_kv_cache_update`` runs the ``kv_insert`` kernel (16-byte vectors per
  (token, KV head) warp) on the layer's post-RoPE key / value.
* Attention: the batch is reordered decodes-first (``reorder_batch_threshold = 1``); decode rows
  run the split-KV decode kernel (``ops.paged_decode``, TMA page ring + tensor-core scores,
  LSE merge), the prefill rows the causal chunked-prefill kernels (``ops.paged_prefill``:
  tcgen05 / TMEM for head_dim 128) reading the same pages.
* CUDA graphs: full graphs of uniform single-token decode batches.  Their split-KV count and
  workspace depend only on the batch size and ``max_model_len``, so every replay matches its
  capture; mixed batches run in vLLM's piecewise graphs with attention eager.

Reference counterparts: the reference's MUSA FlashAttention backend
(vllm_musa/v1/attention/backends/flash_attn.py:238-1537: capabilities, metadata builder with
an AOT scheduler, forward) and its selector (vllm_musa/platform.py:730-836).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from vllm.v1.attention.backend import (AttentionBackend, AttentionCGSupport, AttentionImpl,
                                       AttentionMetadataBuilder, AttentionType,
                                       CommonAttentionMetadata, MultipleOf)

from . import ops

HEAD_SIZES = (64, 128, 256)


class B200AttentionBackend(AttentionBackend):
    supported_dtypes = [torch.bfloat16]
    supported_kv_cache_dtypes = ["auto", "bfloat16"]
    forward_includes_kv_cache_update = False

    @staticmethod
    def get_supported_kernel_block_sizes() -> list:
        # the kernels' page geometry: 16 / 32 / 64-token pages or multiples of 64
        return [16, 32, 64, MultipleOf(64)]

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls():
        return B200AttentionImpl

    @staticmethod
    def get_builder_cls():
        return B200AttentionMetadataBuilder

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple:
        if block_size % 16 or (block_size > 64 and block_size % 64):
            raise ValueError("block size must be 16, 32, 64 or a multiple of 64")
        return (2, num_blocks, num_kv_heads, block_size, head_size)

    @classmethod
    def get_supported_head_sizes(cls) -> list:
        return list(HEAD_SIZES)

    @classmethod
    def supports_head_size(cls, head_size: int) -> bool:
        return head_size in HEAD_SIZES

    @classmethod
    def supports_compute_capability(cls, capability) -> bool:
        return getattr(capability, "major", None) == 10

    @classmethod
    def supports_attn_type(cls, attn_type: str) -> bool:
        return attn_type == AttentionType.DECODER

    @classmethod
    def supports_sink(cls) -> bool:
        return True


@dataclass
class B200AttentionMetadata:
    num_actual_tokens: int
    num_decodes: int
    num_prefills: int
    max_seq_len: int
    query_start_loc: torch.Tensor   # int32 [R + 1]
    seq_lens: torch.Tensor          # int32 [R]
    block_table: torch.Tensor       # int32 [R, W]
    slot_mapping: torch.Tensor      # int64 [T]
    decode_splits: int
    tile_scratch: Optional[torch.Tensor] = None


class B200AttentionMetadataBuilder(AttentionMetadataBuilder[B200AttentionMetadata]):
    _cudagraph_support = AttentionCGSupport.UNIFORM_SINGLE_TOKEN_DECODE

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        self._init_reorder_batch_threshold(1)
        mc = vllm_config.model_config
        pc = vllm_config.parallel_config
        self.num_kv_heads = mc.get_num_kv_heads(pc)
        self.num_heads = mc.get_num_attention_heads(pc)
        self.head_size = mc.get_head_size()
        self.max_model_len = mc.max_model_len
        max_reqs = vllm_config.scheduler_config.max_num_seqs
        self.tile_scratch = torch.zeros(max_reqs + 1, dtype=torch.int32, device=device)
        if device.type == "cuda":
            # split-KV workspace for every decode batch a graph can hold (reserved before any
            # capture: the workspace never grows inside a graph)
            worst = max(b * ops.attention.num_decode_splits(b, self.num_kv_heads,
                                                            self.max_model_len)
                        for b in range(1, max_reqs + 1))
            ops.attention.decode_workspace(device, worst, self.num_heads, self.head_size, 1)

    def _splits(self, nd: int) -> int:
        if self.device.type != "cuda" or nd == 0:
            return 1
        return ops.attention.num_decode_splits(nd, self.num_kv_heads, self.max_model_len)

    def build(self, common_prefix_len: int, common_attn_metadata: CommonAttentionMetadata,
              fast_build: bool = False) -> B200AttentionMetadata:
        cm = common_attn_metadata
        R = cm.num_reqs
        qsl = cm.query_start_loc_cpu[:R + 1]
        q_lens = (qsl[1:] - qsl[:-1]).tolist()
        nd = 0
        while nd < R and q_lens[nd] == 1:
            nd += 1
        return B200AttentionMetadata(
            num_actual_tokens=cm.num_actual_tokens, num_decodes=nd, num_prefills=R - nd,
            max_seq_len=int(cm.max_seq_len),
            query_start_loc=cm.query_start_loc[:R + 1].to(torch.int32),
            seq_lens=cm.seq_lens[:R].to(torch.int32),
            block_table=cm.block_table_tensor[:R].to(torch.int32),
            slot_mapping=cm.slot_mapping.to(torch.int64),
            decode_splits=self._splits(nd), tile_scratch=self.tile_scratch)


class B200AttentionImpl(AttentionImpl):
    def __init__(self, num_heads: int, head_size: int, scale: float,
                 num_kv_heads: Optional[int] = None, alibi_slopes=None,
                 sliding_window: Optional[int] = None, kv_cache_dtype: str = "auto",
                 logits_soft_cap: Optional[float] = None, attn_type: str = AttentionType.DECODER,
                 kv_sharing_target_layer_name: Optional[str] = None,
                 sinks: Optional[torch.Tensor] = None, **unused) -> None:
        if alibi_slopes is not None or (logits_soft_cap or 0) > 0:
            raise NotImplementedError("b200 attention: ALiBi / logit soft-capping not served")
        if attn_type != AttentionType.DECODER:
            raise NotImplementedError("b200 attention: decoder self-attention only")
        if head_size not in HEAD_SIZES:
            raise ValueError(f"b200 attention: head size {head_size} not served")
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = float(scale) if scale else 1.0 / math.sqrt(head_size)
        self.num_kv_heads = num_kv_heads or num_heads
        self.window = int(sliding_window or 0)
        self.kv_cache_dtype = kv_cache_dtype
        self.attn_type = attn_type
        self.sinks = sinks

    def do_kv_cache_update(self, layer, key: torch.Tensor, value: torch.Tensor,
                           kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
        k_cache, v_cache = kv_cache.unbind(0)
        ops.attention.kv_insert(key, value, k_cache, v_cache, slot_mapping)

    def forward(self, layer, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                kv_cache: torch.Tensor, attn_metadata: Optional[B200AttentionMetadata],
                output: torch.Tensor, output_scale=None, output_block_scale=None) -> torch.Tensor:
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("b200 attention: fused output quantisation not served")
        if attn_metadata is None:  # memory-profiling run
            return output.fill_(0)
        m = attn_metadata
        T = m.num_actual_tokens
        q = query[:T].reshape(T, self.num_heads * self.head_size)
        out = output[:T].view(T, self.num_heads * self.head_size)
        k_cache, v_cache = kv_cache.unbind(0)
        sinks = self.sinks.float() if self.sinks is not None else None
        nd, npf = m.num_decodes, m.num_prefills
        if nd:
            ops.paged_decode(q[:nd], k_cache, v_cache, m.block_table[:nd], m.seq_lens[:nd],
                             self.num_heads, self.num_kv_heads, self.scale, m.max_seq_len,
                             out=out[:nd], num_splits=m.decode_splits, sinks=sinks)
        if npf:
            ops.paged_prefill(q, k_cache, v_cache, m.query_start_loc[nd:], m.seq_lens[nd:],
                              m.block_table[nd:], self.num_heads, self.num_kv_heads, self.scale,
                              self.window, out=out, tile_scratch=m.tile_scratch, sinks=sinks)
        return output


def register() -> str:
    """Register the backend as vLLM's CUSTOM attention backend; returns its class path."""
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
    path = f"{B200AttentionBackend.__module__}.{B200AttentionBackend.__qualname__}"
    register_backend(AttentionBackendEnum.CUSTOM, path)
    return path


def serves(cfg) -> bool:
    """Whether an attention selector configuration runs on this backend."""
    return (cfg.dtype == torch.bfloat16 and cfg.head_size in HEAD_SIZES and not cfg.use_mla and
            not cfg.use_sparse and cfg.kv_cache_dtype in (None, "auto", "bfloat16") and
            not cfg.use_mm_prefix and not cfg.use_non_causal and
            cfg.attn_type == AttentionType.DECODER and
            (cfg.block_size is None or cfg.block_size in (16, 32, 64) or cfg.block_size % 64 == 0))
