"""Engine configuration: model architecture, KV cache, scheduler, parallelism.

The reference takes these from upstream vLLM's ``VllmConfig`` and mutates them in platform
hooks (vllm_musa/platform.py:442-720: block size 64 pin, custom-op defaults, compile
ranges).  Here they are plain dataclasses with B200 defaults: 64-token KV pages (one TMA box
per page and head), chunked prefill with an 8K token budget, CUDA graphs for decode batches.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any, Optional

import torch


@dataclass
class ModelConfig:
    arch: str = "llama"  # llama | qwen3 | qwen3_moe | deepseek_v3 | qwen3_next
    vocab_size: int = 32000
    hidden_size: int = 4096
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: Optional[dict] = None
    rotary_dim: Optional[int] = None  # default head_dim
    rope_neox: bool = True
    max_position: int = 8192
    tie_word_embeddings: bool = False
    qk_norm: bool = False
    attention_bias: bool = False
    # mixture of experts
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    shared_expert_intermediate_size: int = 0
    first_k_dense: int = 0
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0
    scoring_func: str = "softmax"
    # multi-head latent attention (DeepSeek)
    q_lora_rank: int = 0
    kv_lora_rank: int = 0
    qk_nope_head_dim: int = 0
    qk_rope_head_dim: int = 0
    v_head_dim: int = 0
    index_n_heads: int = 0
    index_head_dim: int = 0
    index_topk: int = 0
    num_nextn_predict_layers: int = 0
    quant: Optional[str] = None  # None | "fp8_block" | "w4afp8" (int4 experts, fp8 linears)
    # hybrid linear attention (Qwen3-Next)
    full_attention_interval: int = 0
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 0
    linear_value_head_dim: int = 0
    linear_conv_kernel_dim: int = 4
    partial_rotary_factor: float = 1.0
    attn_output_gate: bool = False
    # clamped SwiGLU (gate <= limit, |up| <= limit) in MLPs and experts; 0: plain SwiGLU
    swiglu_limit: float = 0.0
    # KV cache storage: "auto" (model dtype) or a TurboQuant preset (turboquant_k8v4,
    # turboquant_4bit_nc, turboquant_k3v4_nc, turboquant_3bit_nc)
    kv_cache_dtype: str = "auto"
    # Mamba2 (state-space) mixers
    ssm_state_size: int = 0
    mamba_num_heads: int = 0
    mamba_head_dim: int = 0
    mamba_n_groups: int = 1
    mamba_expand: int = 2
    mamba_conv_kernel: int = 4
    mamba_conv_bias: bool = True
    mamba_dt_min: float = 0.0
    mamba_dt_max: float = float("inf")
    eos_token_id: Optional[int] = None
    dtype: torch.dtype = torch.bfloat16
    name: str = ""

    @property
    def rot_dim(self) -> int:
        if self.rotary_dim:
            return self.rotary_dim
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def num_params(self) -> int:
        """Approximate parameter count (dense and MoE decoders)."""
        H, L, V = self.hidden_size, self.num_layers, self.vocab_size
        attn = H * (self.num_heads + 2 * self.num_kv_heads) * self.head_dim + \
            self.num_heads * self.head_dim * H
        if self.is_moe:
            mlp = self.num_experts * 3 * H * self.moe_intermediate_size + H * self.num_experts
            mlp += 3 * H * self.shared_expert_intermediate_size
        else:
            mlp = 3 * H * self.intermediate_size
        emb = V * H * (1 if self.tie_word_embeddings else 2)
        return L * (attn + mlp) + emb

    @staticmethod
    def _from_hf_mamba2(hf: dict, a: str) -> "ModelConfig":
        """transformers' Mamba2Config keys (state_size, expand, head_dim, n_groups, ...)."""
        H = hf["hidden_size"]
        expand = hf.get("expand", 2)
        P = hf.get("head_dim", 64)
        nh = hf.get("num_heads") or expand * H // P
        lim = hf.get("time_step_limit") or (0.0, float("inf"))
        eos = hf.get("eos_token_id")
        return ModelConfig(
            arch="mamba2", vocab_size=hf["vocab_size"], hidden_size=H,
            num_layers=hf["num_hidden_layers"], num_heads=nh, num_kv_heads=nh, head_dim=P,
            intermediate_size=expand * H, rms_norm_eps=hf.get("layer_norm_epsilon", 1e-5),
            max_position=hf.get("max_position_embeddings", 1 << 20),
            tie_word_embeddings=hf.get("tie_word_embeddings", True),
            ssm_state_size=hf.get("state_size", 128), mamba_num_heads=nh, mamba_head_dim=P,
            mamba_n_groups=hf.get("n_groups", 1) or 1, mamba_expand=expand,
            mamba_conv_kernel=hf.get("conv_kernel", 4), mamba_conv_bias=hf.get("use_conv_bias",
                                                                               True),
            mamba_dt_min=float(lim[0]), mamba_dt_max=float(lim[1]),
            eos_token_id=eos[0] if isinstance(eos, list) else eos, name=a)

    @staticmethod
    def from_hf(config: "str | dict") -> "ModelConfig":
        """Build from a HuggingFace ``config.json`` (path, directory or dict)."""
        if isinstance(config, str):
            path = os.path.join(config, "config.json") if os.path.isdir(config) else config
            with open(path) as f:
                hf = json.load(f)
        else:
            hf = dict(config)
        archs = hf.get("architectures") or [""]
        a = archs[0]
        mt = hf.get("model_type", "")
        if "Mamba2" in a or mt == "mamba2":
            return ModelConfig._from_hf_mamba2(hf, a)
        if "Qwen3Next" in a or mt == "qwen3_next":
            arch = "qwen3_next"
        elif "Qwen3Moe" in a or mt == "qwen3_moe":
            arch = "qwen3_moe"
        elif "Qwen3" in a or mt == "qwen3":
            arch = "qwen3"
        elif "Deepseek" in a or mt.startswith("deepseek"):
            arch = "deepseek_v3"
        else:
            arch = "llama"
        H = hf["hidden_size"]
        nh = hf["num_attention_heads"]
        c = ModelConfig(
            arch=arch,
            vocab_size=hf["vocab_size"],
            hidden_size=H,
            num_layers=hf["num_hidden_layers"],
            num_heads=nh,
            num_kv_heads=hf.get("num_key_value_heads", nh),
            head_dim=hf.get("head_dim") or H // nh,
            intermediate_size=hf.get("intermediate_size", 4 * H),
            rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
            rope_theta=hf.get("rope_theta", 10000.0),
            rope_scaling=hf.get("rope_scaling"),
            max_position=hf.get("max_position_embeddings", 8192),
            tie_word_embeddings=hf.get("tie_word_embeddings", False),
            qk_norm=arch in ("qwen3", "qwen3_moe", "qwen3_next"),
            attention_bias=hf.get("attention_bias", False),
            num_experts=hf.get("num_experts", hf.get("n_routed_experts", 0)) or 0,
            num_experts_per_tok=hf.get("num_experts_per_tok", 0) or 0,
            moe_intermediate_size=hf.get("moe_intermediate_size", 0) or 0,
            norm_topk_prob=hf.get("norm_topk_prob", True),
            shared_expert_intermediate_size=hf.get("shared_expert_intermediate_size", 0) or
            (hf.get("n_shared_experts", 0) or 0) * (hf.get("moe_intermediate_size", 0) or 0),
            first_k_dense=hf.get("first_k_dense_replace", 0) or 0,
            n_group=hf.get("n_group", 1) or 1,
            topk_group=hf.get("topk_group", 1) or 1,
            routed_scaling_factor=hf.get("routed_scaling_factor", 1.0) or 1.0,
            scoring_func=hf.get("scoring_func", "softmax"),
            q_lora_rank=hf.get("q_lora_rank", 0) or 0,
            kv_lora_rank=hf.get("kv_lora_rank", 0) or 0,
            qk_nope_head_dim=hf.get("qk_nope_head_dim", 0) or 0,
            qk_rope_head_dim=hf.get("qk_rope_head_dim", 0) or 0,
            v_head_dim=hf.get("v_head_dim", 0) or 0,
            index_n_heads=hf.get("index_n_heads", 0) or 0,
            index_head_dim=hf.get("index_head_dim", 0) or 0,
            index_topk=hf.get("index_topk", 0) or 0,
            num_nextn_predict_layers=hf.get("num_nextn_predict_layers", 0) or 0,
            full_attention_interval=hf.get("full_attention_interval", 0) or 0,
            linear_num_key_heads=hf.get("linear_num_key_heads", 0) or 0,
            linear_num_value_heads=hf.get("linear_num_value_heads", 0) or 0,
            linear_key_head_dim=hf.get("linear_key_head_dim", 0) or 0,
            linear_value_head_dim=hf.get("linear_value_head_dim", 0) or 0,
            linear_conv_kernel_dim=hf.get("linear_conv_kernel_dim", 4) or 4,
            partial_rotary_factor=hf.get("partial_rotary_factor", 1.0) or 1.0,
            attn_output_gate=arch == "qwen3_next",
            swiglu_limit=float(hf.get("swiglu_limit") or 0.0),
            # DeepSeek checkpoints rotate interleaved (even, odd) pairs (HF rope_interleave)
            rope_neox=not (arch == "deepseek_v3" and hf.get("rope_interleave", True)),
            eos_token_id=(hf.get("eos_token_id")[0] if isinstance(hf.get("eos_token_id"), list)
                          else hf.get("eos_token_id")),
            name=a,
        )
        qc = hf.get("quantization_config") or {}
        if qc.get("quant_method") == "fp8" and qc.get("weight_block_size"):
            c.quant = "fp8_block"
        elif qc.get("quant_method") == "w4afp8":
            # packed int4 routed experts (group 128, bf16 scales) beside block-FP8 linears;
            # vllm_musa/model_executor/layers/quantization/w4afp8.py:37-44 sets the same limits
            if int(qc.get("moe_group_size", 128)) != 128:
                raise ValueError("W4AFP8 requires moe_group_size=128")
            if qc.get("activation_scheme", "dynamic") != "dynamic":
                raise ValueError("W4AFP8 requires dynamic FP8 activations")
            c.quant = "w4afp8"
        return c


@dataclass
class CacheConfig:
    block_size: int = 64
    gpu_memory_utilization: float = 0.90
    num_gpu_blocks: Optional[int] = None  # override the memory-derived block count
    kv_dtype: torch.dtype = torch.bfloat16
    enable_prefix_caching: bool = True


@dataclass
class SchedulerConfig:
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    max_model_len: int = 4096
    enable_chunked_prefill: bool = True
    long_prefill_token_threshold: int = 0
    # "fcfs" or "priority" (requests carry an int priority, lower first; vLLM's policy names)
    scheduling_policy: str = "fcfs"

    def __post_init__(self):
        if self.scheduling_policy not in ("fcfs", "priority"):
            raise ValueError("scheduling_policy must be 'fcfs' or 'priority'")


@dataclass
class ParallelConfig:
    tensor_parallel_size: int = 1
    pipeline_parallel_size: int = 1
    data_parallel_size: int = 1
    enable_expert_parallel: bool = False
    # decode context parallelism: shard the (replicated) MLA latent cache by token over the
    # tensor-parallel group; must equal tensor_parallel_size when > 1
    decode_context_parallel_size: int = 1
    distributed_backend: str = "nccl"
    use_custom_allreduce: bool = True


@dataclass
class SpeculativeConfig:
    """Speculative decoding.  ``ngram``: prompt lookup (drafts copied from the continuation of
    the latest earlier occurrence of the context's suffix n-gram, n in [prompt_lookup_min,
    prompt_lookup_max]); ``mtp``: the checkpoint's multi-token-prediction layer (DeepSeek);
    ``eagle3``: an EAGLE-3 head (three target residual streams, own draft vocabulary);
    ``medusa``: Medusa heads on the final hidden state (chains or token trees); model drafters
    chain ``num_speculative_tokens`` > 1 drafts through their layer;
    ``eagle``: an EAGLE-1 head over a dense decoder, loaded from ``model`` (a safetensors
    directory) or, without one, seeded random weights.

    Token trees (``tree_width`` > 1): ``ngram`` merges the continuations of up to
    ``tree_width`` earlier occurrences of the suffix into a trie of at most
    ``num_speculative_tokens`` nodes; ``eagle`` proposes the head's top ``tree_width`` tokens as
    siblings.  vLLM's ``speculative_token_tree`` (a list of child-index paths such as
    ``"[(0,), (1,), (2,)]"``) is accepted for one-level trees and sets ``tree_width``.  The
    whole tree is verified in one step under per-node ancestor masks.

    ``draft_tensor_parallel_size=1`` keeps a whole EAGLE head on every rank of a
    tensor-parallel target (its layer then needs no all-reduce)."""
    method: Optional[str] = None  # None | "ngram" | "mtp" | "eagle" | "eagle3" | "medusa"
    num_speculative_tokens: int = 0
    model: Optional[str] = None
    prompt_lookup_min: int = 1
    prompt_lookup_max: int = 4
    tree_width: int = 1
    speculative_token_tree: Optional[str] = None
    # 1: the draft head runs whole on every rank (no collectives in the draft layer) under a
    # tensor-parallel target; None: sharded like the target
    draft_tensor_parallel_size: Optional[int] = None

    def __post_init__(self):
        if self.speculative_token_tree:
            import ast
            paths = ast.literal_eval(self.speculative_token_tree) \
                if isinstance(self.speculative_token_tree, str) else self.speculative_token_tree
            paths = [tuple(p) for p in paths]
            if not paths or any(len(p) != 1 for p in paths) or \
                    sorted(p[0] for p in paths) != list(range(len(paths))):
                raise ValueError("speculative_token_tree: one-level trees [(0,), (1,), ...] "
                                 "are served")
            self.tree_width = len(paths)
        if self.tree_width < 1:
            raise ValueError("tree_width must be >= 1")
        if self.draft_tensor_parallel_size == 1 and self.method == "mtp":
            raise ValueError("draft_tensor_parallel_size=1 serves EAGLE heads (the MTP layer "
                             "is sharded like the target)")

    @property
    def tree(self) -> bool:
        return self.tree_width > 1

    @staticmethod
    def from_dict(d: Optional[dict]) -> "SpeculativeConfig":
        if not d:
            return SpeculativeConfig()
        return SpeculativeConfig(**{k: v for k, v in d.items()
                                    if k in SpeculativeConfig.__dataclass_fields__})


@dataclass
class LoRAConfig:
    """Multi-LoRA serving: adapters of rank <= max_lora_rank in max_loras device slots."""
    enable_lora: bool = False
    max_loras: int = 4
    max_lora_rank: int = 64


LOGPROBS_MODES = ("raw_logprobs", "raw_logits", "processed_logprobs", "processed_logits")


@dataclass
class EngineConfig:
    model: ModelConfig = field(default_factory=ModelConfig)
    cache: CacheConfig = field(default_factory=CacheConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    device: str = "cuda"
    seed: int = 0
    load_format: str = "dummy"  # dummy (random N(0, init_std)) | safetensors
    model_path: Optional[str] = None
    init_std: float = 0.02
    enforce_eager: bool = False
    cuda_graph_sizes: Optional[list] = None
    speculative: SpeculativeConfig = field(default_factory=SpeculativeConfig)
    lora: LoRAConfig = field(default_factory=lambda: LoRAConfig())
    # what ``logprobs`` report (vLLM's logprobs_mode): raw_logprobs (log_softmax of the model's
    # logits, the default), raw_logits, processed_logprobs / processed_logits (after penalties,
    # logit bias, bad words, token masks and the temperature division)
    logprobs_mode: str = "raw_logprobs"

    def __post_init__(self):
        if self.logprobs_mode not in LOGPROBS_MODES:
            raise ValueError(f"logprobs_mode must be one of {LOGPROBS_MODES}")

    def replace(self, **kw: Any) -> "EngineConfig":
        return dataclasses.replace(self, **kw)
