"""Architecture presets for the benchmark configurations (random-init weights; no network).

Each preset reproduces the named architecture's shapes; weights come from
``load_format="dummy"`` (N(0, init_std), seeded) unless a checkpoint path is given.
"""
from __future__ import annotations

import torch

from ..config import ModelConfig


def tiny_llama() -> ModelConfig:
    """CPU plumbing model: 2 layers, hidden 256, 4q/2kv heads of 64, SwiGLU 688, vocab 1024."""
    return ModelConfig(arch="llama", vocab_size=1024, hidden_size=256, num_layers=2, num_heads=4,
                       num_kv_heads=2, head_dim=64, intermediate_size=688, rms_norm_eps=1e-6,
                       rope_theta=1e4, max_position=2048, dtype=torch.float32, name="tiny-llama")


def llama3_8b() -> ModelConfig:
    return ModelConfig(arch="llama", vocab_size=128256, hidden_size=4096, num_layers=32,
                       num_heads=32, num_kv_heads=8, head_dim=128, intermediate_size=14336,
                       rms_norm_eps=1e-5, rope_theta=5e5, max_position=8192, eos_token_id=128001,
                       name="Llama-3-8B")


def qwen3_30b_a3b() -> ModelConfig:
    return ModelConfig(arch="qwen3_moe", vocab_size=151936, hidden_size=2048, num_layers=48,
                       num_heads=32, num_kv_heads=4, head_dim=128, intermediate_size=6144,
                       rms_norm_eps=1e-6, rope_theta=1e6, max_position=40960, qk_norm=True,
                       num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768,
                       norm_topk_prob=True, eos_token_id=151645, name="Qwen3-30B-A3B")


def deepseek_v32() -> ModelConfig:
    return ModelConfig(arch="deepseek_v3", vocab_size=129280, hidden_size=7168, num_layers=61,
                       num_heads=128, num_kv_heads=128, head_dim=192, intermediate_size=18432,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=163840,
                       num_experts=256, num_experts_per_tok=8, moe_intermediate_size=2048,
                       shared_expert_intermediate_size=2048, first_k_dense=3, n_group=8,
                       topk_group=4, routed_scaling_factor=2.5, scoring_func="sigmoid",
                       q_lora_rank=1536, kv_lora_rank=512, qk_nope_head_dim=128,
                       qk_rope_head_dim=64, v_head_dim=128, index_n_heads=64, index_head_dim=128,
                       index_topk=2048, num_nextn_predict_layers=1, quant="fp8_block",
                       rope_neox=False, eos_token_id=1, name="DeepSeek-V3.2")


def qwen3_next_80b() -> ModelConfig:
    return ModelConfig(arch="qwen3_next", vocab_size=151936, hidden_size=2048, num_layers=48,
                       num_heads=16, num_kv_heads=2, head_dim=256, intermediate_size=5120,
                       rms_norm_eps=1e-6, rope_theta=1e7, max_position=262144, qk_norm=True,
                       num_experts=512, num_experts_per_tok=10, moe_intermediate_size=512,
                       shared_expert_intermediate_size=512, full_attention_interval=4,
                       linear_num_key_heads=16, linear_num_value_heads=32,
                       linear_key_head_dim=128, linear_value_head_dim=128,
                       linear_conv_kernel_dim=4, partial_rotary_factor=0.25,
                       attn_output_gate=True, eos_token_id=151645, name="Qwen3-Next-80B-A3B")


PRESETS = {
    "tiny-llama": tiny_llama,
    "llama3-8b": llama3_8b,
    "qwen3-30b-a3b": qwen3_30b_a3b,
    "deepseek-v3.2": deepseek_v32,
    "qwen3-next-80b-a3b": qwen3_next_80b,
}


def get_preset(name: str) -> ModelConfig:
    key = name.lower()
    if key not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[key]()
