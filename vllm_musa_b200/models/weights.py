"""Weight sources: HuggingFace safetensors checkpoints and seeded random ("dummy") weights.

Both yield ``(hf_name, tensor)`` pairs in HuggingFace naming, so every model has exactly one
loading path (``load_weights``) that shards and fuses.  Random weights are drawn parameter
by parameter from one seeded generator in a fixed order, full logical shape first and then
sharded by the model, so a tensor-parallel run sees the same logical weights as a
single-GPU run.  Reference: upstream vLLM's loader (HF safetensors, ``load_format=dummy``),
used by the reference unchanged.
"""
from __future__ import annotations

import glob
import json
import os
from typing import Iterator, Tuple

import torch

from ..config import ModelConfig


def safetensors_weights(path: str, device: str = "cpu") -> Iterator[Tuple[str, torch.Tensor]]:
    from safetensors import safe_open
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no *.safetensors under {path}")
    for f in files:
        with safe_open(f, framework="pt", device=device) as fh:
            for name in fh.keys():
                yield name, fh.get_tensor(name)


def _mamba2_shapes(cfg: ModelConfig) -> list:
    """transformers' Mamba2ForCausalLM parameter names (``backbone.*``)."""
    H, V = cfg.hidden_size, cfg.vocab_size
    nh, P, G, N = cfg.mamba_num_heads, cfg.mamba_head_dim, cfg.mamba_n_groups, cfg.ssm_state_size
    dI = nh * P
    conv_dim = dI + 2 * G * N
    out = [("backbone.embeddings.weight", (V, H), "w")]
    for i in range(cfg.num_layers):
        p = f"backbone.layers.{i}."
        m = p + "mixer."
        out += [(p + "norm.weight", (H,), "norm"),
                (m + "in_proj.weight", (2 * dI + 2 * G * N + nh, H), "w"),
                (m + "conv1d.weight", (conv_dim, 1, cfg.mamba_conv_kernel), "conv")]
        if cfg.mamba_conv_bias:
            out.append((m + "conv1d.bias", (conv_dim,), "norm0"))
        out += [(m + "dt_bias", (nh,), "norm"),
                (m + "A_log", (nh,), "a_log"),
                (m + "D", (nh,), "norm"),
                (m + "norm.weight", (dI,), "norm"),
                (m + "out_proj.weight", (H, dI), "w")]
    out.append(("backbone.norm_f.weight", (H,), "norm"))
    if not cfg.tie_word_embeddings:
        out.append(("lm_head.weight", (V, H), "w"))
    return out


def hf_param_shapes(cfg: ModelConfig) -> list:
    """Ordered (name, shape, kind) list of the dense/MoE decoder parameters (HF names)."""
    H, D, V = cfg.hidden_size, cfg.head_dim, cfg.vocab_size
    if cfg.arch == "mamba2":
        return _mamba2_shapes(cfg)
    out = [("model.embed_tokens.weight", (V, H), "w")]
    if cfg.arch.startswith("deepseek"):
        return out + _deepseek_shapes(cfg)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        hybrid = cfg.arch == "qwen3_next"
        norm = "norm0" if hybrid else "norm"  # Qwen3-Next stores (1 + w) norms as w
        out.append((p + "input_layernorm.weight", (H,), norm))
        if hybrid and (i + 1) % (cfg.full_attention_interval or 4):
            Hk, Hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
            dk, dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
            conv_dim = 2 * Hk * dk + Hv * dv
            q = p + "linear_attn."
            out += [(q + "in_proj_qkvz.weight", (2 * Hk * dk + 2 * Hv * dv, H), "w"),
                    (q + "in_proj_ba.weight", (2 * Hv, H), "w"),
                    (q + "conv1d.weight", (conv_dim, 1, cfg.linear_conv_kernel_dim), "conv"),
                    (q + "dt_bias", (Hv,), "norm"),
                    (q + "A_log", (Hv,), "a_log"),
                    (q + "norm.weight", (dv,), "norm"),
                    (q + "out_proj.weight", (H, Hv * dv), "w")]
        else:
            qrows = cfg.num_heads * D * (2 if cfg.attn_output_gate else 1)
            out += [
                (p + "self_attn.q_proj.weight", (qrows, H), "w"),
                (p + "self_attn.k_proj.weight", (cfg.num_kv_heads * D, H), "w"),
                (p + "self_attn.v_proj.weight", (cfg.num_kv_heads * D, H), "w"),
                (p + "self_attn.o_proj.weight", (H, cfg.num_heads * D), "w"),
            ]
            if cfg.qk_norm:
                out += [(p + "self_attn.q_norm.weight", (D,), norm),
                        (p + "self_attn.k_norm.weight", (D,), norm)]
        out.append((p + "post_attention_layernorm.weight", (H,), norm))
        if cfg.is_moe:
            E, I = cfg.num_experts, cfg.moe_intermediate_size
            out.append((p + "mlp.gate.weight", (E, H), "w"))
            for e in range(E):
                q = f"{p}mlp.experts.{e}."
                out += [(q + "gate_proj.weight", (I, H), "w"), (q + "up_proj.weight", (I, H), "w"),
                        (q + "down_proj.weight", (H, I), "w")]
            if cfg.shared_expert_intermediate_size:
                Is = cfg.shared_expert_intermediate_size
                q = p + "mlp.shared_expert."
                out += [(q + "gate_proj.weight", (Is, H), "w"), (q + "up_proj.weight", (Is, H), "w"),
                        (q + "down_proj.weight", (H, Is), "w"),
                        (p + "mlp.shared_expert_gate.weight", (1, H), "w")]
        else:
            I = cfg.intermediate_size
            out += [(p + "mlp.gate_proj.weight", (I, H), "w"), (p + "mlp.up_proj.weight", (I, H), "w"),
                    (p + "mlp.down_proj.weight", (H, I), "w")]
    out.append(("model.norm.weight", (H,), "norm0" if cfg.arch == "qwen3_next" else "norm"))
    if not cfg.tie_word_embeddings:
        out.append(("lm_head.weight", (V, H), "w"))
    return out


def _deepseek_shapes(cfg: ModelConfig) -> list:
    """DeepSeek-V2/V3/V3.2 HF names (MLA, optional lightning indexer, grouped MoE, and the
    multi-token-prediction layer at index num_layers)."""
    H, V, Hq = cfg.hidden_size, cfg.vocab_size, cfg.num_heads
    nope, rope, vd = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim
    out = []
    n_mtp = 1 if cfg.num_nextn_predict_layers > 0 else 0
    for i in range(cfg.num_layers + n_mtp):
        p = f"model.layers.{i}."
        if i == cfg.num_layers:
            out += [(p + "enorm.weight", (H,), "norm"), (p + "hnorm.weight", (H,), "norm"),
                    (p + "eh_proj.weight", (H, 2 * H), "w"),
                    (p + "shared_head.norm.weight", (H,), "norm"),
                    (p + "shared_head.head.weight", (V, H), "w")]
        a = p + "self_attn."
        out.append((p + "input_layernorm.weight", (H,), "norm"))
        if cfg.q_lora_rank:
            out += [(a + "q_a_proj.weight", (cfg.q_lora_rank, H), "w"),
                    (a + "q_a_layernorm.weight", (cfg.q_lora_rank,), "norm"),
                    (a + "q_b_proj.weight", (Hq * (nope + rope), cfg.q_lora_rank), "w")]
        else:
            out.append((a + "q_proj.weight", (Hq * (nope + rope), H), "w"))
        out += [(a + "kv_a_proj_with_mqa.weight", (cfg.kv_lora_rank + rope, H), "w"),
                (a + "kv_a_layernorm.weight", (cfg.kv_lora_rank,), "norm"),
                (a + "kv_b_proj.weight", (Hq * (nope + vd), cfg.kv_lora_rank), "w"),
                (a + "o_proj.weight", (H, Hq * vd), "w")]
        if cfg.index_topk:
            x = a + "indexer."
            out += [(x + "wq_b.weight", (cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank), "w"),
                    (x + "wk.weight", (cfg.index_head_dim, H), "w"),
                    (x + "k_norm.weight", (cfg.index_head_dim,), "norm"),
                    (x + "k_norm.bias", (cfg.index_head_dim,), "norm0"),
                    (x + "weights_proj.weight", (cfg.index_n_heads, H), "w")]
        out.append((p + "post_attention_layernorm.weight", (H,), "norm"))
        if cfg.num_experts and i >= cfg.first_k_dense:
            E, I = cfg.num_experts, cfg.moe_intermediate_size
            out += [(p + "mlp.gate.weight", (E, H), "w"),
                    (p + "mlp.gate.e_score_correction_bias", (E,), "norm0")]
            for e in range(E):
                q = f"{p}mlp.experts.{e}."
                out += [(q + "gate_proj.weight", (I, H), "w"), (q + "up_proj.weight", (I, H), "w"),
                        (q + "down_proj.weight", (H, I), "w")]
            if cfg.shared_expert_intermediate_size:
                Is, q = cfg.shared_expert_intermediate_size, p + "mlp.shared_experts."
                out += [(q + "gate_proj.weight", (Is, H), "w"), (q + "up_proj.weight", (Is, H), "w"),
                        (q + "down_proj.weight", (H, Is), "w")]
        else:
            I = cfg.intermediate_size
            out += [(p + "mlp.gate_proj.weight", (I, H), "w"), (p + "mlp.up_proj.weight", (I, H), "w"),
                    (p + "mlp.down_proj.weight", (H, I), "w")]
    out.append(("model.norm.weight", (H,), "norm"))
    if not cfg.tie_word_embeddings:
        out.append(("lm_head.weight", (V, H), "w"))
    return out


def dummy_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02, device: str = "cpu",
                  dtype: torch.dtype | None = None,
                  shapes: list | None = None) -> Iterator[Tuple[str, torch.Tensor]]:
    """N(0, std) matrices and unit norm weights from one generator seeded with ``seed``."""
    dtype = dtype or cfg.dtype
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    for name, shape, kind in (shapes or hf_param_shapes(cfg)):
        if kind == "norm":
            yield name, torch.ones(shape, dtype=dtype, device=device)
        elif kind == "norm0":
            yield name, torch.zeros(shape, dtype=dtype, device=device)
        elif kind == "a_log":  # decay rates A = 1..16 (log-spaced), as HF initialises them
            yield name, torch.log(torch.linspace(1.0, 16.0, shape[0])).to(dtype).to(device)
        elif kind == "conv":
            t = torch.empty(shape, dtype=torch.float32, device=device)
            t.normal_(0.0, 0.3, generator=gen)
            yield name, t.to(dtype)
        else:
            t = torch.empty(shape, dtype=torch.float32, device=device)
            t.normal_(0.0, std, generator=gen)
            yield name, t.to(dtype)


def save_safetensors(weights, path: str, cfg_dict: dict | None = None) -> None:
    """Write ``(name, tensor)`` pairs as one safetensors file (tests / examples)."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    save_file({n: t.contiguous().cpu() for n, t in weights},
              os.path.join(path, "model.safetensors"))
    if cfg_dict is not None:
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(cfg_dict, f)
