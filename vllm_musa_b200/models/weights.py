"""Weight sources: HuggingFace safetensors checkpoints and seeded random ("dummy") weights.

Both yield ``(hf_name, tensor)`` pairs in HuggingFace naming, so every model has exactly one
loading path (``load_weights``) that shards and fuses.  Random weights are drawn parameter
by parameter from one seeded generator in a fixed order, full logical shape first and then
sharded by the model, so a tensor-parallel run sees the same logical weights as a
single-GPU run.  Reference: upstream vLLM's loader (HF safetensors, ``load_format=dummy``),
used by the reference unchanged (checkpoint row).
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


def hf_param_shapes(cfg: ModelConfig) -> list:
    """Ordered (name, shape, kind) list of the dense/MoE decoder parameters (HF names)."""
    H, D, V = cfg.hidden_size, cfg.head_dim, cfg.vocab_size
    out = [("model.embed_tokens.weight", (V, H), "w")]
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (H,), "norm"),
            (p + "self_attn.q_proj.weight", (cfg.num_heads * D, H), "w"),
            (p + "self_attn.k_proj.weight", (cfg.num_kv_heads * D, H), "w"),
            (p + "self_attn.v_proj.weight", (cfg.num_kv_heads * D, H), "w"),
            (p + "self_attn.o_proj.weight", (H, cfg.num_heads * D), "w"),
        ]
        if cfg.qk_norm:
            out += [(p + "self_attn.q_norm.weight", (D,), "norm"),
                    (p + "self_attn.k_norm.weight", (D,), "norm")]
        out.append((p + "post_attention_layernorm.weight", (H,), "norm"))
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
