"""Model registry: architecture name -> implementation class."""
from __future__ import annotations

from ..config import ModelConfig

_REGISTRY = {}


def register_model(arch: str):
    def deco(cls):
        _REGISTRY[arch] = cls
        return cls
    return deco


def get_model_class(cfg: ModelConfig):
    _populate()
    if cfg.arch not in _REGISTRY:
        raise NotImplementedError(f"architecture {cfg.arch!r} is not supported; "
                                  f"supported: {sorted(_REGISTRY)}")
    return _REGISTRY[cfg.arch]


def supported_architectures() -> list:
    _populate()
    return sorted(_REGISTRY)


def _populate():
    if _REGISTRY:
        return
    from .llama import DenseDecoderForCausalLM
    _REGISTRY["llama"] = DenseDecoderForCausalLM
    _REGISTRY["qwen3"] = DenseDecoderForCausalLM
    from .qwen3_moe import Qwen3MoeForCausalLM
    from .qwen3_next import Qwen3NextForCausalLM
    _REGISTRY["qwen3_moe"] = Qwen3MoeForCausalLM
    _REGISTRY["qwen3_next"] = Qwen3NextForCausalLM
    from .deepseek_v2 import DeepseekV2ForCausalLM
    for arch in ("deepseek_v2", "deepseek_v3", "deepseek_v32"):
        _REGISTRY[arch] = DeepseekV2ForCausalLM
    from .mamba2 import Mamba2ForCausalLM
    _REGISTRY["mamba2"] = Mamba2ForCausalLM
