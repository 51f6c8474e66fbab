"""vllm_musa_b200: a Blackwell-native (sm_100a) LLM serving framework.

Public surface (mirrors what a vllm-musa user drives):
  * ``LLM`` / ``SamplingParams`` offline API and ``LLMEngine``;
  * an OpenAI-compatible HTTP server (``python -m vllm_musa_b200.entrypoints.openai.api_server``
    or ``b200-vllm serve``);
  * vLLM plugin entry points ``b200_platform_plugin`` (``vllm.platform_plugins``) and
    ``register_custom_ops`` (``vllm.general_plugins``), reference: vllm_musa/__init__.py:52-193;
  * ``torch.ops.b200.*`` custom ops over the hand-written sm_100a kernels.
"""
from __future__ import annotations

__version__ = "0.1.0"

__all__ = ["LLM", "LLMEngine", "SamplingParams", "StructuredOutputsParams", "LoRARequest",
           "BeamSearchParams", "PoolingParams",
           "EngineConfig", "ModelConfig", "b200_platform_plugin", "register_custom_ops",
           "__version__"]


def __getattr__(name):
    if name == "LLM":
        from .entrypoints.llm import LLM
        return LLM
    if name == "LLMEngine":
        from .engine.llm_engine import LLMEngine
        return LLMEngine
    if name in ("SamplingParams", "StructuredOutputsParams", "BeamSearchParams",
                "PoolingParams"):
        from .sample import sampling_params
        return getattr(sampling_params, name)
    if name == "LoRARequest":
        from .lora import LoRARequest
        return LoRARequest
    if name in ("EngineConfig", "ModelConfig"):
        from . import config
        return getattr(config, name)
    raise AttributeError(name)


def b200_platform_plugin():
    """``vllm.platform_plugins`` entry point: the platform class path when a B200 is present."""
    from .plugin import platform_plugin
    return platform_plugin()


def register_custom_ops():
    """``vllm.general_plugins`` entry point: register torch.ops.b200.* and the vLLM overrides."""
    from .plugin import register_custom_ops as _reg
    return _reg()
