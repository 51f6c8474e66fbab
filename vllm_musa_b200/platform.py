"""vLLM platform class for B200 (sm_100a) with this package's kernels.

Subclasses vLLM's NVML CUDA platform and changes what the reference's MUSAPlatform changes for
its device (vllm_musa/platform.py:245-955): default KV block size 64 (one TMA box per page),
the b200 IR-op providers first in priority, custom ops enabled, the custom all-reduce on, a
device-architecture check at worker start.
"""
from __future__ import annotations

import logging

log = logging.getLogger("vllm_musa_b200")

try:  # pragma: no cover - depends on the installed vLLM
    from vllm.platforms.cuda import NvmlCudaPlatform as _Base
except Exception:  # vLLM missing: a stand-in keeps the module importable for tests
    _Base = object


class B200Platform(_Base):
    device_name: str = "cuda"
    b200_default_block_size: int = 64

    @classmethod
    def get_device_name(cls, device_id: int = 0) -> str:
        try:
            return super().get_device_name(device_id)  # type: ignore[misc]
        except Exception:
            return "NVIDIA B200"

    @classmethod
    def check_and_update_config(cls, vllm_config) -> None:
        if hasattr(super(), "check_and_update_config"):
            super().check_and_update_config(vllm_config)  # type: ignore[misc]
        cache = getattr(vllm_config, "cache_config", None)
        if cache is not None and getattr(cache, "block_size", None) in (None, 16):
            cache.block_size = cls.b200_default_block_size
        comp = getattr(vllm_config, "compilation_config", None)
        if comp is not None and hasattr(comp, "custom_ops") and "all" not in comp.custom_ops:
            comp.custom_ops.append("all")
        from .plugin import register_custom_ops
        register_custom_ops()

    @classmethod
    def get_default_ir_op_priority(cls, vllm_config):
        from vllm.config.kernel import IrOpPriorityConfig
        base = ["b200", "native"]
        return IrOpPriorityConfig.with_default(["native"], rms_norm=base, fused_add_rms_norm=base)

    @classmethod
    def get_pass_manager_cls(cls) -> str:
        return "vllm_musa_b200.compile.vllm_pass_manager.B200PostGradPassManager"

    @classmethod
    def use_custom_allreduce(cls) -> bool:
        return True

    @classmethod
    def check_worker_device(cls) -> None:
        from .native_arch import check_current_device
        check_current_device()
