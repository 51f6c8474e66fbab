"""vLLM platform class for B200 (sm_100a) with this package's kernels.

Subclasses vLLM's NVML CUDA platform and changes what the reference's MUSAPlatform changes for
its device (vllm_musa/platform.py:245-955): default KV block size 64 (one TMA box per page),
the b200 IR-op providers first in priority, custom ops enabled, this package's attention
backend (vllm_backend.py) and device communicator (vllm_comm.py: NVSwitch all-reduce), the
post-grad fusion passes, and its worker (vllm_worker.py: device-architecture check and op
preloading at worker start).
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

    worker_cls: str = "vllm_musa_b200.vllm_worker.B200Worker"

    @classmethod
    def check_and_update_config(cls, vllm_config) -> None:
        par = getattr(vllm_config, "parallel_config", None)
        if par is not None and getattr(par, "worker_cls", None) == "auto":
            par.worker_cls = cls.worker_cls
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
    def get_attn_backend_cls(cls, selected_backend, attn_selector_config, num_heads=None) -> str:
        """This package's paged-attention backend for the decoder attention it serves (bf16,
        head size 64 / 128 / 256, bf16 KV cache, no MLA / sparse / encoder attention) when no
        backend was requested explicitly; vLLM's CUDA selection otherwise.  Reference:
        vllm_musa/platform.py:730-836 (get_valid_backends / get_attn_backend_cls)."""
        from . import vllm_backend
        if selected_backend is None and vllm_backend.serves(attn_selector_config):
            path = vllm_backend.register()
            log.info("attention backend: %s", path)
            return path
        return super().get_attn_backend_cls(selected_backend, attn_selector_config,  # type: ignore[misc]
                                            num_heads)

    @classmethod
    def get_device_communicator_cls(cls) -> str:
        """vLLM's CUDA communicator with the tensor-parallel all-reduce on this package's
        NVSwitch kernels (reference: vllm_musa/platform.py:890-892)."""
        return "vllm_musa_b200.vllm_comm.B200Communicator"

    @classmethod
    def use_custom_allreduce(cls) -> bool:
        return True

    @classmethod
    def check_worker_device(cls) -> None:
        from .native_arch import check_current_device
        check_current_device()
