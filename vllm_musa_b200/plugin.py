"""vLLM plugin entry points.

``platform_plugin`` (group ``vllm.platform_plugins``) returns the B200 platform class path when
an sm_100 device is present; ``register_custom_ops`` (group ``vllm.general_plugins``) registers
this package's kernels with vLLM:
  * IR-op providers ``b200`` for ``rms_norm`` / ``fused_add_rms_norm`` (vllm.ir),
  * CustomOp out-of-tree overrides for ``SiluAndMul``, ``RotaryEmbedding`` and ``QuantFP8``.
Reference counterparts: vllm_musa/__init__.py:52-193 (musa_platform_plugin,
register_custom_ops), vllm_musa/kernels/musa_ops.py:66-241 (IR providers),
vllm_musa/model_executor/layers/activation.py:11-53, rotary_embedding/base.py:8-35.
"""
from __future__ import annotations

import logging
from typing import Optional

from . import envs

log = logging.getLogger("vllm_musa_b200")

PLATFORM_CLASS = "vllm_musa_b200.platform.B200Platform"
PROVIDER = "b200"
_REGISTERED = False


def detect_b200() -> bool:
    """True when NVML reports a compute-capability 10.0 device (no CUDA context is created)."""
    if envs.get("B200_FORCE_PLATFORM"):
        return True
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                if tuple(pynvml.nvmlDeviceGetCudaComputeCapability(h)) == (10, 0):
                    return True
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        return False
    return False


def platform_plugin() -> Optional[str]:
    return PLATFORM_CLASS if detect_b200() else None


def register_ir_providers(ir) -> None:
    """Register the ``b200`` providers on a ``vllm.ir`` module (separate for testing)."""
    from .ir_providers import register
    register(ir)


def make_custom_op_classes():
    """OOT subclasses of vLLM's SiluAndMul and RotaryEmbedding running the b200 kernels."""
    import torch
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.rotary_embedding import RotaryEmbedding

    from . import ops

    use_native = envs.get("B200_CUSTOM_OP_USE_NATIVE")

    class B200SiluAndMul(SiluAndMul):
        def forward_oot(self, x: torch.Tensor) -> torch.Tensor:
            if use_native or not x.is_cuda or x.dtype != torch.bfloat16:
                return self.forward_native(x)
            shp = x.shape
            y = ops.silu_and_mul(x.reshape(-1, shp[-1]))
            return y.reshape(*shp[:-1], shp[-1] // 2)

        forward_cuda = forward_oot

    class B200RotaryEmbedding(RotaryEmbedding):
        def forward_oot(self, positions, query, key=None):
            ok = (not use_native and key is not None and query.is_cuda and
                  query.dtype == torch.bfloat16 and self.head_size in (64, 128, 256) and
                  query.dim() == 2 and key.dim() == 2)
            if not ok:
                return self.forward_native(positions, query, key)
            T = query.shape[0]
            hq, hk = query.shape[1] // self.head_size, key.shape[1] // self.head_size
            qk = torch.cat([query, key, torch.empty_like(key)], dim=1)
            cs = self._b200_cos_sin(query.device)
            ops.rope_kv(qk, positions.to(torch.int32).reshape(-1), cs, None, None,
                        torch.full((T,), -1, dtype=torch.int32, device=query.device), hq, hk,
                        self.rotary_dim, self.is_neox_style, write_k=True)
            query.copy_(qk[:, :hq * self.head_size])
            key.copy_(qk[:, hq * self.head_size:(hq + hk) * self.head_size])
            return query, key

        def _b200_cos_sin(self, device):
            cs = getattr(self, "_b200_cs", None)
            if cs is None or cs.device != device:
                c = self.cos_sin_cache.float()
                # vLLM caches [max_pos, rot] as [cos | sin] halves: same layout as ours
                cs = c.to(device).contiguous()
                self._b200_cs = cs
            return cs

        forward_cuda = forward_oot

    return B200SiluAndMul, B200RotaryEmbedding


def make_quant_fp8_class():
    """OOT subclass of vLLM's QuantFP8: dynamic per-token 1x128 e4m3 group quantisation of bf16
    activations (row-major fp32 scales, amax / 448) on the b200 group-quant kernel; every other
    configuration (static scales, per-tensor / per-token, column-major or TMA-aligned or UE8M0
    scales) stays on vLLM's path.  Reference counterpart: vllm_musa/model_executor/layers/
    quantization/input_quant_fp8.py (the QuantFP8 OOT override over the MUSA group-quant op)."""
    import torch
    from vllm.model_executor.layers.quantization.input_quant_fp8 import QuantFP8

    from . import ops

    use_native = envs.get("B200_CUSTOM_OP_USE_NATIVE")

    class B200QuantFP8(QuantFP8):
        def _b200_serves(self, x, scale) -> bool:
            return (not use_native and self.is_group_quant and not self.static and
                    scale is None and getattr(self, "group_size", 0) == 128 and
                    not self.column_major_scales and not self.tma_aligned_scales and
                    not self.use_ue8m0 and x.dtype == torch.bfloat16 and x.dim() == 2 and
                    x.shape[-1] % 128 == 0 and x.is_contiguous())

        def forward_oot(self, x, scale=None, scale_ub=None, use_triton=False):
            if self._b200_serves(x, scale):
                return ops.activation.group_quant_fp8(x)
            if x.is_cuda:
                return self.forward_cuda(x, scale, scale_ub, use_triton)
            return self.forward_native(x, scale, scale_ub, use_triton)

    return B200QuantFP8


# Modules that register torch.ops.b200.* and the IR providers; they must be imported before
# vLLM traces or compiles a model so the ops exist in every process (workers included).
# Reference counterpart: vllm_musa/custom_op_modules.py:5-27.
CUSTOM_OP_MODULES = ("vllm_musa_b200.ops", "vllm_musa_b200.ir_providers")


def preload_custom_op_modules() -> None:
    import importlib
    for name in CUSTOM_OP_MODULES:
        importlib.import_module(name)
    import torch
    from .ops import _ext
    if torch.cuda.is_available():
        _ext.ops()  # load the extension: registers torch.ops.b200.*


def register_custom_ops() -> None:
    global _REGISTERED
    if _REGISTERED:
        return
    try:
        from vllm import ir
        from vllm.model_executor.custom_op import CustomOp
    except Exception as e:  # vLLM not importable: nothing to register into
        log.info("vLLM not available, skipping plugin registration: %s", e)
        return
    preload_custom_op_modules()
    register_ir_providers(ir)
    silu, rope = make_custom_op_classes()
    CustomOp.register_oot(silu, name="SiluAndMul")
    CustomOp.register_oot(rope, name="RotaryEmbedding")
    try:
        CustomOp.register_oot(make_quant_fp8_class(), name="QuantFP8")
    except Exception as e:  # an older vLLM without QuantFP8
        log.info("QuantFP8 override not registered: %s", e)
    _REGISTERED = True
