"""Check that the running GPU matches the architecture the extension was built for.

Reference counterpart: vllm_musa/native_arch.py:18-47 (built_archs / check_device_arch),
called from the worker's init_device.  The extension is compiled for sm_100a only.
"""
from __future__ import annotations

from typing import Tuple

BUILT_ARCHS = ("sm_100a",)
REQUIRED_CAPABILITY: Tuple[int, int] = (10, 0)


def built_archs() -> Tuple[str, ...]:
    try:
        from .ops import _ext
        mod = _ext.load()
        if mod is not None:
            return (str(mod.BUILT_ARCH),)
    except Exception:  # pragma: no cover
        pass
    return BUILT_ARCHS


def check_device_arch(capability: Tuple[int, int], name: str = "") -> None:
    """Raise if a device of ``capability`` cannot run the sm_100a kernels."""
    if tuple(capability) != REQUIRED_CAPABILITY:
        raise RuntimeError(
            f"device {name or ''} has compute capability {capability[0]}.{capability[1]}; "
            f"vllm_musa_b200 kernels are built for {', '.join(built_archs())} "
            f"(capability {REQUIRED_CAPABILITY[0]}.{REQUIRED_CAPABILITY[1]}, B200)")


def check_current_device() -> None:
    import torch
    if not torch.cuda.is_available():
        return
    d = torch.cuda.current_device()
    check_device_arch(torch.cuda.get_device_capability(d), torch.cuda.get_device_name(d))
