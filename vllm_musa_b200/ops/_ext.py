"""Loader for the native extension ``vllm_musa_b200._C``.

The extension carries every sm_100a kernel (registered as ``torch.ops.b200.*``) and the C++
host runtime (scheduler / KV block pool).  CPU tensors never reach the extension's kernels:
the op wrappers in this package route them to PyTorch reference implementations.  A CUDA
tensor with no extension loaded is an error, never a silent fallback.
"""
from __future__ import annotations

import importlib
from typing import Optional

_EXT = None
_ERR: Optional[BaseException] = None


def load():
    """Import ``vllm_musa_b200._C`` once; returns the module or None."""
    global _EXT, _ERR
    if _EXT is None and _ERR is None:
        try:
            _EXT = importlib.import_module("vllm_musa_b200._C")
        except Exception as e:  # pragma: no cover - depends on the build
            _ERR = e
    return _EXT


def available() -> bool:
    return load() is not None


def require():
    """Return the extension or raise with the import error (used by every CUDA path)."""
    mod = load()
    if mod is None:
        raise RuntimeError(
            "vllm_musa_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_ERR!r})")
    return mod


def ops():
    """``torch.ops.b200`` after making sure the extension registered it."""
    require()
    import torch
    return torch.ops.b200


def check_device_errors(device=None) -> None:
    """Raise if a bounded wait in a kernel on ``device`` recorded a timeout.

    Reads the per-device error word (synchronising the device) and clears it.
    """
    import torch
    mod = require()
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    word = mod.error_word(torch.empty(0, device=dev))
    vals = word.cpu()
    if int(vals[0]) != 0:
        code = int(vals[0])
        word.zero_()
        names = {1: "mbarrier wait timed out", 2: "peer flag wait timed out",
                 3: "bad index detected on device"}
        raise RuntimeError(f"b200 kernel error {code}: {names.get(code, 'unknown')}")
