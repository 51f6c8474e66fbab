"""vLLM GPU worker for B200: vLLM's own worker plus this package's per-process setup.

``B200Platform`` selects it (``parallel_config.worker_cls``).  Every worker process (tensor-
parallel ranks included) checks at device initialisation that it drives an sm_100 device and
that this package's extension was built for it, and loads the custom ops before vLLM builds or
compiles the model.  Reference counterpart: vllm_musa/worker.py:10-35 (the MUSA worker's device
check and op preloading).
"""
from __future__ import annotations

from vllm.v1.worker.gpu_worker import Worker


class B200Worker(Worker):
    def init_device(self):
        super().init_device()
        from .native_arch import check_current_device
        from .plugin import preload_custom_op_modules
        check_current_device()
        preload_custom_op_modules()
