"""vLLM post-grad pass manager with this package's fusion passes appended (returned by
``B200Platform.get_pass_manager_cls``).  Reference counterpart:
vllm_musa/compilation/passes/pass_manager.py:59-83 (MusaPostGradPassManager.configure)."""
from __future__ import annotations

from vllm.compilation.passes.pass_manager import PostGradPassManager

from .passes import AllReduceRMSNormFusionPass, RMSNormQuantFusionPass, SiluMulQuantFusionPass


class _Wrapped:
    """Adapts a graph pass to the interface vLLM's manager iterates over."""

    def __init__(self, p):
        self.p = p

    def is_applicable_for_range(self, compile_range) -> bool:
        return True

    def __call__(self, graph):
        return self.p(graph)

    def uuid(self):
        return self.p.uuid()


def b200_passes() -> list:
    return [_Wrapped(AllReduceRMSNormFusionPass()), _Wrapped(SiluMulQuantFusionPass()),
            _Wrapped(RMSNormQuantFusionPass())]


class B200PostGradPassManager(PostGradPassManager):
    def configure(self, config) -> None:
        super().configure(config)
        self.passes += b200_passes()
