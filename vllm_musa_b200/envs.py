"""Environment flags (``B200_*``), read lazily with typed defaults.

Reference counterpart: vllm_musa/utils/environ.py:6-93 (EnvField / EnvBool / Envs).  Every
flag the framework reads is declared here with its type, default and meaning, so
``collect_env`` can report the effective configuration.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Any, Callable, Dict


@dataclass(frozen=True)
class EnvFlag:
    name: str
    default: Any
    parse: Callable[[str], Any]
    doc: str

    def get(self):
        raw = os.environ.get(self.name)
        if raw is None or raw == "":
            return self.default
        try:
            return self.parse(raw)
        except ValueError as e:
            raise ValueError(f"{self.name}={raw!r}: {e}") from None


def _bool(s: str) -> bool:
    v = s.strip().lower()
    if v in ("1", "true", "yes", "on"):
        return True
    if v in ("0", "false", "no", "off"):
        return False
    raise ValueError("expected a boolean")


FLAGS: Dict[str, EnvFlag] = {f.name: f for f in [
    EnvFlag("B200_DISABLE_CUSTOM_AR", False, _bool,
            "use NCCL instead of the NVSwitch peer-memory all-reduce kernels"),
    EnvFlag("B200_AR_ONE_SHOT_MAX_BYTES", 0, int,
            "largest message (bytes per rank) reduced one-shot; larger ones go two-shot "
            "(0: 2 MiB of peer reads, i.e. 2 MiB / (world - 1) per rank)"),
    EnvFlag("B200_DISABLE_TUNING", False, _bool, "ignore the measured tuning tables"),
    EnvFlag("B200_WORKER_TERMINATION_TIMEOUT_S", 10.0, float,
            "grace period before follower ranks are SIGTERM'd / SIGKILL'd at shutdown"),
    EnvFlag("B200_IDLE_SYNC_S", 1.0, float,
            "server: period of the idle step broadcast that keeps follower ranks alive"),
    EnvFlag("B200_SPMD_ROLE", "replicated", str,
            "multi-rank mode: replicated (torchrun, every rank adds requests), driver, follower"),
    EnvFlag("B200_FORCE_PLATFORM", False, _bool,
            "vLLM plugin: activate the B200 platform even if no sm_100 device is detected"),
    EnvFlag("B200_CUSTOM_OP_USE_NATIVE", False, _bool,
            "vLLM plugin: register the custom ops but route them to the PyTorch implementations"),
    EnvFlag("B200_LOG_LEVEL", "INFO", str, "logging level of the vllm_musa_b200 logger"),
    EnvFlag("B200_TORCH_PROFILER_DIR", "b200_traces", str,
            "directory of the Chrome traces written by LLM.stop_profile()"),
]}


def get(name: str):
    return FLAGS[name].get()


def snapshot() -> Dict[str, Any]:
    """Effective value of every flag (for collect_env / logs)."""
    return {n: f.get() for n, f in FLAGS.items()}
