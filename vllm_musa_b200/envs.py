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
    EnvFlag("B200_DEBUG_BOUNDS", False, _bool,
            "check index tensors (KV slots, block tables, row indices) against the kernels' "
            "bounds at every op call and raise IndexError (synchronises: debugging only)"),
    EnvFlag("B200_MOE_GEMV_MAX_PAIRS", 256, int,
            "bf16 MoE layers with at most this many routed (token, slot) pairs run per-pair "
            "GEMVs instead of align + gather + grouped GEMMs (0: always grouped)"),
    EnvFlag("B200_MOE_SHAPE_INVENTORY", "", str,
            "append one JSON line per eager MoE layer call (shape, dispatch path, routed-token "
            "histogram) to this file; empty: off (synchronises: shape collection only)"),
    EnvFlag("B200_MOE_SHAPE_INVENTORY_MIN_TOKENS", 0, int,
            "smallest token count an MoE call needs to be recorded in the shape inventory"),
    EnvFlag("B200_MOE_SHAPE_INVENTORY_MAX_RECORDS", 64, int,
            "shape inventory records per process (< 0: unlimited)"),
    EnvFlag("B200_MAMBA_CHUNKED", True, _bool,
            "Mamba2 prefill parts of >= 64 tokens through the chunked SSD kernels (off: the "
            "token recurrence for every request)"),
    EnvFlag("B200_SKIP_NVLINK_CHECK", False, _bool,
            "build the peer-memory communicator without the NVML NVLink full-mesh check"),
    EnvFlag("B200_AR_NVLS", True, _bool,
            "allow the NVLS (multimem) all-reduce where every rank got a multicast mapping"),
    EnvFlag("B200_AR_NVLS_MIN_BYTES", None, int,
            "NVLS for messages above this many bytes at every world size (default: the "
            "measured per-world table in parallel/custom_ar.py)"),
    EnvFlag("B200_AR_NVLS_QUANT_MIN_ROWS", None, int,
            "rows from which the NVLS kernel emits the 1x128 e4m3 output itself (default: "
            "per-world table)"),
    EnvFlag("B200_AR_NVLS_ROWS_PER_WARP", 0, int,
            "rows each warp of the NVLS kernel walks (0: one row per warp up to the block cap)"),
    EnvFlag("B200_FUSE_GEMM_RS", False, _bool,
            "row-parallel GEMM with the reduce-scatter in its epilogue (peer stores) + local "
            "reduce / norm / all-gather, instead of GEMM + fused all-reduce"),
    EnvFlag("B200_EP_A2A", True, _bool,
            "MoE expert parallelism over the NVLink dispatch / return all-to-all kernels"),
    EnvFlag("B200_PP_MICRO_BATCHES", 0, int,
            "micro-batches per pipeline-parallel step (0: pipeline_parallel_size)"),
    EnvFlag("B200_ATTN_TC", True, _bool, "tcgen05 prefill attention (head_dim 128)"),
    EnvFlag("B200_ATTN_TC2", True, _bool,
            "two-heads-per-CTA tcgen05 prefill attention where the GQA group allows"),
    EnvFlag("B200_GEMM_PAIR_MIN_ROWS", 2048, int,
            "rows from which untuned GEMM shapes use CTA-pair (cta_group::2) tiles (<= 0: never)"),
    EnvFlag("B200_GEMM_SPLITK_REDUCE", True, _bool,
            "split-K partial sums reduced by a separate grid (PDL) instead of the last CTA"),
    EnvFlag("B200_LOG_LEVEL", "INFO", str, "logging level of the vllm_musa_b200 logger"),
    EnvFlag("B200_TORCH_PROFILER_DIR", "b200_traces", str,
            "directory of the Chrome traces written by LLM.stop_profile()"),
]}


def get(name: str):
    return FLAGS[name].get()


def snapshot() -> Dict[str, Any]:
    """Effective value of every flag (for collect_env / logs)."""
    return {n: f.get() for n, f in FLAGS.items()}
