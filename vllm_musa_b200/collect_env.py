"""Environment report (``b200-vllm collect-env`` / ``b200_collect_env``).

Reference counterpart: vllm_musa/collect_env.py:450-687.  Reports the Python / torch / CUDA /
NCCL / vLLM versions, the GPUs NVML sees (name, capability, clocks, NVLink peer status), the
extension build, and every ``B200_*`` flag.
"""
from __future__ import annotations

import json
import platform
import sys


def get_env_info() -> dict:
    info = {"python": sys.version.split()[0], "platform": platform.platform()}
    try:
        import torch
        info.update(torch=torch.__version__, cuda_runtime=torch.version.cuda,
                    cuda_available=torch.cuda.is_available())
        try:
            info["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
        except Exception:
            pass
    except Exception as e:  # pragma: no cover
        info["torch"] = f"unavailable: {e}"
    try:
        import vllm
        info["vllm"] = vllm.__version__
    except Exception:
        info["vllm"] = None
    from . import __version__, envs
    from .native_arch import built_archs
    info["vllm_musa_b200"] = __version__
    info["built_archs"] = list(built_archs())
    try:
        from .ops import _ext
        info["extension_loaded"] = _ext.available()
    except Exception:
        info["extension_loaded"] = False
    info["flags"] = envs.snapshot()
    gpus = []
    try:
        import pynvml
        pynvml.nvmlInit()
        n = pynvml.nvmlDeviceGetCount()
        for i in range(n):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            g = {"index": i, "name": pynvml.nvmlDeviceGetName(h),
                 "capability": list(pynvml.nvmlDeviceGetCudaComputeCapability(h)),
                 "memory_gib": round(pynvml.nvmlDeviceGetMemoryInfo(h).total / 2**30, 1),
                 "sm_clock_max_mhz": pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)}
            peers = []
            for j in range(n):
                if j == i:
                    continue
                try:
                    hj = pynvml.nvmlDeviceGetHandleByIndex(j)
                    st = pynvml.nvmlDeviceGetP2PStatus(h, hj, pynvml.NVML_P2P_CAPS_INDEX_NVLINK)
                    peers.append({"peer": j, "nvlink_p2p": st == pynvml.NVML_P2P_STATUS_OK})
                except Exception:
                    pass
            g["peers"] = peers
            gpus.append(g)
        pynvml.nvmlShutdown()
    except Exception as e:
        info["nvml"] = f"unavailable: {type(e).__name__}"
    info["gpus"] = gpus
    return info


def main() -> None:
    print(json.dumps(get_env_info(), indent=1, default=str))


if __name__ == "__main__":
    main()
