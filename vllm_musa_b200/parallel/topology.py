"""NVLink topology check for the peer-memory communicator.

The custom all-reduce, NVLS and all-to-all kernels load and store peer memory directly, which is
only fast (and on B200 only what the kernels are tuned for) when every pair of the group's GPUs
talks over NVLink / NVSwitch.  Before the communicator is built, every rank reports its GPU's PCI
bus id, and each rank asks NVML whether it reaches every other rank's GPU over NVLink; the group
uses the custom kernels only if all of them do (the caller's MIN consensus makes that
all-or-none), otherwise it stays on NCCL.  An NVML that cannot answer leaves the kernels on.  Reference counterpart: the MtLink full-connectivity
probe at vllm_musa/platform.py:1139-1163.
"""
from __future__ import annotations

import logging
from typing import List, Optional

import torch

log = logging.getLogger("vllm_musa_b200")


def pci_bus_id(device: torch.device) -> str:
    """NVML-style PCI bus id ("00000000:1B:00.0") of a CUDA device."""
    p = torch.cuda.get_device_properties(device)
    return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"


def nvlink_to_all(mine: str, peers: List[str], nvml=None) -> bool:
    """True when NVML reports NVLink peer-to-peer status OK from GPU ``mine`` to every GPU in
    ``peers`` (bus ids; ``mine`` itself is skipped).  ``nvml``: the pynvml module or a stand-in
    with the same calls (tests)."""
    if nvml is None:
        import pynvml as nvml
    nvml.nvmlInit()
    try:
        h = nvml.nvmlDeviceGetHandleByPciBusId(mine)
        for b in peers:
            if b == mine:
                continue
            hp = nvml.nvmlDeviceGetHandleByPciBusId(b)
            st = nvml.nvmlDeviceGetP2PStatus(h, hp, nvml.NVML_P2P_CAPS_INDEX_NVLINK)
            if st != nvml.NVML_P2P_STATUS_OK:
                log.warning("GPU %s reaches %s without NVLink (status %s)", mine, b, st)
                return False
        return True
    finally:
        nvml.nvmlShutdown()


def group_nvlink_ok(device: torch.device, group, nvml=None) -> bool:
    """This rank's verdict for its group (collective over the Gloo ``group``): False when NVML
    reports a peer GPU reached without NVLink.  When NVML cannot answer (no library, unknown
    bus id) the topology is unknown and the verdict is True: the peer-memory kernels are
    correct over any CUDA peer path, the check only keeps them off slow ones."""
    import torch.distributed as dist
    try:
        mine = pci_bus_id(device)
    except Exception as e:  # pragma: no cover - no CUDA properties
        log.warning("PCI bus id unavailable: %s", e)
        mine = ""
    ids: List[Optional[str]] = [None] * dist.get_world_size(group)
    dist.all_gather_object(ids, mine, group=group)
    if not mine or any(not b for b in ids):
        return True
    try:
        return nvlink_to_all(mine, [str(b) for b in ids], nvml)
    except Exception as e:
        log.warning("NVLink topology unknown (NVML: %s); keeping the peer-memory kernels", e)
        return True
