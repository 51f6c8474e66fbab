"""Failure detection without GPU faults.

CPU (Gloo ranks): the NVSwitch communicator is fail-closed -- if any rank cannot build it, the
MIN consensus makes every rank fall back to NCCL, and the ranks that did build it release it.
GPU (one device): the all-reduce kernel's peer barrier waits on a flag that no rank will ever
set; the bounded wait gives up after its clock budget, records "peer flag wait timed out" in
the device error word, and the context stays usable.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _consensus_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from types import SimpleNamespace
    from vllm_musa_b200.parallel import custom_ar
    dist.init_process_group("gloo", rank=rank, world_size=world)
    closed = []

    class Fake:
        def __init__(self, st, device, max_tokens, hidden):
            if st.rank == 1:
                raise RuntimeError("injected: cudaIpcOpenMemHandle failed")

        def close(self):
            closed.append(True)

    custom_ar.CustomAllReduce = Fake
    st = SimpleNamespace(tp_size=world, rank=rank, tp_rank=rank, tp_cpu_group=None)
    got = custom_ar.maybe_create_custom_allreduce(st, torch.device("cpu"), 16, 64)
    q.put((rank, got is None, bool(closed)))
    dist.destroy_process_group()


def test_custom_allreduce_setup_is_fail_closed():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_consensus_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (none, closed)) for r, none, closed in (q.get(timeout=120) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == (True, True)   # built, then released after the consensus said no
    assert res[1] == (True, False)  # failed to build


@pytest.mark.gpu
def test_peer_barrier_timeout_returns_error_status():
    from vllm_musa_b200.ops import _ext
    mod = _ext.require()
    dev = torch.device("cuda", 0)
    H, T = 1024, 4
    flag_bytes = int(mod.comm_flag_bytes())
    # "rank 0" and a "rank 1" whose process never runs: both buffers live on this GPU and
    # nothing ever writes rank 1's arrival flag into rank 0's flag region
    mine = torch.zeros(4 * T * H * 2 + flag_bytes, dtype=torch.uint8, device=dev)
    ghost = torch.zeros_like(mine)
    slot = T * H * 2

    def bufs(b):
        base = b.data_ptr()
        return base, base + 2 * slot, base + 4 * slot
    s0, o0, f0 = bufs(mine)
    s1, o1, f1 = bufs(ghost)
    epochs = f0 + flag_bytes - 128 * 4
    x = torch.randn(T, H, device=dev).to(torch.bfloat16)
    _ext.check_device_errors()
    mod.fused_allreduce(x, [s0, s1, o0, o1, f0, f1], epochs, 0, 2, T, H, 1, 0, False, None,
                        None, 0.0)
    with pytest.raises(RuntimeError, match="peer flag wait timed out"):
        _ext.check_device_errors()
    # the context still works and the error word was cleared
    y = (x.float() * 2).sum()
    torch.cuda.synchronize()
    assert torch.isfinite(y)
    _ext.check_device_errors()


class _FakeNvml:
    """NVML stand-in: GPUs by bus id; `nvlink` lists the bus-id pairs joined by NVLink."""
    NVML_P2P_CAPS_INDEX_NVLINK = 5
    NVML_P2P_STATUS_OK = 0

    def __init__(self, nvlink):
        self.nvlink = {frozenset(p) for p in nvlink}
        self.inits = 0

    def nvmlInit(self):
        self.inits += 1

    def nvmlShutdown(self):
        self.inits -= 1

    def nvmlDeviceGetHandleByPciBusId(self, b):
        return b

    def nvmlDeviceGetP2PStatus(self, a, b, cap):
        assert cap == self.NVML_P2P_CAPS_INDEX_NVLINK
        return self.NVML_P2P_STATUS_OK if frozenset((a, b)) in self.nvlink else 4


def test_nvlink_topology_check_with_fake_nvml():
    """The communicator's NVLink full-mesh check: OK only if this GPU reaches every peer over
    NVLink (a PCIe-only pair, or an NVML error, keeps the group on NCCL)."""
    from vllm_musa_b200.parallel.topology import nvlink_to_all
    ids = ["0000:1b:00.0", "0000:43:00.0", "0000:52:00.0"]
    full = _FakeNvml([(ids[0], ids[1]), (ids[0], ids[2]), (ids[1], ids[2])])
    assert nvlink_to_all(ids[0], ids, full) and full.inits == 0
    partial = _FakeNvml([(ids[0], ids[1])])
    assert nvlink_to_all(ids[0], ids[:2], partial)
    assert not nvlink_to_all(ids[0], ids, partial)
    assert not nvlink_to_all(ids[2], ids, partial) and partial.inits == 0
