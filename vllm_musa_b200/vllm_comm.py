"""vLLM device communicator whose tensor-parallel all-reduce runs this package's NVSwitch
kernels (``B200Platform.get_device_communicator_cls``).

It is vLLM's CUDA communicator plus one ``CustomAllReduce`` (parallel/custom_ar.py) per
tensor-parallel group: CUDA-IPC peer buffers for the one-shot / two-shot kernels and, where
the GPUs support NVLink multicast, the NVLS buffer for the multimem kernel.  ``all_reduce`` of
a bf16 ``[tokens, hidden]`` activation (the row-parallel projections' outputs) goes through
it; everything else (other shapes, other groups) keeps vLLM's path.  vLLM mixes eager calls and
CUDA-graph replays whose buffer choice was fixed at capture, so this communicator has every
kernel end with a barrier (``end_barrier``): a rank reuses a buffer only after every peer has
left the previous call that read it, whatever the call sequence.

Reference counterpart: the reference routes vLLM's CudaCommunicator to its own
MusaJitCustomAllreduce (vllm_musa/platform.py:890-902, patch 0005,
vllm_musa/distributed/device_communicators/musa_jit_custom_all_reduce.py:1762-1938).
"""
from __future__ import annotations

import logging
from types import SimpleNamespace

import torch

from vllm.distributed.device_communicators.cuda_communicator import CudaCommunicator

log = logging.getLogger("vllm_musa_b200")


class B200Communicator(CudaCommunicator):
    def __init__(self, cpu_group, device=None, device_group=None, unique_name: str = "", *args,
                 **kwargs):
        super().__init__(cpu_group, device, device_group, unique_name, *args, **kwargs)
        self.b200_ar = None
        if "tp" not in unique_name or self.world_size < 2 or device is None or \
                device.type != "cuda":
            return
        try:
            from vllm.config import get_current_vllm_config
            cfg = get_current_vllm_config()
            hidden = cfg.model_config.get_hidden_size()
            max_tokens = cfg.scheduler_config.max_num_batched_tokens
        except Exception as e:  # no model config (unit use of the communicator)
            log.info("b200 all-reduce not configured: %s", e)
            return
        from .parallel.custom_ar import maybe_create_custom_allreduce
        st = SimpleNamespace(tp_size=self.world_size, tp_rank=self.rank_in_group,
                             rank=self.rank, tp_group=device_group, tp_cpu_group=cpu_group,
                             local_rank=device.index)
        self.b200_ar = maybe_create_custom_allreduce(st, device, max_tokens=max_tokens,
                                                     hidden=hidden)
        if self.b200_ar is not None:
            self.b200_ar.end_barrier = True
            log.info("b200 NVSwitch all-reduce on %s (%d ranks, NVLS %s)", unique_name,
                     self.world_size, self.b200_ar.nvls is not None)

    def all_reduce(self, input_: torch.Tensor) -> torch.Tensor:
        ar = self.b200_ar
        if ar is not None and input_.is_cuda and input_.dim() == 2 and ar.can_run(input_) and \
                input_.shape[0] > 0:
            return ar.all_reduce_out_of_place(input_)
        return super().all_reduce(input_)

    def destroy(self):
        if self.b200_ar is not None:
            self.b200_ar.close()
            self.b200_ar = None
        super().destroy()
