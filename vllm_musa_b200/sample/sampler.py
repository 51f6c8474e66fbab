"""Sampler over (possibly vocab-sharded) logits.

Each tensor-parallel rank holds the logits of its vocab shard.  Instead of all-gathering the
full [S, V] logits (the reference's path: patch 0069 IPC all-gather, then top-k/top-p,
vllm_musa/distributed/device_communicators/musa_jit_custom_all_reduce.py:1941-1956), every
rank reduces its shard to one (score, token) candidate per row with the Gumbel-max sampler,
ranks exchange the [S] candidates (one kernel storing them into every peer's candidate region
over NVLink, then an epoch barrier and the merge, when the P2P communicator is up; NCCL
all-gather otherwise), and the max wins: identical on every rank because the
Gumbel noise is a function of (seed, step, global token id).  Rows that use top-k / top-p /
min-p need global order statistics: each rank reduces its shard to at most 128 candidates per
row and the candidate rows (not the logits) cross NVLink, merged into the exact global
filtered draw; only a batch the candidates cannot decide exactly gathers the full logits.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import ops


class Sampler:
    def __init__(self, comm=None, vocab_start: int = 0, tp_size: int = 1):
        self.comm = comm
        self.vocab_start = vocab_start
        self.tp = tp_size

    def __call__(self, logits: torch.Tensor, temperature: Optional[torch.Tensor],
                 top_k: Optional[torch.Tensor], top_p: Optional[torch.Tensor],
                 min_p: Optional[torch.Tensor], seeds: Optional[torch.Tensor],
                 steps: Optional[torch.Tensor], any_filter: bool = False,
                 generator: Optional[torch.Generator] = None) -> torch.Tensor:
        if self.tp == 1:
            return ops.sample_tokens(logits, temperature, top_k, top_p, min_p, seeds, steps,
                                     generator=generator)
        if any_filter:
            custom = getattr(self.comm, "custom", None)
            if logits.is_cuda and custom is not None and temperature is not None:
                # candidate rows exchanged over NVLink instead of the logits; a row the
                # candidates cannot decide exactly (-1, the same on every rank) sends the
                # batch through the gathered path below
                out = custom.sample_topk(logits, temperature, top_k, top_p, min_p, seeds, steps,
                                         self.vocab_start, logits.shape[1] * self.tp)
                if out is not None and int(out.min()) >= 0:
                    return out
            full = self.comm.all_gather(logits, dim=1)
            return ops.sample_tokens(full, temperature, top_k, top_p, min_p, seeds, steps,
                                     generator=generator)
        ids, vals = ops.sample_tokens(logits, temperature, None, None, None, seeds, steps,
                                      vocab_offset=self.vocab_start, return_values=True)
        custom = getattr(self.comm, "custom", None)
        if logits.is_cuda and custom is not None:
            merged = custom.merge_candidates(vals, ids)  # NVLink exchange + merge, one kernel
            if merged is not None:
                return merged
        all_vals = self.comm.all_gather(vals.unsqueeze(0), dim=0)   # [tp, S]
        all_ids = self.comm.all_gather(ids.unsqueeze(0), dim=0)
        if logits.is_cuda:
            out = torch.empty_like(ids)
            torch.ops.b200.merge_candidates(all_vals.contiguous(), all_ids.contiguous(), out)
            return out
        best = torch.argmax(all_vals, dim=0)
        return all_ids.gather(0, best.unsqueeze(0)).squeeze(0)
