"""Token sampling: greedy / temperature (Gumbel-max) with top-k, top-p and min-p filters.

CUDA: csrc/sampling/sampling.cu (radix-select thresholds, Philox Gumbel noise keyed by
(seed, step, vocab index) so vocab-parallel shards agree).  CPU: a PyTorch restatement with
the same filtering semantics (random draws come from torch's generator, so only greedy
results are bit-comparable across devices).  Reference: vllm_musa/v1/sample/
topk_topp_sampler.py:351, csrc/musa/sampler.mu:124, top_p_mask_logits.mu:149.
"""
from __future__ import annotations

import torch

from . import _ext


def _filter_ref(l: torch.Tensor, k: int, p: float, mp: float) -> torch.Tensor:
    keep = torch.ones_like(l, dtype=torch.bool)
    if 0 < k < l.numel():
        kth = torch.topk(l, k).values[-1]
        keep &= l >= kth
    m = l.max()
    if mp > 0:
        keep &= l >= m + torch.log(torch.tensor(mp))
    if p < 1.0:
        e = torch.where(keep, torch.exp(l - m), torch.zeros_like(l))
        vals, order = torch.sort(e, descending=True)
        cum = torch.cumsum(vals, 0)
        target = p * cum[-1]
        # smallest prefix whose mass reaches the target; keep ties of the threshold value
        cut = int(torch.searchsorted(cum, target).clamp(max=l.numel() - 1))
        thr = vals[cut]
        keep &= e >= thr
    return keep


_M64 = (1 << 64) - 1


def _mix64(z: torch.Tensor) -> torch.Tensor:
    """SplitMix64 finaliser on int64 lanes (wrapping arithmetic; logical shifts emulated)."""
    def srl(x, n):
        return (x >> n) & ((1 << (64 - n)) - 1)

    def wrap(v):
        v &= _M64
        return v - (1 << 64) if v >= (1 << 63) else v

    z = (z ^ srl(z, 30)) * wrap(0xBF58476D1CE4E5B9)
    z = (z ^ srl(z, 27)) * wrap(0x94D049BB133111EB)
    return z ^ srl(z, 31)


def _keyed_uniform(seed: int, step: int, idx: torch.Tensor) -> torch.Tensor:
    """U(0,1) noise that is a pure function of (seed, step, global token id): the CPU
    counterpart of the kernel's counter-based generator, so a token drawn at output index
    `step` does not depend on batching, chunking, speculation or the vocab split."""
    key = (seed * 0x9E3779B97F4A7C15 + step * 0xD1B54A32D192ED03) & _M64
    key = key - (1 << 64) if key >= (1 << 63) else key
    z = _mix64(idx * 0x2545F4914F6CDD1D + key)
    return (((z >> 11) & ((1 << 53) - 1)).double() / float(1 << 53)).float()


def sample_tokens(logits: torch.Tensor, temperature: torch.Tensor | None = None,
                  top_k: torch.Tensor | None = None, top_p: torch.Tensor | None = None,
                  min_p: torch.Tensor | None = None, seeds: torch.Tensor | None = None,
                  steps: torch.Tensor | None = None, vocab_offset: int = 0,
                  return_values: bool = False, generator: torch.Generator | None = None):
    """logits [R, V] fp32 -> token ids [R] int64 (global ids = vocab_offset + local index).

    temperature <= 0 means greedy.  With ``return_values`` also returns the winning score
    (logit for greedy, perturbed logit otherwise) for merging vocab shards.
    """
    R = logits.shape[0]
    if logits.is_cuda:
        out_idx = torch.empty(R, dtype=torch.int64, device=logits.device)
        out_val = torch.empty(R, dtype=torch.float32, device=logits.device) if return_values else None
        if R:
            _ext.ops().sample(logits, temperature, top_k, top_p, min_p, seeds, steps,
                              vocab_offset, out_idx, out_val)
        return (out_idx, out_val) if return_values else out_idx
    ids = torch.empty(R, dtype=torch.int64)
    vals = torch.empty(R, dtype=torch.float32)
    for r in range(R):
        l = logits[r].float()
        T = float(temperature[r]) if temperature is not None else 0.0
        if T <= 0:
            i = int(torch.argmax(l))
            ids[r], vals[r] = i + vocab_offset, l[i]
            continue
        l = l / T
        keep = _filter_ref(l, int(top_k[r]) if top_k is not None else 0,
                           float(top_p[r]) if top_p is not None else 1.0,
                           float(min_p[r]) if min_p is not None else 0.0)
        if seeds is not None and steps is not None:
            idx = torch.arange(l.shape[0], dtype=torch.int64) + vocab_offset
            u = _keyed_uniform(int(seeds[r]), int(steps[r]), idx)
        else:
            u = torch.rand(l.shape, generator=generator)
        u = u.clamp(1e-7, 1 - 1e-7)
        g = -torch.log(-torch.log(u))
        sc = torch.where(keep, l + g, torch.full_like(l, float("-inf")))
        i = int(torch.argmax(sc))
        ids[r], vals[r] = i + vocab_offset, sc[i]
    return (ids, vals) if return_values else ids


def apply_penalties(logits: torch.Tensor, entries: torch.Tensor, rep: torch.Tensor,
                    pres: torch.Tensor, freq: torch.Tensor, vocab_offset: int = 0) -> torch.Tensor:
    """Repetition / presence / frequency penalties, in place, on fp32 logits [R, V] of the vocab
    shard starting at ``vocab_offset``.  ``entries`` int32 [n, 3] = (row, global token id,
    occurrences in the row's output); each row lists every token of its prompt and output
    once.  vLLM semantics: a listed token's logit is divided by the repetition penalty when
    positive (multiplied when not), minus frequency x count, minus presence if count > 0."""
    if entries.numel() == 0:
        return logits
    if logits.is_cuda:
        _ext.ops().apply_penalties(logits, entries.contiguous(), rep.contiguous(),
                                   pres.contiguous(), freq.contiguous(), vocab_offset)
        return logits
    V = logits.shape[1]
    for row, tok, cnt in entries.tolist():
        t = tok - vocab_offset
        if not 0 <= t < V:
            continue
        v = float(logits[row, t])
        r = float(rep[row])
        if r != 1.0:
            v = v / r if v > 0 else v * r
        v -= float(freq[row]) * cnt
        if cnt > 0:
            v -= float(pres[row])
        logits[row, t] = v
    return logits


def apply_token_bitmask(logits: torch.Tensor, bitmask: torch.Tensor, rows: torch.Tensor,
                        vocab_offset: int = 0) -> torch.Tensor:
    """Constrained decoding, in place: logits row ``rows[r]`` (fp32 [S, V] of the vocab shard at
    ``vocab_offset``) keeps token t only where bit t % 32 of ``bitmask[r, t // 32]`` (int32) is
    set; the rest become -inf."""
    if rows.numel() == 0:
        return logits
    if logits.is_cuda:
        _ext.ops().apply_token_bitmask(logits, bitmask.contiguous(), rows.contiguous(),
                                       vocab_offset)
        return logits
    V = logits.shape[1]
    t = torch.arange(vocab_offset, vocab_offset + V)
    words = bitmask.shape[1]
    w = (t >> 5).clamp(max=words - 1)
    bits = (bitmask[:, w] >> (t & 31)) & 1
    allowed = (bits == 1) & (t < words * 32)
    for r, row in enumerate(rows.tolist()):
        logits[row].masked_fill_(~allowed[r], float("-inf"))
    return logits


def penalty_entries(rows_tokens) -> torch.Tensor:
    """[(row, prompt token ids, output token ids)] -> int32 [n, 3] (row, token, output count)
    with every token of the prompt and output listed once per row."""
    import numpy as np
    parts = []
    for row, prompt, output in rows_tokens:
        out = np.asarray(output, dtype=np.int64)
        toks = np.unique(np.concatenate([np.asarray(prompt, dtype=np.int64), out]))
        cnt = np.zeros(toks.shape[0], dtype=np.int64)
        if out.size:
            u, c = np.unique(out, return_counts=True)
            cnt[np.searchsorted(toks, u)] = c
        parts.append(np.stack([np.full_like(toks, row), toks, cnt], 1))
    if not parts:
        return torch.zeros(0, 3, dtype=torch.int32)
    return torch.from_numpy(np.concatenate(parts).astype(np.int32))


def token_logprobs(raw: torch.Tensor, tokens: torch.Tensor, k: int, as_logits: bool = False):
    """Log-probabilities from logits rows [n, V]: (top-k ids [n, k], top-k logprobs [n, k],
    the given tokens' logprobs [n], their ranks [n] (1 = most likely)); ``as_logits`` reports
    the logits themselves instead of their log_softmax (same ids and ranks)."""
    lp = raw.float() if as_logits else torch.log_softmax(raw.float(), dim=-1)
    tok_lp = lp.gather(1, tokens.view(-1, 1).long()).squeeze(1)
    rank = (lp > tok_lp.unsqueeze(1)).sum(1) + 1
    if k > 0:
        vals, ids = lp.topk(k, dim=-1)
    else:
        vals = torch.zeros(lp.shape[0], 0, device=lp.device)
        ids = torch.zeros(lp.shape[0], 0, dtype=torch.int64, device=lp.device)
    return ids, vals, tok_lp, rank


def shard_candidates(logits: torch.Tensor, temperature, seeds, steps,
                     vocab_offset: int = 0) -> torch.Tensor:
    """Per-row candidate rows of this vocab shard (CUDA): the <= 128 largest scaled logits with
    their global ids, the shard's max / exp-mass / completeness key and its Gumbel-max winner.
    Returns uint8 [R, cand_row_bytes] (the layout of the CUDA CandRow)."""
    mod = _ext.require()
    R = logits.shape[0]
    out = torch.empty(R, int(mod.cand_row_bytes()), dtype=torch.uint8, device=logits.device)
    if R:
        mod.shard_candidates(logits.contiguous(), temperature, seeds, steps, vocab_offset, out)
    return out


def merge_candidates_local(cands: torch.Tensor, world: int, R: int, temperature, top_k, top_p,
                           min_p, seeds, steps, V_total: int) -> torch.Tensor:
    """Merge candidate rows [world][R] held on this GPU and sample each row; -1 marks a row the
    candidates cannot decide exactly (the caller samples the gathered logits instead)."""
    mod = _ext.require()
    out = torch.empty(R, dtype=torch.int64, device=cands.device)
    if R:
        mod.merge_candidates_local(cands, world, R, temperature, top_k, top_p, min_p, seeds,
                                   steps, V_total, out)
    return out
