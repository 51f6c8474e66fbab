"""Speculative decoding on one GPU: output tokens/s of greedy generation without drafts, with
prompt-lookup chains, with prompt-lookup token tries, and with oracle drafts (the plain run's
own tokens) laid out as a chain and as a tree whose right path sits on non-first branches (so
an accepted step also copies KV rows into place).

On random-init weights the logits are flat: ``--check-logits`` shows verification rows within
bf16 noise of the plain decode rows (a few percent of the largest logit) while the plain
top-1 / top-2 gap is often smaller than that, so greedy continuations part at near-ties and
oracle drafts are rejected from the first parting on.  The oracle rows therefore measure what a
verification step costs next to a decode step (equal step counts: the time ratio is the step
cost ratio); real checkpoints decide the acceptance.

    python benchmarks/spec_decode_bench.py [--model llama3-8b] [--batch 1 16] [--check-logits]

Workload: random-init weights of the named architecture (bf16), prompts that repeat a
64-token random block (so suffix lookups find earlier occurrences), ``--output-len`` tokens
per request, temperature 0, ignore_eos.  Time: wall clock around each generate() with a
device synchronize on both sides (host scheduling and verification included), after one
warm-up pass.  Prints one JSON line per (batch, mode).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, nargs="+", default=[1, 16])
    ap.add_argument("--input-len", type=int, default=512)
    ap.add_argument("--output-len", type=int, default=128)
    ap.add_argument("--num-layers", type=int, default=None)
    ap.add_argument("--check-logits", action="store_true",
                    help="also compare verification-row logits with plain decode logits")
    return ap.parse_args()


def prompts(n, L, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        block = torch.randint(0, vocab, (64,), generator=g).tolist()
        out.append((block * (L // 64 + 1))[:L])
    return out


def oracle_drafts(eng, ref, names, tree):
    """Three right tokens per decode request: a chain, or a tree with wrong siblings whose
    right path is nodes 1 -> 3 -> 4."""
    iids = {eng._by_name[n]: i for i, n in enumerate(names) if n in eng._by_name}
    V = eng.config.model.vocab_size
    for iid in eng.scheduler.decode_request_ids():
        done = len(eng.scheduler.output_tokens(iid))
        right = ref[iids[iid]][done:done + 3]
        if len(right) < 3:
            continue
        if not tree:
            eng.scheduler.set_draft(iid, right)
            continue
        w = [(t + 1) % V for t in right]
        eng.scheduler.set_draft_tree(iid, [w[0], right[0], w[1], right[1], right[2], w[2]],
                                     [-1, -1, 1, 1, 3, 0])


def run(llm, ps, sp, spec, ref=None, tree=False):
    from vllm_musa_b200.config import SpeculativeConfig
    eng = llm.engine
    eng.config.speculative = SpeculativeConfig.from_dict(spec)
    names = [f"q{run.k}_{i}" for i in range(len(ps))]
    run.k += 1
    acc0, prop0, steps0 = eng.scheduler.spec_accepted(), eng.scheduler.spec_proposed(), \
        eng.num_steps
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for n, p in zip(names, ps):
        eng.add_request(n, p, sp)
    outs = {}
    while eng.has_unfinished_requests():
        if ref is not None:
            oracle_drafts(eng, ref, names, tree)
        for o in eng.step():
            if o.finished:
                outs[o.request_id] = o.outputs[0].token_ids
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    toks = [outs[n] for n in names]
    return toks, dt, eng.num_steps - steps0, eng.scheduler.spec_accepted() - acc0, \
        eng.scheduler.spec_proposed() - prop0


run.k = 0


def _step_all(eng, names):
    outs = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                outs[o.request_id] = o.outputs[0].token_ids
    return [outs[n] for n in names]


def check_logits(llm, ps, tree):
    """Teacher-forced comparison of the logits a verification step computes for its rows with
    the logits plain decoding computed for the same token histories: relative max error,
    argmax agreement, and the plain top-1 / top-2 gap (a flip needs error > gap)."""
    from vllm_musa_b200 import SamplingParams
    eng, rn = llm.engine, llm.engine.runner
    n = 4
    sp = SamplingParams(temperature=0.0, max_tokens=n + 1, ignore_eos=True)
    names = [f"lp{check_logits.k}_{i}" for i in range(len(ps))]
    check_logits.k += 1
    rn.record_logits, rn.logits_log = True, []
    for nm, p in zip(names, ps):
        eng.add_request(nm, p, sp)
    toks = _step_all(eng, names)
    plain = rn.logits_log  # step 0: prefill rows, step j: decode rows predicting token j
    rn.logits_log = []
    names2 = [f"lq{check_logits.k}_{i}" for i in range(len(ps))]
    check_logits.k += 1
    sp1 = SamplingParams(temperature=0.0, max_tokens=n + 2, ignore_eos=True)  # room for 3
    for nm, p in zip(names2, ps):
        eng.add_request(nm, p, sp1)
    eng.step()  # prefill: first token
    V = eng.config.model.vocab_size
    rows_of = []  # per request: verification rows predicting tokens 1..3 (None: skipped)
    for i, nm in enumerate(names2):
        iid = eng._by_name[nm]
        if list(eng.scheduler.output_tokens(iid))[:1] != toks[i][:1]:
            rows_of.append(None)
            continue
        t = toks[i]
        if tree:
            w = [(x + 1) % V for x in t[1:4]]
            eng.scheduler.set_draft_tree(iid, [w[0], t[1], w[1], t[2], t[3], w[2]],
                                         [-1, -1, 1, 1, 3, 0])
            rows_of.append([0, 2, 4])
        else:
            eng.scheduler.set_draft(iid, t[1:4])
            rows_of.append([0, 1, 2])
    rn.logits_log = []
    eng.step()
    ver = rn.logits_log[0]
    width = 7 if tree else 4
    errs, agree, gaps, nrow = [], 0, [], 0
    # step rows: one-token decodes first (requests left without drafts), then verifications
    base = sum(r is None for r in rows_of)
    for i, rows in enumerate(rows_of):
        if rows is None:
            continue
        for j, r in enumerate(rows):
            a, b = ver[base + r], plain[j + 1][i]
            errs.append(float((a - b).abs().max() / b.abs().max()))
            agree += int(a.argmax() == b.argmax())
            top = torch.topk(b, 2).values
            gaps.append(float((top[0] - top[1]) / b.abs().max()))
            nrow += 1
        base += width
    _step_all(eng, names2)
    rn.record_logits = False
    gaps.sort()
    errs.sort()
    return {"rows": nrow, "argmax_agree": agree, "rel_err_median": errs[len(errs) // 2],
            "rel_err_max": errs[-1], "rel_gap_median": gaps[len(gaps) // 2],
            "rel_gap_min": gaps[0]}


check_logits.k = 0


def main():
    a = parse()
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.presets import get_preset
    cfg = get_preset(a.model)
    if a.num_layers:
        cfg.num_layers = a.num_layers
    bmax = max(a.batch)
    llm = LLM(cfg, seed=0, max_model_len=a.input_len + a.output_len + 64, max_num_seqs=bmax,
              max_num_batched_tokens=max(2048, bmax * 8), enforce_eager=False)
    sp = SamplingParams(temperature=0.0, max_tokens=a.output_len, ignore_eos=True)
    modes = [("plain", None, False, False),
             ("ngram_chain_k4", {"method": "ngram", "num_speculative_tokens": 4}, False, False),
             ("ngram_tree_k8_w3", {"method": "ngram", "num_speculative_tokens": 8,
                                   "tree_width": 3}, False, False),
             ("oracle_chain_3", None, True, False),
             ("oracle_tree_6nodes_path3", None, True, True)]
    if a.check_logits:
        ps = prompts(4, a.input_len, cfg.vocab_size, seed=99)
        for tree in (False, True):
            print(json.dumps({"model": a.model, "check": "tree" if tree else "chain",
                              **check_logits(llm, ps, tree)}), flush=True)
    for B in a.batch:
        ps = prompts(B, a.input_len, cfg.vocab_size, seed=B)
        run(llm, ps, sp, None)  # warm-up (graphs, allocator)
        ref, base = None, None
        for name, spec, oracle, tree in modes:
            toks, dt, steps, acc, prop = run(llm, ps, sp, spec, ref if oracle else None, tree)
            if name == "plain":
                ref, base = toks, dt
            same = sum(x == y for t, r in zip(toks, ref) for x, y in zip(t, r)) / \
                sum(map(len, ref))
            print(json.dumps({"model": a.model, "batch": B, "mode": name,
                              "output_tok_s": round(B * a.output_len / dt, 1),
                              "speedup_vs_plain": round(base / dt, 3), "engine_steps": steps,
                              "drafts_proposed": prop, "drafts_accepted": acc,
                              "tokens_equal_plain": round(same, 4)}), flush=True)
    llm.shutdown()


if __name__ == "__main__":
    main()
