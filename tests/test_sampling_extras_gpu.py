"""Penalties kernel on a B200 against the PyTorch oracle (full vocab and a vocab shard), and
log-probabilities through the engine on the GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_apply_penalties_kernel_matches_oracle():
    from vllm_musa_b200.ops.sampling import apply_penalties, penalty_entries
    g = torch.Generator().manual_seed(1)
    R, V = 6, 5000
    rows = []
    for r in range(R):
        prompt = torch.randint(0, V, (int(torch.randint(0, 300, (1,), generator=g)),),
                               generator=g).tolist()
        out = torch.randint(0, V, (int(torch.randint(0, 60, (1,), generator=g)),),
                            generator=g).tolist()
        rows.append((r, prompt, out))
    e = penalty_entries(rows)
    logits = torch.randn(R, V, generator=g) * 3
    rep = torch.rand(R, generator=g) + 0.7
    pres = torch.rand(R, generator=g) - 0.5
    freq = torch.rand(R, generator=g)
    want = apply_penalties(logits.clone(), e, rep, pres, freq)
    got = apply_penalties(logits.cuda(), e.cuda(), rep.cuda(), pres.cuda(), freq.cuda())
    torch.testing.assert_close(got.cpu(), want)
    off = 2000
    shard = apply_penalties(logits[:, off:3000].contiguous().cuda(), e.cuda(), rep.cuda(),
                            pres.cuda(), freq.cuda(), vocab_offset=off)
    torch.testing.assert_close(shard.cpu(), want[:, off:3000])


def test_engine_logprobs_on_gpu():
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.presets import tiny_llama
    cfg = tiny_llama()
    cfg.dtype = torch.bfloat16
    llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=32, max_model_len=256, max_num_seqs=4,
              max_num_batched_tokens=256, cuda_graph_sizes=[1, 2, 4])
    g = torch.Generator().manual_seed(2)
    prompts = torch.randint(0, 1024, (3, 30), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True, logprobs=4,
                        repetition_penalty=1.2)
    outs = llm.generate(prompts, sp)
    for o in outs:
        c = o.outputs[0]
        assert len(c.logprobs) == 6
        for t, d in zip(c.token_ids, c.logprobs):
            assert t in d and len(d) >= 4 and all(v.logprob <= 0 for v in d.values())
    llm.shutdown()


def _sampling_batch(R, V, seed):
    g = torch.Generator().manual_seed(seed)
    scale = torch.where(torch.arange(R) % 3 == 0, 12.0, 2.0)  # some rows peaked
    logits = (torch.randn(R, V, generator=g) * scale[:, None]).cuda()
    temp = torch.tensor([0.0 if r % 7 == 0 else (0.7 if r % 2 else 1.0) for r in range(R)]).cuda()
    top_k = torch.tensor([[0, 5, 50, 128, 300][r % 5] for r in range(R)], dtype=torch.int32).cuda()
    top_p = torch.tensor([[1.0, 0.9, 0.5, 1.0][r % 4] for r in range(R)]).cuda()
    min_p = torch.tensor([[0.0, 0.0, 0.05][r % 3] for r in range(R)]).cuda()
    seeds = torch.arange(R, dtype=torch.int64).cuda() * 7919 + 3
    steps = (torch.arange(R, dtype=torch.int32) % 11).cuda()
    return logits, temp, top_k, top_p, min_p, seeds, steps


def test_topk_candidates_merge_matches_full_vocab_sampler():
    """Vocab shards reduced to candidate rows and merged (the single-GPU form of the NVLink
    exchange) draw exactly the token the full-vocab sampler draws, on every row they decide;
    rows with top-k <= 128, greedy rows and unfiltered rows are always decided."""
    from vllm_musa_b200 import ops
    from vllm_musa_b200.ops.sampling import merge_candidates_local, shard_candidates
    R, V, world = 96, 32000, 4
    Vs = V // world
    logits, temp, top_k, top_p, min_p, seeds, steps = _sampling_batch(R, V, 5)
    ref = ops.sample_tokens(logits, temp, top_k, top_p, min_p, seeds, steps)
    cands = torch.cat([shard_candidates(logits[:, s * Vs:(s + 1) * Vs].contiguous(), temp,
                                        seeds, steps, s * Vs) for s in range(world)])
    out = merge_candidates_local(cands, world, R, temp, top_k, top_p, min_p, seeds, steps, V)
    torch.cuda.synchronize()
    decided = out >= 0
    assert torch.equal(out[decided], ref[decided])
    k, t = top_k.cpu(), temp.cpu()
    must = (t == 0) | ((k > 0) & (k <= 128)) | \
        ((k == 0) & (top_p.cpu() == 1.0) & (min_p.cpu() == 0.0))
    assert bool(decided.cpu()[must].all()), (out.cpu()[must], must.nonzero())
    assert decided.float().mean() > 0.6


def test_token_bitmask_kernel_matches_reference():
    """The constrained-decoding mask kernel against the PyTorch bit test, including a vocab
    shard at an offset and tokens past the bitmask."""
    import torch
    from vllm_musa_b200.ops.sampling import apply_token_bitmask
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(6, 5000, generator=g)
    bm = torch.randint(-2**31, 2**31 - 1, (3, 150), generator=g, dtype=torch.int64).to(torch.int32)
    rows = torch.tensor([5, 0, 2], dtype=torch.int32)
    for off in (0, 96):
        want = apply_token_bitmask(logits[:, off:].clone(), bm, rows, vocab_offset=off)
        got = apply_token_bitmask(logits[:, off:].clone().cuda(), bm.cuda(), rows.cuda(),
                                  vocab_offset=off)
        assert torch.equal(got.cpu(), want)


def test_structured_outputs_on_gpu():
    import json
    import os
    import sys
    import torch
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_structured_outputs_cpu import SCHEMA, CharTokenizer, _cfg
    from vllm_musa_b200 import LLM, SamplingParams
    cfg = _cfg()
    cfg.dtype = torch.bfloat16
    llm = LLM(cfg, tokenizer=CharTokenizer(), block_size=64, seed=0, num_gpu_blocks=64,
              max_model_len=512, max_num_seqs=8, max_num_batched_tokens=256)
    sps = [SamplingParams(temperature=0.9, seed=3 + i, max_tokens=120, structured_outputs=so)
           for i, so in enumerate([{"json": SCHEMA, "disable_any_whitespace": True},
                                   {"choice": ["yes", "no"]}])]
    outs = llm.generate([[5, 6, 7], [8, 9, 10]], sps)
    obj = json.loads(outs[0].outputs[0].text)
    assert obj["color"] in ("red", "green") and isinstance(obj["ok"], bool)
    assert outs[1].outputs[0].text in ("yes", "no")
