"""Speculative decoding on CPU: prompt-lookup (n-gram) drafts verified in one step per
request.  Every position's token is drawn with the same per-(seed, output index) noise as
without speculation and drafts are accepted only while they equal the drawn token, so the
outputs must be identical to plain decoding, greedy and sampled; repetitive prompts must
actually get drafts accepted."""
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama


def _prompts():
    g = torch.Generator().manual_seed(5)
    base = torch.randint(0, 1024, (12,), generator=g).tolist()
    rep = (base * 4)[:40]                       # repetitive: n-gram lookup hits
    rnd = torch.randint(0, 1024, (33,), generator=g).tolist()
    return [rep, rnd, rep[:25]]


def _run(spec, temperature, budget=256):
    llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
              max_model_len=128, max_num_seqs=4, max_num_batched_tokens=budget,
              speculative_config=spec)
    sp = SamplingParams(temperature=temperature, max_tokens=24, ignore_eos=True, seed=11)
    outs = [o.outputs[0].token_ids for o in llm.generate(_prompts(), sp)]
    return outs, llm.engine.scheduler


def test_ngram_spec_decode_greedy_matches_plain():
    plain, _ = _run(None, 0.0)
    spec, sch = _run({"method": "ngram", "num_speculative_tokens": 3}, 0.0)
    assert spec == plain
    assert sch.spec_proposed() > 0


def test_spec_decode_sampled_matches_plain():
    """Temperature sampling with drafts that are partly right (the plain run's own tokens
    with every third one corrupted): accepted and rejected drafts must both leave the sampled
    sequence unchanged."""
    plain, _ = _run(None, 0.8)
    llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
              max_model_len=128, max_num_seqs=4, max_num_batched_tokens=48)
    eng = llm.engine
    sp = SamplingParams(temperature=0.8, max_tokens=24, ignore_eos=True, seed=11)
    names = []
    for i, p in enumerate(_prompts()):
        eng.add_request(f"r{i}", p, sp)
        names.append(f"r{i}")
    iids = {eng._by_name[n]: k for k, n in enumerate(names)}
    outs = {}
    step = 0
    while eng.has_unfinished_requests():
        for iid in eng.scheduler.decode_request_ids():
            k = iids[iid]
            done = len(eng.scheduler.output_tokens(iid))
            d = list(plain[k][done:done + 3])
            if d and (done + step) % 3 == 0:
                d[-1] = (d[-1] + 1) % 1024
            eng.scheduler.set_draft(iid, d)
        for o in eng.step():
            outs[o.request_id] = o.outputs[0].token_ids
        step += 1
    assert [outs[n] for n in names] == plain
    sch = eng.scheduler
    assert 0 < sch.spec_accepted() < sch.spec_proposed()


def test_ngram_accepts_drafts_on_repetition():
    # a model that copies: greedy on a strongly repetitive prompt with random weights does
    # not copy, so check acceptance directly with drafts equal to the model's own outputs
    plain, _ = _run(None, 0.0)
    llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
              max_model_len=128, max_num_seqs=4, max_num_batched_tokens=256)
    eng = llm.engine
    sp = SamplingParams(temperature=0.0, max_tokens=24, ignore_eos=True)
    eng.add_request("a", _prompts()[0], sp)
    outs = []
    while eng.has_unfinished_requests():
        for iid in eng.scheduler.decode_request_ids():
            done = len(eng.scheduler.output_tokens(iid))
            eng.scheduler.set_draft(iid, plain[0][done:done + 3])   # oracle drafts
        outs += eng.step()
    assert outs[-1].outputs[0].token_ids == plain[0]
    assert eng.scheduler.spec_accepted() == eng.scheduler.spec_proposed() > 0
    assert eng.num_steps < 24 - 10  # several tokens per step


def test_mtp_spec_decode_matches_plain_deepseek():
    """DeepSeek multi-token prediction: the MTP layer (checkpoint layer num_layers) drafts one
    token per step from the main model's hidden states; verified outputs equal plain
    decoding."""
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_deepseek_cpu import tiny_ds
    cfg = tiny_ds(True, 128)
    cfg.num_nextn_predict_layers = 1
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (30, 70)]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    kw = dict(device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
              max_num_seqs=4, max_num_batched_tokens=64)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **kw).generate(prompts, sp)]
    for k in (1, 2):  # 2: the MTP layer chained on its own output
        llm = LLM(cfg, speculative_config={"method": "mtp", "num_speculative_tokens": k}, **kw)
        outs = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
        assert outs == plain
        assert llm.engine.drafter.proposed > 0
        assert llm.engine.scheduler.spec_proposed() > 0
