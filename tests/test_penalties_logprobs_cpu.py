"""Repetition / presence / frequency penalties and per-token log-probabilities through the
engine on the tiny CPU Llama, against a greedy loop over the pure-PyTorch reference decoder
that applies vLLM's penalty rules to its logits and reports log_softmax of the raw logits."""
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights
from vllm_musa_b200.ops.sampling import apply_penalties, penalty_entries


def _prompts(n=3, length=20, seed=9):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 1024, (n, length), generator=g).tolist()


def _penalised(l, prompt, out, rep, pres, freq):
    l = l.clone()
    seen = set(prompt) | set(out)
    for t in seen:
        v = float(l[t])
        if rep != 1.0:
            v = v / rep if v > 0 else v * rep
        c = out.count(t)
        v -= freq * c
        if c:
            v -= pres
        l[t] = v
    return l


def test_penalty_entries_and_op():
    e = penalty_entries([(0, [5, 7, 5], [7, 9, 9]), (1, [], [3])])
    rows = {(r, t): c for r, t, c in e.tolist()}
    assert rows == {(0, 5): 0, (0, 7): 1, (0, 9): 2, (1, 3): 1}
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(2, 12, generator=g)
    ref = torch.stack([_penalised(logits[0], [5, 7, 5], [7, 9, 9], 1.3, 0.5, 0.25),
                       _penalised(logits[1], [], [3], 1.0, -0.5, 1.0)])
    got = apply_penalties(logits.clone(), e, torch.tensor([1.3, 1.0]),
                          torch.tensor([0.5, -0.5]), torch.tensor([0.25, 1.0]))
    torch.testing.assert_close(got, ref)
    # a vocab shard only touches its own columns
    shard = apply_penalties(logits[:, 6:].clone(), e, torch.tensor([1.3, 1.0]),
                            torch.tensor([0.5, -0.5]), torch.tensor([0.25, 1.0]), vocab_offset=6)
    torch.testing.assert_close(shard, ref[:, 6:])


def _llm():
    return LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
               max_model_len=128, max_num_seqs=4, max_num_batched_tokens=256)


def test_penalties_match_reference_greedy():
    cfg = tiny_llama()
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    prompts = _prompts()
    rep, pres, freq = 1.4, 0.3, 0.2
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True, repetition_penalty=rep,
                        presence_penalty=pres, frequency_penalty=freq)
    outs = _llm().generate(prompts, sp)
    plain = _llm().generate(prompts, SamplingParams(temperature=0.0, max_tokens=10,
                                                    ignore_eos=True))
    assert any(a.outputs[0].token_ids != b.outputs[0].token_ids for a, b in zip(outs, plain))
    for o, p in zip(outs, prompts):
        toks = []
        for _ in range(10):
            l = ref.logits(p + toks)[-1]
            toks.append(int(torch.argmax(_penalised(l, p, toks, rep, pres, freq))))
        assert o.outputs[0].token_ids == toks


def test_logprobs_of_raw_logits():
    cfg = tiny_llama()
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    prompts = _prompts(2, 16, seed=10)
    outs = _llm().generate(prompts, SamplingParams(temperature=0.0, max_tokens=5,
                                                   ignore_eos=True, logprobs=3))
    for o, p in zip(outs, prompts):
        c = o.outputs[0]
        assert len(c.logprobs) == len(c.token_ids) == 5
        cum = 0.0
        for k, (t, d) in enumerate(zip(c.token_ids, c.logprobs)):
            lp = torch.log_softmax(ref.logits(p + c.token_ids[:k])[-1], -1)
            top = torch.topk(lp, 3)
            assert d[t].rank == 1  # greedy picks the most likely token
            assert abs(d[t].logprob - float(lp[t])) < 1e-4
            assert set(top.indices.tolist()) <= set(d)
            for j, i in enumerate(top.indices.tolist()):
                assert abs(d[i].logprob - float(top.values[j])) < 1e-4
            cum += float(lp[t])
        assert abs(c.cumulative_logprob - cum) < 1e-3
    # without the request, no log-probabilities are computed or returned
    plain = _llm().generate(prompts[:1], SamplingParams(temperature=0.0, max_tokens=2))
    assert plain[0].outputs[0].logprobs is None


def test_special_requests_beside_speculative_decoding():
    """With n-gram speculation configured, requests with penalties or log-probabilities run
    without drafts in the same batches as drafted requests: every output equals its run
    without speculation, and the plain repetitive request still gets drafts accepted."""
    g = torch.Generator().manual_seed(5)
    base = torch.randint(0, 1024, (12,), generator=g).tolist()
    rep = (base * 4)[:40]
    prompts = [rep, _prompts(1, 20, seed=3)[0], rep[:30]]
    params = [SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True),
              SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True,
                             repetition_penalty=1.3, presence_penalty=0.2),
              SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True, logprobs=2)]

    def run(spec):
        llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
                  max_model_len=128, max_num_seqs=4, max_num_batched_tokens=256,
                  speculative_config=spec)
        outs = llm.generate(prompts, params)
        return outs, llm.engine.scheduler

    plain, _ = run(None)
    spec, sch = run({"method": "ngram", "num_speculative_tokens": 3})
    for a, b in zip(plain, spec):
        assert a.outputs[0].token_ids == b.outputs[0].token_ids
    for x, y in zip(plain[2].outputs[0].logprobs, spec[2].outputs[0].logprobs):
        assert x.keys() == y.keys()
        for t in x:
            assert abs(x[t].logprob - y[t].logprob) < 1e-4
    assert sch.spec_accepted() > 0


def test_logprobs_modes():
    """logprobs_mode: raw_logits reports the model's logits; processed_logprobs the
    log_softmax of the logits after the penalties; processed_logits those logits divided by
    the temperature."""
    cfg = tiny_llama()
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    p = _prompts(1, 16, seed=12)[0]

    def run(mode, sp):
        llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
                  max_model_len=128, max_num_seqs=4, max_num_batched_tokens=256,
                  logprobs_mode=mode)
        return llm.generate([p], sp)[0].outputs[0]

    c = run("raw_logits", SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True,
                                         logprobs=2))
    for k, (t, d) in enumerate(zip(c.token_ids, c.logprobs)):
        l = ref.logits(p + c.token_ids[:k])[-1]
        assert abs(d[t].logprob - float(l[t])) < 1e-4 and d[t].rank == 1
    rep = 1.5
    c = run("processed_logprobs", SamplingParams(temperature=0.0, max_tokens=4,
                                                 ignore_eos=True, logprobs=2,
                                                 repetition_penalty=rep))
    for k, (t, d) in enumerate(zip(c.token_ids, c.logprobs)):
        l = _penalised(ref.logits(p + c.token_ids[:k])[-1], p, c.token_ids[:k], rep, 0.0, 0.0)
        lp = torch.log_softmax(l, -1)
        assert abs(d[t].logprob - float(lp[t])) < 1e-4
    temp = 0.7
    c = run("processed_logits", SamplingParams(temperature=temp, max_tokens=4, seed=4,
                                               ignore_eos=True, logprobs=1,
                                               repetition_penalty=rep))
    for k, (t, d) in enumerate(zip(c.token_ids, c.logprobs)):
        l = _penalised(ref.logits(p + c.token_ids[:k])[-1], p, c.token_ids[:k], rep, 0.0, 0.0)
        assert abs(d[t].logprob - float(l[t]) / temp) < 1e-4
    import pytest
    with pytest.raises(ValueError):
        run("softmax", SamplingParams(max_tokens=1))


def test_prompt_logprobs_match_reference():
    """prompt_logprobs: every prompt position after the first carries the log_softmax of the
    reference logits at the previous position (the prompt token's own entry plus the top k),
    also when the prompt is prefilled in chunks and when a prefix of it is cached by another
    request (the request recomputes its whole prompt)."""
    cfg = tiny_llama()
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    p = _prompts(1, 40, seed=13)[0]
    for budget in (256, 16):
        llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
                  max_model_len=128, max_num_seqs=4, max_num_batched_tokens=budget)
        llm.generate([p], SamplingParams(temperature=0.0, max_tokens=2))  # caches the prefix
        o = llm.generate([p], SamplingParams(temperature=0.0, max_tokens=3, prompt_logprobs=2))[0]
        plp = o.prompt_logprobs
        assert len(plp) == len(p) and plp[0] is None
        lp = torch.log_softmax(ref.logits(p), -1)  # row j predicts token j + 1
        for j in range(1, len(p)):
            d = plp[j]
            assert abs(d[p[j]].logprob - float(lp[j - 1, p[j]])) < 1e-4
            assert d[p[j]].rank == int((lp[j - 1] > lp[j - 1, p[j]]).sum()) + 1
            top = torch.topk(lp[j - 1], 2).indices.tolist()
            assert set(top) <= set(d)
        plain = llm.generate([p], SamplingParams(temperature=0.0, max_tokens=3))[0]
        assert plain.prompt_logprobs is None
        assert o.outputs[0].token_ids == plain.outputs[0].token_ids


def test_truncate_prompt_tokens():
    p = _prompts(1, 40, seed=14)[0]
    sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True, truncate_prompt_tokens=12)
    got = _llm().generate([p], sp)[0]
    want = _llm().generate([p[-12:]], SamplingParams(temperature=0.0, max_tokens=4,
                                                      ignore_eos=True))[0]
    assert got.prompt_token_ids == p[-12:]
    assert got.outputs[0].token_ids == want.outputs[0].token_ids
