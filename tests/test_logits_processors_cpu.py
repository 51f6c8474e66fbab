"""logit_bias, allowed_token_ids and bad_words (vLLM / OpenAI logits processors) through the
engine on the tiny CPU Llama, against greedy loops over the pure-PyTorch reference decoder
that apply the same rule to its logits; at TP=1 and with the vocabulary sharded over two Gloo
ranks (each rank biases / masks its own columns)."""
import os
import socket

import torch
import torch.multiprocessing as mp

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights


class DigitTokenizer:
    """Token id t <-> the text str(t) + ' ' (enough to name bad words by their ids)."""

    def encode(self, s):
        return [int(w) for w in s.split()]

    def decode(self, ids, skip_special_tokens=True):
        return "".join(f"{i} " for i in ids)


def _prompts():
    g = torch.Generator().manual_seed(21)
    return torch.randint(0, 1024, (3, 18), generator=g).tolist()


def _llm(**kw):
    return LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
               max_model_len=128, max_num_seqs=4, max_num_batched_tokens=256, **kw)


def _ref():
    cfg = tiny_llama()
    return ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))


def _greedy(ref, prompt, n, rule):
    toks = []
    for _ in range(n):
        l = rule(ref.logits(prompt + toks)[-1].clone(), toks)
        toks.append(int(torch.argmax(l)))
    return toks


def test_logit_bias_and_allowed_tokens_match_reference():
    ref = _ref()
    prompts = _prompts()
    free = [o.outputs[0].token_ids for o in _llm().generate(
        prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))]
    # push the second free token of each prompt down, and a fixed token up a little
    bias = {free[0][1]: -100.0, 77: 2.5, 500: -3.0}
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True, logit_bias=bias)
    got = [o.outputs[0].token_ids for o in _llm().generate(prompts, sp)]

    def add_bias(l, toks):
        for t, v in bias.items():
            l[t] += v
        return l

    for p, g in zip(prompts, got):
        assert g == _greedy(ref, p, 8, add_bias)
    assert got[0] != free[0]
    allowed = [3, 9, 77, 500, 901]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True,
                        allowed_token_ids=allowed)
    got = [o.outputs[0].token_ids for o in _llm().generate(prompts, sp)]

    def only(l, toks):
        m = torch.full_like(l, float("-inf"))
        m[allowed] = l[allowed]
        return m

    for p, g in zip(prompts, got):
        assert set(g) <= set(allowed)
        assert g == _greedy(ref, p, 8, only)
    # sampled rows stay inside the allowed set too
    sp = SamplingParams(temperature=1.0, max_tokens=16, ignore_eos=True, seed=3,
                        allowed_token_ids=allowed)
    for o in _llm().generate(prompts, sp):
        assert set(o.outputs[0].token_ids) <= set(allowed)


def test_bad_words_never_completed():
    ref = _ref()
    prompts = _prompts()
    llm = _llm(tokenizer=DigitTokenizer())
    free = [o.outputs[0].token_ids for o in llm.generate(
        prompts, SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True))]
    # ban the free continuation's 3rd token outright, and the 5th token after the 4th
    one = str(free[0][2])
    two = f"{free[1][3]} {free[1][4]}"
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True, bad_words=[one, two])
    got = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    seqs = [[int(one)], [free[1][3], free[1][4]]]

    def ban(l, toks):
        for s in seqs:
            pre = s[:-1]
            if not pre or toks[len(toks) - len(pre):] == pre:
                l[s[-1]] = float("-inf")
        return l

    for p, g in zip(prompts, got):
        assert g == _greedy(ref, p, 10, ban)
        assert int(one) not in g
        assert all(g[i:i + 2] != seqs[1] for i in range(len(g) - 1))
    assert got[0] != free[0] and got[1] != free[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from vllm_musa_b200.parallel.state import destroy_distributed
    llm = _llm(tensor_parallel_size=world)
    sps = [SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True,
                          logit_bias={5: 40.0, 1000: 3.0}),
           SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True,
                          allowed_token_ids=[4, 600, 1001]),
           SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)]
    outs = llm.generate(_prompts(), sps)
    q.put((rank, [o.outputs[0].token_ids for o in outs]))
    destroy_distributed()


def test_logits_processors_vocab_parallel_tp2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1]
    assert res[0][0] == [5] * 6  # a +40 bias wins every step
    assert set(res[0][1]) <= {4, 600, 1001}
    one = [o.outputs[0].token_ids for o in _llm().generate(
        _prompts(), [SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True,
                                    logit_bias={5: 40.0, 1000: 3.0}),
                     SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True,
                                    allowed_token_ids=[4, 600, 1001]),
                     SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)])]
    assert res[0] == one
