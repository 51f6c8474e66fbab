"""Structured outputs (xgrammar) through the engine on the tiny CPU Llama with a character-level
vocabulary: sampled outputs always parse as the requested choice / regex / JSON schema and end
with EOS, under temperature sampling, at TP=1 and TP=2 (gloo, vocab-parallel sampling)."""
import json
import os
import re
import socket
import string

import pytest
import torch
import torch.multiprocessing as mp

pytest.importorskip("xgrammar")

from vllm_musa_b200 import LLM, SamplingParams  # noqa: E402
from vllm_musa_b200.models.presets import tiny_llama  # noqa: E402

VOCAB = ["<eos>"] + list(string.printable[:95]) + ["true", "false", "null", '{"', '":', '",',
                                                   "red", "green", "yes", "no"]
VOCAB += [f"<unused{i}>" for i in range(1024 - len(VOCAB))]


class CharTokenizer:
    b200_vocab = VOCAB

    def decode(self, ids, skip_special_tokens=True):
        return "".join(VOCAB[i] for i in ids if i != 0)

    def encode(self, s):
        return [VOCAB.index(c) for c in s]


def _cfg():
    c = tiny_llama()
    c.eos_token_id = 0
    return c


def _llm(tp=1):
    return LLM(_cfg(), device="cpu", tokenizer=CharTokenizer(), block_size=16, seed=0,
               num_gpu_blocks=64, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256,
               tensor_parallel_size=tp)


SCHEMA = {"type": "object", "properties": {"color": {"enum": ["red", "green"]},
                                           "ok": {"type": "boolean"}},
          "required": ["color", "ok"], "additionalProperties": False}


def _requests():
    prompts = [[5 + i, 17, 40, 3] for i in range(6)]
    sps = [SamplingParams(temperature=0.9, seed=11 + i, max_tokens=120, structured_outputs=so)
           for i, so in enumerate([{"choice": ["yes", "no", "maybe"]},
                                   {"regex": r"[0-9]{3}-[a-z]{2}"},
                                   {"json": SCHEMA, "disable_any_whitespace": True},
                                   {"choice": ["alpha", "beta"]},
                                   {"regex": r"(ab|cd)+x"},
                                   {"grammar": 'root ::= "<" [a-c]+ ">"'}])]
    return prompts, sps


def _check(texts, reasons):
    assert texts[0] in ("yes", "no", "maybe")
    assert re.fullmatch(r"[0-9]{3}-[a-z]{2}", texts[1])
    obj = json.loads(texts[2])
    assert set(obj) == {"color", "ok"} and obj["color"] in ("red", "green") and \
        isinstance(obj["ok"], bool)
    assert texts[3] in ("alpha", "beta")
    assert re.fullmatch(r"(ab|cd)+x", texts[4])
    assert re.fullmatch(r"<[a-c]+>", texts[5])
    assert all(r == "stop" for r in reasons)


def test_structured_outputs_tp1():
    prompts, sps = _requests()
    outs = _llm().generate(prompts, sps)
    _check([o.outputs[0].text for o in outs], [o.outputs[0].finish_reason for o in outs])
    # unconstrained sampling of the same random model does not produce these
    free = _llm().generate(prompts[:1], SamplingParams(temperature=0.9, seed=11, max_tokens=8))
    assert free[0].outputs[0].text not in ("yes", "no", "maybe")


def test_token_bitmask_op():
    from vllm_musa_b200.ops.sampling import apply_token_bitmask
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(4, 70, generator=g)
    bm = torch.randint(-2**31, 2**31 - 1, (2, 3), generator=g, dtype=torch.int64).to(torch.int32)
    out = apply_token_bitmask(logits.clone(), bm, torch.tensor([3, 1], dtype=torch.int32))
    for r, row in ((0, 3), (1, 1)):
        for t in range(70):
            allowed = (int(bm[r, t // 32]) >> (t % 32)) & 1
            assert (out[row, t] == float("-inf")) == (not allowed)
    assert torch.equal(out[0], logits[0]) and torch.equal(out[2], logits[2])
    # a vocab shard (offset 32): tokens past the bitmask are masked
    sh = apply_token_bitmask(logits[:, 32:].clone(), bm[:1], torch.tensor([0], dtype=torch.int32),
                             vocab_offset=32)
    for t in range(32, 70):
        allowed = t < 96 and (int(bm[0, t // 32]) >> (t % 32)) & 1
        assert (sh[0, t - 32] == float("-inf")) == (not allowed)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from vllm_musa_b200.parallel.state import destroy_distributed
    prompts, sps = _requests()
    outs = _llm(tp=world).generate(prompts, sps)
    q.put((rank, [o.outputs[0].text for o in outs], [o.outputs[0].finish_reason for o in outs]))
    destroy_distributed()


def test_structured_outputs_tp2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (t, f)) for r, t, f in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1], "ranks diverged"
    _check(*res[0])


def test_stop_strings():
    """A stop string ends the request as soon as the output text contains it; the text is cut
    before it (or keeps it with include_stop_str_in_output), finish_reason "stop"."""
    llm = _llm()
    prompt = [[7, 30, 44, 2]]
    free = llm.generate(prompt, SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True))
    text = free[0].outputs[0].text
    stop = text[5:7]
    at = text.find(stop)
    out = llm.generate(prompt, SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True,
                                              stop=[stop, "\x00never"]))[0].outputs[0]
    assert out.text == text[:at] and out.finish_reason == "stop" and out.stop_reason == stop
    assert len(out.token_ids) < 30
    kept = llm.generate(prompt, SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True,
                                               stop=stop, include_stop_str_in_output=True))
    assert kept[0].outputs[0].text == text[:at + len(stop)]
