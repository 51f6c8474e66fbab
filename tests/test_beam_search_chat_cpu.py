"""LLM.beam_search against a beam search over the pure-PyTorch reference decoder (same
expansion and ranking rules, fp32 logits), and LLM.chat through a chat template."""
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights
from vllm_musa_b200.sample.sampling_params import BeamSearchParams


def _llm(**kw):
    return LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=128,
               max_model_len=128, max_num_seqs=16, max_num_batched_tokens=512, **kw)


def _ref_beams(ref, prompt, w, n, eos, lp_pen, ignore_eos):
    live, done = [([], 0.0)], []
    for _ in range(n):
        cands = []
        for gen, cum in live:
            lp = torch.log_softmax(ref.logits(prompt + gen)[-1], -1)
            top = torch.topk(lp, 2 * w)
            for t, v in zip(top.indices.tolist(), top.values.tolist()):
                cands.append((gen + [t], cum + v))
        cands.sort(key=lambda c: c[1], reverse=True)
        live = []
        for c in cands:
            if not ignore_eos and c[0][-1] == eos:
                done.append(c)
            else:
                live.append(c)
            if len(live) == w:
                break
    allb = done + live

    def score(c):
        L = len(prompt) + len(c[0]) - (1 if c[0][-1] == eos and not ignore_eos else 0)
        return c[1] / L ** lp_pen
    allb.sort(key=score, reverse=True)
    return allb[:w]


def test_beam_search_matches_reference():
    cfg = tiny_llama()
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    g = torch.Generator().manual_seed(4)
    prompts = torch.randint(0, 1024, (2, 12), generator=g).tolist()
    llm = _llm()
    # make a likely token the EOS so some beams finish early
    eos = int(torch.argmax(ref.logits(prompts[0])[-1]))
    llm.engine.config.model.eos_token_id = eos
    for ignore_eos, pen in ((False, 1.0), (True, 0.5)):
        outs = llm.beam_search(prompts, BeamSearchParams(beam_width=3, max_tokens=4,
                                                         ignore_eos=ignore_eos,
                                                         length_penalty=pen))
        for p, o in zip(prompts, outs):
            want = _ref_beams(ref, p, 3, 4, eos, pen, ignore_eos)
            assert len(o.sequences) == 3
            for s, (gen, cum) in zip(o.sequences, want):
                assert s.tokens == p + gen
                assert abs(s.cum_logprob - cum) < 1e-3


def test_chat_renders_template_and_generates():
    class T:
        chat_template = "x"

        def apply_chat_template(self, msgs, add_generation_prompt=True, tokenize=True):
            ids = []
            for m in msgs:
                ids += [1 if m["role"] == "user" else 2] + [ord(c) % 1000 + 10 for c in m["content"]]
            return ids + ([3] if add_generation_prompt else [])

        def encode(self, s):
            return [ord(c) % 1000 for c in s]

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr(65 + i % 26) for i in ids)

    llm = _llm(tokenizer=T())
    conv = [{"role": "user", "content": "hi there"}]
    sp = SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True)
    got = llm.chat(conv, sp)[0]
    ids = T().apply_chat_template(conv)
    assert got.prompt_token_ids == ids
    assert got.outputs[0].token_ids == llm.generate([ids], sp)[0].outputs[0].token_ids
    two = llm.chat([conv, conv + [{"role": "assistant", "content": "yo"}]], sp)
    assert len(two) == 2 and two[0].outputs[0].token_ids == got.outputs[0].token_ids
