"""Engine request options on a B200 (tiny Llama, bf16), checked against the fp32 PyTorch
reference decoder: logit_bias and allowed_token_ids (bias entries and allowed-token bitmasks on
the device logits), prompt_logprobs (LM head over the prompt rows), embeddings (pooled final
hidden states).  The file sorts after every other GPU test so that a stop-at-first-failure run
has executed them all first."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg():
    from vllm_musa_b200.models.presets import tiny_llama
    c = tiny_llama()
    c.dtype = torch.bfloat16
    return c


def _llm():
    from vllm_musa_b200 import LLM
    return LLM(_cfg(), block_size=64, seed=0, num_gpu_blocks=32, max_model_len=512,
               max_num_seqs=8, max_num_batched_tokens=512, enforce_eager=True)


def _ref():
    from vllm_musa_b200.models.presets import tiny_llama
    from vllm_musa_b200.models.reference import ReferenceDecoder
    from vllm_musa_b200.models.weights import dummy_weights
    cfg = tiny_llama()
    W = {k: v.cpu() for k, v in dummy_weights(cfg, seed=0, std=0.02, device="cuda")}
    return ReferenceDecoder(cfg, W)


def _prompts():
    g = torch.Generator().manual_seed(31)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (20, 70)]


def test_logit_bias_and_allowed_tokens_on_gpu():
    from vllm_musa_b200 import SamplingParams
    llm = _llm()
    ps = _prompts()
    outs = llm.generate(ps, [SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True,
                                            logit_bias={321: 100.0}),
                             SamplingParams(temperature=0.8, max_tokens=8, ignore_eos=True,
                                            seed=2, allowed_token_ids=[7, 70, 700])])
    assert outs[0].outputs[0].token_ids == [321] * 5
    assert set(outs[1].outputs[0].token_ids) <= {7, 70, 700}
    llm.shutdown()


def test_prompt_logprobs_on_gpu_track_reference():
    from vllm_musa_b200 import SamplingParams
    llm = _llm()
    p = _prompts()[1]
    o = llm.generate([p], SamplingParams(temperature=0.0, max_tokens=2, prompt_logprobs=1))[0]
    llm.shutdown()
    lp = torch.log_softmax(_ref().logits(p), -1)
    assert o.prompt_logprobs[0] is None and len(o.prompt_logprobs) == len(p)
    for j in range(1, len(p)):
        got = o.prompt_logprobs[j][p[j]].logprob
        assert abs(got - float(lp[j - 1, p[j]])) < 0.15, (j, got, float(lp[j - 1, p[j]]))


def test_embeddings_on_gpu_track_reference():
    from vllm_musa_b200.sample.sampling_params import PoolingParams
    llm = _llm()
    ps = _prompts()
    ref = _ref()
    for kind in ("last", "mean"):
        outs = llm.embed(ps, PoolingParams(pooling_type=kind))
        for p, o in zip(ps, outs):
            h = ref.hidden(p)
            want = h[-1] if kind == "last" else h.mean(0)
            got = torch.tensor(o.outputs.embedding)
            cos = float(torch.nn.functional.cosine_similarity(got, want / want.norm(), dim=0))
            assert cos > 0.99, (kind, cos)
    llm.shutdown()


def test_eagle3_head_on_gpu_keeps_tokens():
    """EAGLE-3 over the bf16 tiny Llama with CUDA graphs: the model records three residual
    streams per step into a static buffer (graph replays included) and the head drafts from
    them; every emitted token is the fp32 reference argmax up to bf16 resolution."""
    from vllm_musa_b200 import LLM, SamplingParams
    cfg = _cfg()
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (20, 90)]
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
    llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=32, max_model_len=512,
              max_num_seqs=8, max_num_batched_tokens=512,
              speculative_config={"method": "eagle3", "num_speculative_tokens": 1})
    got = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert llm.engine.drafter.proposed > 0
    llm.shutdown()
    ref = _ref()
    for p, toks in zip(prompts, got):
        assert len(toks) == 12
        for k, t in enumerate(toks):
            want = ref.logits(p + toks[:k])[-1]
            gap = float(want.max() - want[t]) / float(want.abs().max())
            assert gap < 0.03, (k, gap)


def test_eagle_chained_drafts_on_gpu_keep_tokens():
    """EAGLE-1 with three chained drafts per step (slots reserved ahead of the verification
    step, the head fed its own output): every emitted token is the fp32 reference argmax up to
    bf16 resolution."""
    from vllm_musa_b200 import LLM, SamplingParams
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (20, 90)]
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
    llm = LLM(_cfg(), block_size=64, seed=0, num_gpu_blocks=32, max_model_len=512,
              max_num_seqs=8, max_num_batched_tokens=512,
              speculative_config={"method": "eagle", "num_speculative_tokens": 3})
    got = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert llm.engine.drafter.proposed > 0
    llm.shutdown()
    ref = _ref()
    for p, toks in zip(prompts, got):
        assert len(toks) == 12
        for k, t in enumerate(toks):
            want = ref.logits(p + toks[:k])[-1]
            gap = float(want.max() - want[t]) / float(want.abs().max())
            assert gap < 0.03, (k, gap)


def test_medusa_on_gpu_keeps_tokens():
    """Medusa heads (chained and tree drafts) over the bf16 tiny Llama with CUDA graphs: every
    emitted token is the fp32 reference argmax up to bf16 resolution."""
    from vllm_musa_b200 import LLM, SamplingParams
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (20, 90)]
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
    ref = _ref()
    for spec in ({"method": "medusa", "num_speculative_tokens": 3},
                 {"method": "medusa", "num_speculative_tokens": 6, "tree_width": 2}):
        llm = LLM(_cfg(), block_size=64, seed=0, num_gpu_blocks=32, max_model_len=512,
                  max_num_seqs=8, max_num_batched_tokens=512, speculative_config=spec)
        got = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
        assert llm.engine.drafter.proposed > 0
        llm.shutdown()
        for p, toks in zip(prompts, got):
            assert len(toks) == 12
            for k, t in enumerate(toks):
                want = ref.logits(p + toks[:k])[-1]
                gap = float(want.max() - want[t]) / float(want.abs().max())
                assert gap < 0.03, (spec, k, gap)
