"""The flagship dense decoder on a B200 through the engine: the logits of the first steps
(prefill, then decode over the paged cache) track the fp32 CPU reference decoder at bf16
resolution, for the tiny Llama and for two layers of the Llama-3-8B shape (hidden 4096,
32 / 8 heads of 128, intermediate 14336, vocab 128256), and CUDA-graph decode produces the same
tokens as eager decode."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _tiny():
    from vllm_musa_b200.models.presets import tiny_llama
    c = tiny_llama()
    c.dtype = torch.bfloat16
    return c


def _llama8b_2layers():
    from vllm_musa_b200.models.presets import llama3_8b
    c = llama3_8b()
    c.num_layers = 2
    return c


@pytest.mark.parametrize("make", [_tiny, _llama8b_2layers], ids=["tiny", "llama3-8b-2l"])
def test_llama_logits_track_reference(make):
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.reference import ReferenceDecoder
    from vllm_musa_b200.models.weights import dummy_weights
    cfg = make()
    g = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, cfg.vocab_size, (150,), generator=g).tolist()
    n_out = 3
    llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=32, max_model_len=512, max_num_seqs=4,
              max_num_batched_tokens=512, enforce_eager=True)
    llm.engine.runner.record_logits = True
    out = llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=n_out,
                                                ignore_eos=True))
    toks = out[0].outputs[0].token_ids
    got = [lg[0] for lg in llm.engine.runner.logits_log]
    llm.shutdown()
    assert len(got) == n_out
    ref_cfg = make()
    ref_cfg.dtype = torch.float32
    # the engine draws its random weights with the CUDA generator: the same stream in fp32
    W = {k: v.cpu() for k, v in dummy_weights(ref_cfg, seed=0, std=0.02, device="cuda")}
    ref = ReferenceDecoder(ref_cfg, W)
    for k in range(n_out):
        want = ref.logits(prompt + toks[:k])[-1]
        err = float((got[k] - want).abs().max() / want.abs().max())
        assert err < 0.05, (k, err)  # bf16 weights / activations vs the fp32 reference


def test_llama_graph_decode_matches_eager():
    from vllm_musa_b200 import LLM, SamplingParams
    cfg = _tiny()
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (3, 70, 130)]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    res = {}
    for eager in (True, False):
        llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=32, max_model_len=512,
                  max_num_seqs=4, max_num_batched_tokens=512, enforce_eager=eager,
                  cuda_graph_sizes=[1, 2, 4])
        res[eager] = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
        llm.shutdown()
    assert res[True] == res[False]
