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


def test_lora_on_gpu_tracks_merged_reference(tmp_path):
    """Two adapters and the base model in one batch on B200 (adapter deltas through this
    package's GEMMs): teacher-forced against the fp32 reference on merged weights, every
    greedy token is the argmax up to bf16 resolution."""
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_lora_cpu import make_adapter, merged_reference
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.lora import LoRARequest
    from vllm_musa_b200.models.reference import ReferenceDecoder
    from vllm_musa_b200.models.weights import dummy_weights
    cfg = _tiny()
    ref_cfg = _tiny()
    ref_cfg.dtype = torch.float32
    ta = make_adapter(str(tmp_path / "a"), ref_cfg, 8, 16, 1)
    tb = make_adapter(str(tmp_path / "b"), ref_cfg, 4, 4, 2)
    W = {k: v.cpu() for k, v in dummy_weights(ref_cfg, seed=0, std=0.02, device="cuda")}

    def merged(t, r, alpha):
        w = dict(W)
        for name, a in t.items():
            if name.endswith("lora_A.weight"):
                b = t[name.replace("lora_A", "lora_B")]
                key = name.replace("base_model.model.", "").replace(".lora_A.weight", ".weight")
                w[key] = w[key] + (alpha / r) * b @ a
        return ReferenceDecoder(ref_cfg, w)
    refs = [merged(ta, 8, 16), merged(tb, 4, 4), ReferenceDecoder(ref_cfg, W)]
    loras = [LoRARequest("a", 1, str(tmp_path / "a")), LoRARequest("b", 2, str(tmp_path / "b")),
             None]
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (30, 70, 12)]
    llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=64, max_model_len=512, max_num_seqs=8,
              max_num_batched_tokens=256, enable_lora=True, max_loras=2, max_lora_rank=16)
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True),
                        lora_request=loras)
    for ref, p, o in zip(refs, prompts, outs):
        toks = o.outputs[0].token_ids
        for k, t in enumerate(toks):
            want = ref.logits(p + toks[:k])[-1]
            assert float(want.max() - want[t]) / float(want.abs().max()) < 0.03, k
