"""Tiny DeepSeek-V3.2-style model (block-FP8 linears and experts, MLA, lightning indexer) on
B200 through the engine: CUDA-graph decode matches eager, and the first-step logits track the
fp32 CPU reference at bf16/fp8 resolution."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg(dtype, quant):
    import sys, os
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_deepseek_cpu import tiny_ds
    c = tiny_ds(True, 128)
    c.dtype, c.quant, c.name = dtype, quant, "tiny-ds-gpu"
    # FP8 GEMM inputs are quantised in 1x128 groups: every GEMM K must be a multiple of 128
    c.moe_intermediate_size = c.shared_expert_intermediate_size = 128
    return c


def test_tiny_deepseek_engine_graph_vs_eager():
    from vllm_musa_b200 import LLM, SamplingParams
    cfg = _cfg(torch.bfloat16, "fp8_block")
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 90, 200)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    outs = {}
    for eager in (True, False):
        llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=64, max_model_len=512,
                  max_num_seqs=8, max_num_batched_tokens=256, enforce_eager=eager,
                  cuda_graph_sizes=[1, 2, 4, 8])
        outs[eager] = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
        llm.shutdown()
    assert outs[True] == outs[False]


@pytest.mark.parametrize("quant", [None, "fp8_block", "w4afp8"])
def test_tiny_deepseek_logits_track_reference(quant):
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.reference import DeepseekReferenceDecoder
    from vllm_musa_b200.models.weights import dummy_weights
    cfg = _cfg(torch.bfloat16, quant)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, 512, (150,), generator=g).tolist()
    llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=64, max_model_len=512, max_num_seqs=4,
              max_num_batched_tokens=256, enforce_eager=True)
    llm.engine.runner.record_logits = True
    llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True))
    got = llm.engine.runner.logits_log[0][0]
    llm.shutdown()
    ref_cfg = _cfg(torch.float32, None)
    # the engine draws its random weights with the CUDA generator: use the same stream
    W = {k: v.cpu() for k, v in dummy_weights(ref_cfg, seed=0, std=0.02, device="cuda")}
    ref = DeepseekReferenceDecoder(ref_cfg, W)
    want = ref.logits(prompt)[-1]
    err = (got - want).abs().max() / want.abs().max()
    assert err < (0.25 if quant else 0.06), float(err)  # fp8: weights and activations rounded
