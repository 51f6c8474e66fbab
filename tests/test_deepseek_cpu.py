"""DeepSeek-V3.2-style tiny model on CPU (fp32): absorbed MLA over the latent cache, the
lightning indexer's causal top-k, sigmoid grouped-top-k MoE with shared experts, through the
engine (chunked prefill, batching) vs the expanded whole-sequence HF-layout reference."""
import pytest
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.config import ModelConfig
from vllm_musa_b200.models.reference import DeepseekReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights


def tiny_ds(sparse=True, q_lora=128):
    return ModelConfig(arch="deepseek_v3", vocab_size=512, hidden_size=256, num_layers=3,
                       num_heads=4, num_kv_heads=4, head_dim=192, intermediate_size=256,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=512,
                       num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                       shared_expert_intermediate_size=64, first_k_dense=1, n_group=4,
                       topk_group=2, routed_scaling_factor=2.5, scoring_func="sigmoid",
                       q_lora_rank=q_lora, kv_lora_rank=512, qk_nope_head_dim=128,
                       qk_rope_head_dim=64, v_head_dim=128,
                       index_n_heads=64 if sparse else 0, index_head_dim=128 if sparse else 0,
                       index_topk=64 if sparse else 0, rope_neox=False, dtype=torch.float32,
                       name="tiny-ds")


def _prompts(n, length, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 512, (n, length), generator=g).tolist()


@pytest.mark.parametrize("sparse,q_lora,budget", [(True, 128, 256), (True, 128, 40),
                                                   (False, 0, 256)])
def test_tiny_deepseek_matches_reference(sparse, q_lora, budget):
    cfg = tiny_ds(sparse, q_lora)
    prompts = _prompts(2, 90, seed=1)  # longer than the indexer's top-64: sparse selection
    llm = LLM(cfg, device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
              max_num_seqs=4, max_num_batched_tokens=budget)
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))
    ref = DeepseekReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    for i, p in enumerate(prompts):
        toks, _ = ref.greedy(p, 4)
        assert outs[i].outputs[0].token_ids == toks, f"request {i} diverged"


def test_tiny_deepseek_w4afp8_experts():
    """W4AFP8: the engine keeps routed experts packed int4 and quantises activations per token;
    its first-step logits match the fp32 reference run on the int4-rounded expert weights."""
    from vllm_musa_b200.ops.w4afp8 import dequant_w4, quantize_w4
    cfg = tiny_ds(False, 0)
    cfg.moe_intermediate_size = 128  # int4 groups of 128 along every expert K
    cfg.quant = "w4afp8"
    prompt = _prompts(1, 40, seed=5)[0]
    llm = LLM(cfg, device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
              max_num_seqs=4, max_num_batched_tokens=256)
    L = llm.engine.runner.model.layers[1]
    assert L.w4 is not None and L.w4[0].dtype == torch.int8 and L.experts_gu is None
    llm.engine.runner.record_logits = True
    llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True))
    got = llm.engine.runner.logits_log[0][0]
    ref_cfg = tiny_ds(False, 0)
    ref_cfg.moe_intermediate_size = 128
    W = dict(dummy_weights(ref_cfg, seed=0, std=0.02))
    for k in list(W):
        if ".experts." in k:
            q, s = quantize_w4(W[k][None])
            W[k] = dequant_w4(q, s)[0]
    want = DeepseekReferenceDecoder(ref_cfg, W).logits(prompt)[-1]
    err = (got - want).abs().max() / want.abs().max()
    assert 0 < err < 0.02, float(err)  # only the per-token e4m3 activation rounding differs


def test_tiny_deepseek_swiglu_clamp():
    """swiglu_limit clamps the dense MLPs' gate (<= limit) and up (|up| <= limit): a large limit
    is the plain SwiGLU, a small one changes the logits."""
    def logits(limit):
        cfg = tiny_ds(False, 0)
        cfg.num_experts = 0
        cfg.swiglu_limit = limit
        llm = LLM(cfg, device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
                  max_model_len=128, max_num_seqs=4, max_num_batched_tokens=256)
        llm.engine.runner.record_logits = True
        llm.generate([_prompts(1, 12, seed=8)[0]],
                     SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True))
        return llm.engine.runner.logits_log[0][0]
    plain, big, small = logits(0.0), logits(1e4), logits(1e-3)
    torch.testing.assert_close(big, plain, rtol=1e-4, atol=1e-5)
    assert (small - plain).abs().max() > 1e-4
