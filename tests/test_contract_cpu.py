"""Optimisation contract: signatures and preferences for each family / execution shape, and
the fail-closed validation."""
import pytest
import torch

from vllm_musa_b200 import plan
from vllm_musa_b200.config import EngineConfig, ModelConfig, ParallelConfig, SpeculativeConfig
from vllm_musa_b200.models.presets import get_preset

F = plan.Feature


def _cfg(model, tp=1, **kw):
    return EngineConfig(model=model, parallel=ParallelConfig(tensor_parallel_size=tp), **kw)


def test_dense_tp1_and_tp8():
    m = get_preset("llama3-8b")
    c = plan.resolve(_cfg(m))
    assert c.prefers(F.CUDA_GRAPH_DECODE) and c.prefers(F.PREFIX_CACHING)
    assert c.prefers(F.PREFILL_TCGEN05) and c.prefers(F.PREFILL_TWO_HEADS)
    assert not c.supports(F.FUSED_AR_RMSNORM)
    assert c.profile == "dense-bfloat16-tp1"
    c8 = plan.resolve(_cfg(m, 8))
    assert c8.prefers(F.FUSED_AR_RMSNORM) and c8.prefers(F.VOCAB_PARALLEL_SAMPLING)
    assert c8.supports(F.GEMM_RS_EPILOGUE) and not c8.prefers(F.GEMM_RS_EPILOGUE)
    # 32 q heads / 8 kv heads over 8 ranks: GQA group 4 per rank is even
    assert c8.prefers(F.PREFILL_TWO_HEADS)


def test_recurrent_models_disable_prefix_caching():
    m = ModelConfig(arch="mamba2", ssm_state_size=128, mamba_num_heads=8, mamba_head_dim=64)
    c = plan.resolve(_cfg(m))
    assert c.model.recurrent_state and not c.prefers(F.PREFIX_CACHING)
    assert plan.resolve(_cfg(ModelConfig(arch="qwen3_next"))).model.recurrent_state


def test_deepseek_features_and_validation():
    m = ModelConfig(arch="deepseek_v3", kv_lora_rank=512, index_topk=2048, quant="fp8_block",
                    dtype=torch.bfloat16, num_experts=256)
    c = plan.resolve(_cfg(m, speculative=SpeculativeConfig(method="mtp",
                                                          num_speculative_tokens=1)))
    assert {F.NORM_QUANT_FP8, F.SPARSE_INDEXER, F.MTP} <= c.preferred
    plan.validate(c)
    bad = _cfg(get_preset("llama3-8b"), 2)
    bad.parallel.decode_context_parallel_size = 2
    with pytest.raises(ValueError):
        plan.validate(plan.resolve(bad))
    with pytest.raises(ValueError):
        plan.validate(plan.resolve(_cfg(get_preset("llama3-8b"), speculative=SpeculativeConfig(
            method="mtp", num_speculative_tokens=1))))
