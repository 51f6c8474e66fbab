"""HuggingFace safetensors checkpoints through ``LLM(path)`` on CPU.

* A Llama checkpoint stored in bf16 (``config.json`` + ``model.safetensors``, written by
  ``save_safetensors``) loads through ``ModelConfig.from_hf`` and the safetensors reader and
  decodes the same greedy tokens as the fp32 reference run on the bf16-rounded weights.
* A DeepSeek-V3-style checkpoint in the block-FP8 layout (e4m3 ``weight`` + fp32
  ``weight_scale_inv`` per 128 x 128 block for every projection, ``quantization_config``
  ``{"quant_method": "fp8", "weight_block_size": [128, 128]}``) loads through the same path
  (dequantised for the CPU fp32 run) and tracks the fp32 reference on the dequantised
  weights.
"""
import os
import sys

import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import DeepseekReferenceDecoder, ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights, save_safetensors

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def _prompts(n, length, vocab, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, length), generator=g).tolist()


def _llm(path):
    return LLM(path, device="cpu", dtype=torch.float32, block_size=16, seed=0, num_gpu_blocks=64,
               max_model_len=128, max_num_seqs=4, max_num_batched_tokens=256)


def test_llama_bf16_safetensors_round_trip(tmp_path):
    cfg = tiny_llama()
    W = {n: t for n, t in dummy_weights(cfg, seed=0, std=0.02, dtype=torch.bfloat16)}
    hf = {"architectures": ["LlamaForCausalLM"], "model_type": "llama",
          "vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size,
          "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
          "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
          "intermediate_size": cfg.intermediate_size, "rms_norm_eps": cfg.rms_norm_eps,
          "rope_theta": cfg.rope_theta, "max_position_embeddings": cfg.max_position,
          "tie_word_embeddings": False, "torch_dtype": "bfloat16"}
    save_safetensors(W.items(), str(tmp_path), hf)
    llm = _llm(str(tmp_path))
    assert llm.engine.config.load_format == "safetensors"
    prompts = _prompts(3, 24, cfg.vocab_size, seed=4)
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    ref = ReferenceDecoder(cfg, {n: t.float() for n, t in W.items()})
    for o, p in zip(outs, prompts):
        toks, _ = ref.greedy(p, 8)
        assert o.outputs[0].token_ids == toks


def _fp8_checkpoint(cfg):
    """Random DeepSeek weights with every projection stored as e4m3 + 128x128 scale_inv;
    returns (checkpoint tensors, dequantised fp32 weights for the reference)."""
    from vllm_musa_b200.ops import fp8 as fp8_ops
    ckpt, deq = {}, {}
    for n, t in dummy_weights(cfg, seed=0, std=0.02):
        if n.endswith("proj.weight") or n.endswith("proj_with_mqa.weight"):
            q, s = fp8_ops.quantize_weight_block(t.float())
            assert q.dtype == torch.float8_e4m3fn
            ckpt[n], ckpt[n[:-len("weight")] + "weight_scale_inv"] = q, s.float()
            deq[n] = fp8_ops.dequantize_weight_block(q, s.float())
        else:
            ckpt[n], deq[n] = t, t
    return ckpt, deq


def test_deepseek_block_fp8_checkpoint(tmp_path):
    from test_deepseek_cpu import tiny_ds
    cfg = tiny_ds(sparse=False, q_lora=128)
    cfg.moe_intermediate_size = cfg.shared_expert_intermediate_size = 128
    ckpt, deq = _fp8_checkpoint(cfg)
    hf = {"architectures": ["DeepseekV3ForCausalLM"], "model_type": "deepseek_v3",
          "vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size,
          "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
          "num_key_value_heads": cfg.num_kv_heads, "intermediate_size": cfg.intermediate_size,
          "moe_intermediate_size": cfg.moe_intermediate_size, "n_routed_experts": cfg.num_experts,
          "n_shared_experts": 1, "num_experts_per_tok": cfg.num_experts_per_tok,
          "first_k_dense_replace": cfg.first_k_dense, "n_group": cfg.n_group,
          "topk_group": cfg.topk_group, "routed_scaling_factor": cfg.routed_scaling_factor,
          "scoring_func": "sigmoid", "norm_topk_prob": True, "q_lora_rank": cfg.q_lora_rank,
          "kv_lora_rank": cfg.kv_lora_rank, "qk_nope_head_dim": cfg.qk_nope_head_dim,
          "qk_rope_head_dim": cfg.qk_rope_head_dim, "v_head_dim": cfg.v_head_dim,
          "rms_norm_eps": cfg.rms_norm_eps, "rope_theta": cfg.rope_theta,
          "max_position_embeddings": cfg.max_position, "tie_word_embeddings": False,
          "quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128],
                                  "activation_scheme": "dynamic", "fmt": "e4m3"}}
    save_safetensors(ckpt.items(), str(tmp_path), hf)
    llm = _llm(str(tmp_path))
    mc = llm.engine.config.model
    assert mc.quant == "fp8_block" and mc.arch == "deepseek_v3" and not mc.rope_neox
    llm.engine.runner.record_logits = True
    prompt = _prompts(1, 40, cfg.vocab_size, seed=6)[0]
    out = llm.generate([prompt], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))
    got = llm.engine.runner.logits_log[0][0]
    ref = DeepseekReferenceDecoder(cfg, deq)
    want = ref.logits(prompt)[-1]
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-4)
    toks, _ = ref.greedy(prompt, 4)
    assert out[0].outputs[0].token_ids == toks
