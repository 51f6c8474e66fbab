"""Qwen3-Next hybrid (Gated DeltaNet + gated attention + MoE) on CPU: the GDN ops against
plain token loops, and a tiny model through the engine (C++ scheduler, per-request state
slots, chunked prefill, batching) matching the whole-sequence HF-layout reference."""
import torch
import torch.nn.functional as F

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.config import ModelConfig
from vllm_musa_b200.models.reference import HybridReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights
from vllm_musa_b200.ops import gdn


def tiny_next():
    return ModelConfig(arch="qwen3_next", vocab_size=512, hidden_size=128, num_layers=4,
                       num_heads=4, num_kv_heads=2, head_dim=64, intermediate_size=256,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=512, qk_norm=True,
                       num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                       shared_expert_intermediate_size=64, full_attention_interval=4,
                       linear_num_key_heads=2, linear_num_value_heads=4,
                       linear_key_head_dim=128, linear_value_head_dim=128,
                       partial_rotary_factor=0.25, attn_output_gate=True,
                       dtype=torch.float32, name="tiny-next")


def test_causal_conv1d_chunks_equal_whole_sequence():
    g = torch.Generator().manual_seed(0)
    C, L = 16, 11
    x = torch.randn(L, C + 5, generator=g)  # extra trailing channels are ignored
    w = torch.randn(C, 4, generator=g)
    ref = F.silu(F.conv1d(F.pad(x[:, :C].t().unsqueeze(0), (3, 0)), w.unsqueeze(1), groups=C)[0]).t()
    state = torch.zeros(2, C, 3)
    outs, done = [], 0
    for chunk in (4, 1, 6):  # prefill chunk, one decode token, rest
        seg = x[done:done + chunk]
        done += chunk
        outs.append(gdn.causal_conv1d(seg, w, state, torch.tensor([0, chunk]),
                                      torch.tensor([done]), torch.tensor([1])))
    torch.testing.assert_close(torch.cat(outs), ref, rtol=1e-5, atol=1e-5)


def test_gdn_recurrent_chunks_equal_whole_sequence():
    g = torch.Generator().manual_seed(1)
    Hk, Hv, L = 1, 2, 9
    qkv = torch.randn(L, 2 * Hk * 128 + Hv * 128, generator=g)
    ba = torch.randn(L, 2 * Hv, generator=g)
    A_log = torch.log(torch.tensor([1.0, 4.0]))
    dt_bias = torch.tensor([0.5, -0.5])
    whole = gdn.gdn_recurrent(qkv, ba, A_log, dt_bias, torch.zeros(1, Hv, 128, 128),
                              torch.tensor([0, L]), torch.tensor([L]), torch.tensor([0]), Hk, Hv)
    state = torch.zeros(3, Hv, 128, 128)
    parts, done = [], 0
    for chunk in (5, 1, 3):
        done += chunk
        parts.append(gdn.gdn_recurrent(qkv[done - chunk:done], ba[done - chunk:done], A_log,
                                       dt_bias, state, torch.tensor([0, chunk]),
                                       torch.tensor([done]), torch.tensor([2]), Hk, Hv))
    torch.testing.assert_close(torch.cat(parts), whole, rtol=1e-5, atol=1e-5)


def _run(max_batched_tokens, prompts, n_out):
    cfg = tiny_next()
    llm = LLM(cfg, device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
              max_num_seqs=4, max_num_batched_tokens=max_batched_tokens)
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=n_out, ignore_eos=True))
    return cfg, llm, outs


def _prompts(n, length, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 512, (n, length), generator=g).tolist()


def test_tiny_qwen3_next_matches_reference():
    prompts = _prompts(3, 20)
    cfg, llm, outs = _run(256, prompts, 6)
    ref = HybridReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    for i, p in enumerate(prompts):
        toks, _ = ref.greedy(p, 6)
        assert outs[i].outputs[0].token_ids == toks, f"request {i} diverged"


def test_tiny_qwen3_next_chunked_prefill_carries_state():
    # a 24-token budget splits the 30-token prompts into chunks: conv and recurrent state must
    # carry across steps through each request's state slot
    prompts = _prompts(2, 30, seed=3)
    cfg, llm, outs = _run(24, prompts, 5)
    ref = HybridReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    for i, p in enumerate(prompts):
        toks, _ = ref.greedy(p, 5)
        assert outs[i].outputs[0].token_ids == toks, f"request {i} diverged"
