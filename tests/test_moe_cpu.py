"""MoE on CPU: router semantics, fused-MoE reference, and a tiny Qwen3-MoE model through the
engine matching a dense per-token evaluation of the same weights."""
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.config import ModelConfig
from vllm_musa_b200.models.weights import dummy_weights
from vllm_musa_b200.ops import moe as moe_ops
from vllm_musa_b200 import ops


def tiny_moe(shared=0):
    return ModelConfig(arch="qwen3_moe", vocab_size=512, hidden_size=128, num_layers=2,
                       num_heads=4, num_kv_heads=2, head_dim=64, intermediate_size=256,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=512, qk_norm=True,
                       num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                       shared_expert_intermediate_size=shared, dtype=torch.float32,
                       name="tiny-moe")


def test_topk_softmax_and_grouped_topk_semantics():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(5, 16, generator=g)
    ids, w = moe_ops.topk_softmax(logits, 3, renorm=True)
    ref = torch.softmax(logits, -1).topk(3, -1)
    assert torch.equal(ids.long(), ref.indices)
    torch.testing.assert_close(w.sum(-1), torch.ones(5))
    ids, w = moe_ops.grouped_topk(logits, 4, n_group=4, topk_group=2, sigmoid=True, scale=2.5)
    groups = (ids.long() // 4)
    for r in range(5):
        assert len(set(groups[r].tolist())) <= 2
    torch.testing.assert_close(w.sum(-1), torch.full((5,), 2.5))


def test_fused_moe_reference_matches_dense_loop():
    g = torch.Generator().manual_seed(1)
    T, H, I, E, k = 6, 32, 16, 4, 2
    x = torch.randn(T, H, generator=g)
    gate = [torch.randn(I, H, generator=g) * 0.1 for _ in range(E)]
    up = [torch.randn(I, H, generator=g) * 0.1 for _ in range(E)]
    down = [torch.randn(H, I, generator=g) * 0.1 for _ in range(E)]
    w_gu = torch.cat([ops.interleave_gate_up(gate[e], up[e]) for e in range(E)])
    w_dn = torch.cat(down)
    ids, w = moe_ops.topk_softmax(torch.randn(T, E, generator=g), k)
    out = moe_ops.fused_moe(x, w_gu, w_dn, ids, w, E)
    ref = torch.zeros(T, H)
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            h = torch.nn.functional.silu(x[t] @ gate[e].t()) * (x[t] @ up[e].t())
            ref[t] += w[t, j] * (h @ down[e].t())
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)


def _dense_forward(cfg, W, tokens):
    """Whole-sequence reference forward of the tiny Qwen3-MoE model (no paging)."""
    from vllm_musa_b200.models.reference import ReferenceDecoder
    ref = ReferenceDecoder(cfg, {k: v for k, v in W.items()})
    # reuse the reference attention; swap the MLP for the MoE block
    import torch.nn.functional as F
    orig = F.silu

    S = len(tokens)
    w = ref.w
    h = w["model.embed_tokens.weight"][torch.tensor(tokens)]
    D = cfg.head_dim
    G = cfg.num_heads // cfg.num_kv_heads
    pos = torch.arange(S)
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        x = ref._rms(h, w[p + "input_layernorm.weight"])
        q = (x @ w[p + "self_attn.q_proj.weight"].t()).view(S, cfg.num_heads, D)
        k = (x @ w[p + "self_attn.k_proj.weight"].t()).view(S, cfg.num_kv_heads, D)
        v = (x @ w[p + "self_attn.v_proj.weight"].t()).view(S, cfg.num_kv_heads, D)
        q = ref._rms(q, w[p + "self_attn.q_norm.weight"])
        k = ref._rms(k, w[p + "self_attn.k_norm.weight"])
        q, k = ref._rope(q, pos), ref._rope(k, pos)
        k, v = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) / D ** 0.5
        a = torch.einsum("hqk,khd->qhd", torch.softmax(s.masked_fill(mask[None], float("-inf")), -1), v)
        h = h + a.reshape(S, -1) @ w[p + "self_attn.o_proj.weight"].t()
        x = ref._rms(h, w[p + "post_attention_layernorm.weight"])
        probs = torch.softmax(x @ w[p + "mlp.gate.weight"].t(), -1)
        tw, ti = probs.topk(cfg.num_experts_per_tok, -1)
        tw = tw / tw.sum(-1, keepdim=True)
        mo = torch.zeros_like(x)
        for t in range(S):
            for j in range(cfg.num_experts_per_tok):
                e = int(ti[t, j])
                q_ = f"{p}mlp.experts.{e}."
                hh = orig(x[t] @ w[q_ + "gate_proj.weight"].t()) * (x[t] @ w[q_ + "up_proj.weight"].t())
                mo[t] += tw[t, j] * (hh @ w[q_ + "down_proj.weight"].t())
        h = h + mo
    h = ref._rms(h, w["model.norm.weight"])
    return h @ w["lm_head.weight"].t()


def test_tiny_qwen3_moe_engine_matches_dense_reference():
    cfg = tiny_moe()
    W = dict(dummy_weights(cfg, seed=0, std=0.02))
    llm = LLM(cfg, device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
              max_num_seqs=4, max_num_batched_tokens=128)
    llm.engine.runner.record_logits = True
    prompt = torch.randint(0, 512, (20,), generator=torch.Generator().manual_seed(3)).tolist()
    out = llm.generate([prompt], SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))[0]
    toks = list(prompt)
    for step in range(4):
        lg = _dense_forward(cfg, W, toks)[-1]
        torch.testing.assert_close(llm.engine.runner.logits_log[step][0], lg, rtol=1e-3, atol=1e-4)
        toks.append(int(lg.argmax()))
    assert out.outputs[0].token_ids == toks[len(prompt):]
