"""EAGLE speculative decoding on the tiny CPU Llama: verified outputs equal plain greedy
decoding, and every draft the head proposes equals a pure-PyTorch EAGLE-1 forward over the
whole sequence (fc over [embed(t_{p+1}); h_p], one decoder layer without input norm, the
target's LM head), with random and with safetensors-loaded head weights."""
import torch
import torch.nn.functional as F
import pytest

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.eagle import eagle_param_shapes
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights, save_safetensors

KW = dict(device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
          max_num_seqs=4, max_num_batched_tokens=64)


def _prompts():
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (23, 40, 9)]


def eagle_logits(ref: ReferenceDecoder, ew: dict, tokens: list) -> torch.Tensor:
    """Draft logits [n-1, V]: row p predicts token p+2 of ``tokens``."""
    cfg, w, D = ref.cfg, ref.w, ref.D
    ew = {k: v.float() for k, v in ew.items()}
    n = len(tokens)
    hid = ref.hidden(tokens)[:n - 1]
    e = w["model.embed_tokens.weight"][torch.tensor(tokens[1:])]
    x = torch.cat([e, hid], -1) @ ew["fc.weight"].t()
    if "fc.bias" in ew:
        x = x + ew["fc.bias"]
    P = n - 1
    a = "layers.0.self_attn."
    q = (x @ ew[a + "q_proj.weight"].t()).view(P, cfg.num_heads, D)
    k = (x @ ew[a + "k_proj.weight"].t()).view(P, cfg.num_kv_heads, D)
    v = (x @ ew[a + "v_proj.weight"].t()).view(P, cfg.num_kv_heads, D)
    pos = torch.arange(P)
    q, k = ref._rope(q, pos), ref._rope(k, pos)
    G = cfg.num_heads // cfg.num_kv_heads
    k, v = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
    s = torch.einsum("qhd,khd->hqk", q, k) / D ** 0.5
    s = s.masked_fill(torch.triu(torch.ones(P, P, dtype=torch.bool), 1)[None], float("-inf"))
    h = x + torch.einsum("hqk,khd->qhd", s.softmax(-1), v).reshape(P, -1) @ \
        ew[a + "o_proj.weight"].t()
    y = ref._rms(h, ew["layers.0.post_attention_layernorm.weight"])
    m = "layers.0.mlp."
    h = h + (F.silu(y @ ew[m + "gate_proj.weight"].t()) * (y @ ew[m + "up_proj.weight"].t())) \
        @ ew[m + "down_proj.weight"].t()
    if "norm.weight" in ew:
        h = ref._rms(h, ew["norm.weight"])
    return h @ w.get("lm_head.weight", w["model.embed_tokens.weight"]).t()


class _Recorder:
    """Scheduler proxy recording (tokens so far, draft) at every ``set_draft``."""

    def __init__(self, inner):
        self._inner = inner
        self.drafts = []

    def __getattr__(self, name):
        return getattr(self._inner, name)

    def set_draft(self, rid, toks):
        n = self._inner.num_tokens(rid)
        self.drafts.append((self._inner.tokens_range(rid, 0, n), list(toks)))
        return self._inner.set_draft(rid, toks)


def _check_drafts(rec, ref, ew):
    assert rec.drafts
    for toks, draft in rec.drafts:
        lg = eagle_logits(ref, ew, toks)[-1]
        top = torch.topk(lg, 2)
        if int(top.indices[0]) != draft[0]:
            # only a near-tie may differ in argmax between the two paths
            assert float(top.values[0] - lg[draft[0]]) < 1e-3


def test_eagle_spec_decode_matches_plain_and_reference_drafts():
    cfg = tiny_llama()
    prompts = _prompts()
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **KW).generate(prompts, sp)]
    llm = LLM(cfg, speculative_config={"method": "eagle", "num_speculative_tokens": 1}, **KW)
    rec = _Recorder(llm.engine.scheduler)
    llm.engine.scheduler = rec
    outs = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert outs == plain
    assert llm.engine.drafter.proposed > 0 and rec.spec_proposed() > 0
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    ew = dict(dummy_weights(cfg, seed=1, std=0.02, shapes=eagle_param_shapes(cfg)))
    _check_drafts(rec, ref, ew)


def test_eagle_head_from_safetensors(tmp_path):
    """A checkpoint with fc bias and a final norm (and an unused embedding copy)."""
    cfg = tiny_llama()
    g = torch.Generator().manual_seed(3)
    ew = {n: (torch.randn(s, generator=g) * 0.05 if k == "w" else
              1.0 + 0.1 * torch.randn(s, generator=g))
          for n, s, k in eagle_param_shapes(cfg)}
    ew["fc.bias"] = 0.05 * torch.randn(cfg.hidden_size, generator=g)
    ew["norm.weight"] = 1.0 + 0.1 * torch.randn(cfg.hidden_size, generator=g)
    ew["embed_tokens.weight"] = torch.zeros(cfg.vocab_size, cfg.hidden_size)
    save_safetensors(ew.items(), str(tmp_path))
    del ew["embed_tokens.weight"]
    prompts = _prompts()[:2]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    llm = LLM(cfg, speculative_config={"method": "eagle", "num_speculative_tokens": 1,
                                       "model": str(tmp_path)}, **KW)
    rec = _Recorder(llm.engine.scheduler)
    llm.engine.scheduler = rec
    outs = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    assert outs == [ref.greedy(p, 6)[0] for p in prompts]
    _check_drafts(rec, ref, ew)


def test_eagle_contract():
    from vllm_musa_b200.config import EngineConfig, SpeculativeConfig
    from vllm_musa_b200.plan import contract as C
    cfg = tiny_llama()
    e = EngineConfig(model=cfg, device="cpu",
                     speculative=SpeculativeConfig(method="eagle", num_speculative_tokens=1))
    k = C.resolve(e)
    C.validate(k)
    assert C.Feature.EAGLE in k.preferred
    with pytest.raises(ValueError):  # chained drafts are verified as chains, not trees
        LLM(cfg, speculative_config={"method": "eagle", "num_speculative_tokens": 2,
                                     "tree_width": 2}, **KW)
    with pytest.raises(ValueError):
        LLM(cfg, speculative_config={"method": "lookahead", "num_speculative_tokens": 1}, **KW)


def _head_layer(ref, ew, X):
    """The EAGLE-1 decoder layer over post-fc inputs X [P, H]: (pre-norm output, logits)."""
    cfg, w, D = ref.cfg, ref.w, ref.D
    P = X.shape[0]
    a = "layers.0.self_attn."
    q = (X @ ew[a + "q_proj.weight"].t()).view(P, cfg.num_heads, D)
    k = (X @ ew[a + "k_proj.weight"].t()).view(P, cfg.num_kv_heads, D)
    v = (X @ ew[a + "v_proj.weight"].t()).view(P, cfg.num_kv_heads, D)
    pos = torch.arange(P)
    q, k = ref._rope(q, pos), ref._rope(k, pos)
    G = cfg.num_heads // cfg.num_kv_heads
    k, v = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
    s = torch.einsum("qhd,khd->hqk", q, k) / D ** 0.5
    s = s.masked_fill(torch.triu(torch.ones(P, P, dtype=torch.bool), 1)[None], float("-inf"))
    h = X + torch.einsum("hqk,khd->qhd", s.softmax(-1), v).reshape(P, -1) @ \
        ew[a + "o_proj.weight"].t()
    y = ref._rms(h, ew["layers.0.post_attention_layernorm.weight"])
    m = "layers.0.mlp."
    h = h + (F.silu(y @ ew[m + "gate_proj.weight"].t()) * (y @ ew[m + "up_proj.weight"].t())) \
        @ ew[m + "down_proj.weight"].t()
    out = ref._rms(h, ew["norm.weight"]) if "norm.weight" in ew else h
    return h, out @ w.get("lm_head.weight", w["model.embed_tokens.weight"]).t()


def eagle_chain(ref, ew, tokens, k):
    """k chained EAGLE-1 drafts after ``tokens``: positions 0..n-2 read the target's hidden
    states, later ones the head's own previous pre-norm output and the previous draft."""
    ew = {n: v.float() for n, v in ew.items()}
    w = ref.w
    n = len(tokens)
    hid = ref.hidden(tokens)[:n - 1]
    emb = w["model.embed_tokens.weight"]

    def fc(e, h):
        x = torch.cat([e, h], -1) @ ew["fc.weight"].t()
        return x + ew["fc.bias"] if "fc.bias" in ew else x

    X = fc(emb[torch.tensor(tokens[1:])], hid)
    drafts = []
    for _ in range(k):
        h, lg = _head_layer(ref, ew, X)
        d = int(torch.argmax(lg[-1]))
        drafts.append(d)
        X = torch.cat([X, fc(emb[d].unsqueeze(0), h[-1:])], 0)
    return drafts


def test_eagle_chained_drafts_match_reference():
    """num_speculative_tokens = 3: each step's three chained drafts equal the pure-PyTorch
    chain, and outputs equal plain greedy decoding."""
    cfg = tiny_llama()
    prompts = _prompts()
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **KW).generate(prompts, sp)]
    llm = LLM(cfg, speculative_config={"method": "eagle", "num_speculative_tokens": 3}, **KW)
    rec = _Recorder(llm.engine.scheduler)
    llm.engine.scheduler = rec
    outs = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert outs == plain
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    ew = dict(dummy_weights(cfg, seed=1, std=0.02, shapes=eagle_param_shapes(cfg)))
    assert rec.drafts and any(len(d) == 3 for _, d in rec.drafts)
    for toks, draft in rec.drafts:
        assert draft == eagle_chain(ref, ew, toks, len(draft))
