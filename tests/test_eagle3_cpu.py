"""EAGLE-3 speculative decoding on a 6-layer tiny CPU Llama: verified outputs equal plain greedy
decoding, and every draft equals the argmax of a pure-PyTorch EAGLE-3 forward (three residual
streams of the target -> fc -> [norm(embed); norm(g)] -> one decoder layer -> norm -> draft
head, mapped to target ids through d2t), with random and with safetensors-loaded weights
including a reduced draft vocabulary."""
import pytest
import torch
import torch.nn.functional as F

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.eagle import eagle3_aux_layers, eagle3_param_shapes
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights, save_safetensors

KW = dict(device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
          max_num_seqs=4, max_num_batched_tokens=64)


def _cfg():
    c = tiny_llama()
    c.num_layers = 6
    return c


def _prompts():
    g = torch.Generator().manual_seed(7)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (21, 37, 9)]


def eagle3_draft(ref, ew, tokens):
    """Target id drafted after ``tokens`` (the head at the last position whose next token is
    the last token of ``tokens``)."""
    cfg, w, D = ref.cfg, ref.w, ref.D
    ew = {k: (v.float() if v.is_floating_point() else v) for k, v in ew.items()}
    n = len(tokens)
    streams = {}
    ref.hidden(tokens, streams)
    aux = torch.cat([streams[l] for l in eagle3_aux_layers(cfg.num_layers)], -1)[:n - 1]
    e = w["model.embed_tokens.weight"][torch.tensor(tokens[1:])]
    g = aux @ ew["fc.weight"].t()
    x = torch.cat([ref._rms(e, ew["midlayer.input_layernorm.weight"]),
                   ref._rms(g, ew["midlayer.hidden_norm.weight"])], -1)
    P = n - 1
    a = "midlayer.self_attn."
    q = (x @ ew[a + "q_proj.weight"].t()).view(P, cfg.num_heads, D)
    k = (x @ ew[a + "k_proj.weight"].t()).view(P, cfg.num_kv_heads, D)
    v = (x @ ew[a + "v_proj.weight"].t()).view(P, cfg.num_kv_heads, D)
    pos = torch.arange(P)
    q, k = ref._rope(q, pos), ref._rope(k, pos)
    G = cfg.num_heads // cfg.num_kv_heads
    k, v = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
    s = torch.einsum("qhd,khd->hqk", q, k) / D ** 0.5
    s = s.masked_fill(torch.triu(torch.ones(P, P, dtype=torch.bool), 1)[None], float("-inf"))
    h = g + torch.einsum("hqk,khd->qhd", s.softmax(-1), v).reshape(P, -1) @ \
        ew[a + "o_proj.weight"].t()
    y = ref._rms(h, ew["midlayer.post_attention_layernorm.weight"])
    m = "midlayer.mlp."
    h = h + (F.silu(y @ ew[m + "gate_proj.weight"].t()) * (y @ ew[m + "up_proj.weight"].t())) \
        @ ew[m + "down_proj.weight"].t()
    lg = ref._rms(h, ew["norm.weight"]) @ ew["lm_head.weight"].t()
    d = int(torch.argmax(lg[-1]))
    return d + int(ew["d2t"][d]) if "d2t" in ew else d


class _Recorder:
    def __init__(self, inner):
        self._inner = inner
        self.drafts = []

    def __getattr__(self, name):
        return getattr(self._inner, name)

    def set_draft(self, rid, toks):
        n = self._inner.num_tokens(rid)
        self.drafts.append((self._inner.tokens_range(rid, 0, n), list(toks)))
        return self._inner.set_draft(rid, toks)


def _run(spec):
    cfg = _cfg()
    prompts = _prompts()
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **KW).generate(prompts, sp)]
    llm = LLM(cfg, speculative_config=spec, **KW)
    rec = _Recorder(llm.engine.scheduler)
    llm.engine.scheduler = rec
    outs = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert outs == plain
    assert rec.drafts and llm.engine.drafter.proposed > 0
    return rec, ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))


def test_eagle3_random_head_matches_reference_drafts():
    rec, ref = _run({"method": "eagle3", "num_speculative_tokens": 1})
    ew = dict(dummy_weights(_cfg(), seed=1, std=0.02, shapes=eagle3_param_shapes(_cfg())))
    for toks, draft in rec.drafts:
        assert draft == [eagle3_draft(ref, ew, toks)]


def test_eagle3_safetensors_reduced_vocab(tmp_path):
    cfg = _cfg()
    g = torch.Generator().manual_seed(11)
    Vd = 300
    ew = {n: (torch.randn(s, generator=g) * 0.05 if k == "w" else
              1.0 + 0.1 * torch.randn(s, generator=g))
          for n, s, k in eagle3_param_shapes(cfg, Vd)}
    # draft id d -> target id d + d2t[d]: a scattered subset of the target vocabulary
    tgt = torch.randperm(cfg.vocab_size, generator=g)[:Vd].sort().values
    ew["d2t"] = tgt - torch.arange(Vd)
    save_safetensors(ew.items(), str(tmp_path))
    rec, ref = _run({"method": "eagle3", "num_speculative_tokens": 1, "model": str(tmp_path)})
    allowed = set(tgt.tolist())
    for toks, draft in rec.drafts:
        assert draft[0] in allowed
        assert draft == [eagle3_draft(ref, ew, toks)]


def test_eagle3_contract():
    with pytest.raises(ValueError):
        LLM(_cfg(), speculative_config={"method": "eagle3", "num_speculative_tokens": 1},
            kv_cache_dtype="fp8", **KW)


def test_eagle3_sibling_tree_matches_plain():
    cfg = _cfg()
    prompts = _prompts()
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **KW).generate(prompts, sp)]
    llm = LLM(cfg, speculative_config={"method": "eagle3", "num_speculative_tokens": 1,
                                       "speculative_token_tree": "[(0,), (1,), (2,)]"}, **KW)
    assert [o.outputs[0].token_ids for o in llm.generate(prompts, sp)] == plain
    assert llm.engine.drafter.proposed > 0


def test_eagle3_chained_drafts_keep_outputs():
    """num_speculative_tokens = 3: the chained steps feed the head's own pre-norm output back
    (3H features only at the first draft); verified outputs equal plain decoding."""
    cfg = _cfg()
    prompts = _prompts()
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **KW).generate(prompts, sp)]
    llm = LLM(cfg, speculative_config={"method": "eagle3", "num_speculative_tokens": 3}, **KW)
    rec = _Recorder(llm.engine.scheduler)
    llm.engine.scheduler = rec
    assert [o.outputs[0].token_ids for o in llm.generate(prompts, sp)] == plain
    assert any(len(d) == 3 for _, d in rec.drafts)
