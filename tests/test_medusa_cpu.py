"""Medusa heads on the tiny CPU Llama: chained and tree drafts keep plain greedy outputs, and
every chain equals the pure-PyTorch heads (residual SiLU block + LM head per head) applied to
the reference decoder's final hidden state; a checkpoint without LM heads shares the target's
LM head."""
import torch
import torch.nn.functional as F

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.medusa import medusa_param_shapes
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights, save_safetensors

KW = dict(device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
          max_num_seqs=4, max_num_batched_tokens=64)


def _prompts():
    g = torch.Generator().manual_seed(17)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (19, 33, 8)]


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


def _ref_chain(ref, mw, tokens, k, shared=None):
    h = ref.hidden(tokens)[len(tokens) - 2]
    out = []
    for i in range(k):
        p = f"blocks.{i}.layers.0."
        r = h + F.silu(h @ mw[p + "weight"].float().t() + mw[p + "bias"].float())
        lm = mw.get(f"lm_heads.{i}.weight", shared).float()
        out.append(int(torch.argmax(r @ lm.t())))
    return out


def _run(spec):
    cfg = tiny_llama()
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **KW).generate(_prompts(), sp)]
    llm = LLM(cfg, speculative_config=spec, **KW)
    rec = _Recorder(llm.engine.scheduler)
    llm.engine.scheduler = rec
    assert [o.outputs[0].token_ids for o in llm.generate(_prompts(), sp)] == plain
    assert llm.engine.drafter.proposed > 0
    return rec, ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))


def test_medusa_chain_matches_reference_heads():
    rec, ref = _run({"method": "medusa", "num_speculative_tokens": 3})
    mw = dict(dummy_weights(tiny_llama(), seed=1, std=0.02,
                            shapes=medusa_param_shapes(tiny_llama(), 3)))
    assert rec.drafts
    for toks, d in rec.drafts:
        assert d == _ref_chain(ref, mw, toks, 3)


def test_medusa_tree_keeps_outputs():
    rec, _ = _run({"method": "medusa", "num_speculative_tokens": 6, "tree_width": 2})
    assert rec.spec_proposed() > 0


def test_medusa_checkpoint_sharing_the_target_head(tmp_path):
    cfg = tiny_llama()
    g = torch.Generator().manual_seed(2)
    mw = {n: torch.randn(s, generator=g) * 0.05 for n, s, k in medusa_param_shapes(cfg, 2)
          if not n.startswith("lm_heads")}
    save_safetensors(mw.items(), str(tmp_path))
    rec, ref = _run({"method": "medusa", "num_speculative_tokens": 2, "model": str(tmp_path)})
    head = ref.w.get("lm_head.weight", ref.w["model.embed_tokens.weight"])
    for toks, d in rec.drafts:
        assert d == _ref_chain(ref, mw, toks, 2, shared=head)
