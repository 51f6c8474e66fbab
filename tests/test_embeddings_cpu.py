"""Embeddings (PoolingParams: last / mean / cls pooling, L2 normalisation, Matryoshka
truncation) through LLM.embed, against the pure-PyTorch reference decoder's final hidden
states; with chunked prefill and a cached prefix; and through the server's /v1/embeddings,
/tokenize and /detokenize."""
import pytest
import torch

from vllm_musa_b200 import LLM
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights
from vllm_musa_b200.sample.sampling_params import PoolingParams


def _llm(budget=256, **kw):
    return LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=128,
               max_model_len=128, max_num_seqs=8, max_num_batched_tokens=budget, **kw)


def _prompts():
    g = torch.Generator().manual_seed(8)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (9, 40, 70)]


@pytest.mark.parametrize("budget", [256, 16])
def test_embed_matches_reference_hidden(budget):
    cfg = tiny_llama()
    ref = ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))
    prompts = _prompts()
    llm = _llm(budget)
    llm.embed(prompts[1][:33])  # caches a prefix of prompt 1
    for kind in ("last", "mean", "cls"):
        outs = llm.embed(prompts, PoolingParams(pooling_type=kind))
        for p, o in zip(prompts, outs):
            hid = ref.hidden(p)  # final (normalised) hidden states [n, H]
            v = {"last": hid[-1], "mean": hid.mean(0), "cls": hid[0]}[kind]
            v = v / v.norm()
            got = torch.tensor(o.outputs.embedding)
            torch.testing.assert_close(got, v, rtol=1e-4, atol=1e-5)
    raw = llm.embed(prompts[0], PoolingParams(normalize=False, dimensions=16))[0]
    assert len(raw.outputs.embedding) == 16
    torch.testing.assert_close(torch.tensor(raw.outputs.embedding), ref.hidden(prompts[0])[-1][:16],
                               rtol=1e-4, atol=1e-5)


def test_embeddings_endpoint():
    from fastapi.testclient import TestClient

    from vllm_musa_b200.engine.async_llm import AsyncLLM
    from vllm_musa_b200.entrypoints.openai.api_server import build_app

    class Tok:
        chat_template = None

        def encode(self, s):
            return [ord(c) % 1000 + 3 for c in s]

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr((i - 3) % 1000) for i in ids)

    llm = _llm(tokenizer=Tok())
    alm = AsyncLLM(llm.engine)
    app = build_app(alm, "tiny", 128)
    try:
        with TestClient(app) as c:
            r = c.post("/v1/embeddings", json={"input": ["hello", "world!"]}).json()
            assert [d["index"] for d in r["data"]] == [0, 1]
            want = _llm().embed([Tok().encode("hello"), Tok().encode("world!")])
            for d, w in zip(r["data"], want):
                torch.testing.assert_close(torch.tensor(d["embedding"]),
                                           torch.tensor(w.outputs.embedding))
            assert r["usage"]["prompt_tokens"] == 11
            t = c.post("/tokenize", json={"prompt": "abc"}).json()
            assert t["tokens"] == Tok().encode("abc") and t["count"] == 3
            assert c.post("/detokenize", json={"tokens": t["tokens"]}).json()["prompt"] == "abc"
            assert c.post("/v1/embeddings", json={"input": "x" * 200}).status_code == 400
    finally:
        alm.shutdown()
