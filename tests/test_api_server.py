"""OpenAI-compatible server on the tiny CPU model: completions (token ids and text through a
toy tokenizer), streaming, chat, n > 1, stop strings, models / health / metrics."""
import json

import pytest
import torch

from vllm_musa_b200 import LLM
from vllm_musa_b200.engine.async_llm import AsyncLLM
from vllm_musa_b200.entrypoints.openai.api_server import build_app
from vllm_musa_b200.models.presets import tiny_llama


class ToyTokenizer:
    """Byte-level toy tokenizer over the tiny model's 1024-token vocabulary."""
    chat_template = None

    def encode(self, text):
        return [b % 1024 for b in text.encode()]

    def decode(self, ids, skip_special_tokens=True):
        return "".join(chr(32 + (i % 90)) for i in ids)


@pytest.fixture(scope="module")
def client():
    from fastapi.testclient import TestClient
    llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=128,
              max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256,
              tokenizer=ToyTokenizer())
    alm = AsyncLLM(llm.engine)
    app = build_app(alm, "tiny", 256)
    with TestClient(app) as c:
        yield c, llm
    alm.shutdown()


def test_models_health_metrics(client):
    c, _ = client
    assert c.get("/health").status_code == 200
    assert c.get("/v1/models").json()["data"][0]["id"] == "tiny"
    m = c.get("/metrics").text
    for name in ("b200_request_success_total", "b200_kv_cache_usage_perc",
                 "b200_prefix_cache_hits_total", "b200_spec_decode_num_accepted_tokens_total",
                 "b200_engine_steps_total"):
        assert name in m


def test_completion_token_ids_matches_offline(client):
    c, llm = client
    prompt = list(range(10, 40))
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 6, "temperature": 0,
                                        "ignore_eos": True}).json()
    assert r["usage"]["completion_tokens"] == 6
    ref = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
              max_model_len=256, max_num_seqs=4, max_num_batched_tokens=256)
    from vllm_musa_b200 import SamplingParams
    want = ref.generate([prompt], SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
    assert r["choices"][0]["token_ids"] == want[0].outputs[0].token_ids


def test_text_prompt_n2_and_stop(client):
    c, _ = client
    r = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 5, "n": 2,
                                        "temperature": 1.0, "seed": 3, "ignore_eos": True}).json()
    assert len(r["choices"]) == 2 and all(len(ch["text"]) == 5 for ch in r["choices"])
    full = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 8, "temperature": 0,
                                           "ignore_eos": True}).json()["choices"][0]["text"]
    stop = full[3:5]
    r = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 8, "temperature": 0,
                                        "ignore_eos": True, "stop": [stop]}).json()
    assert r["choices"][0]["text"] == full[:full.find(stop)]
    assert r["choices"][0]["finish_reason"] == "stop"


def test_streaming_and_chat(client):
    c, _ = client
    with c.stream("POST", "/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4,
                                                  "temperature": 0, "ignore_eos": True,
                                                  "stream": True}) as r:
        events = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert events[-1] == "data: [DONE]"
    text = "".join(json.loads(e[6:])["choices"][0]["text"] for e in events[:-1])
    assert len(text) == 4
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                             "max_tokens": 3, "temperature": 0,
                                             "ignore_eos": True}).json()
    assert r["choices"][0]["message"]["role"] == "assistant"
    assert r["usage"]["completion_tokens"] == 3


def test_bad_request(client):
    c, _ = client
    r = c.post("/v1/completions", json={"prompt": list(range(300)), "max_tokens": 4})
    assert r.status_code == 400


def test_completion_logits_processors_and_prompt_logprobs(client):
    """logit_bias (string keys, OpenAI), allowed_token_ids and prompt_logprobs through the
    server: a +100 bias wins every step, allowed ids bound the output, prompt_logprobs lists
    None then one entry per later prompt token."""
    c, _ = client
    prompt = list(range(50, 70))
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 4, "temperature": 0,
                                        "ignore_eos": True, "logit_bias": {"321": 100}}).json()
    assert r["choices"][0]["token_ids"] == [321] * 4
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 5, "temperature": 0.9,
                                        "ignore_eos": True, "allowed_token_ids": [7, 8, 9],
                                        "prompt_logprobs": 1}).json()
    ch = r["choices"][0]
    assert set(ch["token_ids"]) <= {7, 8, 9}
    plp = ch["prompt_logprobs"]
    assert len(plp) == len(prompt) and plp[0] is None
    assert all(str(t) in d for t, d in zip(prompt[1:], plp[1:]))
    bad = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 2,
                                          "logit_bias": {"5000": 1}})
    assert bad.status_code == 400


def test_engine_failure_reports_dead():
    """A step that raises stops the engine loop: open and later requests fail (HTTP 500 / 503
    style errors instead of hanging) and /health answers 503."""
    from fastapi.testclient import TestClient
    llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
              max_model_len=256, max_num_seqs=4, max_num_batched_tokens=256)
    alm = AsyncLLM(llm.engine)

    def boom():
        raise RuntimeError("injected step failure")

    llm.engine.step = boom
    app = build_app(alm, "tiny", 256)
    with TestClient(app, raise_server_exceptions=False) as c:
        r = c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 2})
        assert r.status_code >= 500
        assert c.get("/health").status_code == 503
        r2 = c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 2})
        assert r2.status_code >= 500
    alm._stop = True


def test_streaming_with_speculation_and_usage():
    """Streaming under n-gram speculation: a step can add several tokens and every one of
    them reaches a chunk; stream_options.include_usage adds the final usage chunk."""
    from fastapi.testclient import TestClient
    llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=128,
              max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256,
              tokenizer=ToyTokenizer(),
              speculative_config={"method": "ngram", "num_speculative_tokens": 4})
    alm = AsyncLLM(llm.engine)
    app = build_app(alm, "tiny", 256)
    g = torch.Generator().manual_seed(5)
    base = torch.randint(0, 1024, (12,), generator=g).tolist()
    prompt = (base * 4)[:40]
    try:
        with TestClient(app) as c:
            full = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 16,
                                                   "temperature": 0, "ignore_eos": True}).json()
            with c.stream("POST", "/v1/completions",
                          json={"prompt": prompt, "max_tokens": 16, "temperature": 0,
                                "ignore_eos": True, "stream": True,
                                "stream_options": {"include_usage": True}}) as r:
                events = [json.loads(l[6:]) for l in r.iter_lines()
                          if l.startswith("data: ") and l != "data: [DONE]"]
        ids = [t for e in events if e["choices"] for t in e["choices"][0]["token_ids"]]
        assert ids == full["choices"][0]["token_ids"]
        assert events[-1]["choices"] == [] and events[-1]["usage"]["completion_tokens"] == 16
        assert llm.engine.scheduler.spec_accepted() > 0
    finally:
        alm.shutdown()
