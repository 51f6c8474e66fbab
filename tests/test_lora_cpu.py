"""Multi-LoRA serving on the tiny CPU Llama: a batch mixing two PEFT adapters (rank 8 and 4,
every linear targeted) and the base model gives, per request, the greedy tokens of the
pure-PyTorch reference decoder run on the merged weights W + (alpha / r) B A; also under TP=2
(gloo) and PP=2, and adapters are evicted / reloaded by slot."""
import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.lora import LoRARequest
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.models.reference import ReferenceDecoder
from vllm_musa_b200.models.weights import dummy_weights

MODS = {"q": "self_attn", "k": "self_attn", "v": "self_attn", "o": "self_attn",
        "gate": "mlp", "up": "mlp", "down": "mlp"}


def make_adapter(path, cfg, r, alpha, seed):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    H, D = cfg.hidden_size, cfg.head_dim
    dims = {"q": (cfg.num_heads * D, H), "k": (cfg.num_kv_heads * D, H),
            "v": (cfg.num_kv_heads * D, H), "o": (H, cfg.num_heads * D),
            "gate": (cfg.intermediate_size, H), "up": (cfg.intermediate_size, H),
            "down": (H, cfg.intermediate_size)}
    t = {}
    for i in range(cfg.num_layers):
        for m, blk in MODS.items():
            N, K = dims[m]
            pre = f"base_model.model.model.layers.{i}.{blk}.{m}_proj."
            t[pre + "lora_A.weight"] = torch.randn(r, K, generator=g) * 0.05
            t[pre + "lora_B.weight"] = torch.randn(N, r, generator=g) * 0.05
    os.makedirs(path, exist_ok=True)
    save_file(t, os.path.join(path, "adapter_model.safetensors"))
    with open(os.path.join(path, "adapter_config.json"), "w") as f:
        json.dump({"r": r, "lora_alpha": alpha, "target_modules": [m + "_proj" for m in MODS]}, f)
    return t


def merged_reference(cfg, tensors, r, alpha):
    w = dict(dummy_weights(cfg, seed=0, std=0.02))
    for name, a in tensors.items():
        if not name.endswith("lora_A.weight"):
            continue
        b = tensors[name.replace("lora_A", "lora_B")]
        key = name.replace("base_model.model.", "").replace(".lora_A.weight", ".weight")
        w[key] = (w[key].float() + (alpha / r) * b @ a).to(w[key].dtype)
    return ReferenceDecoder(cfg, w)


KW = dict(device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
          max_num_seqs=8, max_num_batched_tokens=64, enable_lora=True, max_loras=2,
          max_lora_rank=16)


def _prompts():
    g = torch.Generator().manual_seed(4)
    return [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (21, 9, 40, 13)]


def _expected(tmp):
    cfg = tiny_llama()
    ta = make_adapter(os.path.join(tmp, "a"), cfg, 8, 16, 1)
    tb = make_adapter(os.path.join(tmp, "b"), cfg, 4, 4, 2)
    refs = [merged_reference(cfg, ta, 8, 16), merged_reference(cfg, tb, 4, 4),
            ReferenceDecoder(cfg, dict(dummy_weights(cfg, seed=0, std=0.02)))]
    la = LoRARequest("a", 1, os.path.join(tmp, "a"))
    lb = LoRARequest("b", 2, os.path.join(tmp, "b"))
    which = [0, 1, 2, 0]  # adapter a, adapter b, base, adapter a
    loras = [[la, lb, None][k] for k in which]
    want = [refs[k].greedy(p, 6)[0] for k, p in zip(which, _prompts())]
    return cfg, loras, want


def test_lora_mixed_batch_matches_merged_reference(tmp_path):
    cfg, loras, want = _expected(str(tmp_path))
    llm = LLM(cfg, **KW)
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    got = [o.outputs[0].token_ids for o in llm.generate(_prompts(), sp, lora_request=loras)]
    assert got == want
    # a third adapter evicts the least recently used idle one; reloading a works again
    cfg2 = tiny_llama()
    make_adapter(str(tmp_path / "c"), cfg2, 8, 8, 3)
    lc = LoRARequest("c", 3, str(tmp_path / "c"))
    llm.generate(_prompts()[:1], sp, lora_request=lc)
    again = llm.generate(_prompts()[:1], sp, lora_request=loras[0])
    assert again[0].outputs[0].token_ids == want[0]
    with pytest.raises(ValueError):
        LLM(cfg, **{**KW, "enable_lora": False}).generate(_prompts()[:1], sp,
                                                          lora_request=loras[0])


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, tmp, tp, pp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    from vllm_musa_b200.parallel.state import destroy_distributed
    cfg, loras, want = _expected(tmp)
    llm = LLM(cfg, tensor_parallel_size=tp, pipeline_parallel_size=pp, **KW)
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    got = [o.outputs[0].token_ids for o in llm.generate(_prompts(), sp, lora_request=loras)]
    q.put((rank, got == want))
    destroy_distributed()


@pytest.mark.parametrize("tp,pp", [(2, 1), (1, 2)])
def test_lora_tensor_and_pipeline_parallel(tmp_path, tp, pp):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = tp * pp
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, str(tmp_path), tp, pp))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(res.values())


def test_lora_through_openai_server(tmp_path):
    """An adapter served under its own model name (--lora-modules name=path)."""
    from fastapi.testclient import TestClient
    from vllm_musa_b200.engine.async_llm import AsyncLLM
    from vllm_musa_b200.entrypoints.openai.api_server import build_app, parse_lora_modules
    cfg, loras, want = _expected(str(tmp_path))
    llm = LLM(cfg, **KW)
    mods = parse_lora_modules([f"ad={loras[0].lora_path}"])
    alm = AsyncLLM(llm.engine)
    app = build_app(alm, "tiny", 128, mods)
    try:
        with TestClient(app) as c:
            names = [m["id"] for m in c.get("/v1/models").json()["data"]]
            assert names == ["tiny", "ad"]
            body = {"prompt": _prompts()[0], "max_tokens": 6, "temperature": 0,
                    "ignore_eos": True}
            r = c.post("/v1/completions", json={**body, "model": "ad"}).json()
            assert r["choices"][0]["token_ids"] == want[0]
            base = c.post("/v1/completions", json={**body, "model": "tiny"}).json()
            assert base["choices"][0]["token_ids"] != want[0]
            assert c.post("/v1/completions", json={**body, "model": "nope"}).status_code == 400
    finally:
        alm.shutdown()
