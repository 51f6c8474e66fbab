"""Tensor parallelism on CPU Gloo ranks: TP=2 shards (heads, intermediate, vocab), the
all-reduce + fused norm path and the vocab-parallel sampler must reproduce TP=1 outputs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model(name):
    if name == "tiny-llama":
        from vllm_musa_b200.models.presets import tiny_llama
        return tiny_llama()
    if name == "tiny-moe":
        from test_moe_cpu import tiny_moe
        return tiny_moe(shared=64)
    if name in ("tiny-ds-dense", "tiny-ds-nomoe"):
        from test_deepseek_cpu import tiny_ds
        c = tiny_ds(sparse=False)
        if name == "tiny-ds-nomoe":
            c.first_k_dense = c.num_layers  # every layer a dense MLP: no expert routing
        return c
    from test_qwen3_next_cpu import tiny_next
    return tiny_next()


def _worker(rank, world, port, q, temperature, model="tiny-llama", ep=False, dcp=1, dp=1,
            pp=1, spec=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.parallel.state import destroy_distributed
    cfg = _model(model)
    llm = LLM(cfg, device="cpu", tensor_parallel_size=world // (dp * pp),
              pipeline_parallel_size=pp, data_parallel_size=dp,
              block_size=16, seed=0,
              num_gpu_blocks=64, max_model_len=128, max_num_seqs=4, max_num_batched_tokens=64,
              enable_expert_parallel=ep, decode_context_parallel_size=dcp,
              speculative_config=spec)
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, min(1024, cfg.vocab_size), (3, 20), generator=g).tolist()
    outs = llm.generate(prompts, SamplingParams(temperature=temperature, max_tokens=8,
                                                ignore_eos=True, seed=7 if temperature else None))
    if pp > 1:  # this rank holds only its stage's layers and cache
        m = llm.engine.model
        assert m.l1 - m.l0 < cfg.num_layers
        assert len(llm.engine.runner.kv_caches) == m.l1 - m.l0
        assert (m.embed is not None) == (m.l0 == 0)
    if spec is not None and spec.get("method") == "eagle":
        head = llm.engine.model.draft_head
        assert llm.engine.drafter.proposed > 0
        assert head.replicated == (spec.get("draft_tensor_parallel_size") == 1 and world > 1)
        if head.replicated:  # whole head, own cache with every KV head
            assert head.own_kv[0].shape[1] == cfg.num_kv_heads
            assert len(llm.engine.runner.kv_caches) == cfg.num_layers
    q.put((rank, [o.outputs[0].token_ids for o in outs]))
    destroy_distributed()


def _run(world, temperature=0.0, model="tiny-llama", ep=False, dcp=1, dp=1, pp=1, spec=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker,
                         args=(r, world, port, q, temperature, model, ep, dcp, dp, pp, spec))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_tp2_greedy_matches_tp1():
    one = _run(1)[0]
    two = _run(2)
    assert two[0] == two[1], "ranks diverged"
    assert two[0] == one


@pytest.mark.parametrize("model,ep", [("tiny-moe", False), ("tiny-moe", True),
                                      ("tiny-next", False), ("tiny-next", True)])
def test_tp2_moe_and_hybrid_match_tp1(model, ep):
    """TP=2 attention with tensor-sharded experts, or with expert parallelism (each rank keeps
    half of the experts whole), reproduces the single-rank tokens."""
    one = _run(1, model=model)[0]
    two = _run(2, model=model, ep=ep)
    assert two[0] == two[1], "ranks diverged"
    assert two[0] == one


def test_tp2_spawned_followers_match_tp1():
    """LLM(tensor_parallel_size=2) without a launcher: the driver spawns a follower rank and
    broadcasts request operations each step."""
    import subprocess
    import sys
    code = r'''
import torch, os
torch.set_num_threads(1)
from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama
llm = LLM(tiny_llama(), device="cpu", tensor_parallel_size=2, block_size=16, seed=0,
          num_gpu_blocks=64, max_model_len=128, max_num_seqs=4, max_num_batched_tokens=64)
g = torch.Generator().manual_seed(0)
prompts = torch.randint(0, 1024, (3, 20), generator=g).tolist()
outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
print("TOKENS", [o.outputs[0].token_ids for o in outs])
outs2 = llm.generate(prompts[:1], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))
print("TOKENS2", [o.outputs[0].token_ids for o in outs2])
# a request the driver rejects never reaches the follower (ids stay in lock-step)
try:
    llm.generate(prompts[:1], SamplingParams(max_tokens=2, logit_bias={5000: 1.0}))
except ValueError:
    print("REJECTED")
outs3 = llm.generate(prompts[:1], SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))
print("TOKENS3", [o.outputs[0].token_ids for o in outs3])
llm.shutdown()
'''
    env = dict(os.environ)
    env.pop("WORLD_SIZE", None)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       env=env, cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr[-4000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("TOKENS ")][0]
    toks = eval(line[len("TOKENS "):])
    one = _run(1)[0]
    assert toks == one
    line2 = [l for l in r.stdout.splitlines() if l.startswith("TOKENS2 ")][0]
    assert eval(line2[len("TOKENS2 "):])[0] == one[0][:4]
    assert "REJECTED" in r.stdout
    line3 = [l for l in r.stdout.splitlines() if l.startswith("TOKENS3 ")][0]
    assert eval(line3[len("TOKENS3 "):])[0] == one[0][:4]


@pytest.mark.parametrize("dcp", [1, 2])
def test_tp2_deepseek_mla_matches_tp1(dcp):
    """DeepSeek MLA at TP=2 (vocab-sharded head: the sampler offsets each rank's candidates by
    its vocab start) reproduces TP=1; with decode context parallelism (dcp=2) the latent cache
    is sharded by token over the two ranks (every rank attends all heads over its tokens, then
    an LSE-weighted reduce-scatter of the partials), through chunked prefill and decode."""
    one = _run(1, model="tiny-ds-dense")[0]
    two = _run(2, model="tiny-ds-dense", dcp=dcp)
    assert two[0] == two[1], "ranks diverged"
    assert two[0] == one


@pytest.mark.parametrize("world,dp", [(2, 2), (4, 2)])
def test_data_parallel_replicas_match_single(world, dp):
    """Data parallelism: dp engine replicas (each TP = world / dp) split the prompts and every
    rank returns all outputs in prompt order, equal to the single-engine run."""
    one = _run(1, temperature=0.7)[0]
    res = _run(world, temperature=0.7, dp=dp)
    for r in range(world):
        assert res[r] == one


@pytest.mark.parametrize("world,pp,model", [(2, 2, "tiny-llama"), (4, 2, "tiny-llama"),
                                            (2, 2, "tiny-moe")])
def test_pipeline_parallel_matches_single(world, pp, model):
    """Pipeline stages (layers split across ranks, micro-batched residual hand-off, tokens
    broadcast from the last stage), alone and combined with TP=2, reproduce one process:
    greedy and seeded sampling."""
    for temperature in (0.0, 0.8):
        one = _run(1, temperature, model)[0]
        got = _run(world, temperature, model, pp=pp)
        assert all(got[r] == got[0] for r in got), "ranks diverged"
        assert got[0] == one


@pytest.mark.parametrize("draft_tp", [None, 1])
def test_tp2_eagle_drafts_match_tp1(draft_tp):
    """EAGLE under TP=2 with the head sharded like the target, or whole on every rank
    (draft_tensor_parallel_size=1: no collectives in the draft layer, its own all-head cache):
    the verified tokens equal plain TP=1 decoding and both ranks stay in lock-step."""
    plain = _run(1)[0]
    spec = {"method": "eagle", "num_speculative_tokens": 1}
    if draft_tp is not None:
        spec["draft_tensor_parallel_size"] = draft_tp
    two = _run(2, spec=spec)
    assert two[0] == two[1], "ranks diverged"
    assert two[0] == plain
