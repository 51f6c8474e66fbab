"""Priority scheduling (vLLM's scheduling_policy="priority", lower values first): admission
follows (priority, arrival); when blocks run out the running request that sorts last is
preempted; outputs stay those of FCFS scheduling."""
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama


def _prompts(n=4, L=20):
    g = torch.Generator().manual_seed(6)
    return torch.randint(0, 1024, (n, L), generator=g).tolist()


def _llm(policy, **kw):
    a = dict(device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
             max_num_seqs=1, max_num_batched_tokens=256, scheduling_policy=policy)
    a.update(kw)
    return LLM(tiny_llama(), **a)


def test_admission_follows_priority():
    sp = SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True)
    prompts = _prompts()
    prios = [5, 0, 3, 0]
    llm = _llm("priority")
    eng = llm.engine
    for i, (p, pr) in enumerate(zip(prompts, prios)):
        eng.add_request(f"r{i}", p, sp, priority=pr)
    order = []
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                order.append(o.request_id)
    assert order == ["r1", "r3", "r2", "r0"]  # by priority, ties by arrival
    fcfs = [o.outputs[0].token_ids for o in _llm("fcfs").generate(prompts, sp)]
    again = _llm("priority").generate(prompts, sp, priority=prios)
    assert [o.outputs[0].token_ids for o in again] == fcfs


def test_preemption_takes_the_lowest_priority():
    sp = SamplingParams(temperature=0.0, max_tokens=40, ignore_eos=True)
    prompts = _prompts(3, 30)
    kw = dict(max_num_seqs=3, num_gpu_blocks=8)
    fcfs = [o.outputs[0].token_ids for o in _llm("fcfs", **kw).generate(prompts, sp)]
    llm = _llm("priority", **kw)
    eng = llm.engine
    prios = [1, 9, 0]
    for i, (p, pr) in enumerate(zip(prompts, prios)):
        eng.add_request(f"r{i}", p, sp, priority=pr)
    iid = {f"r{i}": eng._by_name[f"r{i}"] for i in range(3)}
    pre = {k: 0 for k in iid}
    outs = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                outs[o.request_id] = o.outputs[0].token_ids
        for k, v in iid.items():
            info = eng.scheduler.request_info(v)
            if info:
                pre[k] = max(pre[k], info["num_preemptions"])
    assert pre["r1"] > 0 and pre["r2"] == 0  # the priority-9 request gives way first
    assert [outs[f"r{i}"] for i in range(3)] == fcfs


def test_tight_pool_never_deadlocks_with_prefix_caching():
    """Regression: a waiting request whose admission fails must not keep the prefix-cache
    blocks it pinned (three preempted requests used to hold the whole pool while nothing ran).
    Bounded step loop: the test fails instead of hanging."""
    sp = SamplingParams(temperature=0.0, max_tokens=40, ignore_eos=True)
    for policy in ("fcfs", "priority"):
        llm = _llm(policy, max_num_seqs=3, num_gpu_blocks=8)
        eng = llm.engine
        for i, p in enumerate(_prompts(3, 30)):
            eng.add_request(f"r{i}", p, sp, priority=i)
        steps = 0
        while eng.has_unfinished_requests():
            eng.step()
            steps += 1
            assert steps < 400, "scheduler made no progress"
            if eng.scheduler.num_running() == 0:
                assert eng.scheduler.num_free_blocks() == 8 or eng.scheduler.num_waiting() == 0
