"""Sleep mode (weights offloaded or discarded, KV cache released, then restored) and the
profiler hooks, on the tiny CPU Llama: outputs after waking equal those before sleeping."""
import os

import pytest
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama


def _llm():
    return LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=64,
               max_model_len=128, max_num_seqs=4, max_num_batched_tokens=256)


def _gen(llm):
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, 1024, (3, 24), generator=g).tolist()
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))
    return [o.outputs[0].token_ids for o in outs]


@pytest.mark.parametrize("level", [1, 2])
def test_sleep_wake_up_round_trip(level):
    llm = _llm()
    before = _gen(llm)
    eng = llm.engine
    held = sum(t.numel() for t in eng._weight_tensors())
    assert held > 0
    llm.sleep(level)
    assert eng.sleep_level == level
    assert sum(t.numel() for t in eng._weight_tensors()) == 0  # every weight released
    assert eng.runner.kv_caches == []
    llm.wake_up()
    assert eng.sleep_level == 0
    assert sum(t.numel() for t in eng._weight_tensors()) == held
    assert _gen(llm) == before


def test_sleep_refuses_bad_level():
    llm = _llm()
    with pytest.raises(ValueError):
        llm.sleep(3)


def test_profiler_writes_trace(tmp_path, monkeypatch):
    monkeypatch.setenv("B200_TORCH_PROFILER_DIR", str(tmp_path))
    llm = _llm()
    llm.start_profile()
    _gen(llm)
    path = llm.stop_profile()
    assert path and os.path.exists(path) and os.path.getsize(path) > 0
    assert llm.stop_profile() is None


def test_sleep_keeps_shared_storage_aliased():
    """Views that share one storage (a fused weight and a slice of it held as another
    attribute) are offloaded once and come back as views of one restored storage."""
    llm = _llm()
    before = _gen(llm)
    eng = llm.engine
    L = eng.model.layers[0]
    L.extra = L.qkv_w[8:24]
    ref = L.extra.clone()
    llm.sleep(1)
    assert L.qkv_w.numel() == 0 and L.extra.numel() == 0
    llm.wake_up()
    assert L.extra.untyped_storage().data_ptr() == L.qkv_w.untyped_storage().data_ptr()
    assert torch.equal(L.extra, ref)
    L.qkv_w[8].add_(1.0)  # an in-place update through one view reaches the other
    assert torch.equal(L.extra[0], ref[0] + 1.0)
    L.qkv_w[8].sub_(1.0)
    assert _gen(llm) == before


def test_sleep_wake_with_spawned_follower_ranks():
    """LLM(tensor_parallel_size=2) without a launcher: sleep() / wake_up() on the driver are
    forwarded to the follower rank (both release and restore their shards), and the outputs
    after waking equal those before sleeping, at both sleep levels."""
    import subprocess
    import sys
    code = r'''
import torch
torch.set_num_threads(1)
from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama
llm = LLM(tiny_llama(), device="cpu", tensor_parallel_size=2, block_size=16, seed=0,
          num_gpu_blocks=64, max_model_len=128, max_num_seqs=4, max_num_batched_tokens=64)
g = torch.Generator().manual_seed(0)
prompts = torch.randint(0, 1024, (3, 20), generator=g).tolist()
sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
def gen():
    return [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
a = gen()
llm.sleep(1); llm.wake_up(); b = gen()
llm.sleep(2); llm.wake_up(); c = gen()
print("SAME", a == b == c)
llm.shutdown()
'''
    env = dict(os.environ)
    env.pop("WORLD_SIZE", None)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                       env=env, cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr[-4000:]
    assert "SAME True" in r.stdout, r.stdout[-2000:]
