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
