"""MoE shape inventory and dispatch counters on the tiny CPU Qwen3-MoE: every eager MoE call is
counted on its path, the JSON-lines inventory holds one record per recorded call with the
layer's shape, and its routed-token histogram sums to tokens x top-k and equals a bincount of
the router's own top-k over the same hidden states."""
import json

import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.config import ModelConfig
from vllm_musa_b200.ops import moe as moe_ops
from vllm_musa_b200.utils import moe_inventory


def tiny_moe():
    return ModelConfig(arch="qwen3_moe", vocab_size=512, hidden_size=128, num_layers=2,
                       num_heads=4, num_kv_heads=2, head_dim=64, intermediate_size=256,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=512, qk_norm=True,
                       num_experts=8, num_experts_per_tok=2, moe_intermediate_size=64,
                       dtype=torch.float32, name="tiny-moe")


def _run(monkeypatch, tmp_path, **env):
    dest = tmp_path / "inv" / "moe.jsonl"
    monkeypatch.setenv("B200_MOE_SHAPE_INVENTORY", str(dest))
    for k, v in env.items():
        monkeypatch.setenv(k, str(v))
    moe_inventory.reset()
    cfg = tiny_moe()
    llm = LLM(cfg, device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
              max_num_seqs=4, max_num_batched_tokens=128)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (20, 9)]
    llm.generate(prompts, SamplingParams(temperature=0, max_tokens=3, ignore_eos=True))
    lines = dest.read_text().splitlines() if dest.exists() else []
    return cfg, [json.loads(l) for l in lines]


def test_inventory_records_shapes_and_histograms(monkeypatch, tmp_path):
    cfg, recs = _run(monkeypatch, tmp_path, B200_MOE_SHAPE_INVENTORY_MAX_RECORDS=-1)
    counts = moe_inventory.dispatch_counts()
    assert counts.get("cpu", 0) == len(recs) > 0
    assert [r["record_index"] for r in recs] == list(range(len(recs)))
    for r in recs:
        st = r["routed_token_stats"]
        assert r["path"] == "cpu" and r["hidden_size"] == cfg.hidden_size
        assert r["top_k"] == cfg.num_experts_per_tok
        assert r["num_local_experts"] == cfg.num_experts
        assert sum(st["histogram"]) == r["num_tokens"] * r["top_k"]
        assert [sum(c) for c in zip(*st["slot_histograms"])] == st["histogram"]
        assert st["outside_count"] == 0
        assert st["nonzero_experts"] == sum(1 for c in st["histogram"] if c)
    # the prefill step routes both prompts' tokens (29) through every MoE layer
    assert max(r["num_tokens"] for r in recs) == 29


def test_inventory_limits(monkeypatch, tmp_path):
    _, recs = _run(monkeypatch, tmp_path, B200_MOE_SHAPE_INVENTORY_MAX_RECORDS=3)
    assert len(recs) == 3
    _, recs = _run(monkeypatch, tmp_path / "b", B200_MOE_SHAPE_INVENTORY_MIN_TOKENS=10)
    assert recs and all(r["num_tokens"] >= 10 for r in recs)


def test_histogram_matches_router_and_offsets():
    g = torch.Generator().manual_seed(0)
    ids, _ = moe_ops.topk_softmax(torch.randn(40, 16, generator=g), 4)
    st = moe_inventory.routed_histogram(ids, 16)
    assert st["histogram"] == torch.bincount(ids.flatten().long(), minlength=16).tolist()
    # this rank holds experts [8, 16): the other half is counted as outside
    half = moe_inventory.routed_histogram(ids, 8, expert_offset=8)
    assert half["histogram"] == st["histogram"][8:]
    assert half["outside_count"] == sum(st["histogram"][:8])
