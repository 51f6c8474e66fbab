"""Debug bounds checks (B200_DEBUG_BOUNDS): with the checks on, index tensors outside what a
kernel assumes raise IndexError at the op boundary (before any kernel runs); a whole engine
run passes them; off, nothing is checked."""
import pytest
import torch

from vllm_musa_b200 import LLM, SamplingParams, ops
from vllm_musa_b200.models.presets import tiny_llama
from vllm_musa_b200.ops import _bounds


@pytest.fixture
def bounds_on():
    _bounds.set_enabled(True)
    yield
    _bounds.set_enabled(False)


def test_bad_indices_raise(bounds_on):
    kc = torch.zeros(4, 2, 16, 64)
    vc = torch.zeros_like(kc)
    kv = torch.randn(3, 2, 64)
    ops.attention.kv_insert(kv, kv, kc, vc, torch.tensor([0, -1, 63]))  # in range / skipped
    with pytest.raises(IndexError, match="kv_insert: slot_mapping holds 64"):
        ops.attention.kv_insert(kv, kv, kc, vc, torch.tensor([0, 5, 64]))
    q = torch.randn(2, 4 * 64)
    bt = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32)
    ops.paged_decode(q, kc, vc, bt, torch.tensor([20, 5], dtype=torch.int32), 4, 2, 0.125, 32)
    with pytest.raises(IndexError, match="block_tables holds 9"):
        ops.paged_decode(q, kc, vc, torch.tensor([[0, 9], [2, 3]], dtype=torch.int32),
                         torch.tensor([20, 5], dtype=torch.int32), 4, 2, 0.125, 32)
    # a page past the sequence's length is never read, so it is not checked
    ops.paged_decode(q, kc, vc, torch.tensor([[0, 9], [2, 3]], dtype=torch.int32),
                     torch.tensor([16, 5], dtype=torch.int32), 4, 2, 0.125, 32)
    with pytest.raises(IndexError, match="seq_lens holds 40"):
        ops.paged_decode(q, kc, vc, bt, torch.tensor([40, 5], dtype=torch.int32), 4, 2, 0.125, 64)
    with pytest.raises(IndexError, match="gather_rows: idx holds 7"):
        ops.gather_rows(torch.randn(7, 8), torch.tensor([1, 7], dtype=torch.int32))


def test_engine_run_passes_checks(bounds_on):
    llm = LLM(tiny_llama(), device="cpu", block_size=16, seed=0, num_gpu_blocks=32,
              max_model_len=128, max_num_seqs=4, max_num_batched_tokens=64)
    outs = llm.generate([[1, 2, 3, 4] * 5, [9] * 30],
                        SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True))
    assert all(len(o.outputs[0].token_ids) == 5 for o in outs)


def test_checks_off_by_default():
    assert not _bounds.enabled()
    _bounds.check("op", "x", torch.tensor([10**9]), 1)  # no-op when off
