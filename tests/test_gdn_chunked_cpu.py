"""The chunked (matrix-form) gated delta rule equals the token recurrence: the algorithm the
chunked prefill kernels implement, checked on CPU with state carry and ragged chunks."""
import torch

from vllm_musa_b200.ops import gdn


def _inputs(T, Hk, Hv, seed):
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(T, 2 * Hk * 128 + Hv * 128, generator=g)).to(torch.bfloat16)
    ba = torch.randn(T, 2 * Hv, generator=g).to(torch.bfloat16)
    A_log = torch.randn(Hv, generator=g) * 0.5
    dt_bias = torch.randn(Hv, generator=g) * 0.5
    return qkv, ba, A_log, dt_bias


def test_chunked_matches_recurrent_with_state_carry():
    Hk, Hv = 2, 4
    lens = [70, 1, 130, 64]
    ctx = [0, 5, 40, 0]           # tokens already processed (state slot carries them)
    T = sum(lens)
    qkv, ba, A_log, dt_bias = _inputs(T, Hk, Hv, 0)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0)), dtype=torch.int32)
    sl = torch.tensor([c + n for c, n in zip(ctx, lens)], dtype=torch.int32)
    slots = torch.tensor([3, 0, 2, 1], dtype=torch.int32)
    g = torch.Generator().manual_seed(9)
    st0 = torch.randn(4, Hv, 128, 128, generator=g) * 0.1
    s1, s2 = st0.clone(), st0.clone()
    ref = gdn.gdn_recurrent(qkv, ba, A_log, dt_bias, s1, cu, sl, slots, Hk, Hv)
    got = gdn.gdn_chunked_ref(qkv, ba, A_log, dt_bias, s2, cu, sl, slots, Hk, Hv, chunk=64)
    torch.testing.assert_close(got.float(), ref.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(s2, s1, rtol=1e-3, atol=1e-3)
