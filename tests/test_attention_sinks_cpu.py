"""Attention sinks and non-causal / encoder attention on CPU: the restatements against direct
softmax formulas written independently."""
import math

import torch

from vllm_musa_b200 import ops
from vllm_musa_b200.attention import MMEncoderAttention


def test_sink_is_a_valueless_softmax_column():
    g = torch.Generator().manual_seed(0)
    Hq, Hkv, D, n = 4, 2, 64, 9
    q = torch.randn(1, Hq, D, generator=g)
    k = torch.randn(n, Hkv, D, generator=g)
    v = torch.randn(n, Hkv, D, generator=g)
    sinks = torch.tensor([0.0, 1.5, -2.0, 3.0])
    got = ops.attention._attend_ref(q, k, v, torch.tensor([n - 1]), 0.125, 0, sinks)
    for h in range(Hq):
        kv = h // (Hq // Hkv)
        s = (k[:, kv] @ q[0, h]) * 0.125
        e = torch.exp(s - s.max())
        den = e.sum() + torch.exp(sinks[h] - s.max())
        want = (e[:, None] * v[:, kv]).sum(0) / den
        torch.testing.assert_close(got[0, h], want, rtol=1e-5, atol=1e-5)
    # a very negative sink is no sink
    none = ops.attention._attend_ref(q, k, v, torch.tensor([n - 1]), 0.125, 0, None)
    far = ops.attention._attend_ref(q, k, v, torch.tensor([n - 1]), 0.125, 0,
                                    torch.full((Hq,), -1e4))
    torch.testing.assert_close(far, none)


def test_encoder_attention_is_bidirectional_per_sequence():
    g = torch.Generator().manual_seed(1)
    H, D = 2, 64
    lens = [5, 1, 12]
    T = sum(lens)
    q, k, v = (torch.randn(T, H * D, generator=g) for _ in range(3))
    cu = torch.tensor([0, 5, 6, 18], dtype=torch.int32)
    out = MMEncoderAttention(H, D).forward(q, k, v, cu)
    for a, b in ((0, 5), (5, 6), (6, 18)):
        for h in range(H):
            qs, ks, vs = (x[a:b, h * D:(h + 1) * D] for x in (q, k, v))
            p = torch.softmax(qs @ ks.T / math.sqrt(D), -1)
            torch.testing.assert_close(out[a:b, h * D:(h + 1) * D], p @ vs, rtol=1e-4, atol=1e-5)
