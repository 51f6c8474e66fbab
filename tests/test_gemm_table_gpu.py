"""Every plan of the measured GEMM table (vllm_musa_b200/tuning/gemm_bf16.json) against the
fp32 product: for each tuned (N, K) and each measured M bucket, the bucket's own M and an M
just inside it (not a multiple of 8, so the non-swapped path runs too) go through
``ops.linear`` -- and, for the fused gate/up shapes, ``ops.linear_silu_mul`` -- with whatever
plan the table picks (one-CTA, CTA-pair, cluster split-K, swapped)."""
import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _table():
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with open(os.path.join(here, "vllm_musa_b200", "tuning", "gemm_bf16.json")) as f:
        return json.load(f)["entries"]


def _cases():
    by_nk = {}
    for e in _table():
        by_nk.setdefault((e["n"], e["k"]), set()).add(e["m"])
    out = []
    for (n, k), ms in sorted(by_nk.items()):
        lo = 0
        for m in sorted(ms):
            if n >= 16000 and m > 1024:  # LM-head shapes: sampled rows only
                continue
            out.append((m, n, k))
            inside = m - 5
            if inside > lo:
                out.append((inside, n, k))
            lo = m
    return out


CASES = _cases()


@pytest.mark.parametrize("N,K", sorted({(n, k) for _, n, k in CASES}))
def test_table_plans_match_fp32(N, K):
    from vllm_musa_b200 import ops
    g = torch.Generator(device=DEV).manual_seed(N * 7 + K)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    for M in sorted({m for m, n, k in CASES if (n, k) == (N, K)}):
        x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
        ref = x.float() @ w.float().t()
        out = ops.linear(x, w)
        torch.cuda.synchronize()
        err = float((out.float() - ref).abs().max())
        tol = 2e-2 * float(ref.abs().max()) / 4 + 1e-2
        assert err <= tol, (M, N, K, err, tol)


@pytest.mark.parametrize("I", [14336, 7168, 3584, 1792])
def test_table_plans_silu_mul_match_fp32(I):
    from vllm_musa_b200 import ops
    K = 4096
    g = torch.Generator(device=DEV).manual_seed(I)
    gate = (torch.randn(I, K, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    up = (torch.randn(I, K, generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    w = ops.interleave_gate_up(gate, up)
    for M in sorted({m for m, n, k in CASES if (n, k) == (2 * I, K)}):
        x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
        ref = torch.nn.functional.silu(x.float() @ gate.float().t()) * (x.float() @ up.float().t())
        out = ops.linear_silu_mul(x, w)
        torch.cuda.synchronize()
        err = float((out.float() - ref).abs().max())
        tol = 2e-2 * float(ref.abs().max()) / 4 + 2e-2
        assert err <= tol, (M, I, err, tol)
