"""W4AFP8 routed experts on a B200: the int4 expansion kernel against the CPU unpack, and the
whole op (row e4m3 round trips, tcgen05 grouped GEMMs, combine) against the fp32 restatement."""
import pytest
import torch

from vllm_musa_b200.ops import _ext
from vllm_musa_b200.ops import w4afp8 as W

from test_w4afp8_cpu import case

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _loaded():
    _ext.require()  # registers torch.ops.b200 (fails loudly without the CUDA extension)


def test_w4_dequant_kernel_skips_idle_experts():
    g = torch.Generator().manual_seed(3)
    E, N, K = 3, 256, 384
    v = torch.randint(-8, 8, (E, N, K), generator=g, dtype=torch.int8)
    s = (torch.rand(E, N, K // 128, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    p = W.pack_int4(v).cuda()
    out = torch.full((E * N, K), 7.0, dtype=torch.bfloat16, device="cuda")
    offsets = torch.tensor([0, 128, 128, 256], dtype=torch.int32, device="cuda")
    torch.ops.b200.w4_dequant(out, p, s.cuda(), offsets)
    want = W.dequant_w4(W.pack_int4(v), s).to(torch.bfloat16).reshape(E * N, K)
    out = out.cpu()
    assert torch.equal(out[:N], want[:N]) and torch.equal(out[2 * N:], want[2 * N:])
    assert (out[N:2 * N] == 7.0).all()  # expert 1 received no rows: left untouched


def test_row_fp8_qdq_kernel():
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(37, 2 * 512, generator=g) * 3).to(torch.bfloat16)
    out = torch.empty(37, 512, dtype=torch.bfloat16, device="cuda")
    torch.ops.b200.row_fp8_qdq(out, x.cuda(), True, 2.0, None)
    gt, up = x.float().chunk(2, -1)
    a = (torch.nn.functional.silu(gt.clamp(max=2.0)) * up.clamp(-2, 2)).to(torch.bfloat16)
    torch.testing.assert_close(out.cpu().float(), W._fp8_round_trip(a).to(torch.bfloat16).float(),
                               rtol=0.07, atol=1e-3)
    plain = torch.empty(37, 1024, dtype=torch.bfloat16, device="cuda")
    torch.ops.b200.row_fp8_qdq(plain, x.cuda(), False, 0.0, None)
    torch.testing.assert_close(plain.cpu().float(), W._fp8_round_trip(x).to(torch.bfloat16).float(),
                               rtol=0.07, atol=1e-3)


@pytest.mark.parametrize("T,routing", [(1, "local"), (7, "mapped"), (64, "hot"), (300, "local"),
                                       (5, "all_remote")])
def test_w4afp8_moe_matches_reference(T, routing):
    x, gu, dn, sgu, sdn, w, ids, emap = case(T, routing)
    want = W.w4afp8_moe_ref(x, W.pack_int4(gu), W.pack_int4(dn), sgu, sdn, w, ids, emap, 10.0)
    dev = [t.cuda() if t is not None else None
           for t in (x, W.pack_int4(gu), W.pack_int4(dn), sgu, sdn, w, ids, emap)]
    got = W.w4afp8_moe(*dev, swiglu_limit=10.0)
    torch.cuda.synchronize()
    torch.testing.assert_close(got.cpu().float(), want.float(), rtol=0.04, atol=0.008)
