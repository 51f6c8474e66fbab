"""Block-scaled FP8 GEMM: weight block quantisation round trip and the fp32 reference on CPU;
the tcgen05 kernel (with and without split-K) against that reference on B200."""
import pytest
import torch

from vllm_musa_b200.ops import fp8


def test_block_quant_roundtrip_and_reference():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(300, 260, generator=g) * 0.05
    q, s = fp8.quantize_weight_block(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (3, 3)
    back = fp8.dequantize_weight_block(q, s)
    # e4m3 keeps 3 mantissa bits: relative error <= 2^-4 (plus subnormal spacing)
    assert ((back - w).abs() <= w.abs() * 2 ** -4 + s.max() * 2 ** -9).all()
    x = torch.randn(5, 256, generator=g).to(torch.bfloat16)
    xq, xs = fp8.group_quant_fp8(x)
    wq, ws = fp8.quantize_weight_block(torch.randn(64, 256, generator=g) * 0.05)
    ref = fp8.gemm_fp8_ref(xq, xs, wq, ws)
    dense = (xq.float() * xs.repeat_interleave(128, 1)) @ fp8.dequantize_weight_block(wq, ws).t()
    torch.testing.assert_close(ref, dense, rtol=1e-4, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 576, 7168), (37, 1536, 512), (128, 7168, 2048),
                                   (300, 2048 + 128, 1536), (1024, 4096, 7168)])
@pytest.mark.parametrize("splits", [0, 1])
def test_gemm_fp8_gpu(M, N, K, splits):
    from vllm_musa_b200.ops import _ext
    g = torch.Generator().manual_seed(M + N + K)
    x = (torch.randn(M, K, generator=g)).to(torch.bfloat16)
    wq, ws = fp8.quantize_weight_block(torch.randn(N, K, generator=g) * 0.05)
    xq, xs = fp8.group_quant_fp8(x)
    ref = fp8.gemm_fp8_ref(xq, xs, wq, ws)
    out = fp8.gemm_fp8(xq.cuda(), xs.cuda(), wq.cuda(), ws.cuda(), splits=splits)
    torch.cuda.synchronize()
    _ext.check_device_errors()
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)
    # the full path: on-device activation quantisation + GEMM (the GPU quantiser may round a
    # few values to the neighbouring e4m3 code, so its own output is the reference input)
    y = fp8.linear_fp8(x.cuda(), wq.cuda(), ws.cuda())
    gq, gs = fp8.group_quant_fp8(x.cuda())
    ref2 = fp8.gemm_fp8_ref(gq.cpu(), gs.cpu(), wq, ws)
    torch.testing.assert_close(y.float().cpu(), ref2, rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("T,E,k,H,I,off,limit", [(1, 8, 2, 256, 128, 0, 0.0),
                                                  (77, 16, 4, 512, 256, 8, 0.0),
                                                  (300, 32, 8, 1024, 256, 0, 0.0),
                                                  (77, 16, 4, 512, 256, 0, 0.5)])
def test_fused_moe_fp8_gpu(T, E, k, H, I, off, limit):
    """limit > 0: clamped SwiGLU between the expert GEMMs."""
    from vllm_musa_b200.ops import moe as moe_ops
    g = torch.Generator().manual_seed(T + E + off)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    gus, gss, dws, dss = [], [], [], []
    for _ in range(E):
        q, s = fp8.quantize_weight_block(torch.randn(2 * I, H, generator=g) * 0.05)
        gus.append(q)
        gss.append(s)
        q, s = fp8.quantize_weight_block(torch.randn(H, I, generator=g) * 0.05)
        dws.append(q)
        dss.append(s)
    w_gu, s_gu, w_dn, s_dn = torch.cat(gus), torch.cat(gss), torch.cat(dws), torch.cat(dss)
    ids, w = moe_ops.topk_softmax(torch.randn(T, 2 * E, generator=g), k)  # half are other ranks'
    shared = (torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16)
    ref = moe_ops.fused_moe_fp8(x, w_gu, s_gu, w_dn, s_dn, ids, w, E, shared, expert_offset=off,
                                swiglu_limit=limit)
    out = moe_ops.fused_moe_fp8(x.cuda(), w_gu.cuda(), s_gu.cuda(), w_dn.cuda(), s_dn.cuda(),
                                ids.cuda(), w.cuda(), E, shared.cuda(), expert_offset=off,
                                swiglu_limit=limit)
    torch.cuda.synchronize()
    # activations are re-quantised to e4m3 twice on the GPU path: compare at fp8 resolution
    torch.testing.assert_close(out.float().cpu(), ref.float(), rtol=6e-2, atol=6e-2)


def test_swiglu_clamp_quant_cpu():
    from vllm_musa_b200.ops.activation import group_quant_fp8, silu_mul_fp8_quant
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(6, 512, generator=g) * 3).to(torch.bfloat16)
    q, s = silu_mul_fp8_quant(x, 1.5)
    gt, up = x.float().chunk(2, -1)
    a = (torch.nn.functional.silu(gt.clamp(max=1.5)) * up.clamp(-1.5, 1.5)).to(torch.bfloat16)
    rq, rs = group_quant_fp8(a)
    assert torch.equal(q.view(torch.uint8), rq.view(torch.uint8)) and torch.equal(s, rs)
    assert float(q.float().mul(s.repeat_interleave(128, 1)).abs().max()) <= 1.5 * 1.5 + 1e-3


@pytest.mark.gpu
def test_swiglu_clamp_quant_gpu():
    from vllm_musa_b200.ops.activation import silu_mul_fp8_quant
    g = torch.Generator().manual_seed(6)
    x = (torch.randn(33, 1024, generator=g) * 3).to(torch.bfloat16)
    q, s = silu_mul_fp8_quant(x.cuda(), 2.0)
    rq, rs = silu_mul_fp8_quant(x, 2.0)
    sc = s.cpu().repeat_interleave(128, 1)
    deq = q.float().cpu() * sc
    ref = rq.float() * rs.repeat_interleave(128, 1)
    # fp32 SiLU on the device vs the bf16-rounded CPU activation: codes may differ by one e4m3
    # step (3 mantissa bits: at most 1/8 relative, 2^-9 of the scale in the subnormal range)
    assert bool(((deq - ref).abs() <= 0.126 * ref.abs() + sc * 2.0 ** -9 + 1e-6).all())
    # the clamp holds: |silu(min(gate, 2)) * clamp(up, -2, 2)| <= 2 * silu(2) (+ one fp8 step)
    assert float(deq.abs().max()) <= 2.0 * 1.7616 * 1.126
