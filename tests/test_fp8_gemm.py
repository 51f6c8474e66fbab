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
    # the full path: on-device activation quantisation + GEMM
    y = fp8.linear_fp8(x.cuda(), wq.cuda(), ws.cuda())
    torch.testing.assert_close(y.float().cpu(), ref, rtol=5e-2, atol=5e-2)
