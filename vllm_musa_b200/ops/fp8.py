"""Block-scaled FP8 linear layers (DeepSeek-style e4m3 quantisation) on the tcgen05 kernel in
csrc/gemm/gemm_fp8.cu.

Weights: e4m3 [N, K] with fp32 scales per 128 x 128 block ([ceil(N/128), ceil(K/128)]), the
layout of HF "fp8" checkpoints with ``weight_block_size = [128, 128]`` (``weight_scale_inv``).
Activations: quantised per token in 1 x 128 groups (fp32 scales [M, ceil(K/128)]).
y = sum_kb sa[m, kb] * sb[n/128, kb] * (A_kb . B_kb^T), output bf16.

Reference counterparts: vllm_musa/model_executor/layers/quantization/utils/fp8_utils.py:33
(per_token_group_quant_fp8), vllm_musa/kernels/fp8_block_gemm.py:18 and
vllm_musa/model_executor/layers/quantization/kernels/linear/scaled_mm/deep_gemm.py:92-198.
"""
from __future__ import annotations

import torch

from . import _ext
from .activation import group_quant_fp8
from .gemm import _counters, _workspace

E4M3_MAX = 448.0


def quantize_weight_block(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16/fp32 [N, K] -> (e4m3 [N, K], fp32 scales [ceil(N/b), ceil(K/b)]), scale = amax/448."""
    N, K = w.shape
    nb, kb = -(-N // block), -(-K // block)
    wp = torch.zeros(nb * block, kb * block, dtype=torch.float32, device=w.device)
    wp[:N, :K] = w.float()
    blocks = wp.view(nb, block, kb, block)
    s = blocks.abs().amax(dim=(1, 3)).clamp(min=1e-12) / E4M3_MAX
    q = (blocks / s[:, None, :, None]).view(nb * block, kb * block)[:N, :K]
    return q.to(torch.float8_e4m3fn).contiguous(), s.contiguous()


def dequantize_weight_block(q: torch.Tensor, s: torch.Tensor, block: int = 128) -> torch.Tensor:
    N, K = q.shape
    rs = s.repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return q.float() * rs


def gemm_fp8_ref(a: torch.Tensor, sa: torch.Tensor, b: torch.Tensor, sb: torch.Tensor) -> torch.Tensor:
    """fp32 reference of the block-scaled GEMM (per-K-block promotion, same order of scaling)."""
    M, K = a.shape
    N = b.shape[0]
    out = torch.zeros(M, N, dtype=torch.float32, device=a.device)
    af, bf = a.float(), b.float()
    for kb in range(-(-K // 128)):
        k0, k1 = kb * 128, min(K, kb * 128 + 128)
        part = af[:, k0:k1] @ bf[:, k0:k1].t()
        scale = sa[:M, kb:kb + 1] * sb[:, kb].repeat_interleave(128)[:N].unsqueeze(0)
        out += part * scale
    return out


def gemm_fp8(a: torch.Tensor, sa: torch.Tensor, b: torch.Tensor, sb: torch.Tensor,
             out: torch.Tensor | None = None, splits: int = 0) -> torch.Tensor:
    """a e4m3 [M, K] (scales sa [M, K/128]) x b e4m3 [N, K] (scales sb [N/128, K/128]) -> bf16."""
    M, N = a.shape[0], b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    if M == 0:
        return out
    if not a.is_cuda:
        out.copy_(gemm_fp8_ref(a, sa, b, sb).to(out.dtype))
        return out
    mod = _ext.require()
    K = a.shape[1]
    if splits <= 0:
        splits, need, _ = mod.gemm_fp8_plan(M, N, K)
    else:
        need = splits * M * N if splits > 1 else 0
    ws = _workspace(a.device, need) if need > 0 else None
    cnt = _counters(a.device) if need > 0 else None
    torch.ops.b200.gemm_fp8(a, sa, b, sb, out, splits, ws, cnt)
    return out


def linear_fp8(x: torch.Tensor, w_q: torch.Tensor, w_s: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 x [M, K] -> per-token 1x128 e4m3 quantisation -> block-scaled GEMM -> bf16 [M, N].
    K must be a multiple of 128 (every DeepSeek projection's input width is)."""
    q, s = group_quant_fp8(x)
    return gemm_fp8(q, s, w_q, w_s, out)
