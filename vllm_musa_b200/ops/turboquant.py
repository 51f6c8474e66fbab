"""TurboQuant-style quantised KV cache: formats, store / decode / dequant ops.

Cache dtypes: ``fp8`` / ``fp8_e4m3`` (e4m3 keys and values, one fp16 scale per vector: vLLM's
fp8 KV cache surface, reference flash_attn.py:349-370) and the names the reference's TurboQuant
backend accepts (vllm_musa/v1/attention/backends/
turboquant.py:69-75): ``turboquant_k8v4`` (e4m3 keys, 4-bit values), ``turboquant_4bit_nc``,
``turboquant_k3v4_nc``, ``turboquant_3bit_nc`` (Lloyd-Max keys after a randomised Hadamard
rotation, uniform values, norm correction).  The slot format, the rotation and the level
tables are defined in csrc/attention/turboquant.cu; this module restates them in PyTorch for
the CPU path and as the numerics oracle of the CUDA kernels.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _ext

# name -> (key bits, value bits, norm correction)
PRESETS = {
    # e4m3 keys and values with one fp16 scale per vector: the "fp8" KV cache
    "fp8": (8, 8, False),
    "fp8_e4m3": (8, 8, False),
    "turboquant_k8v4": (8, 4, False),
    "turboquant_4bit_nc": (4, 4, True),
    "turboquant_k3v4_nc": (3, 4, True),
    "turboquant_3bit_nc": (3, 3, True),
}

# Lloyd-Max levels of N(0, 1) (the same literals as the CUDA constant tables).
LEVELS = {
    3: [-2.1519457, -1.3439093, -0.7560053, -0.2450942,
        0.2450942, 0.7560053, 1.3439093, 2.1519457],
    4: [-2.7325896, -2.0690172, -1.6180464, -1.2562312, -0.9423405, -0.6567591, -0.3880483,
        -0.1283950, 0.1283950, 0.3880483, 0.6567591, 0.9423405, 1.2562312, 1.6180464,
        2.0690172, 2.7325896],
}


def is_turboquant(kv_cache_dtype: str | None) -> bool:
    return bool(kv_cache_dtype) and kv_cache_dtype in PRESETS


@dataclass(frozen=True)
class TQFormat:
    head_dim: int
    key_bits: int
    value_bits: int
    norm_correction: bool

    @property
    def key_bytes(self) -> int:
        return self.head_dim * self.key_bits // 8

    @property
    def value_bytes(self) -> int:
        return self.head_dim * self.value_bits // 8

    @property
    def meta_offset(self) -> int:
        return self.key_bytes + self.value_bytes

    @property
    def slot_bytes(self) -> int:
        return (self.meta_offset + 6 + 15) // 16 * 16


def tq_format(kv_cache_dtype: str, head_dim: int) -> TQFormat:
    if kv_cache_dtype not in PRESETS:
        raise ValueError(f"unknown TurboQuant cache dtype {kv_cache_dtype!r}; "
                         f"expected one of {sorted(PRESETS)}")
    if head_dim not in (64, 128, 256):
        raise ValueError("TurboQuant cache: head_dim must be 64, 128 or 256")
    kb, vb, nc = PRESETS[kv_cache_dtype]
    return TQFormat(head_dim, kb, vb, nc)


def lloyd_max_normal(levels: int, iters: int = 5000) -> list:
    """Lloyd-Max quantiser of the standard normal: boundaries at the midpoints of adjacent
    levels, each level the conditional mean of its interval (Max, 1960)."""
    def pdf(x):
        return math.exp(-x * x / 2) / math.sqrt(2 * math.pi) if math.isfinite(x) else 0.0

    def cdf(x):
        if not math.isfinite(x):
            return 1.0 if x > 0 else 0.0
        return 0.5 * (1 + math.erf(x / math.sqrt(2)))
    c = [-2 + 4 * (i + 0.5) / levels for i in range(levels)]
    for _ in range(iters):
        b = [-math.inf] + [(c[i] + c[i + 1]) / 2 for i in range(levels - 1)] + [math.inf]
        c = [(pdf(b[i]) - pdf(b[i + 1])) / (cdf(b[i + 1]) - cdf(b[i])) for i in range(levels)]
    return c


# ----------------------------------------------------------------------------- rotation
def _fmix32(h: int) -> int:
    h &= 0xFFFFFFFF
    h ^= h >> 16
    h = (h * 0x85EBCA6B) & 0xFFFFFFFF
    h ^= h >> 13
    h = (h * 0xC2B2AE35) & 0xFFFFFFFF
    h ^= h >> 16
    return h


def rotation_signs(D: int) -> torch.Tensor:
    return torch.tensor([-1.0 if _fmix32(i + 0x9E3779B9) & 1 else 1.0 for i in range(D)])


def hadamard(D: int) -> torch.Tensor:
    H = torch.ones(1, 1)
    while H.shape[0] < D:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    return H


def rotate(x: torch.Tensor) -> torch.Tensor:
    """y = H (s . x) / sqrt(D) over the last dim (fp32)."""
    D = x.shape[-1]
    return (x.float() * rotation_signs(D).to(x.device)) @ hadamard(D).to(x.device) / math.sqrt(D)


def unrotate(y: torch.Tensor) -> torch.Tensor:
    D = y.shape[-1]
    return (y.float() @ hadamard(D).to(y.device) / math.sqrt(D)) * rotation_signs(D).to(y.device)


# ----------------------------------------------------------------------- packing helpers
def _pack(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """[N, D] ints -> [N, D*bits/8] uint8, code i at bits [i*bits, i*bits+bits)."""
    N, D = codes.shape
    shifts = torch.arange(bits, device=codes.device)
    bitarr = ((codes.long()[..., None] >> shifts) & 1).reshape(N, D * bits // 8, 8)
    return (bitarr << torch.arange(8, device=codes.device)).sum(-1).to(torch.uint8)


def _unpack(packed: torch.Tensor, bits: int, D: int) -> torch.Tensor:
    N = packed.shape[0]
    bitarr = (packed.long()[..., None] >> torch.arange(8, device=packed.device)) & 1
    bitarr = bitarr.reshape(N, D, bits)
    return (bitarr << torch.arange(bits, device=packed.device)).sum(-1)


def _f16_bytes(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float16).reshape(-1, 1).view(torch.uint8)


def _f16_from(b: torch.Tensor) -> torch.Tensor:
    return b.contiguous().view(torch.float16).reshape(-1).float()


def quantize_vectors(k: torch.Tensor, v: torch.Tensor, fmt: TQFormat) -> torch.Tensor:
    """k, v [N, D] -> slots uint8 [N, slot_bytes] (CPU / oracle path)."""
    D = fmt.head_dim
    k = k.float()
    v = v.float()
    N = k.shape[0]
    if fmt.key_bits == 8:
        amax = k.abs().amax(-1)
        ksc = (amax / 448.0).to(torch.float16).float()
        safe = torch.where(ksc > 0, ksc, torch.ones_like(ksc))
        x = torch.where(ksc[:, None] > 0, k / safe[:, None], torch.zeros_like(k))
        kcodes = x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
    else:
        lv = torch.tensor(LEVELS[fmt.key_bits], dtype=torch.float32, device=k.device)
        bounds = 0.5 * (lv[:-1] + lv[1:])
        norm = k.norm(dim=-1)
        y = rotate(k)
        zmul = torch.where(norm > 0, math.sqrt(D) / norm.clamp_min(1e-30), torch.zeros_like(norm))
        idx = torch.bucketize(y * zmul[:, None], bounds)
        c = lv[idx]
        cs = c.pow(2).sum(-1)
        if fmt.norm_correction:
            ksc = torch.where(cs > 0, norm / cs.clamp_min(1e-30).sqrt(), torch.zeros_like(norm))
        else:
            ksc = norm / math.sqrt(D)
        ksc = ksc.to(torch.float16).float()
        kcodes = _pack(idx, fmt.key_bits)
    if fmt.value_bits == 8:  # e4m3 values, per-vector scale amax / 448
        vsc = (v.abs().amax(-1) / 448.0).to(torch.float16).float()
        vz = torch.zeros_like(vsc)
        safe = torch.where(vsc > 0, vsc, torch.ones_like(vsc))
        x = torch.where(vsc[:, None] > 0, v / safe[:, None], torch.zeros_like(v))
        vcodes = x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
    else:
        L = (1 << fmt.value_bits) - 1
        vmin, vmax = v.amin(-1), v.amax(-1)
        vsc = ((vmax - vmin) / L).to(torch.float16).float()
        vz = vmin.to(torch.float16).float()
        safe = torch.where(vsc > 0, vsc, torch.ones_like(vsc))
        vc = torch.round((v - vz[:, None]) / safe[:, None]).clamp(0, L)
        vc = torch.where(vsc[:, None] > 0, vc, torch.zeros_like(vc)).long()
        vcodes = _pack(vc, fmt.value_bits)
    out = torch.zeros(N, fmt.slot_bytes, dtype=torch.uint8, device=k.device)
    out[:, :fmt.key_bytes] = kcodes
    out[:, fmt.key_bytes:fmt.meta_offset] = vcodes
    m = fmt.meta_offset
    out[:, m:m + 2] = _f16_bytes(ksc)
    out[:, m + 2:m + 4] = _f16_bytes(vsc)
    out[:, m + 4:m + 6] = _f16_bytes(vz)
    return out


def dequantize_slots(slots: torch.Tensor, fmt: TQFormat, rotated_keys: bool = False):
    """slots [N, slot_bytes] -> k, v fp32 [N, D] (keys in the original space unless
    ``rotated_keys``)."""
    D, m = fmt.head_dim, fmt.meta_offset
    ksc = _f16_from(slots[:, m:m + 2])
    vsc = _f16_from(slots[:, m + 2:m + 4])
    vz = _f16_from(slots[:, m + 4:m + 6])
    if fmt.key_bits == 8:
        k = slots[:, :fmt.key_bytes].contiguous().view(torch.float8_e4m3fn).float() * ksc[:, None]
    else:
        lv = torch.tensor(LEVELS[fmt.key_bits], dtype=torch.float32, device=slots.device)
        k = lv[_unpack(slots[:, :fmt.key_bytes], fmt.key_bits, D)] * ksc[:, None]
        if not rotated_keys:
            k = unrotate(k)
    if fmt.value_bits == 8:
        v = slots[:, fmt.key_bytes:m].contiguous().view(torch.float8_e4m3fn).float() * vsc[:, None]
        return k, v
    vc = _unpack(slots[:, fmt.key_bytes:m], fmt.value_bits, D).float()
    return k, vc * vsc[:, None] + vz[:, None]


# --------------------------------------------------------------------------------- ops
def tq_store(k: torch.Tensor, v: torch.Tensor, cache: torch.Tensor, slot_mapping: torch.Tensor,
             fmt: TQFormat) -> None:
    """k, v [T, >= Hkv*D] rows -> cache [num_blocks, Hkv, block_size, slot] at ``slot_mapping``
    (slot = block * block_size + offset; < 0 skips)."""
    T = k.shape[0]
    if T == 0:
        return
    Hkv, bs = cache.shape[1], cache.shape[2]
    D = fmt.head_dim
    if k.is_cuda:
        _ext.ops().tq_store(k[:, :Hkv * D], v, cache, slot_mapping, fmt.key_bits,
                            fmt.value_bits, fmt.norm_correction)
        return
    sl = slot_mapping[:T].long()
    ok = sl >= 0
    kk = k[:T, :Hkv * D][ok].reshape(-1, D)
    vv = v[:T, :Hkv * D][ok].reshape(-1, D)
    slots = quantize_vectors(kk, vv, fmt).reshape(-1, Hkv, fmt.slot_bytes)
    blk, off = sl[ok] // bs, sl[ok] % bs
    cache[blk, :, off] = slots


def _gather_slots(cache: torch.Tensor, table: torch.Tensor, n: int) -> torch.Tensor:
    bs = cache.shape[2]
    nb = (n + bs - 1) // bs
    blocks = cache[table[:nb].long()]  # [nb, Hkv, bs, slot]
    return blocks.permute(0, 2, 1, 3).reshape(nb * bs, cache.shape[1], cache.shape[3])[:n]


def tq_decode(q: torch.Tensor, cache: torch.Tensor, block_tables: torch.Tensor,
              seq_lens: torch.Tensor, num_q_heads: int, scale: float, fmt: TQFormat,
              out: torch.Tensor | None = None, num_splits: int | None = None) -> torch.Tensor:
    """One query token per sequence over the quantised cache.  q [B, >= Hq*D] -> [B, Hq*D]."""
    B, D, Hq = q.shape[0], fmt.head_dim, num_q_heads
    Hkv = cache.shape[1]
    if out is None:
        out = torch.empty(B, Hq * D, dtype=q.dtype, device=q.device)
    if B == 0:
        return out
    if q.is_cuda:
        if num_splits is None:
            num_splits = decode_splits(B, Hkv, int(block_tables.shape[1] * cache.shape[2]))
        ws_o = ws_l = None
        if num_splits > 1:
            from .attention import decode_workspace
            ws_o, ws_l = decode_workspace(q.device, B, Hq, D, num_splits)
        _ext.ops().tq_decode(q, out, cache, block_tables, seq_lens, Hq, D, scale, fmt.key_bits,
                             fmt.value_bits, num_splits, ws_o, ws_l)
        return out
    G = Hq // Hkv
    for b in range(B):
        n = int(seq_lens[b])
        slots = _gather_slots(cache, block_tables[b], n)          # [n, Hkv, slot]
        k, v = dequantize_slots(slots.reshape(-1, fmt.slot_bytes), fmt)
        k = k.reshape(n, Hkv, D).repeat_interleave(G, 1)
        v = v.reshape(n, Hkv, D).repeat_interleave(G, 1)
        qb = q[b, :Hq * D].float().reshape(Hq, D)
        p = torch.softmax(torch.einsum("hd,shd->hs", qb, k) * scale, -1)
        out[b, :Hq * D] = torch.einsum("hs,shd->hd", p, v).reshape(-1).to(out.dtype)
    return out


def decode_splits(B: int, Hkv: int, max_seq_len: int) -> int:
    """Split the context so that B * Hkv * splits covers the 148 SMs about twice, with at least
    256 tokens per split."""
    want = max(1, -(-296 // max(1, B * Hkv)))
    return int(max(1, min(16, want, -(-max_seq_len // 256))))


def tq_dequant_pages(cache: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor,
                     fmt: TQFormat, num_pages: int):
    """Dequantise the first ``num_pages`` block-table pages of every row into fresh bf16 caches
    [R * num_pages, Hkv, block_size, D]; row r's page w lands at r * num_pages + w.  Returns
    (k_cache, v_cache, block_tables) for the bf16 paged prefill kernel."""
    R = block_tables.shape[0]
    Hkv, bs, D = cache.shape[1], cache.shape[2], fmt.head_dim
    dev = cache.device
    k_out = torch.zeros(R * num_pages, Hkv, bs, D, dtype=torch.bfloat16, device=dev)
    v_out = torch.zeros_like(k_out)
    bt = torch.arange(R * num_pages, dtype=torch.int32, device=dev).reshape(R, num_pages)
    if R == 0 or num_pages == 0:
        return k_out, v_out, bt
    if cache.is_cuda:
        _ext.ops().tq_dequant(cache, block_tables, seq_lens, k_out, v_out, D, fmt.key_bits,
                              fmt.value_bits)
        return k_out, v_out, bt
    for r in range(R):
        n = min(int(seq_lens[r]), num_pages * bs)
        slots = _gather_slots(cache, block_tables[r], n)
        k, v = dequantize_slots(slots.reshape(-1, fmt.slot_bytes), fmt)
        k = k.reshape(n, Hkv, D)
        v = v.reshape(n, Hkv, D)
        for t in range(n):
            k_out[r * num_pages + t // bs, :, t % bs] = k[t].to(torch.bfloat16)
            v_out[r * num_pages + t // bs, :, t % bs] = v[t].to(torch.bfloat16)
    return k_out, v_out, bt
