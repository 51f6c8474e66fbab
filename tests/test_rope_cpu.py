"""RoPE reference paths on CPU: standard rotation and multimodal RoPE (sectioned and
interleaved frequency-to-position assignment)."""
import torch

from vllm_musa_b200 import ops
from vllm_musa_b200.ops.rope import _mrope_cos_sin


def _naive_mrope(cos_sin, pos3, rot_dim, section, interleaved):
    half = rot_dim // 2
    T = pos3.shape[1]
    out = torch.empty(T, rot_dim)
    for t in range(T):
        for f in range(half):
            if interleaved:
                c = 1 if (f % 3 == 1 and f < 3 * section[1]) else \
                    2 if (f % 3 == 2 and f < 3 * section[2]) else 0
            else:
                c = 0 if f < section[0] else 1 if f < section[0] + section[1] else 2
            p = int(pos3[c, t])
            out[t, f] = cos_sin[p, f]
            out[t, half + f] = cos_sin[p, half + f]
    return out


def test_mrope_cos_sin_matches_naive():
    cs = ops.build_cos_sin_cache(128, 512, 1e6)
    g = torch.Generator().manual_seed(0)
    pos3 = torch.randint(0, 512, (3, 9), generator=g, dtype=torch.int32)
    for sec, inter in (([16, 24, 24], False), ([24, 20, 20], True)):
        got = _mrope_cos_sin(cs, pos3, 128, sec, inter)
        torch.testing.assert_close(got, _naive_mrope(cs, pos3, 128, sec, inter))


def test_mrope_with_equal_rows_is_plain_rope():
    """Text tokens carry the same position in all three rows: M-RoPE must reduce to RoPE."""
    T, Hq, Hkv, D = 5, 4, 2, 128
    cs = ops.build_cos_sin_cache(D, 256, 1e6)
    g = torch.Generator().manual_seed(1)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 256, (T,), generator=g, dtype=torch.int32)
    slots = torch.full((T,), -1, dtype=torch.int32)
    a, b = qkv.clone(), qkv.clone()
    ops.rope_kv(a, pos, cs, None, None, slots, Hq, Hkv, D, neox=True, write_k=True, head_dim=D)
    ops.rope_kv(b, pos.unsqueeze(0).repeat(3, 1), cs, None, None, slots, Hq, Hkv, D, neox=True,
                write_k=True, head_dim=D, mrope_section=[16, 24, 24])
    torch.testing.assert_close(a.float(), b.float())
