"""W4AFP8 routed experts on CPU: int4 packing round trip, the fp32 restatement against a
per-token loop written independently (dynamic per-token e4m3, clamped SwiGLU, expert map)."""
import pytest
import torch
import torch.nn.functional as F

from vllm_musa_b200.ops import w4afp8 as W


def _fp8(v):
    s = v.float().abs().amax(-1, keepdim=True).clamp_min(1e-4) / 448.0
    return (v.float() / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s


def _per_token(x, gu, dn, sgu, sdn, w, ids, emap, limit):
    gu = gu.float() * sgu.float().repeat_interleave(128, -1)
    dn = dn.float() * sdn.float().repeat_interleave(128, -1)
    out = torch.zeros(x.shape, dtype=torch.float32)
    xq = _fp8(x)
    for t in range(x.shape[0]):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            if emap is not None:
                e = int(emap[e])
            if e < 0:
                continue
            p = (xq[t] @ gu[e].T).to(torch.bfloat16).float()
            g, u = p.chunk(2)
            a = (F.silu(g.clamp(max=limit)) * u.clamp(-limit, limit)).to(torch.bfloat16)
            out[t] += (_fp8(a) @ dn[e].T).to(torch.bfloat16).float() * w[t, j]
    return out.to(torch.bfloat16)


def case(T, routing, E=4, H=256, I=256, seed=0):
    g = torch.Generator().manual_seed(seed + T)
    x = (torch.randn(T, H, generator=g) * 0.3).to(torch.bfloat16)
    gu = torch.randint(-8, 8, (E, 2 * I, H), generator=g, dtype=torch.int8)
    dn = torch.randint(-8, 8, (E, H, I), generator=g, dtype=torch.int8)
    sgu = (torch.rand(E, 2 * I, H // 128, generator=g) * 0.01 + 0.002).to(torch.bfloat16)
    sdn = (torch.rand(E, H, I // 128, generator=g) * 0.01 + 0.002).to(torch.bfloat16)
    mapped = routing in ("mapped", "all_remote")
    total = 2 * E if mapped else E
    ids = torch.stack([torch.randperm(total, generator=g)[:2] for _ in range(T)]).to(torch.int32)
    if routing == "all_remote":
        ids.remainder_(E)
    elif routing == "hot":
        ids.zero_()
    w = torch.softmax(torch.randn(T, 2, generator=g), -1)
    emap = torch.cat((torch.full((E,), -1), torch.arange(E))).to(torch.int32) if mapped else None
    return x, gu, dn, sgu, sdn, w, ids, emap


def test_pack_round_trip():
    v = torch.randint(-8, 8, (3, 5, 256), dtype=torch.int8)
    p = W.pack_int4(v)
    assert p.shape == (3, 5, 128) and p.dtype == torch.int8
    assert torch.equal(W.unpack_int4(p), v)
    # element 2j in the low nibble
    assert int(p[0, 0, 0]) & 15 == int(v[0, 0, 0]) & 15


@pytest.mark.parametrize("T,routing", [(1, "local"), (9, "mapped"), (17, "hot"), (5, "all_remote")])
def test_ref_matches_per_token_loop(T, routing):
    x, gu, dn, sgu, sdn, w, ids, emap = case(T, routing)
    want = _per_token(x, gu, dn, sgu, sdn, w, ids, emap, 10.0)
    got = W.w4afp8_moe(x, W.pack_int4(gu), W.pack_int4(dn), sgu, sdn, w, ids, emap,
                       swiglu_limit=10.0)
    torch.testing.assert_close(got.float(), want.float(), rtol=1e-2, atol=2e-3)
    if routing == "all_remote":
        assert not got.float().abs().any()


def test_shape_checks():
    x, gu, dn, sgu, sdn, w, ids, emap = case(2, "local")
    with pytest.raises(ValueError):
        W.w4afp8_moe(x, W.pack_int4(gu), W.pack_int4(dn)[:, :128], sgu, sdn, w, ids)
