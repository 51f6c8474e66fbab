"""MLA / DeepSeek sparse-attention kernels on B200 vs the fp32 PyTorch loops of ops.mla:
latent-cache prep, absorbed attention (dense prefix and index lists, with KV splits), the
lightning indexer's scores and the radix top-k."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_musa_b200.ops import _ext, mla
from vllm_musa_b200.ops.rope import build_cos_sin_cache


@pytest.fixture(autouse=True)
def _errs():
    yield
    torch.cuda.synchronize()
    _ext.check_device_errors()


def _layout(q_lens, hist, bs, g, nblk=64):
    R = len(q_lens)
    seq = [q + h for q, h in zip(q_lens, hist)]
    per = [(s + bs - 1) // bs for s in seq]
    perm = torch.randperm(nblk, generator=g)
    bt = torch.zeros(R, max(per), dtype=torch.int32)
    k = 0
    for r in range(R):
        bt[r, :per[r]] = perm[k:k + per[r]].to(torch.int32)
        k += per[r]
    cu = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    return bt, cu, torch.tensor(seq, dtype=torch.int32)


def test_mla_prep():
    g = torch.Generator().manual_seed(0)
    T, H, bs = 37, 16, 64
    q = torch.randn(T, H * 192, generator=g).to(torch.bfloat16)
    kv = torch.randn(T, 576 + 64, generator=g).to(torch.bfloat16)[:, :576]
    w = torch.rand(512, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), generator=g, dtype=torch.int32)
    cs = build_cos_sin_cache(64, 4096, 1e4, None)
    slots = torch.randperm(64 * bs, generator=g)[:T].to(torch.int32)
    slots[3] = -1
    cache = torch.zeros(64, bs, 576, dtype=torch.bfloat16)
    qc, cc = q.clone(), cache.clone()
    mla.mla_prep(qc, kv, w, 1e-6, pos, cs, cc, slots, H)
    qg, cg = q.cuda(), cache.cuda()
    mla.mla_prep(qg, kv.cuda(), w.cuda(), 1e-6, pos.cuda(), cs.cuda(), cg, slots.cuda(), H)
    torch.testing.assert_close(qg.cpu().float(), qc.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(cg.cpu().float(), cc.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("H,sparse,splits", [(16, False, 1), (16, False, 3), (40, True, 1),
                                             (16, True, 4), (128, False, 2)])
def test_mla_attention(H, sparse, splits):
    g = torch.Generator().manual_seed(H + splits + sparse)
    bs = 64
    q_lens, hist = [1, 1, 5, 70, 1], [200, 0, 30, 0, 1000]
    bt, cu, seq = _layout(q_lens, hist, bs, g)
    T = int(cu[-1])
    cache = (torch.randn(64, bs, 576, generator=g) * 0.5).to(torch.bfloat16)
    q_lat = torch.randn(T, H, 512, generator=g).to(torch.bfloat16)
    q_pe = torch.randn(T, H, 64 + 8, generator=g).to(torch.bfloat16)[:, :, :64]  # strided
    idx = None
    if sparse:
        topk = 128
        idx = torch.full((T, topk), -1, dtype=torch.int32)
        for t, (r, count) in enumerate(mla._req_of_tokens(cu, seq)):
            n = min(topk, count)
            idx[t, :n] = torch.randperm(count, generator=g)[:n].to(torch.int32)
    scale = 192 ** -0.5
    ref = torch.zeros(T, H, 512, dtype=torch.bfloat16)
    mla.mla_attention(q_lat, q_pe, cache, bt, cu, seq, idx, ref, scale)
    out = torch.empty(T, H, 512, dtype=torch.bfloat16, device="cuda")
    ws = None
    if splits > 1:
        ws = (torch.empty(splits * T * H * 512, device="cuda"), torch.empty(splits * T * H, device="cuda"))
    mla.mla_attention(q_lat.cuda(), q_pe.cuda(), cache.cuda(), bt.cuda(), cu.cuda(), seq.cuda(),
                      idx.cuda() if idx is not None else None, out, scale, splits, ws)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_indexer_scores_and_topk():
    g = torch.Generator().manual_seed(3)
    bs = 64
    q_lens, hist = [1, 9, 1, 300], [700, 0, 40, 0]
    bt, cu, seq = _layout(q_lens, hist, bs, g)
    T = int(cu[-1])
    k_raw = torch.randn(T, 128, generator=g).to(torch.bfloat16)
    ln_w = torch.rand(128, generator=g).to(torch.bfloat16)
    ln_b = (torch.randn(128, generator=g) * 0.1).to(torch.bfloat16)
    cs = build_cos_sin_cache(64, 4096, 1e4, None)
    positions = torch.cat([torch.arange(int(seq[r]) - q_lens[r], int(seq[r])) for r in range(4)]).to(torch.int32)
    slots = torch.cat([bt[r][(positions[cu[r]:cu[r + 1]] // bs).long()] * bs +
                       positions[cu[r]:cu[r + 1]] % bs for r in range(4)]).to(torch.int32)
    icache = (torch.randn(64, bs, 128, generator=g) * 0.5).to(torch.bfloat16)
    ic_ref = icache.clone()
    mla.indexer_k_prep(k_raw, ln_w, ln_b, 1e-6, positions, cs, ic_ref, slots)
    ic = icache.cuda()
    mla.indexer_k_prep(k_raw.cuda(), ln_w.cuda(), ln_b.cuda(), 1e-6, positions.cuda(), cs.cuda(),
                       ic, slots.cuda())
    torch.testing.assert_close(ic.cpu().float(), ic_ref.float(), rtol=2e-2, atol=2e-2)
    q = torch.randn(T, 64 * 128, generator=g).to(torch.bfloat16)
    w = torch.randn(T, 64, generator=g) * 0.1
    L = 1024
    ref = torch.empty(T, L)
    mla.indexer_scores(q, w, ic_ref, bt, cu, seq, ref)
    got = torch.empty(T, L, device="cuda")
    mla.indexer_scores(q.cuda(), w.cuda(), ic_ref.cuda(), bt.cuda(), cu.cuda(), seq.cuda(), got)
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(got.cpu()), fin)
    torch.testing.assert_close(got.cpu()[fin], ref[fin], rtol=2e-2, atol=5e-2)
    k = 256
    idx = mla.topk_indices(got, cu.cuda(), seq.cuda(), k).cpu()
    for t, (r, count) in enumerate(mla._req_of_tokens(cu, seq)):
        row = idx[t]
        if count <= k:
            assert sorted(row[:count].tolist()) == list(range(count)) and (row[count:] == -1).all()
        else:
            sel = set(row.tolist())
            assert len(sel) == k and -1 not in sel
            thresh = got.cpu()[t, :count].topk(k).values[-1]
            assert (got.cpu()[t, row.long()] >= thresh).all()


@pytest.mark.parametrize("dcp,splits", [(2, 1), (4, 3)])
def test_mla_attention_dcp_partials_combine(dcp, splits):
    """Decode context parallelism, emulated on one GPU: each virtual rank's cache holds the
    tokens p % dcp == rank at local index p // dcp; the kernel attends those (dcp params) and
    reports the log2-sum-exp; the LSE-weighted combine of the partials equals full attention."""
    g = torch.Generator().manual_seed(7 + dcp)
    bs, H = 16, 32
    q_lens, hist = [1, 1, 5, 70, 1], [200, 0, 30, 0, 1000]
    bt, cu, seq = _layout(q_lens, hist, bs, g, nblk=128)
    T = int(cu[-1])
    cache = (torch.randn(128, bs, 576, generator=g) * 0.5).to(torch.bfloat16)
    q_lat = torch.randn(T, H, 512, generator=g).to(torch.bfloat16)
    q_pe = torch.randn(T, H, 64, generator=g).to(torch.bfloat16)
    scale = 192 ** -0.5
    ref = torch.zeros(T, H, 512, dtype=torch.bfloat16)
    mla.mla_attention(q_lat, q_pe, cache, bt, cu, seq, None, ref, scale)
    flat = cache.view(-1, 576)
    outs, lses = [], []
    for r in range(dcp):
        # local cache of virtual rank r: token p (p % dcp == r) at local index p // dcp
        loc = torch.zeros(128, bs, 576, dtype=torch.bfloat16)
        lbt = torch.zeros_like(bt)
        nb = 0
        for i, L in enumerate(seq.tolist()):
            n_loc = (L - r + dcp - 1) // dcp if L > r else 0
            for b in range((n_loc + bs - 1) // bs):
                lbt[i, b] = nb
                nb += 1
            for li in range(n_loc):
                p = li * dcp + r
                src = int(bt[i, p // bs]) * bs + p % bs
                loc[int(lbt[i, li // bs]), li % bs] = flat[src]
        o = torch.empty(T, H, 512, dtype=torch.bfloat16, device="cuda")
        lse = torch.empty(T, H, dtype=torch.float32, device="cuda")
        ws = None
        if splits > 1:
            ws = (torch.empty(splits * T * H * 512, device="cuda"),
                  torch.empty(splits * T * H, device="cuda"))
        mla.mla_attention(q_lat.cuda(), q_pe.cuda(), loc.cuda(), lbt.cuda(), cu.cuda(),
                          seq.cuda(), None, o, scale, splits, ws, dcp=(dcp, r), lse_out=lse)
        outs.append(o.float().cpu())
        lses.append(lse.cpu())
    L = torch.stack(lses)                                   # [dcp, T, H]
    m = L.max(0).values
    w = torch.exp2(L - m)
    comb = (torch.stack(outs) * w.unsqueeze(-1)).sum(0) / w.sum(0).unsqueeze(-1)
    torch.testing.assert_close(comb, ref.float(), rtol=2e-2, atol=2e-2)
