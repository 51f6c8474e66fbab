"""Numerics of the sm_100a kernels against plain PyTorch fp32 references of the same op."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_musa_b200 import ops
from vllm_musa_b200.ops import _ext

DEV = "cuda"


@pytest.fixture(autouse=True)
def _check_errors():
    yield
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        _ext.check_device_errors()


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(DEV)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (7, 4096, 4096), (128, 512, 256), (200, 1000, 4096),
                                   (256, 6144, 4096), (1024, 2048, 1024), (4096, 4096, 4096),
                                   (300, 128256 // 8, 4096)])
def test_gemm_bf16(M, N, K):
    a, b = _bf(M, K, seed=1), _bf(N, K, seed=2, scale=0.05)
    ref = a.float() @ b.float().t()
    out = ops.linear(a, b)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2 * ref.abs().max().item() / 4 + 1e-2)


@pytest.mark.parametrize("bn,splits,mt", [(64, 1, 1), (128, 1, 1), (256, 1, 1), (128, 3, 1),
                                          (256, 4, 1), (64, 8, 1), (208, 1, 1), (48, 2, 1),
                                          (128, 1, 2), (256, 1, 2), (176, 3, 2), (16, 1, 2)])
def test_gemm_bf16_forced_plans(bn, splits, mt):
    M, N, K = 250, 768 + 16, 2048
    a, b = _bf(M, K, seed=3), _bf(N, K, seed=4, scale=0.05)
    ref = a.float() @ b.float().t()
    out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm._run(a, b, out, 0, bn, splits, mt)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("bn,splits,mt", [(208, 1, 1), (128, 1, 2), (96, 2, 2), (256, 1, 2)])
def test_gemm_silu_forced_plans(bn, splits, mt):
    M, I, K = 300, 1024, 1024
    x = _bf(M, K, seed=17)
    g, u = _bf(I, K, seed=18, scale=0.05), _bf(I, K, seed=19, scale=0.05)
    w = ops.interleave_gate_up(g, u)
    out = torch.empty(M, I, dtype=torch.bfloat16, device=DEV)
    ops.gemm._run(x, w, out, 1, bn, splits, mt)
    ref = torch.nn.functional.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("M,N,K,bn,mode,splits", [
    (256, 512, 1024, 256, 0, 1), (1000, 784, 2048, 256, 0, 1), (2048, 4096, 4096, 192, 0, 1),
    (777, 1024, 512, 128, 1, 1), (4096, 2000, 1024, 224, 2, 1), (300, 96, 256, 64, 0, 1),
    (256, 4096, 4096, 256, 0, 4), (200, 1024, 2048, 128, 1, 3), (512, 2000, 1024, 192, 2, 2)])
def test_gemm_bf16_cta_pair(M, N, K, bn, mode, splits):
    """CTA-pair (cta_group::2) tiles: 256 x bn per 2-CTA cluster, forced with mt=4, with and
    without split-K."""
    a = _bf(M, K, seed=21)
    if mode == 1:
        g, u = _bf(N // 2, K, seed=22, scale=0.05), _bf(N // 2, K, seed=23, scale=0.05)
        b = ops.interleave_gate_up(g, u)
        ref = torch.nn.functional.silu(a.float() @ g.float().t()) * (a.float() @ u.float().t())
        out = torch.empty(M, N // 2, dtype=torch.bfloat16, device=DEV)
    else:
        b = _bf(N, K, seed=24, scale=0.05)
        ref = a.float() @ b.float().t()
        out = torch.empty(M, N, dtype=torch.float32 if mode == 2 else torch.bfloat16, device=DEV)
    ops.gemm._run(a, b, out, mode, bn, splits, 4)
    torch.cuda.synchronize()
    _ext.check_device_errors()
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("M,N,K,bn,splits,mt,mode", [
    (256, 4096, 1024, 256, 1, 1, 0), (64, 1024, 2048, 64, 4, 1, 0), (8, 768, 512, 16, 2, 1, 0),
    (256, 2048, 4096, 256, 3, 2, 0), (128, 1024, 1024, 128, 1, 1, 1), (40, 784, 1024, 48, 2, 1, 1),
    (200, 1056, 512, 208, 1, 2, 1)])
def test_gemm_bf16_swapped(M, N, K, bn, splits, mt, mode):
    """Swap-AB plans: C^T = W X^T computed with the tokens in the MMA's N dimension and stored
    transposed through shared memory (with and without split-K, store and SwiGLU)."""
    a = _bf(M, K, seed=31)
    if mode == 1:
        g, u = _bf(N // 2, K, seed=32, scale=0.05), _bf(N // 2, K, seed=33, scale=0.05)
        b = ops.interleave_gate_up(g, u)
        ref = torch.nn.functional.silu(a.float() @ g.float().t()) * (a.float() @ u.float().t())
        out = torch.empty(M, N // 2, dtype=torch.bfloat16, device=DEV)
    else:
        b = _bf(N, K, seed=34, scale=0.05)
        ref = a.float() @ b.float().t()
        out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    ops.gemm.reserve_workspace(a.device, 16 << 20)
    ops.gemm._run(a, b, out, mode, bn, splits, mt, swap=True)
    torch.cuda.synchronize()
    _ext.check_device_errors()
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=3e-2)


def test_gemm_fp32_out_and_strided_a():
    M, N, K = 64, 1000, 512
    big = _bf(M, K + 64, seed=5)
    a = big[:, 32:32 + K]
    b = _bf(N, K, seed=6, scale=0.05)
    out = ops.linear(a, b, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    torch.testing.assert_close(out, a.float() @ b.float().t(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("M,I,K", [(5, 688, 256), (256, 1792, 4096), (1000, 512, 1024)])
def test_gemm_silu_mul_epilogue(M, I, K):
    x = _bf(M, K, seed=7)
    g, u = _bf(I, K, seed=8, scale=0.05), _bf(I, K, seed=9, scale=0.05)
    w = ops.interleave_gate_up(g, u)
    out = ops.linear_silu_mul(x, w)
    ref = torch.nn.functional.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())
    torch.testing.assert_close(out[:, :I].float(), ref, rtol=2e-2, atol=2e-2)
    assert out.shape[1] >= I


@pytest.mark.parametrize("rows,H", [(1, 256), (33, 4096), (256, 2048), (7, 7168), (4, 5120)])
def test_rms_norm_and_fused_add(rows, H):
    x, r, w = _bf(rows, H, seed=1), _bf(rows, H, seed=2), _bf(H, seed=3)
    y = ops.rms_norm(x, w, 1e-6)
    ref = ops.norm._rms_ref(x.cpu(), w.cpu(), 1e-6, False)
    torch.testing.assert_close(y.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)
    x2, r2 = x.clone(), r.clone()
    ops.fused_add_rms_norm(x2, r2, w, 1e-6)
    xc, rc = x.cpu().clone(), r.cpu().clone()
    ops.fused_add_rms_norm(xc, rc, w.cpu(), 1e-6)
    torch.testing.assert_close(r2.cpu(), rc, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(x2.cpu().float(), xc.float(), rtol=2e-2, atol=2e-2)


def test_rms_norm_gated():
    x, z, w = _bf(8, 4096, seed=1), _bf(8, 4096, seed=2), _bf(128, seed=3)
    y = ops.rms_norm_gated(x, z, w, 128, 1e-6)
    ref = ops.rms_norm_gated(x.cpu(), z.cpu(), w.cpu(), 128, 1e-6)
    torch.testing.assert_close(y.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_act_and_mul():
    x = _bf(17, 2 * 768, seed=4)
    for kind in (0, 1):
        y = ops.act_and_mul(x, kind)
        ref = ops.act_and_mul(x.cpu(), kind)
        torch.testing.assert_close(y.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def _make_cache(nb, Hkv, bs, D, seed=0):
    k = _bf(nb, Hkv, bs, D, seed=seed)
    v = _bf(nb, Hkv, bs, D, seed=seed + 1)
    return k, v


@pytest.mark.parametrize("D,Hq,Hkv,rot,neox,qknorm", [(128, 32, 8, 128, True, False),
                                                      (128, 32, 4, 128, True, True),
                                                      (64, 4, 2, 64, True, False),
                                                      (256, 16, 2, 64, True, True),
                                                      (128, 8, 8, 64, False, False)])
def test_rope_kv(D, Hq, Hkv, rot, neox, qknorm):
    T, bs, nb = 37, 16, 8
    qkv = _bf(T, (Hq + 2 * Hkv) * D, seed=5)
    pos = torch.randint(0, 500, (T,), dtype=torch.int32)
    slots = torch.randperm(nb * bs)[:T].to(torch.int32)
    slots[3] = -1
    cs = ops.build_cos_sin_cache(rot, 1024, 10000.0)
    qn = _bf(D, seed=6) if qknorm else None
    kn = _bf(D, seed=7) if qknorm else None
    kc, vc = torch.zeros(nb, Hkv, bs, D, dtype=torch.bfloat16), torch.zeros(nb, Hkv, bs, D, dtype=torch.bfloat16)
    q_cpu = qkv.cpu().clone()
    ops.rope_kv(q_cpu, pos, cs, kc, vc, slots, Hq, Hkv, rot, neox,
                qn.cpu() if qn is not None else None, kn.cpu() if kn is not None else None)
    kg, vg = kc.zero_().to(DEV), vc.zero_().to(DEV)
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    ops.rope_kv(q_cpu.clone(), pos, cs, kc2, vc2, slots, Hq, Hkv, rot, neox,
                qn.cpu() if qn is not None else None, kn.cpu() if kn is not None else None)
    q_gpu = qkv.clone()
    ops.rope_kv(q_gpu, pos.to(DEV), cs.to(DEV), kg, vg, slots.to(DEV), Hq, Hkv, rot, neox, qn, kn)
    torch.testing.assert_close(q_gpu[:, :Hq * D].cpu().float(), q_cpu[:, :Hq * D].float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(kg.cpu().float(), kc2.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(vg.cpu().float(), vc2.float(), rtol=0, atol=0)


def _random_tables(B, lens, bs, nb, seed=0):
    g = torch.Generator().manual_seed(seed)
    maxb = max((l + bs - 1) // bs for l in lens)
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(B, maxb + 3, dtype=torch.int32)
    used = 0
    for b, l in enumerate(lens):
        n = (l + bs - 1) // bs
        bt[b, :n] = perm[used:used + n].to(torch.int32)
        used += n
    return bt


@pytest.mark.parametrize("D,Hq,Hkv,bs", [(128, 32, 8, 64), (128, 32, 4, 16), (64, 4, 2, 32),
                                          (256, 16, 2, 64), (128, 64, 8, 128)])
@pytest.mark.parametrize("splits", [1, 4])
def test_paged_decode(D, Hq, Hkv, bs, splits):
    lens = [1, 5, 64, 65, 200, 1000, 129, 3]
    B = len(lens)
    nb = sum((l + bs - 1) // bs for l in lens) + 4
    kc, vc = _make_cache(nb, Hkv, bs, D, seed=11)
    bt = _random_tables(B, lens, bs, nb)
    sl = torch.tensor(lens, dtype=torch.int32)
    q = _bf(B, (Hq + 2 * Hkv) * D, seed=12)
    scale = 1.0 / math.sqrt(D)
    ref = ops.paged_decode(q.cpu(), kc.cpu(), vc.cpu(), bt, sl, Hq, Hkv, scale, 1024)
    out = ops.paged_decode(q, kc, vc, bt.to(DEV), sl.to(DEV), Hq, Hkv, scale, 1024, num_splits=splits)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("D,Hq,Hkv,bs,window", [(128, 32, 8, 64, 0), (128, 8, 2, 16, 0), (64, 4, 4, 32, 0),
                                                 (256, 16, 2, 64, 0), (128, 8, 2, 64, 100)])
def test_paged_prefill_chunked(D, Hq, Hkv, bs, window):
    # (context already cached, new tokens) per request
    reqs = [(0, 1), (0, 70), (64, 64), (100, 3), (900, 130), (5, 1)]
    R = len(reqs)
    lens = [c + n for c, n in reqs]
    nb = sum((l + bs - 1) // bs for l in lens) + 4
    kc, vc = _make_cache(nb, Hkv, bs, D, seed=21)
    bt = _random_tables(R, lens, bs, nb, seed=3)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor([n for _, n in reqs]), 0)), dtype=torch.int32)
    T = int(cu[-1])
    q = _bf(T, (Hq + 2 * Hkv) * D, seed=22)
    sl = torch.tensor(lens, dtype=torch.int32)
    scale = 1.0 / math.sqrt(D)
    ref = ops.paged_prefill(q.cpu(), kc.cpu(), vc.cpu(), cu, sl, bt, Hq, Hkv, scale, window)
    out = ops.paged_prefill(q, kc, vc, cu.to(DEV), sl.to(DEV), bt.to(DEV), Hq, Hkv, scale, window)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("bs,window,qscale", [(64, 0, 1.0), (16, 0, 4.0), (128, 0, 8.0),
                                               (64, 300, 4.0)])
@pytest.mark.parametrize("tc", ["tc2", "tc", "sync"])
def test_paged_prefill_long(bs, window, qscale, tc):
    """Long prompts and cached contexts on the head_dim-128 prefill kernels (tcgen05 with two
    heads per CTA, tcgen05 with one head, and the mma.sync one): several 128-key blocks, partial
    tiles, large logits (lazy rescaling of O in TMEM), sliding window."""
    D, Hq, Hkv = 128, 16, 4
    reqs = [(0, 1024), (300, 700), (2000, 257), (0, 129), (127, 1)]
    R = len(reqs)
    lens = [c + n for c, n in reqs]
    nb = sum((l + bs - 1) // bs for l in lens) + 4
    kc, vc = _make_cache(nb, Hkv, bs, D, seed=41)
    bt = _random_tables(R, lens, bs, nb, seed=5)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor([n for _, n in reqs]), 0)), dtype=torch.int32)
    T = int(cu[-1])
    q = (_bf(T, (Hq + 2 * Hkv) * D, seed=42).float() * qscale).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32)
    scale = 1.0 / math.sqrt(D)
    ref = ops.paged_prefill(q.cpu(), kc.cpu(), vc.cpu(), cu, sl, bt, Hq, Hkv, scale, window)
    mod = _ext.require()
    mod.set_prefill_tc(tc != "sync")
    mod.set_prefill_tc2(tc == "tc2")
    try:
        out = ops.paged_prefill(q, kc, vc, cu.to(DEV), sl.to(DEV), bt.to(DEV), Hq, Hkv, scale,
                                window)
        torch.cuda.synchronize()
    finally:
        mod.set_prefill_tc(True)
        mod.set_prefill_tc2(True)
    _ext.check_device_errors()
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_sampling_greedy_and_shards():
    R, V = 64, 50000
    logits = torch.randn(R, V, device=DEV) * 3
    ids = ops.sample_tokens(logits)
    assert torch.equal(ids.cpu(), logits.argmax(-1).cpu())
    # vocab-parallel: 4 shards, merged candidates equal the unsharded draw (random and greedy)
    temp = torch.full((R,), 0.8, device=DEV)
    temp[::3] = 0
    seeds = torch.arange(R, dtype=torch.int64, device=DEV) * 7919
    steps = torch.full((R,), 5, dtype=torch.int32, device=DEV)
    full = ops.sample_tokens(logits, temp, seeds=seeds, steps=steps)
    shard = V // 4
    vals, idxs = [], []
    for s in range(4):
        i, v = ops.sample_tokens(logits[:, s * shard:(s + 1) * shard].contiguous(), temp,
                                 seeds=seeds, steps=steps, vocab_offset=s * shard, return_values=True)
        vals.append(v)
        idxs.append(i)
    merged = torch.empty(R, dtype=torch.int64, device=DEV)
    torch.ops.b200.merge_candidates(torch.stack(vals), torch.stack(idxs), merged)
    assert torch.equal(merged, full)


def test_sampling_distribution_and_filters():
    V = 64
    base = torch.randn(V) * 2
    R = 4096
    logits = base.repeat(R, 1).to(DEV)
    temp = torch.full((R,), 1.0, device=DEV)
    seeds = torch.arange(R, dtype=torch.int64, device=DEV)
    steps = torch.zeros(R, dtype=torch.int32, device=DEV)
    ids = ops.sample_tokens(logits, temp, seeds=seeds, steps=steps).cpu()
    freq = torch.bincount(ids, minlength=V).float() / R
    p = torch.softmax(base, -1)
    assert (freq - p).abs().max() < 0.04
    # top-k = 5: only the 5 largest appear
    tk = torch.full((R,), 5, dtype=torch.int32, device=DEV)
    ids = ops.sample_tokens(logits, temp, top_k=tk, seeds=seeds, steps=steps).cpu()
    assert set(ids.tolist()) <= set(torch.topk(base, 5).indices.tolist())
    # top-p = 0.5: support is the smallest prefix reaching 0.5 mass
    tp = torch.full((R,), 0.5, device=DEV)
    ids = ops.sample_tokens(logits, temp, top_p=tp, seeds=seeds, steps=steps).cpu()
    keep = ops.sampling._filter_ref(base, 0, 0.5, 0.0)
    assert set(ids.tolist()) <= set(torch.nonzero(keep).flatten().tolist())
    # min-p
    mp = torch.full((R,), 0.2, device=DEV)
    ids = ops.sample_tokens(logits, temp, min_p=mp, seeds=seeds, steps=steps).cpu()
    keep = ops.sampling._filter_ref(base, 0, 1.0, 0.2)
    assert set(ids.tolist()) <= set(torch.nonzero(keep).flatten().tolist())


def test_embedding_and_gather():
    table = _bf(1000, 256, seed=1)
    ids = torch.randint(0, 1000, (77,), dtype=torch.int32, device=DEV)
    out = ops.embedding(ids, table)
    assert torch.equal(out, table[ids.long()])
    shard = ops.embedding(ids, table[500:].contiguous(), vocab_start=500)
    ref = torch.where((ids.long() >= 500)[:, None], table[ids.long()], torch.zeros_like(out))
    assert torch.equal(shard, ref)
    x = _bf(50, 4096, seed=2)
    idx = torch.tensor([0, 49, 3, 3], dtype=torch.int32, device=DEV)
    assert torch.equal(ops.gather_rows(x, idx), x[idx.long()])


@pytest.mark.parametrize("rows,H,add,want", [(1, 7168, True, False), (37, 4096, False, True),
                                             (256, 1536, True, True), (5, 128, False, False)])
def test_rms_norm_quant_fp8(rows, H, add, want):
    """Fused (residual add +) RMSNorm + 1x128 e4m3 quantisation against the PyTorch path."""
    x = _bf(rows, H, seed=61, scale=2.0)
    w = (_bf(H, 1, seed=62).view(H) * 0.2 + 1).to(torch.bfloat16)
    res = _bf(rows, H, seed=63) if add else None
    q, s, y = ops.rms_norm_quant_fp8(x, w, 1e-6, residual=res.clone() if add else None,
                                     want_bf16=want)
    rq, rs, ry = ops.rms_norm_quant_fp8(x.cpu(), w.cpu(), 1e-6,
                                        residual=res.cpu().clone() if add else None,
                                        want_bf16=True)
    torch.cuda.synchronize()
    _ext.check_device_errors()
    torch.testing.assert_close(s.cpu(), rs, rtol=1e-2, atol=1e-6)
    deq = q.cpu().float().view(rows, H // 128, 128) * s.cpu().unsqueeze(-1)
    torch.testing.assert_close(deq.view(rows, H), ry.float(), rtol=0.07, atol=0.02)
    if want:
        torch.testing.assert_close(y.cpu().float(), ry.float(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("section,interleaved,neox", [([16, 24, 24], False, True),
                                                      ([24, 20, 20], True, True),
                                                      ([8, 12, 12], False, False)])
def test_rope_kv_mrope(section, interleaved, neox):
    """Multimodal RoPE in the fused rope/KV-insert kernel against the PyTorch reference."""
    T, Hq, Hkv, D, bs = 37, 8, 2, 128, 16
    rot = 2 * sum(section) if not interleaved else 128
    cs = ops.build_cos_sin_cache(rot, 4096, 1e6)
    g = torch.Generator().manual_seed(7)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    pos3 = torch.randint(0, 4096, (3, T + 5), generator=g, dtype=torch.int32)
    nb = (T + bs - 1) // bs + 2
    kc = torch.zeros(nb, Hkv, bs, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nb * bs, generator=g)[:T].to(torch.int32)
    ref_qkv, rk, rv = qkv.clone(), kc.clone(), vc.clone()
    ops.rope_kv(ref_qkv, pos3, cs, rk, rv, slots, Hq, Hkv, rot, neox=neox,
                mrope_section=section, mrope_interleaved=interleaved)
    gq, gk, gv = qkv.to(DEV), kc.to(DEV), vc.to(DEV)
    ops.rope_kv(gq, pos3.to(DEV), cs.to(DEV), gk, gv, slots.to(DEV), Hq, Hkv, rot, neox=neox,
                mrope_section=section, mrope_interleaved=interleaved)
    torch.cuda.synchronize()
    _ext.check_device_errors()
    torch.testing.assert_close(gq.cpu().float(), ref_qkv.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(gk.cpu().float(), rk.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(gv.cpu().float(), rv.float())


@pytest.mark.parametrize("splits", [1, 4])
def test_paged_decode_sinks(splits):
    D, Hq, Hkv, bs = 64, 8, 2, 64
    lens = [1, 70, 600, 33]
    B = len(lens)
    nb = sum((l + bs - 1) // bs for l in lens) + 4
    kc, vc = _make_cache(nb, Hkv, bs, D, seed=51)
    bt = _random_tables(B, lens, bs, nb, seed=9)
    sl = torch.tensor(lens, dtype=torch.int32)
    q = _bf(B, (Hq + 2 * Hkv) * D, seed=52)
    sinks = torch.linspace(-3.0, 4.0, Hq)
    scale = 1.0 / math.sqrt(D)
    ref = ops.paged_decode(q.cpu(), kc.cpu(), vc.cpu(), bt, sl, Hq, Hkv, scale, 1024, sinks=sinks)
    out = ops.paged_decode(q, kc, vc, bt.to(DEV), sl.to(DEV), Hq, Hkv, scale, 1024,
                           num_splits=splits, sinks=sinks.to(DEV))
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("causal,sinks", [(True, True), (False, False), (False, True)])
def test_paged_prefill_sinks_noncausal(causal, sinks):
    """Sinks and bidirectional attention run on the mma.sync prefill kernel (the tcgen05 ones
    serve the causal sink-free case)."""
    D, Hq, Hkv, bs = 128, 8, 2, 64
    reqs = [(0, 70), (64, 64), (300, 130), (5, 1)]
    R = len(reqs)
    lens = [c + n for c, n in reqs]
    nb = sum((l + bs - 1) // bs for l in lens) + 4
    kc, vc = _make_cache(nb, Hkv, bs, D, seed=61)
    bt = _random_tables(R, lens, bs, nb, seed=4)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor([n for _, n in reqs]), 0)), dtype=torch.int32)
    T = int(cu[-1])
    q = _bf(T, (Hq + 2 * Hkv) * D, seed=62)
    sl = torch.tensor(lens, dtype=torch.int32)
    sk = torch.linspace(-1.0, 2.0, Hq) if sinks else None
    scale = 1.0 / math.sqrt(D)
    ref = ops.paged_prefill(q.cpu(), kc.cpu(), vc.cpu(), cu, sl, bt, Hq, Hkv, scale, 0,
                            sinks=sk, causal=causal)
    out = ops.paged_prefill(q, kc, vc, cu.to(DEV), sl.to(DEV), bt.to(DEV), Hq, Hkv, scale, 0,
                            sinks=sk.to(DEV) if sk is not None else None, causal=causal)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_encoder_varlen_attention():
    from vllm_musa_b200.attention import MMEncoderAttention
    H, D = 16, 64
    lens = [1024, 1, 300, 64, 577]
    T = sum(lens)
    q, k, v = (_bf(T, H * D, seed=s) for s in (71, 72, 73))
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0)), dtype=torch.int32)
    attn = MMEncoderAttention(H, D)
    ref = attn.forward(q.cpu(), k.cpu(), v.cpu(), cu)
    out = attn.forward(q, k, v, cu.to(DEV))
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_paged_prefill_tree_mask_with_causal_rows():
    """A tree-verification step batching prefill chunks: zero mask rows are causal (a chunk of
    150 queries, longer than the 64 mask bits, and a short one) beside two draft trees."""
    from vllm_musa_b200.ops.attention import tree_ancestor_masks
    D, Hq, Hkv, bs = 128, 8, 2, 64
    trees = [[-1, -1, 0, 1, 1, 2], None, [-1, 0, 0], None]
    qlens = [7, 150, 4, 9]
    ctxs = [90, 40, 200, 0]
    R = len(qlens)
    lens = [c + q for c, q in zip(ctxs, qlens)]
    nb = sum((l + bs - 1) // bs for l in lens) + 4
    kc, vc = _make_cache(nb, Hkv, bs, D, seed=85)
    bt = _random_tables(R, lens, bs, nb, seed=7)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(qlens), 0)), dtype=torch.int32)
    T = int(cu[-1])
    parts = []
    for t, ql in zip(trees, qlens):
        if t is None:
            parts.append(torch.zeros(ql, dtype=torch.int64))
        else:  # step token 0 = the pending token, then the drafts
            parts.append(torch.cat([torch.ones(1, dtype=torch.int64),
                                    (tree_ancestor_masks(t) << 1) | 1]))
    masks = torch.cat(parts)
    q = _bf(T, (Hq + 2 * Hkv) * D, seed=86)
    sl = torch.tensor(lens, dtype=torch.int32)
    scale = 1.0 / math.sqrt(D)
    ref = ops.paged_prefill(q.cpu(), kc.cpu(), vc.cpu(), cu, sl, bt, Hq, Hkv, scale,
                            tree_mask=masks)
    plain = ops.paged_prefill(q.cpu(), kc.cpu(), vc.cpu(), cu, sl, bt, Hq, Hkv, scale)
    torch.testing.assert_close(ref[7:157], plain[7:157])  # zero rows = causal (oracle check)
    out = ops.paged_prefill(q, kc, vc, cu.to(DEV), sl.to(DEV), bt.to(DEV), Hq, Hkv, scale,
                            tree_mask=masks.to(DEV))
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_paged_prefill_tree_mask():
    """Speculative token trees on the prefill kernel: per-row ancestor masks over the drafts."""
    from vllm_musa_b200.ops.attention import tree_ancestor_masks
    D, Hq, Hkv, bs = 128, 8, 2, 64
    g = torch.Generator().manual_seed(81)
    trees = [[-1], [-1, 0, 0, 1, 1, 2], [-1] + [int(torch.randint(0, i, (1,), generator=g))
                                               for i in range(1, 64)], [-1, 0, 1, -1]]
    ctxs = [0, 70, 300, 5]
    R = len(trees)
    lens = [c + len(t) for c, t in zip(ctxs, trees)]
    nb = sum((l + bs - 1) // bs for l in lens) + 4
    kc, vc = _make_cache(nb, Hkv, bs, D, seed=82)
    bt = _random_tables(R, lens, bs, nb, seed=6)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor([len(t) for t in trees]), 0)),
                      dtype=torch.int32)
    T = int(cu[-1])
    masks = torch.cat([tree_ancestor_masks(t) for t in trees])
    q = _bf(T, (Hq + 2 * Hkv) * D, seed=83)
    sl = torch.tensor(lens, dtype=torch.int32)
    scale = 1.0 / math.sqrt(D)
    ref = ops.paged_prefill(q.cpu(), kc.cpu(), vc.cpu(), cu, sl, bt, Hq, Hkv, scale,
                            tree_mask=masks)
    out = ops.paged_prefill(q, kc, vc, cu.to(DEV), sl.to(DEV), bt.to(DEV), Hq, Hkv, scale,
                            tree_mask=masks.to(DEV))
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2e-2, atol=2e-2)
