"""TurboQuant KV cache kernels (csrc/attention/turboquant.cu) against the PyTorch oracle in
vllm_musa_b200/ops/turboquant.py: store (slot bytes), paged decode (split and unsplit, GQA),
prefill-page dequantisation, and the tiny Llama through the engine on a quantised cache."""
import pytest
import torch

from vllm_musa_b200.ops import _ext
from vllm_musa_b200.ops import turboquant as tq

pytestmark = pytest.mark.gpu

PRESETS = sorted(tq.PRESETS)


def _filled_cache(name, D, Hkv, bs, T, seed=0):
    fmt = tq.tq_format(name, D)
    g = torch.Generator().manual_seed(seed)
    k = (torch.randn(T, Hkv * D, generator=g) * 2).to(torch.bfloat16)
    v = torch.randn(T, Hkv * D, generator=g).to(torch.bfloat16)
    nblk = (T + bs - 1) // bs + 3
    perm = torch.randperm(nblk, generator=g)[: (T + bs - 1) // bs].to(torch.int32)
    slots = (perm.repeat_interleave(bs)[:T] * bs + torch.arange(T) % bs).to(torch.int32)
    cache = torch.zeros(nblk, Hkv, bs, fmt.slot_bytes, dtype=torch.uint8, device="cuda")
    tq.tq_store(k.cuda(), v.cuda(), cache, slots.cuda(), fmt)
    return fmt, k, v, perm, slots, cache


@pytest.mark.parametrize("name", PRESETS)
@pytest.mark.parametrize("D", [64, 128, 256])
def test_tq_store_matches_oracle(name, D):
    Hkv, bs, T = 2, 16, 100
    fmt, k, v, perm, slots, cache = _filled_cache(name, D, Hkv, bs, T)
    torch.cuda.synchronize()
    _ext.check_device_errors()
    ref = torch.zeros(cache.shape, dtype=torch.uint8)
    tq.tq_store(k.float(), v.float(), ref, slots, fmt)
    got = cache.cpu()
    sl = slots.long()
    g_slots = got[sl // bs, :, sl % bs].reshape(-1, fmt.slot_bytes)
    r_slots = ref[sl // bs, :, sl % bs].reshape(-1, fmt.slot_bytes)
    same = (g_slots == r_slots).all(-1).float().mean().item()
    assert same > 0.97, same  # rare code flips at level boundaries (rounding order)
    gk, gv = tq.dequantize_slots(g_slots, fmt)
    rk, rv = tq.dequantize_slots(r_slots, fmt)
    rel = lambda a, b: ((a - b).norm() / b.norm()).item()  # noqa: E731
    assert rel(gk, rk) < 2e-2 and rel(gv, rv) < 2e-2


@pytest.mark.parametrize("name", PRESETS)
@pytest.mark.parametrize("D,Hq,Hkv", [(128, 32, 8), (64, 8, 8), (256, 16, 2)])
@pytest.mark.parametrize("splits", [1, 4])
def test_tq_decode_matches_oracle(name, D, Hq, Hkv, splits):
    bs = 16
    lens = [1, 37, 300, 129]
    B = len(lens)
    T = sum(lens)
    fmt, k, v, perm, slots, cache = _filled_cache(name, D, Hkv, bs, T, seed=3)
    # request b owns a contiguous run of the stored tokens
    W = max((n + bs - 1) // bs for n in lens) + 1
    bt = torch.zeros(B, W, dtype=torch.int32)
    # rebuild per-request tables: token j of request b is stored token start_b + j, whose
    # block is perm[(start_b + j) // bs]; use a fresh cache where requests start on page edges
    starts, s = [], 0
    for n in lens:
        starts.append(s)
        s += (n + bs - 1) // bs * bs
    Tp = s
    g = torch.Generator().manual_seed(5)
    kk = (torch.randn(Tp, Hkv * D, generator=g) * 2).to(torch.bfloat16).cuda()
    vv = torch.randn(Tp, Hkv * D, generator=g).to(torch.bfloat16).cuda()
    nblk = Tp // bs + 2
    cache = torch.zeros(nblk, Hkv, bs, fmt.slot_bytes, dtype=torch.uint8, device="cuda")
    pages = torch.randperm(nblk, generator=g)[:Tp // bs].to(torch.int32)
    sm = (pages.repeat_interleave(bs) * bs + torch.arange(Tp) % bs).to(torch.int32)
    tq.tq_store(kk, vv, cache, sm.cuda(), fmt)
    for b, (st, n) in enumerate(zip(starts, lens)):
        npg = (n + bs - 1) // bs
        bt[b, :npg] = pages[st // bs: st // bs + npg]
    q = torch.randn(B, Hq * D, generator=g).to(torch.bfloat16)
    seq = torch.tensor(lens, dtype=torch.int32)
    scale = D ** -0.5
    out = tq.tq_decode(q.cuda(), cache, bt.cuda(), seq.cuda(), Hq, scale, fmt,
                       num_splits=splits)
    torch.cuda.synchronize()
    _ext.check_device_errors()
    ref = tq.tq_decode(q.float(), cache.cpu(), bt, seq, Hq, scale, fmt)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("name", PRESETS)
def test_tq_dequant_pages_matches_oracle(name):
    D, Hkv, bs = 128, 4, 16
    fmt, k, v, perm, slots, cache = _filled_cache(name, D, Hkv, bs, 70, seed=7)
    bt = torch.zeros(2, 8, dtype=torch.int32)
    bt[0, :5] = perm[:5]
    bt[1, :2] = perm[:2]
    seq = torch.tensor([70, 20], dtype=torch.int32)
    kd, vd, bt2 = tq.tq_dequant_pages(cache, bt.cuda(), seq.cuda(), fmt, 5)
    torch.cuda.synchronize()
    _ext.check_device_errors()
    rk, rv, _ = tq.tq_dequant_pages(cache.cpu(), bt, seq, fmt, 5)
    torch.testing.assert_close(kd.float().cpu(), rk.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(vd.float().cpu(), rv.float(), rtol=2e-2, atol=2e-2)
    assert bt2.cpu().tolist() == [[0, 1, 2, 3, 4], [5, 6, 7, 8, 9]]


@pytest.mark.parametrize("name", ["turboquant_k8v4", "turboquant_4bit_nc", "fp8"])
def test_tiny_llama_generates_on_turboquant_cache(name):
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.presets import tiny_llama
    cfg = tiny_llama()
    cfg.dtype = torch.bfloat16
    outs = {}
    for kv in ("auto", name):
        llm = LLM(cfg, device="cuda", block_size=64, num_gpu_blocks=64, max_model_len=256,
                  max_num_seqs=8, max_num_batched_tokens=512, cuda_graph_sizes=[1, 2, 4, 8],
                  kv_cache_dtype=kv)
        o = llm.generate([list(range(1, 40)), list(range(100, 230))],
                         SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
        torch.cuda.synchronize()
        _ext.check_device_errors()
        outs[kv] = [r.outputs[0].token_ids for r in o]
        llm.shutdown()
    assert all(len(t) == 8 and all(0 <= x < cfg.vocab_size for x in t) for t in outs[name])
