"""Per-kernel timings of the hot sm_100a kernels against the measured roofline.

Each case times one kernel (CUDA events on the launching stream, after warm-up, averaged over
a back-to-back loop) on inputs larger than L2 (126 MB) or cycling through copies whose total
exceeds it, and reports achieved bytes/s and FLOP/s with their fractions of the measured
copy bandwidth / cuBLAS bf16 peak in MEASURED_PEAKS.json ("of measured").

    python benchmarks/kernel_bench.py                 # every case
    python benchmarks/kernel_bench.py --only gemm_decode,attn_decode --iters 20

The same command with --iters small is what the committed ncu summaries under profiles/ were
captured on (one kernel, few launches).
"""
import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from vllm_musa_b200 import ops  # noqa: E402
from vllm_musa_b200.ops import _ext  # noqa: E402

L2 = 126 << 20


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12
    return 6.65e12, 1.59e15


def timed(fn, iters):
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / iters  # us


def copies(make, nbytes):
    n = max(2, -(-3 * L2 // max(nbytes, 1)))
    return [make() for _ in range(n)]


def report(name, shape, us, nbytes, flops):
    bw, pk = peaks()
    rec = {"kernel": name, "shape": shape, "us": round(us, 2),
           "TBps": round(nbytes / us / 1e6, 3), "TFLOPs": round(flops / us / 1e6, 1),
           "frac_hbm_of_measured": round(nbytes / (us * 1e-6) / bw, 3),
           "frac_bf16_of_measured": round(flops / (us * 1e-6) / pk, 3)}
    print(json.dumps(rec), flush=True)


def bf16(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


# ------------------------------------------------------------------------------------ cases
def gemm(M, N, K, iters, name):
    ws = copies(lambda: bf16(N, K, scale=0.02), N * K * 2)
    x = bf16(M, K)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    us = timed(lambda i: ops.linear(x, ws[i % len(ws)], out=out), iters)
    report(name, [M, N, K], us, (M * K + N * K + M * N) * 2, 2 * M * N * K)


def case_gemm_decode(it):
    gemm(256, 28672, 4096, it, "gemm_bf16_decode_gate_up")
    gemm(256, 4096, 14336, it, "gemm_bf16_decode_down")


def case_gemm_decode_all(it):
    """Every Llama-3-8B TP=1 linear at the bench's decode batch (M = 256)."""
    for name, N, K in (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 28672, 4096),
                       ("down", 4096, 14336)):
        gemm(256, N, K, it, f"gemm_bf16_decode_{name}")


def case_gemm_decode_qkv(it):
    gemm(256, 6144, 4096, it, "gemm_bf16_decode_qkv")


def case_gemm_prefill(it):
    gemm(8192, 28672, 4096, it, "gemm_bf16_prefill_gate_up")
    gemm(8192, 4096, 4096, it, "gemm_bf16_prefill_o")


def case_gemm_pair(it):
    """1-CTA 128 x 256 tiles (mt=1) vs CTA-pair 256 x bn tiles (mt=4) on prefill shapes."""
    for M, N, K in ((8192, 28672, 4096), (8192, 4096, 14336), (8192, 6144, 4096),
                    (8192, 4096, 4096)):
        ws = copies(lambda: bf16(N, K, scale=0.02), N * K * 2)
        x = bf16(M, K)
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        for mt, bn in ((1, 256), (4, 0)):
            us = timed(lambda i: ops.gemm._run(x, ws[i % len(ws)], out, 0, bn, 1, mt), it)
            report(f"gemm_bf16_{'pair' if mt == 4 else 'single'}", [M, N, K], us,
                   (M * K + N * K + M * N) * 2, 2 * M * N * K)


def case_gemm_fp8(it):
    from vllm_musa_b200.ops import fp8
    for M, N, K in ((64, 24576, 7168), (4096, 7168, 2048)):
        mk = lambda: fp8.quantize_weight_block(torch.randn(N, K, device="cuda") * 0.02)  # noqa
        ws = copies(mk, N * K)
        xq, xs = fp8.group_quant_fp8(bf16(M, K))
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        us = timed(lambda i: fp8.gemm_fp8(xq, xs, *ws[i % len(ws)], out), it)
        report("gemm_fp8_block", [M, N, K], us, M * K + N * K + M * N * 2, 2 * M * N * K)


def _paged(B, ctx, Hkv, D, bs=64):
    per = -(-ctx // bs)
    nblk = B * per
    k = bf16(nblk, Hkv, bs, D)
    v = bf16(nblk, Hkv, bs, D)
    bt = torch.randperm(nblk, device="cuda", dtype=torch.int32).view(B, per)
    return k, v, bt


def case_attn_decode(it):
    B, ctx, Hq, Hkv, D = 256, 1152, 32, 8, 128
    k, v, bt = _paged(B, ctx, Hkv, D)
    q = bf16(B, Hq * D)
    seq = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq * D, dtype=torch.bfloat16, device="cuda")
    splits = ops.attention.num_decode_splits(B, Hkv, ctx)
    ops.attention.decode_workspace(q.device, B, Hq, D, splits)
    us = timed(lambda i: ops.paged_decode(q, k, v, bt, seq, Hq, Hkv, D ** -0.5, ctx, out=out,
                                          num_splits=splits), it)
    report("paged_decode", [B, ctx, Hq, Hkv, D], us, 2 * B * ctx * Hkv * D * 2,
           4 * B * ctx * Hq * D)


def case_tq_decode(it):
    """TurboQuant-cache decode (turboquant_4bit_nc, 144-byte slots): bytes = packed slots read."""
    from vllm_musa_b200.ops import turboquant as tq
    B, ctx, Hq, Hkv, D, bs = 256, 1152, 32, 8, 128, 64
    fmt = tq.tq_format("turboquant_4bit_nc", D)
    nb = B * ctx // bs
    cache = torch.randint(0, 256, (nb, Hkv, bs, fmt.slot_bytes), dtype=torch.uint8,
                          device="cuda")
    m = fmt.meta_offset  # valid fp16 scales in every slot
    cache[..., m:m + 6] = torch.tensor([0.01, 0.02, -0.1], dtype=torch.float16).view(
        torch.uint8).cuda()
    bt = torch.arange(nb, dtype=torch.int32, device="cuda").reshape(B, ctx // bs)
    q = bf16(B, Hq * D)
    seq = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq * D, dtype=torch.bfloat16, device="cuda")
    splits = tq.decode_splits(B, Hkv, ctx)
    ops.attention.decode_workspace(q.device, B, Hq, D, splits)
    us = timed(lambda i: tq.tq_decode(q, cache, bt, seq, Hq, D ** -0.5, fmt, out=out,
                                      num_splits=splits), it)
    report("tq_decode", [B, ctx, Hq, Hkv, D], us, B * ctx * Hkv * fmt.slot_bytes,
           4 * B * ctx * Hq * D)


def case_attn_prefill(it):
    R, L, Hq, Hkv, D = 8, 1024, 32, 8, 128
    k, v, bt = _paged(R, L, Hkv, D)
    T = R * L
    qkv = bf16(T, (Hq + 2 * Hkv) * D)
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device="cuda")
    seq = torch.full((R,), L, dtype=torch.int32, device="cuda")
    out = torch.empty(T, Hq * D, dtype=torch.bfloat16, device="cuda")
    us = timed(lambda i: ops.paged_prefill(qkv, k, v, cu, seq, bt, Hq, Hkv, D ** -0.5,
                                           out=out), it)
    report("paged_prefill", [R, L, Hq, Hkv, D], us, (T * (Hq + 2 * Hkv) * D + T * Hq * D) * 2,
           2 * R * L * L * Hq * D)  # causal: half of 4*L^2*Hq*D


def case_mla_decode(it):
    from vllm_musa_b200.ops import mla
    B, ctx, H, bs = 64, 8192, 16, 64
    per = ctx // bs
    cache = bf16(B * per, bs, 576)
    bt = torch.randperm(B * per, device="cuda", dtype=torch.int32).view(B, per)
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    seq = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    q_lat, q_pe = bf16(B, H, 512), bf16(B, H, 64)
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device="cuda")
    for sparse in (False, True):
        idx = None
        keys = ctx
        if sparse:
            keys = 2048
            idx = torch.stack([torch.randperm(ctx, device="cuda")[:keys] for _ in range(B)]).to(torch.int32)
        splits = mla.choose_splits(B * ((H + 15) // 16), keys)
        ws = (torch.empty(splits * B * H * 512, device="cuda"), torch.empty(splits * B * H, device="cuda"))
        us = timed(lambda i: mla.mla_attention(q_lat, q_pe, cache, bt, cu, seq, idx, out,
                                               192 ** -0.5, splits, ws), it)
        report("mla_decode_sparse2048" if sparse else "mla_decode_dense", [B, keys, H], us,
               B * keys * 576 * 2, 2 * B * keys * H * (576 + 512))


def case_gdn_decode(it):
    from vllm_musa_b200.ops import gdn
    B, Hk, Hv = 256, 16, 32
    state = torch.randn(B, Hv, 128, 128, device="cuda") * 0.01
    qkv = bf16(B, (2 * Hk + Hv) * 128)
    ba = bf16(B, 2 * Hv)
    A, dt = torch.zeros(Hv, device="cuda"), torch.zeros(Hv, device="cuda")
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    seq = torch.full((B,), 100, dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hv * 128, dtype=torch.bfloat16, device="cuda")
    for single in (True, False):
        us = timed(lambda i: gdn.gdn_recurrent(qkv, ba, A, dt, state, cu, seq, slots, Hk, Hv, out,
                                               single_token=single), it)
        report("gdn_decode" if single else "gdn_recurrent_decode", [B, Hk, Hv], us,
               2 * B * Hv * 128 * 128 * 4, 4 * B * Hv * 128 * 128)


def case_gdn_prefill(it):
    """Gated delta rule over 2 x 4096 new tokens (Qwen3-Next 16 QK / 32 V heads at TP=1):
    chunked kernels (prep + tensor-core scan) and, for comparison, the token recurrence."""
    from vllm_musa_b200.ops import gdn
    R, L, Hk, Hv = 2, 4096, 16, 32
    T = R * L
    state = torch.zeros(R, Hv, 128, 128, device="cuda")
    qkv = bf16(T, (2 * Hk + Hv) * 128)
    ba = bf16(T, 2 * Hv)
    A, dt = torch.zeros(Hv, device="cuda"), torch.zeros(Hv, device="cuda")
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device="cuda")
    seq = torch.full((R,), L, dtype=torch.int32, device="cuda")
    slots = torch.arange(R, dtype=torch.int32, device="cuda")
    out = torch.empty(T, Hv * 128, dtype=torch.bfloat16, device="cuda")
    # matrix-form FLOPs per chunk and head: K K^T, Q K^T (2 C^2 d), solve (C^2 2d),
    # W S^T, Qg S^T, U^T Kt (3 C d^2), Mq U (C^2 d)
    C, d = 64, 128
    flops = 2 * (T // C) * Hv * (2 * C * C * d + C * C * 2 * d + 3 * C * d * d + C * C * d)
    nbytes = T * (2 * Hk + Hv) * 128 * 2 + T * Hv * 128 * 2
    us = timed(lambda i: gdn.gdn_chunked(qkv, ba, A, dt, state, cu, seq, slots, Hk, Hv, out), it)
    report("gdn_chunked_prefill", [R, L, Hk, Hv], us, nbytes, flops)
    us = timed(lambda i: gdn.gdn_recurrent(qkv, ba, A, dt, state, cu, seq, slots, Hk, Hv, out),
               max(2, it // 4))
    report("gdn_recurrent_prefill", [R, L, Hk, Hv], us, nbytes, flops)


def case_moe(it):
    from vllm_musa_b200.ops import moe
    T, E, k, H, I = 256, 128, 8, 2048, 768
    w_gu = bf16(E * 2 * I, H, scale=0.02)
    w_dn = bf16(E * H, I, scale=0.02)
    x = bf16(T, H)
    ids, w = moe.topk_softmax(torch.randn(T, E, device="cuda"), k)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    us = timed(lambda i: moe.fused_moe(x, w_gu, w_dn, ids, w, E, None, out=out), it)
    report("fused_moe_decode", [T, E, k, H, I], us, (w_gu.numel() + w_dn.numel()) * 2,
           2 * T * k * 3 * H * I)


def case_moe_small(it):
    """Routed bf16 experts at decode batch sizes (Qwen3-30B-A3B at TP1: 128 experts, top-8,
    hidden 2048, expert intermediate 768): per-pair GEMVs against align + gather + grouped
    GEMMs, for the dispatch threshold."""
    import os
    from vllm_musa_b200.ops import moe
    E, k, H, I = 128, 8, 2048, 768
    w_gu = bf16(E * 2 * I, H, scale=0.02)
    w_dn = bf16(E * H, I, scale=0.02)
    for T in (1, 2, 4, 8, 16, 32, 64):
        x = bf16(T, H)
        # 16 routings in turn: the experts they touch (1.2 GB in all) do not stay in L2
        routes = [moe.topk_softmax(torch.randn(T, E, device="cuda"), k) for _ in range(16)]
        live = sum(int(torch.unique(r[0]).numel()) for r in routes) / len(routes)
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        nbytes = live * 3 * H * I * 2
        for name, limit in (("gemv", 1 << 20), ("grouped", 0)):
            os.environ["B200_MOE_GEMV_MAX_PAIRS"] = str(limit)
            us = timed(lambda i: moe.fused_moe(x, w_gu, w_dn, routes[i % 16][0], routes[i % 16][1],
                                               E, None, out=out), it)
            report(f"fused_moe_{name}", [T, E, k, H, I, round(live, 1)], us, nbytes,
                   2 * T * k * 3 * H * I)
    os.environ.pop("B200_MOE_GEMV_MAX_PAIRS", None)


def case_rope_kv(it):
    """Fused RoPE + paged KV insert over one 8192-token prefill chunk (Llama-3-8B heads)."""
    T, Hq, Hkv, D, bs = 8192, 32, 8, 128, 64
    qkv = bf16(T, (Hq + 2 * Hkv) * D)
    cs = ops.build_cos_sin_cache(D, 16384, 5e5, device="cuda")
    pos = (torch.arange(T, device="cuda") % 8192).to(torch.int32)
    nb = T // bs + 8
    kc = bf16(nb, Hkv, bs, D)
    vc = bf16(nb, Hkv, bs, D)
    slots = torch.randperm(nb * bs, device="cuda")[:T].to(torch.int32)
    us = timed(lambda i: ops.rope_kv(qkv, pos, cs, kc, vc, slots, Hq, Hkv, D, True), it)
    # read q, k, v; write q back, k and v into the cache
    report("rope_kv_prefill", [T, Hq, Hkv, D], us, T * (Hq + 2 * Hkv) * D * 2 * 2, 0)


def case_silu_fp8(it):
    """SwiGLU + 1x128 e4m3 quantisation of a gate/up output (DeepSeek dense MLP, 4096 tokens)."""
    T, I = 4096, 18432 // 8
    x = bf16(T, 2 * I)
    us = timed(lambda i: ops.activation.silu_mul_fp8_quant(x), it)
    report("silu_mul_fp8_quant", [T, I], us, T * 2 * I * 2 + T * I + T * I // 128 * 4, 0)


def case_routers(it):
    from vllm_musa_b200.ops import moe
    T = 8192
    lg = torch.randn(T, 128, device="cuda")
    us = timed(lambda i: moe.topk_softmax(lg, 8), it)
    report("topk_softmax_router", [T, 128, 8], us, T * 128 * 4 + T * 8 * 8, 0)
    lg2 = torch.randn(T, 256, device="cuda")
    bias = torch.randn(256, device="cuda") * 0.1
    us = timed(lambda i: moe.grouped_topk(lg2, 8, 8, 4, bias=bias, sigmoid=True), it)
    report("grouped_topk_router", [T, 256, 8], us, T * 256 * 4 + T * 8 * 8, 0)


def case_indexer(it):
    """Lightning-indexer scores + top-2048 for 64 decode rows over 8192-token contexts."""
    from vllm_musa_b200.ops import mla
    B, L, bs, k = 64, 8192, 64, 2048
    per = L // bs
    cache = bf16(B * per, bs, 128)
    bt = torch.arange(B * per, dtype=torch.int32, device="cuda").view(B, per)
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    seq = torch.full((B,), L, dtype=torch.int32, device="cuda")
    q = bf16(B, 64 * 128)
    w = torch.randn(B, 64, device="cuda") * 0.1
    scores = torch.empty(B, L, device="cuda")
    us = timed(lambda i: mla.indexer_scores(q, w, cache, bt, cu, seq, scores), it)
    report("indexer_scores_decode", [B, L, 64, 128], us, B * L * 128 * 2 + B * L * 4,
           2 * B * L * 64 * 128)
    us = timed(lambda i: mla.topk_indices(scores, cu, seq, k), it)
    report("indexer_topk_2048", [B, L, k], us, B * L * 4, 0)


def case_conv1d(it):
    """Causal conv1d (kernel 4) + SiLU over a prefill chunk of Qwen3-Next GDN channels."""
    from vllm_musa_b200.ops import gdn
    T, C = 8192, 2 * 16 * 128 + 32 * 128
    x = bf16(T, C)
    wt = bf16(C, 4)
    state = bf16(4, C, 3)
    cu = torch.tensor([0, T // 2, T], dtype=torch.int32, device="cuda")
    seq = torch.tensor([T // 2 + 10, T // 2], dtype=torch.int32, device="cuda")
    slots = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    out = torch.empty(T, C, dtype=torch.bfloat16, device="cuda")
    us = timed(lambda i: gdn.causal_conv1d(x, wt, state, cu, seq, slots, out), it)
    report("causal_conv1d", [T, C], us, 2 * T * C * 2, 8 * T * C)


def case_mamba2(it):
    """Mamba2 SSD recurrence, one decode step for 256 sequences (Mamba2-2.7B heads)."""
    from vllm_musa_b200.ops import mamba as M
    B, H, G, P, N = 256, 80, 1, 64, 128
    xbc = bf16(B, H * P + 2 * G * N)
    dt = bf16(B, H)
    dtb, Alog, D = (torch.rand(H, device="cuda") for _ in range(3))
    st = torch.randn(B, H, P, N, device="cuda") * 0.1
    cu = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    sl = torch.full((B,), 100, dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    out = torch.empty(B, H * P, dtype=torch.bfloat16, device="cuda")
    us = timed(lambda i: M.mamba2_scan(xbc, H * P, H * P + G * N, dt, dtb, Alog, D, st, cu, sl,
                                       slots, H, G, P, N, out=out), it)
    report("mamba2_decode", [B, H, P, N], us, 2 * B * H * P * N * 4, 6 * B * H * P * N)


def case_mamba2_prefill(it):
    """Mamba2 SSD over 2 x 4096 new tokens (Mamba2-2.7B: 80 heads of 64, state 128, 1 group):
    chunked kernels (chunk states, state pass, chunk scan) and, for comparison, the token
    recurrence."""
    from vllm_musa_b200.ops import mamba as M
    R, L, H, G, P, N = 2, 4096, 80, 1, 64, 128
    T = R * L
    xbc = bf16(T, H * P + 2 * G * N, scale=0.5)
    dt = bf16(T, H)
    dtb, Alog, D = (torch.rand(H, device="cuda") for _ in range(3))
    st = torch.zeros(R, H, P, N, device="cuda")
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device="cuda")
    sl = torch.full((R,), L, dtype=torch.int32, device="cuda")
    slots = torch.arange(R, dtype=torch.int32, device="cuda")
    out = torch.empty(T, H * P, dtype=torch.bfloat16, device="cuda")
    # matrix-form FLOPs per chunk and head: Sc = x^T B (C P N), C S0^T (C N P), C B^T (C^2 N),
    # G x (C^2 P)
    C = 64
    flops = 2 * (T // C) * H * (2 * C * P * N + C * C * N + C * C * P)
    nbytes = T * (H * P + 2 * G * N + H) * 2 + T * H * P * 2
    us = timed(lambda i: M.mamba2_chunked(xbc, H * P, H * P + G * N, dt, dtb, Alog, D, st, cu,
                                          sl, slots, H, G, P, N, out=out), it)
    report("mamba2_chunked_prefill", [R, L, H, P, N], us, nbytes, flops)
    us = timed(lambda i: M.mamba2_scan(xbc, H * P, H * P + G * N, dt, dtb, Alog, D, st, cu, sl,
                                       slots, H, G, P, N, out=out), max(2, it // 4))
    report("mamba2_recurrent_prefill", [R, L, H, P, N], us, nbytes, flops)


def case_rmsnorm(it):
    T, H = 32768, 4096
    x, r = bf16(T, H), bf16(T, H)
    w = bf16(H)
    us = timed(lambda i: ops.fused_add_rms_norm(x, r, w, 1e-5), it)
    report("fused_add_rms_norm", [T, H], us, 4 * T * H * 2, 0)


def case_sample(it):
    B, V = 256, 128256
    logits = torch.randn(B, V, device="cuda")
    t = torch.ones(B, device="cuda")
    seeds = torch.arange(B, dtype=torch.int64, device="cuda")
    steps = torch.zeros(B, dtype=torch.int32, device="cuda")
    us = timed(lambda i: ops.sample_tokens(logits, t, None, None, None, seeds, steps), it)
    report("gumbel_sample", [B, V], us, B * V * 4, 0)


CASES = {n[5:]: f for n, f in globals().items() if n.startswith("case_")}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=",".join(CASES))
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    _ext.require()
    ops.gemm.reserve_workspace(torch.device("cuda"), 64 << 20)
    for name in a.only.split(","):
        CASES[name](a.iters)
    torch.cuda.synchronize()
    _ext.check_device_errors()


if __name__ == "__main__":
    main()
