"""Sweep the tcgen05 BF16 GEMM's plans (tile width BN x split-K x row tiles: MT = 1 or 2
128-row tiles per CTA, 3 = one 128-row tile per CTA with the K splits reduced inside a
cluster, or 4 = a CTA pair on a 256-row tile) for a model's linear shapes
and write the fastest plan per (N, K, M) to vllm_musa_b200/tuning/gemm_bf16.json.

Timing: a loop of launches cycling through copies of the weight whose total exceeds L2 (every
launch reads its weight from HBM) is captured in a CUDA graph and replayed; CUDA events around
the replay, averaged over the loop; median of --reps.  Also reports cuBLAS (torch.matmul) for the same
shape as a yardstick and the achieved TB/s of weight streaming (decode) / TFLOP/s.

    python benchmarks/tune_gemm_bf16.py --model llama3-8b --tp 1 [--write]
"""
import argparse
import json
import os
import statistics
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from vllm_musa_b200 import ops  # noqa: E402
from vllm_musa_b200.models.presets import get_preset  # noqa: E402
from vllm_musa_b200.tuning import path_of  # noqa: E402

M_BUCKETS = [1, 8, 16, 32, 64, 128, 192, 256, 384, 512, 1024, 2048, 4096, 8192]


def model_shapes(name, tp):
    c = get_preset(name)
    H, D = c.hidden_size, c.head_dim
    hq, hkv = c.num_heads // tp, max(1, c.num_kv_heads // tp)
    I = c.intermediate_size // tp
    I_pad = (I + 31) // 32 * 32
    return {"qkv": ((hq + 2 * hkv) * D, H, 0), "o": (H, hq * D, 0), "gate_up": (2 * I_pad, H, 1),
            "down": (H, I_pad, 0), "lm_head": (c.vocab_size // tp, H, 2)}


L2_BYTES = 126 << 20


def s_ok(M):
    """CTA-pair plans (256-row tiles) are tried above one 128-row tile."""
    return M > 128


def timed(fn, ws, reps):
    """Median per-launch device time of ``fn(w)`` cycling through weight copies ``ws`` whose
    total size exceeds L2, so every launch streams its weights from HBM (as consecutive layers
    do in a decode step).  The loop of launches is captured once in a CUDA graph and replayed,
    so the number is the kernels' back-to-back device time (with programmatic dependent launch
    overlap between neighbours, as in the engine's captured decode steps), not the host's
    per-call dispatch time."""
    for w in ws:
        fn(w)
    torch.cuda.synchronize()
    loop = max(16, len(ws))
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for i in range(loop):
                fn(ws[i % len(ws)])
    torch.cuda.current_stream().wait_stream(st)
    g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e) * 1e3 / loop)
    del g
    return statistics.median(ts)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--reps", type=int, default=7)
    ap.add_argument("--m", type=str, default=",".join(map(str, M_BUCKETS)))
    ap.add_argument("--write", action="store_true")
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    mod = ops._ext.require()
    ops.gemm.reserve_workspace(torch.device("cuda"), 64 << 20)
    entries, report = [], []
    for lname, (N, K, mode) in model_shapes(a.model, a.tp).items():
        copies = max(2, -(-3 * L2_BYTES // (N * K * 2)))
        ws = [(torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(copies)]
        for M in map(int, a.m.split(",")):
            x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
            out = torch.empty(M, N // 2 if mode == 1 else N, device="cuda",
                              dtype=torch.float32 if mode == 2 else torch.bfloat16)
            auto = mod.gemm_plan(M, N, K)
            t_auto = timed(lambda w: ops.gemm._run(x, w, out, mode, auto[0], auto[1], auto[3]),
                           ws, a.reps)
            best = (t_auto, auto[0], auto[1], auto[3])
            kb = (K + 63) // 64
            for mt in ((1, 2, 4, 3) if M > 128 else (1, 3) if M <= 512 else (1,)):
                for bn in (256, 224, 208, 192, 176, 160, 144, 128, 112, 96, 64, 48, 32):
                    if mt == 4 and (bn % 32 or bn < 128):  # CTA pairs: 256-row tiles
                        continue
                    if mt == 4 and s_ok(M) is False:
                        continue
                    if M >= 1024 and mt != 4 and (bn % 64 or mt * bn * 2 > 512):
                        continue
                    # mt 3: one-CTA tiles whose 2-4 K splits reduce inside a cluster
                    for s in ((1,) if M >= 1024 else (1, 2, 3, 4) if mt == 4 else
                              (2, 3, 4) if mt == 3 else (1, 2, 3, 4, 6, 8)):
                        if s > 1 and kb // s < 4:
                            continue
                        if s * M * N > (64 << 20):
                            continue
                        t = timed(lambda w: ops.gemm._run(x, w, out, mode, bn, s, mt), ws, a.reps)
                        if t < best[0]:
                            best = (t, bn, s, mt)
            # swapped plans (C^T = W X^T): tokens in the MMA's N dimension, one token tile
            swap_best = None
            if mode in (0, 1) and M <= 256 and M % 8 == 0:
                sbn = (M + 15) // 16 * 16
                for smt in (1, 2):
                    for s in (1, 2, 3, 4, 6, 8):
                        if s > 1 and kb // s < 4:
                            continue
                        t = timed(lambda w: ops.gemm._run(x, w, out, mode, sbn, s, smt, swap=True),
                                  ws, a.reps)
                        if swap_best is None or t < swap_best[0]:
                            swap_best = (t, sbn, s, smt)
            t_cublas = timed(lambda w: torch.matmul(x, w.t()), ws, a.reps)
            tb = (N * K * 2 + M * K * 2 + M * N * 2) / (best[0] * 1e-6) / 1e12
            tf = 2 * M * N * K / (best[0] * 1e-6) / 1e12
            report.append(dict(layer=lname, M=M, N=N, K=K, auto=[auto[0], auto[1], auto[3]],
                               t_auto_us=round(t_auto, 1), best_bn=best[1], best_splits=best[2],
                               best_mt=best[3], t_best_us=round(best[0], 1),
                               swap_us=round(swap_best[0], 1) if swap_best else None,
                               cublas_us=round(t_cublas, 1), TBps=round(tb, 2), TFLOPs=round(tf, 1)))
            print(json.dumps(report[-1]), flush=True)
            entries.append({"n": N, "k": K, "m": M, "bn": best[1], "splits": best[2],
                            "mt": best[3], "us": round(best[0], 2)})
            if swap_best is not None:
                entries.append({"n": N, "k": K, "m": M, "bn": swap_best[1],
                                "splits": swap_best[2], "mt": swap_best[3], "swap": 1,
                                "us": round(swap_best[0], 2)})
    table = {"device": torch.cuda.get_device_name(), "model": a.model, "tp": str(a.tp),
             "entries": entries}
    if a.write:
        path = a.out or path_of("gemm_bf16")
        old = {"entries": []}
        if os.path.exists(path):
            old = json.load(open(path))
            tps = set(str(old.get("tp", "")).split(",")) | {str(a.tp)}
            table["tp"] = ",".join(sorted((t for t in tps if t), key=int))
        fresh = {(x["n"], x["k"], x["m"]) for x in entries}
        keep = [e for e in old["entries"] if (e["n"], e["k"], e["m"]) not in fresh]
        table["entries"] = keep + entries
        with open(path, "w") as f:
            json.dump(table, f, indent=1)
        print("wrote", path)


if __name__ == "__main__":
    main()
