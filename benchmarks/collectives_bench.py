"""Fused compute + collective paths over NVLink, timed on the device (CUDA events, max over
ranks), against their NVLink roofline and against the NCCL path they replace.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/collectives_bench.py

Cases (hidden 4096, bf16, every rank holds its partial sums):
  ar_norm    fused all-reduce + residual + RMSNorm (one-shot / two-shot by size) vs
             NCCL all_reduce followed by the fused add + RMSNorm kernel
  gemm_rs    row-parallel GEMM [T, K/N] x [H, K/N]^T whose epilogue stores into the owners'
             staging slots + the local-source reduce (+ residual + RMSNorm + all-gather) vs
             GEMM + fused all-reduce kernel
  cand       vocab-parallel sampling candidate exchange (one kernel) vs two NCCL all_gathers

Calls are captured into CUDA graphs and replayed (as the engine's decode steps are), so the
times are device times without per-call host overhead.
Roofline: the bytes a rank must move over NVLink (one direction, the larger of send / receive)
divided by the measured peer-copy bandwidth (770 GB/s per direction); for gemm_rs the slower of
that and the GEMM's FLOPs at the measured bf16 peak.  Prints one JSON line per case and size on
rank 0.
"""
from __future__ import annotations

import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

LINK_BPS = 770e9     # measured peer copy, per direction per GPU
BF16_FLOPS = 1.639e15  # measured cuBLAS bf16 burst


def _time(fn, iters, group, graph=True):
    """Per-call device time, max over ranks.  With ``graph`` the calls are captured once into a
    CUDA graph (20 back-to-back calls) and replayed, so host launch overhead (one Python
    dispatch per call on each of N processes) does not enter the number, as in the engine's
    captured decode steps."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = None
    per = 20
    if graph:
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                for _ in range(per):
                    fn()
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        g.replay()
        torch.cuda.synchronize()
    dist.barrier(group=group)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(1, iters // per) if graph else iters
    s.record()
    for _ in range(reps):
        if graph:
            g.replay()
        else:
            fn()
    e.record()
    torch.cuda.synchronize()
    n = reps * (per if graph else 1)
    t = torch.tensor([s.elapsed_time(e) * 1e3 / n], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    del g
    return float(t)


def main():
    from vllm_musa_b200 import ops
    from vllm_musa_b200.parallel.custom_ar import maybe_create_custom_allreduce
    from vllm_musa_b200.parallel.state import init_distributed
    world = int(os.environ["WORLD_SIZE"])
    st = init_distributed(tp_size=world)
    dev = torch.device("cuda", st.local_rank)
    H, eps = 4096, 1e-6
    ar = maybe_create_custom_allreduce(st, dev, max_tokens=8192, hidden=H)
    assert ar is not None, "P2P communicator did not initialise"
    ops.gemm.reserve_workspace(dev, 64 << 20)
    w = torch.ones(H, dtype=torch.bfloat16, device=dev)
    out = []

    def emit(d):
        if st.rank == 0:
            d.update(world=world)
            print(json.dumps(d), flush=True)
            out.append(d)

    nv = ar.nvls
    emit(dict(case="setup", nvls=nv is not None))
    for T in (1, 8, 64, 256, 1024, 4096, 8192):
        x = torch.randn(T, H, device=dev).to(torch.bfloat16)
        res = torch.randn(T, H, device=dev).to(torch.bfloat16)
        two_shot, _ = ar._plan(T)

        def p2p():  # peer-to-peer kernel (one- or two-shot by size), NVLS switched off
            ar.nvls = None
            stg = ar.staging_view(T)
            ar.allreduce_add_rmsnorm(stg, res, w, eps)
            ar.nvls = nv

        def nccl():
            y = x.clone()
            dist.all_reduce(y, group=st.tp_group)
            ops.fused_add_rms_norm(y, res, w, eps)

        it = 200 if T <= 256 else 50
        tf, tn = _time(p2p, it, st.tp_group), _time(nccl, it, st.tp_group)
        nbytes = T * H * 2
        # one-shot: read the other ranks' full slots; two-shot: read (N-1)/N of each peer's
        # slot for the owned chunk, then write the owned normalised chunk to N-1 peers
        link = (world - 1) * nbytes if not two_shot else (world - 1) * nbytes / world
        roof = link / LINK_BPS * 1e6
        rec = dict(case="ar_norm", T=T, H=H, two_shot=two_shot, us=round(tf, 2),
                   nccl_us=round(tn, 2), speedup_vs_nccl=round(tn / tf, 2),
                   roofline_us=round(roof, 2), frac_of_roofline=round(roof / tf, 3))
        if nv is not None and T >= world:
            k_fn = {}
            for shot in (True, False):
                def f(shot=shot):
                    ar._run_nvls(nv.staging[ar.parity][:T], res, w, eps, two_shot=shot)
                k_fn[shot] = _time(f, it, st.tp_group)
            # NVLS two-shot: each rank's link carries ~one message copy per direction
            # (ld_reduce of the owned rows from every rank + multimem.st of them to every rank)
            nroof = nbytes / LINK_BPS * 1e6
            rec.update(nvls2_us=round(k_fn[True], 2), nvls1_us=round(k_fn[False], 2),
                       nvls_roofline_us=round(nroof, 2),
                       nvls2_frac_of_roofline=round(nroof / k_fn[True], 3))
        emit(rec)

    if nv is not None:
        # rows per warp of the NVLS two-shot kernel at large messages (1: every warp loads,
        # then stores, in lock-step; 2+: the next row's reduce overlaps the current stores)
        import vllm_musa_b200.parallel.custom_ar as car
        for T in (1024, 4096, 8192):
            res = torch.randn(T, H, device=dev).to(torch.bfloat16)
            rec = dict(case="nvls_rows_per_warp", T=T, H=H)
            for rpw in (1, 2, 4, 0):
                car.NVLS_ROWS_PER_WARP = rpw

                def f():
                    ar._run_nvls(nv.staging[ar.parity][:T], res, w, eps, two_shot=True)
                rec[f"rpw{rpw}_us" if rpw else "default_us"] = round(_time(f, 50, st.tp_group), 2)
            car.NVLS_ROWS_PER_WARP = 0
            emit(rec)

    if nv is not None and H % 256 == 0:
        for T in (8, 256, 2048):
            x = torch.randn(T, H, device=dev).to(torch.bfloat16)
            res = torch.randn(T, H, device=dev).to(torch.bfloat16)

            def fused_q():
                ar.allreduce_add_rmsnorm_quant(ar.staging_view(T)[:T], res, w, eps)

            def unfused_q():
                o, _ = ar.allreduce_add_rmsnorm(ar.staging_view(T), res, w, eps)
                ops.activation.group_quant_fp8(o)

            tq, tu = _time(fused_q, 100, st.tp_group), _time(unfused_q, 100, st.tp_group)
            emit(dict(case="ar_norm_fp8", T=T, H=H, us=round(tq, 2), unfused_us=round(tu, 2),
                      speedup_vs_unfused=round(tu / tq, 2)))

    K = 14336
    for T in (256, 1024, 4096):
        if not ar._plan(T)[0]:  # the epilogue reduce-scatter pairs with the two-shot kernel
            continue
        Kr = K // world
        x = (torch.randn(T, Kr, device=dev) * 0.1).to(torch.bfloat16)
        wt = (torch.randn(H, Kr, device=dev) * 0.02).to(torch.bfloat16)
        res = torch.randn(T, H, device=dev).to(torch.bfloat16)

        def fused_rs():  # consecutive calls alternate the buffer parity by themselves
            ar.linear_allreduce_add_rmsnorm(x, wt, res, w, eps)

        def unfused():
            stg = ar.staging_view(T)
            ops.linear(x, wt, out=stg)
            ar.allreduce_add_rmsnorm(stg, res, w, eps)

        it = 50
        tf, tu = _time(fused_rs, it, st.tp_group), _time(unfused, it, st.tp_group)
        flops = 2 * T * H * Kr
        link = 2 * (world - 1) * T * H * 2 / world  # reduce-scatter out + all-gather out
        roof = max(flops / BF16_FLOPS, link / LINK_BPS) * 1e6
        emit(dict(case="gemm_rs", T=T, H=H, K_per_rank=Kr, us=round(tf, 2),
                  unfused_us=round(tu, 2), speedup_vs_unfused=round(tu / tf, 2),
                  roofline_us=round(roof, 2), frac_of_roofline=round(roof / tf, 3)))

    for R in (8, 64, 256):
        vals = torch.randn(R, device=dev)
        ids = torch.randint(0, 1 << 20, (R,), device=dev)

        def p2p():
            ar.merge_candidates(vals, ids)

        def nccl_gather():
            av = [torch.empty_like(vals) for _ in range(world)]
            ai = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(av, vals, group=st.tp_group)
            dist.all_gather(ai, ids, group=st.tp_group)
            torch.stack(av).argmax(0)

        tp, tn = _time(p2p, 200, st.tp_group), _time(nccl_gather, 200, st.tp_group)
        emit(dict(case="cand", rows=R, us=round(tp, 2), nccl_us=round(tn, 2),
                  speedup_vs_nccl=round(tn / tp, 2)))
    ops._ext.check_device_errors()
    ar.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
