"""Where a serving step's time goes: per-step device / host time by step kind, and a per-kernel
breakdown of decode and mixed (prefill + decode) steps on rank 0.

    python benchmarks/step_profile.py                       # 1 GPU
    torchrun --nproc-per-node N --master-addr 127.0.0.1 benchmarks/step_profile.py

Workload: the bench.py configuration 2 shape (Llama-3-8B architecture, random weights,
256 requests x 1024 prompt tokens -> 256 output tokens, temperature 1.0, ignore_eos),
tensor-parallel over the launched ranks.  Pass 1 steps the engine through the whole workload
and records, per engine step, the CUDA-event device time of ModelRunner.execute and the host
wall time of LLMEngine.step (max over ranks per step kind).  Pass 2 repeats the workload with
torch.profiler (CUDA activity) switched on for a few mixed steps and a few late decode steps,
and prints every kernel's share of those steps, grouped by family, plus the fraction of the
profiled span in which rank 0's GPU ran no kernel at all (launch / host / barrier gaps).
Prints JSON lines on rank 0.
"""
from __future__ import annotations

import argparse
import collections
import json
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

FAMILIES = [  # (family, substrings of the kernel name)
    ("allreduce", ("fused_ar", "cand_exchange", "ncclDevKernel", "ncclKernel", "ep_")),
    ("gemm", ("gemm_bf16", "gemm_fp8", "splitk", "gemm::")),
    ("attention", ("attn::", "decode_kernel", "prefill", "mla", "tile_offsets")),
    ("rope_kv", ("rope",)),
    ("norm", ("norm::", "rmsnorm")),
    ("sampling", ("sampling::", "sample_")),
    ("embed/gather", ("embedding", "gather_rows")),
]


def family(name: str) -> str:
    for fam, keys in FAMILIES:
        if any(k in name for k in keys):
            return fam
    return "other"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--num-requests", type=int, default=256)
    ap.add_argument("--input-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--max-num-batched-tokens", type=int, default=8192)
    ap.add_argument("--profile-decode-steps", type=int, default=6)
    ap.add_argument("--profile-mixed-steps", type=int, default=2)
    ap.add_argument("--num-layers", type=int, default=None)
    return ap.parse_args()


def run_workload(llm, prompts, sp, on_step=None):
    """Drive the engine step by step.  Returns [(kind, host_ms)] per step."""
    eng = llm.engine
    for i, p in enumerate(prompts):
        eng.add_request(f"r{llm._counter}-{i}", p, sp)
    llm._counter += 1
    rec = []
    k = 0
    while eng.has_unfinished_requests():
        if on_step is not None:
            on_step(k, "pre")
        t0 = time.perf_counter()
        eng.step()
        rec.append(time.perf_counter() - t0)
        if on_step is not None:
            on_step(k, "post")
        k += 1
    return rec


def main():
    args = parse()
    from vllm_musa_b200 import LLM, SamplingParams

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    n, il, ol = args.num_requests, args.input_len, args.output_len
    llm = LLM(args.model, tensor_parallel_size=world, max_num_seqs=n,
              max_num_batched_tokens=args.max_num_batched_tokens, max_model_len=il + ol + 64,
              block_size=64, seed=0, num_layers=args.num_layers)
    eng = llm.engine
    vocab = eng.config.model.vocab_size
    sp = SamplingParams(temperature=1.0, top_p=1.0, max_tokens=ol, ignore_eos=True)

    def prompts(step):
        g = torch.Generator().manual_seed(1000 + step)
        return torch.randint(0, vocab, (n, il), generator=g).tolist()

    llm.generate(prompts(0), sp)  # warm-up
    runner = eng.runner
    runner.timing = True

    # ---- pass 1: per-step device and host time by kind
    runner.step_times.clear()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    host = run_workload(llm, prompts(1), sp)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    kinds = [k for k, _, _ in runner.step_times]
    dev = [s.elapsed_time(e) for _, s, e in runner.step_times]
    agg = {}
    for kind in ("decode", "mixed"):
        idx = [i for i, k in enumerate(kinds) if k == kind]
        agg[kind] = [len(idx), sum(dev[i] for i in idx), sum(host[i] for i in idx) * 1e3]
    t = torch.tensor([agg["decode"][1], agg["decode"][2], agg["mixed"][1], agg["mixed"][2], wall],
                     dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        nd, nm = agg["decode"][0], agg["mixed"][0]
        print(json.dumps({
            "what": "per-step time by kind (max over ranks)", "tp": world,
            "decode_steps": nd, "decode_dev_ms_mean": round(float(t[0]) / max(nd, 1), 3),
            "decode_host_ms_mean": round(float(t[1]) / max(nd, 1), 3),
            "mixed_steps": nm, "mixed_dev_ms_mean": round(float(t[2]) / max(nm, 1), 3),
            "mixed_host_ms_mean": round(float(t[3]) / max(nm, 1), 3),
            "workload_wall_s": round(float(t[4]), 3),
            "output_tok_s_wall": round(n * ol / float(t[4]), 1)}), flush=True)

    # ---- pass 2: kernels of a few mixed and late decode steps
    runner.step_times.clear()
    mixed_idx = [i for i, k in enumerate(kinds) if k == "mixed"]
    dec_idx = [i for i, k in enumerate(kinds) if k == "decode"]
    prof_steps = set(mixed_idx[len(mixed_idx) // 2:len(mixed_idx) // 2 + args.profile_mixed_steps])
    late = dec_idx[-(len(dec_idx) // 4) - args.profile_decode_steps:-(len(dec_idx) // 4)] \
        if len(dec_idx) > 8 else dec_idx[:args.profile_decode_steps]
    prof_steps |= set(late)
    import torch.profiler as tp
    windows = []  # (kind, profiler)
    state = {}

    def on_step(k, when):
        if k not in prof_steps:
            return
        if when == "pre":
            torch.cuda.synchronize()
            p = tp.profile(activities=[tp.ProfilerActivity.CUDA])
            p.__enter__()
            state["p"] = p
        else:
            torch.cuda.synchronize()
            p = state.pop("p")
            p.__exit__(None, None, None)
            windows.append((kinds[k] if k < len(kinds) else "?", p))

    run_workload(llm, prompts(2), sp, on_step)
    if rank == 0:
        for kind in ("decode", "mixed"):
            per_kernel = collections.defaultdict(lambda: [0, 0.0])
            busy = span = 0.0
            nsteps = 0
            for kd, p in windows:
                if kd != kind:
                    continue
                nsteps += 1
                evs = [e for e in p.events()
                       if getattr(e, "device_type", None) == torch.autograd.DeviceType.CUDA]
                iv = []
                for e in evs:
                    d = e.time_range.end - e.time_range.start
                    per_kernel[e.name][0] += 1
                    per_kernel[e.name][1] += d
                    iv.append((e.time_range.start, e.time_range.end))
                if iv:
                    iv.sort()
                    span += iv[-1][1] - iv[0][0]
                    cur_s, cur_e = iv[0]
                    for s, e in iv[1:]:
                        if s > cur_e:
                            busy += cur_e - cur_s
                            cur_s, cur_e = s, e
                        else:
                            cur_e = max(cur_e, e)
                    busy += cur_e - cur_s
            if not nsteps:
                continue
            fam = collections.defaultdict(float)
            for name, (c, us) in per_kernel.items():
                fam[family(name)] += us
            tot = sum(fam.values())
            print(json.dumps({
                "what": f"{kind} step kernel time by family (rank 0, per step)", "tp": world,
                "steps": nsteps, "kernel_us_per_step": round(tot / nsteps, 1),
                "gpu_span_us_per_step": round(span / nsteps, 1),
                "gpu_idle_frac_in_span": round(1 - busy / span, 3) if span else None,
                "families_us": {k: round(v / nsteps, 1) for k, v in
                                sorted(fam.items(), key=lambda x: -x[1])}}), flush=True)
            top = sorted(per_kernel.items(), key=lambda x: -x[1][1])[:25]
            for name, (c, us) in top:
                print(json.dumps({"kind": kind, "kernel": name[:110], "calls_per_step": c / nsteps,
                                  "us_per_step": round(us / nsteps, 1),
                                  "us_per_call": round(us / c, 2)}), flush=True)
    llm.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
