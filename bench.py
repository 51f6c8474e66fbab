"""Headline benchmark: serving throughput of a Llama-3-8B-architecture model on 1..8 B200s.

Metric: output tokens/s of the whole box (max over ranks), plus p50 TTFT and
p50 TPOT.  Config 2: Llama-3-8B architecture, bf16, random N(0, 0.02) weights, 256 concurrent
requests of 1024 token ids drawn uniformly over the vocabulary, 256 output tokens each with
ignore_eos, temperature 1.0.  With N GPUs the model runs tensor-parallel over N ranks (one
process per GPU, launched by torchrun); the workload is fixed, so scaling is "strong".

One bench step = serving the whole 256-request workload through ``LLM.generate`` (fresh
random prompts every step, so the prefix cache cannot skip any prefill).  W warm-up steps are
not timed; K steps are timed between a barrier + synchronize on both sides, with CUDA events
on the compute stream; the maximum over ranks is reported.

  value     output tokens / sum of device time of the engine's model steps (CUDA events
            around each step's H2D inputs + forward + sampling + D2H result): kernel-level rate
  e2e       output tokens / CUDA-event time of the LLM.generate() call (host scheduling
            included), with the per-step host->device / device->host byte counts

Other BASELINE configurations (same metric, their own model and workload; the default is
configuration 2):  --config 3  Qwen3-30B-A3B MoE, 128 x 2048 -> 512, experts expert-parallel
over the GPUs;  --config 5  Qwen3-Next-80B-A3B hybrid, 32 x 32768 -> 512;  --config 4
DeepSeek-V3.2 (fp8), 64 x 8192 -> 1024 (needs the memory of 8 GPUs).

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config C]
        torchrun --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

BASELINE_METRIC = "output tok/s (whole box, max over ranks) at 1/2/4/8 B200; p50 TTFT, p50 TPOT"
REFERENCE_UNAVAILABLE = (
    "the reference (MooreThreads/vllm-musa) cannot be installed or run on CUDA: its setup.py "
    "imports torchada/torch_musa and builds with the MUSA compiler (pip install fails with "
    "ModuleNotFoundError: No module named 'torchada')")


# BASELINE.json configurations 2..5: preset, concurrent requests, input / output lengths
CONFIGS = {
    2: dict(model="llama3-8b", requests=256, input=1024, output=256, ep=False),
    3: dict(model="qwen3-30b-a3b", requests=128, input=2048, output=512, ep=True),
    4: dict(model="deepseek-v3.2", requests=64, input=8192, output=1024, ep=True),
    5: dict(model="qwen3-next-80b-a3b", requests=32, input=32768, output=512, ep=False),
}


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--model", default=None)
    ap.add_argument("--num-requests", type=int, default=None)
    ap.add_argument("--input-len", type=int, default=None)
    ap.add_argument("--output-len", type=int, default=None)
    ap.add_argument("--max-num-batched-tokens", type=int, default=8192)
    ap.add_argument("--num-layers", type=int, default=None, help="debug only: fewer layers")
    ap.add_argument("--enforce-eager", action="store_true")
    a = ap.parse_args()
    c = CONFIGS[a.config]
    a.model = a.model or c["model"]
    a.num_requests = a.num_requests or c["requests"]
    a.input_len = a.input_len or c["input"]
    a.output_len = a.output_len or c["output"]
    a.ep = c["ep"]
    return a


def main():
    args = parse()
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": REFERENCE_UNAVAILABLE}))
        return 0

    import torch
    import torch.distributed as dist

    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.ops import _ext
    from vllm_musa_b200.utils.clocks import ClockSampler

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)

    n_req, in_len, out_len = args.num_requests, args.input_len, args.output_len
    llm = LLM(args.model, tensor_parallel_size=args.gpus, max_num_seqs=n_req,
              max_num_batched_tokens=args.max_num_batched_tokens,
              max_model_len=in_len + out_len + 64, block_size=64, seed=0,
              enforce_eager=args.enforce_eager, num_layers=args.num_layers,
              enable_expert_parallel=args.ep and args.gpus > 1)
    eng = llm.engine
    vocab = eng.config.model.vocab_size
    sp = SamplingParams(temperature=1.0, top_p=1.0, max_tokens=out_len, ignore_eos=True)

    def prompts(step):
        g = torch.Generator().manual_seed(1000 + step)
        return torch.randint(0, vocab, (n_req, in_len), generator=g).tolist()

    def barrier():
        if world > 1:
            dist.barrier()

    for w in range(args.warmup):
        llm.generate(prompts(w), sp)

    mod = _ext.require()
    runner = eng.runner
    runner.timing = True
    stream = torch.cuda.current_stream()
    e2e_ms, dev_ms, toks, ttfts, tpots, engine_steps = [], [], 0, [], [], 0
    h2d0, d2h0 = runner.h2d_bytes, runner.d2h_bytes
    launches0 = mod.launch_count()
    replay_launches = 0
    clocks = ClockSampler(gpu_index=local)
    clocks.start()
    for k in range(args.steps):
        ps = prompts(args.warmup + k)
        runner.step_times.clear()
        steps0 = eng.num_steps
        barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        outs = llm.generate(ps, sp)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms.append(ev0.elapsed_time(ev1))
        dev_ms.append(sum(s.elapsed_time(e) for _, s, e in runner.step_times))
        engine_steps += eng.num_steps - steps0
        toks += sum(len(o.outputs[0].token_ids) for o in outs)
        for o in outs:
            if o.metrics.ttft is not None:
                ttfts.append(o.metrics.ttft * 1e3)
            t = o.tpot()
            if t is not None:
                tpots.append(t * 1e3)
    clocks.stop()
    replay_launches = getattr(runner, "graph_launches_replayed", 0)
    launches = mod.launch_count() - launches0 + replay_launches

    tot = torch.tensor([sum(e2e_ms), sum(dev_ms)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    e2e_total, dev_total = float(tot[0]), float(tot[1])
    K = args.steps
    value = toks / (dev_total / 1e3)
    e2e_value = toks / (e2e_total / 1e3)
    ck = clocks.summary()
    rec = {
        "metric": BASELINE_METRIC,
        "value": round(value, 1),
        "unit": "output tok/s",
        "n_gpus": args.gpus,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(dev_total / K, 2),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: token ids uniform over the vocab, fresh prompts every step; "
                "random-init N(0,0.02) weights",
        "config": {"model": eng.config.model.name + (f" ({args.num_layers} layers)" if args.num_layers else ""),
                   "global_batch": n_req, "seq_len": in_len, "output_len": out_len,
                   "parallelism": f"tp{args.gpus}" + (f"+ep{args.gpus}" if args.ep and args.gpus > 1 else ""),
                   "sampling": "temperature 1.0, ignore_eos",
                   "max_num_batched_tokens": args.max_num_batched_tokens,
                   "l2": "inputs larger than L2: every step streams the model's weights (GBs) and "
                         "the KV cache from HBM"},
        "p50_ttft_ms": round(statistics.median(ttfts), 1) if ttfts else None,
        "p50_tpot_ms": round(statistics.median(tpots), 3) if tpots else None,
        "engine_steps_per_step": engine_steps / K,
        "e2e": {"value": round(e2e_value, 1), "unit": "output tok/s",
                "ms_per_step": round(e2e_total / K, 2),
                "h2d_bytes_per_step": int((runner.h2d_bytes - h2d0) / K),
                "d2h_bytes_per_step": int((runner.d2h_bytes - d2h0) / K)},
        "gpu_launches": int(launches),
        "clocks": ck,
    }
    if rank == 0:
        print(json.dumps(rec), flush=True)
    llm.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
