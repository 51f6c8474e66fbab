"""Worker for the multi-GPU tests (run under torchrun by tests/test_tp_gpu.py).

--mode ar   : fused all-reduce + residual + RMSNorm kernel vs NCCL all-reduce + PyTorch math,
              one-shot and two-shot sizes, several calls in a row (parity / epoch reuse).
--mode topk : vocab-parallel top-k / top-p / min-p sampling through the NVLink candidate
              exchange vs sampling the gathered logits.
--mode llm  : greedy generation of a small Llama-architecture model at TP = WORLD_SIZE;
              writes tokens and first-step logits (gathered to full vocab) as JSON.
"""
import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def small_cfg():
    from vllm_musa_b200.config import ModelConfig
    return ModelConfig(arch="llama", vocab_size=4096, hidden_size=1024, num_layers=3,
                       num_heads=16, num_kv_heads=4, head_dim=64, intermediate_size=2816,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=2048, name="tp-test")


def mode_ar(out_path):
    from vllm_musa_b200 import ops
    from vllm_musa_b200.parallel.custom_ar import maybe_create_custom_allreduce
    from vllm_musa_b200.parallel.state import init_distributed
    world = int(os.environ["WORLD_SIZE"])
    st = init_distributed(tp_size=world)
    dev = torch.device("cuda", st.local_rank)
    H = 4096
    import vllm_musa_b200.parallel.custom_ar as car
    # numerics of every kernel: NVLS two-shot above 64 KiB, peer-to-peer below
    car.NVLS_MIN_BYTES = {w: 64 << 10 for w in (2, 4, 8)}
    car.NVLS_QUANT_MIN_ROWS = {w: 1 for w in (2, 4, 8)}
    # up to 4096 rows: at TP=2 the NVLS kernel's warps then walk two rows each (pipelined)
    ar = maybe_create_custom_allreduce(st, dev, max_tokens=4096, hidden=H)
    assert ar is not None, "custom all-reduce did not initialise"
    errs = []
    g = torch.Generator(device="cpu").manual_seed(123)
    w = (torch.randn(H, generator=g) * 0.1 + 1).to(torch.bfloat16).to(dev)
    # (rows, NVLS threshold for this call): NVLS one-shot below `world` rows, two-shot above
    # 64 KiB, peer-to-peer one- / two-shot where the threshold is None or not reached
    cases = [(1, 0), (7, 64 << 10), (32, 64 << 10), (256, 64 << 10), (1000, 64 << 10),
             (2048, None), (5, None), (1, None), (3, 0), (4096, 0)]
    for it, (T, lim) in enumerate(cases):
        car.NVLS_MIN_BYTES = {w: lim for w in (2, 4, 8)}
        ar.begin_forward() if it % 2 == 0 else None
        gen = torch.Generator(device="cpu").manual_seed(1000 * it + st.rank)
        x = torch.randn(T, H, generator=gen).to(torch.bfloat16).to(dev)
        gres = torch.Generator(device="cpu").manual_seed(77 + it)
        res = torch.randn(T, H, generator=gres).to(torch.bfloat16).to(dev)
        # reference: NCCL sum then fused norm math in fp32
        ref_sum = x.float().clone()
        dist.all_reduce(ref_sum, group=st.tp_group)
        ref_res = (ref_sum + res.float()).to(torch.bfloat16)
        ref_out = ops.norm._rms_ref(ref_res, w, 1e-6, False)
        stg = ar.staging_view(T)
        stg.copy_(x)
        nvls = ar.use_nvls(T)
        out, res2 = ar.allreduce_add_rmsnorm(stg, res.clone(), w, 1e-6)
        torch.cuda.synchronize()
        two_shot = nvls == 2 or (not nvls and ar._plan(T)[0])
        q_err = None
        if ar.can_quant(x):
            # the fused fp8 output (1x128 e4m3 groups) against quantising the reference rows
            stg = ar.staging_view(T)
            stg.copy_(x)
            q, s = ar.allreduce_add_rmsnorm_quant(stg, res.clone(), w, 1e-6)
            torch.cuda.synchronize()
            rq, rs = ops.activation.group_quant_fp8(ref_out)
            deq = q.float().view(T, -1, 128) * s.unsqueeze(-1)
            rdeq = rq.float().view(T, -1, 128) * rs.unsqueeze(-1)
            q_err = ((deq - rdeq).abs().max() / rdeq.abs().max()).item()
        if two_shot:
            per = (T + world - 1) // world
            r0, r1 = min(T, st.rank * per), min(T, st.rank * per + per)
            dres = (res2[r0:r1].float() - ref_res[r0:r1].float()).abs().max().item() if r1 > r0 else 0.0
        else:
            dres = (res2.float() - ref_res.float()).abs().max().item()
        dout = (out.float() - ref_out.float()).abs().max().item()
        errs.append({"T": T, "two_shot": two_shot, "nvls": nvls, "dout": dout, "dres": dres,
                     "q_err": q_err})
    ops._ext.check_device_errors()
    ar.close()
    if st.rank == 0:
        with open(out_path, "w") as f:
            json.dump(errs, f)
    dist.barrier()
    dist.destroy_process_group()


def mode_topk(out_path):
    """Vocab-parallel top-k / top-p / min-p sampling over NVLink (candidate rows exchanged and
    merged in one kernel) against sampling the gathered logits on every rank."""
    from vllm_musa_b200 import ops
    from vllm_musa_b200.parallel.custom_ar import maybe_create_custom_allreduce
    from vllm_musa_b200.parallel.state import init_distributed
    world = int(os.environ["WORLD_SIZE"])
    st = init_distributed(tp_size=world)
    dev = torch.device("cuda", st.local_rank)
    ar = maybe_create_custom_allreduce(st, dev, max_tokens=1024, hidden=1024)
    assert ar is not None
    res = []
    for it, (R, V) in enumerate([(64, 16000), (200, 32000), (7, 8000)]):
        g = torch.Generator().manual_seed(40 + it)
        scale = torch.where(torch.arange(R) % 3 == 0, 12.0, 2.0)
        logits = (torch.randn(R, V, generator=g) * scale[:, None]).to(dev)
        temp = torch.tensor([0.0 if r % 7 == 0 else 0.8 for r in range(R)], device=dev)
        top_k = torch.tensor([[0, 5, 50, 128][r % 4] for r in range(R)], dtype=torch.int32,
                             device=dev)
        top_p = torch.tensor([[1.0, 0.9, 0.5][r % 3] for r in range(R)], device=dev)
        min_p = torch.tensor([[0.0, 0.05][r % 2] for r in range(R)], device=dev)
        seeds = torch.arange(R, dtype=torch.int64, device=dev) * 31 + 1
        steps = torch.arange(R, dtype=torch.int32, device=dev) % 5
        Vs = V // world
        shard = logits[:, st.rank * Vs:(st.rank + 1) * Vs].contiguous()
        ref = ops.sample_tokens(logits, temp, top_k, top_p, min_p, seeds, steps)
        out = ar.sample_topk(shard, temp, top_k, top_p, min_p, seeds, steps, st.rank * Vs, V)
        torch.cuda.synchronize()
        dec = out >= 0
        must = (temp == 0) | (top_k > 0)
        res.append({"R": R, "V": V, "decided": float(dec.float().mean()),
                    "mismatch": int((out[dec] != ref[dec]).sum()),
                    "undecided_topk": int((~dec & must).sum())})
    ops._ext.check_device_errors()
    ar.close()
    if st.rank == 0:
        with open(out_path, "w") as f:
            json.dump(res, f)
    dist.barrier()
    dist.destroy_process_group()


def mode_gemm_rs(out_path):
    os.environ["B200_FUSE_GEMM_RS"] = "1"
    import vllm_musa_b200.parallel.custom_ar as car
    car.FUSE_GEMM_RS = True
    """Row-parallel GEMM with the reduce-scatter in its tcgen05 epilogue (NVLink stores into
    the owners' staging slots) + local reduce / residual / RMSNorm / all-gather, against NCCL
    all-reduce of a plain GEMM."""
    from vllm_musa_b200 import ops
    from vllm_musa_b200.parallel.custom_ar import maybe_create_custom_allreduce
    from vllm_musa_b200.parallel.state import init_distributed
    world = int(os.environ["WORLD_SIZE"])
    st = init_distributed(tp_size=world)
    dev = torch.device("cuda", st.local_rank)
    H, K = 4096, 1024
    ar = maybe_create_custom_allreduce(st, dev, max_tokens=2048, hidden=H)
    assert ar is not None
    ops.gemm.reserve_workspace(dev, 64 << 20)
    g = torch.Generator(device="cpu").manual_seed(5)
    nw = (torch.randn(H, generator=g) * 0.1 + 1).to(torch.bfloat16).to(dev)
    errs = []
    for it, T in enumerate([300, 1000, 2048, 77, 513]):
        ar.begin_forward()
        gen = torch.Generator(device="cpu").manual_seed(100 * it + st.rank)
        x = (torch.randn(T, K, generator=gen)).to(torch.bfloat16).to(dev)
        w = (torch.randn(H, K, generator=gen) * 0.03).to(torch.bfloat16).to(dev)
        gres = torch.Generator(device="cpu").manual_seed(7 + it)
        res = torch.randn(T, H, generator=gres).to(torch.bfloat16).to(dev)
        ref_sum = ops.linear(x, w).float()
        dist.all_reduce(ref_sum, group=st.tp_group)
        ref_res = (ref_sum + res.float()).to(torch.bfloat16)
        ref_out = ops.norm._rms_ref(ref_res, nw, 1e-6, False)
        fused = ar.can_fuse_gemm(T)
        r2 = res.clone()
        out, r2 = ar.linear_allreduce_add_rmsnorm(x, w, r2, nw, 1e-6) if fused else (None, None)
        torch.cuda.synchronize()
        if not fused:
            errs.append({"T": T, "fused": False})
            continue
        per = (T + world - 1) // world
        r0, r1 = min(T, st.rank * per), min(T, st.rank * per + per)
        dres = (r2[r0:r1].float() - ref_res[r0:r1].float()).abs().max().item() if r1 > r0 else 0.0
        dout = (out.float() - ref_out.float()).abs().max().item()
        errs.append({"T": T, "fused": True, "dout": dout, "dres": dres})
    ops._ext.check_device_errors()
    ar.close()
    if st.rank == 0:
        with open(out_path, "w") as f:
            json.dump(errs, f)
    dist.barrier()
    dist.destroy_process_group()


def mode_cand(out_path):
    """Vocab-parallel sampling candidate exchange (NVLink stores + epoch barrier + merge in one
    kernel) against NCCL all-gather + argmax, with ties broken toward the smaller token id."""
    from vllm_musa_b200.parallel.custom_ar import maybe_create_custom_allreduce
    from vllm_musa_b200.parallel.state import init_distributed
    world = int(os.environ["WORLD_SIZE"])
    st = init_distributed(tp_size=world)
    dev = torch.device("cuda", st.local_rank)
    ar = maybe_create_custom_allreduce(st, dev, max_tokens=512, hidden=1024)
    assert ar is not None
    bad = 0
    for it, R in enumerate([1, 5, 256, 300, 512, 2]):
        g = torch.Generator(device="cpu").manual_seed(10 * it + st.rank)
        vals = torch.randint(0, 4, (R,), generator=g).float().to(dev)  # many ties across ranks
        ids = (torch.randint(0, 1000, (R,), generator=g) + 1000 * st.rank).to(dev)
        got = ar.merge_candidates(vals, ids)
        av = [torch.empty_like(vals) for _ in range(world)]
        ai = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(av, vals, group=st.tp_group)
        dist.all_gather(ai, ids, group=st.tp_group)
        V, I = torch.stack(av).cpu(), torch.stack(ai).cpu()
        key = torch.where(V == V.max(0).values, I, torch.full_like(I, 1 << 40))
        ref = key.min(0).values
        bad += int((got.cpu() != ref).sum())
    from vllm_musa_b200 import ops
    ops._ext.check_device_errors()
    ar.close()
    if st.rank == 0:
        with open(out_path, "w") as f:
            json.dump({"mismatches": bad}, f)
    dist.barrier()
    dist.destroy_process_group()


def moe_cfg():
    from vllm_musa_b200.config import ModelConfig
    return ModelConfig(arch="qwen3_moe", vocab_size=4096, hidden_size=1024, num_layers=3,
                       num_heads=16, num_kv_heads=4, head_dim=64, intermediate_size=2816,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=2048, qk_norm=True,
                       num_experts=16, num_experts_per_tok=4, moe_intermediate_size=256,
                       name="tp-moe-test")


def ds_cfg():
    """Small dense-MLA DeepSeek (no sparse indexer) for the decode-context-parallel check."""
    from vllm_musa_b200.config import ModelConfig
    return ModelConfig(arch="deepseek_v3", vocab_size=4096, hidden_size=1024, num_layers=3,
                       num_heads=16, num_kv_heads=16, head_dim=192, intermediate_size=2048,
                       rms_norm_eps=1e-6, rope_theta=1e4, max_position=2048,
                       num_experts=16, num_experts_per_tok=2, moe_intermediate_size=256,
                       shared_expert_intermediate_size=256, first_k_dense=1, n_group=4,
                       topk_group=2, routed_scaling_factor=2.5, scoring_func="sigmoid",
                       q_lora_rank=256, kv_lora_rank=512, qk_nope_head_dim=128,
                       qk_rope_head_dim=64, v_head_dim=128, index_n_heads=0, index_head_dim=0,
                       index_topk=0, rope_neox=False, name="tp-ds-test")


def mode_llm(out_path, tp, eager, model="dense", ep=False, dcp=1, pp=1):
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.parallel.state import destroy_distributed, get_parallel_state
    cfg = moe_cfg() if model == "moe" else ds_cfg() if model == "ds" else small_cfg()
    llm = LLM(cfg, tensor_parallel_size=tp, pipeline_parallel_size=pp, block_size=64, seed=0,
              num_gpu_blocks=256,
              max_model_len=1024, max_num_seqs=16, max_num_batched_tokens=1024,
              enforce_eager=eager, cuda_graph_sizes=[1, 2, 4, 8, 16],
              enable_expert_parallel=ep, decode_context_parallel_size=dcp)
    if ep and tp > 1:
        assert llm.engine.comm.ep_a2a is not None, "EP all-to-all did not initialise"
    llm.engine.runner.record_logits = True
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (7, 100, 300, 64)]
    outs = llm.generate(prompts, SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True))
    st = get_parallel_state()
    log = llm.engine.runner.logits_log
    first = log[0].cuda() if log else torch.zeros(1, 1, device="cuda")  # last stage only (PP)
    if st.tp_size > 1:
        parts = [torch.empty_like(first) for _ in range(st.tp_size)]
        dist.all_gather(parts, first, group=st.tp_group)
        first = torch.cat(parts, dim=1)
    res = {"tokens": [o.outputs[0].token_ids for o in outs], "logits0": first.cpu().tolist(),
           "rank": st.rank}
    ops_ext = __import__("vllm_musa_b200.ops._ext", fromlist=["check_device_errors"])
    ops_ext.check_device_errors()
    with open(f"{out_path}.{st.rank}", "w") as f:
        json.dump(res, f)
    llm.shutdown()
    destroy_distributed()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["ar", "gemm_rs", "cand", "topk", "llm"], required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--model", default="dense")
    ap.add_argument("--ep", action="store_true")
    ap.add_argument("--dcp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    a = ap.parse_args()
    if a.mode == "ar":
        mode_ar(a.out)
    elif a.mode == "gemm_rs":
        mode_gemm_rs(a.out)
    elif a.mode == "cand":
        mode_cand(a.out)
    elif a.mode == "topk":
        mode_topk(a.out)
    else:
        mode_llm(a.out, a.tp, a.eager, a.model, a.ep, a.dcp, a.pp)
