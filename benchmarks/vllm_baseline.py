"""Stock-vLLM baseline on the same box and workload as bench.py (configuration 2).

The reference (a MUSA-only plugin) cannot be built for CUDA, so the practical on-box
comparison is the installed vLLM's own CUDA path (NCCL, cuBLAS, FlashAttention/FlashInfer,
torch.compile) on an identical Llama-3-8B-architecture model with random weights
(``load_format="dummy"``) and the same synthetic workload: 256 requests x 1024 uniform-random
token ids -> 256 tokens, temperature 1.0, ignore_eos.  Output tokens / wall time of
``LLM.generate`` (which blocks until every request finishes).

    python benchmarks/vllm_baseline.py [--tp N] [--steps K] [--warmup W]
"""
import argparse
import json
import os
import statistics
import tempfile
import time

LLAMA3_8B = {
    "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
    "intermediate_size": 14336, "num_hidden_layers": 32, "num_attention_heads": 32,
    "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 128256, "rms_norm_eps": 1e-5,
    "rope_theta": 500000.0, "max_position_embeddings": 8192, "tie_word_embeddings": False,
    "torch_dtype": "bfloat16", "bos_token_id": 128000, "eos_token_id": 128001,
    "hidden_act": "silu", "attention_bias": False, "mlp_bias": False,
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--num-requests", type=int, default=256)
    ap.add_argument("--input-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=256)
    a = ap.parse_args()
    import torch
    from vllm import LLM, SamplingParams
    d = tempfile.mkdtemp(prefix="llama3_8b_cfg_")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(LLAMA3_8B, f)
    llm = LLM(model=d, load_format="dummy", skip_tokenizer_init=True, tensor_parallel_size=a.tp,
              max_num_seqs=a.num_requests, max_num_batched_tokens=8192,
              max_model_len=a.input_len + a.output_len + 64, seed=0, dtype="bfloat16",
              gpu_memory_utilization=0.9)
    sp = SamplingParams(temperature=1.0, max_tokens=a.output_len, ignore_eos=True,
                        detokenize=False)

    def prompts(step):
        g = torch.Generator().manual_seed(1000 + step)
        ids = torch.randint(0, LLAMA3_8B["vocab_size"], (a.num_requests, a.input_len), generator=g)
        return [{"prompt_token_ids": r} for r in ids.tolist()]

    for w in range(a.warmup):
        llm.generate(prompts(w), sp, use_tqdm=False)
    times, toks = [], 0
    for k in range(a.steps):
        ps = prompts(a.warmup + k)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        outs = llm.generate(ps, sp, use_tqdm=False)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
        toks += sum(len(o.outputs[0].token_ids) for o in outs)
    print(json.dumps({"impl": "stock-vllm", "model": "Llama-3-8B (random weights)", "tp": a.tp,
                      "output_tok_s": round(toks / sum(times), 1),
                      "s_per_step": round(statistics.mean(times), 3), "steps": a.steps,
                      "warmup": a.warmup, "requests": a.num_requests, "input_len": a.input_len,
                      "output_len": a.output_len, "timing": "wall clock around LLM.generate"}))


if __name__ == "__main__":
    main()
