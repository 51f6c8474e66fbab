"""Penalties kernel on a B200 against the PyTorch oracle (full vocab and a vocab shard), and
log-probabilities through the engine on the GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_apply_penalties_kernel_matches_oracle():
    from vllm_musa_b200.ops.sampling import apply_penalties, penalty_entries
    g = torch.Generator().manual_seed(1)
    R, V = 6, 5000
    rows = []
    for r in range(R):
        prompt = torch.randint(0, V, (int(torch.randint(0, 300, (1,), generator=g)),),
                               generator=g).tolist()
        out = torch.randint(0, V, (int(torch.randint(0, 60, (1,), generator=g)),),
                            generator=g).tolist()
        rows.append((r, prompt, out))
    e = penalty_entries(rows)
    logits = torch.randn(R, V, generator=g) * 3
    rep = torch.rand(R, generator=g) + 0.7
    pres = torch.rand(R, generator=g) - 0.5
    freq = torch.rand(R, generator=g)
    want = apply_penalties(logits.clone(), e, rep, pres, freq)
    got = apply_penalties(logits.cuda(), e.cuda(), rep.cuda(), pres.cuda(), freq.cuda())
    torch.testing.assert_close(got.cpu(), want)
    off = 2000
    shard = apply_penalties(logits[:, off:3000].contiguous().cuda(), e.cuda(), rep.cuda(),
                            pres.cuda(), freq.cuda(), vocab_offset=off)
    torch.testing.assert_close(shard.cpu(), want[:, off:3000])


def test_engine_logprobs_on_gpu():
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.presets import tiny_llama
    cfg = tiny_llama()
    cfg.dtype = torch.bfloat16
    llm = LLM(cfg, block_size=64, seed=0, num_gpu_blocks=32, max_model_len=256, max_num_seqs=4,
              max_num_batched_tokens=256, cuda_graph_sizes=[1, 2, 4])
    g = torch.Generator().manual_seed(2)
    prompts = torch.randint(0, 1024, (3, 30), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True, logprobs=4,
                        repetition_penalty=1.2)
    outs = llm.generate(prompts, sp)
    for o in outs:
        c = o.outputs[0]
        assert len(c.logprobs) == 6
        for t, d in zip(c.token_ids, c.logprobs):
            assert t in d and len(d) >= 4 and all(v.logprob <= 0 for v in d.values())
    llm.shutdown()
