"""Speculative decoding on B200 (tiny Llama, bf16): drafts verified in multi-token steps
(prefill attention kernel) give the same tokens as plain decoding up to bf16 near-ties, and
verification steps run whole requests' drafts at once."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_oracle_drafts_cut_steps_and_keep_tokens():
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.presets import tiny_llama
    cfg = tiny_llama()
    cfg.dtype = torch.bfloat16
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (20, 64, 100)]
    sp = SamplingParams(temperature=0.0, max_tokens=32, ignore_eos=True)
    kw = dict(block_size=64, seed=0, num_gpu_blocks=64, max_model_len=512, max_num_seqs=8,
              max_num_batched_tokens=256, enforce_eager=True)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **kw).generate(prompts, sp)]
    llm = LLM(cfg, **kw)
    eng = llm.engine
    for i, p in enumerate(prompts):
        eng.add_request(f"r{i}", p, sp)
    iids = {eng._by_name[f"r{i}"]: i for i in range(3)}
    outs = {}
    while eng.has_unfinished_requests():
        for iid in eng.scheduler.decode_request_ids():
            done = len(eng.scheduler.output_tokens(iid))
            eng.scheduler.set_draft(iid, plain[iids[iid]][done:done + 4])
        for o in eng.step():
            outs[o.request_id] = o.outputs[0].token_ids
    got = [outs[f"r{i}"] for i in range(3)]
    agree = sum(a == b for x, y in zip(got, plain) for a, b in zip(x, y)) / sum(map(len, plain))
    assert agree > 0.9, agree
    assert eng.num_steps < 32  # several tokens accepted per verification step
    assert eng.scheduler.spec_accepted() > 0


def test_eagle_head_on_gpu_keeps_tokens():
    """EAGLE head over the bf16 tiny Llama: the draft layer runs the GEMM / RoPE-KV /
    paged-attention kernels on its extra cache layer after every step, and the verified outputs
    stay a greedy continuation of the target: teacher-forced against the fp32 reference, every
    emitted token is the argmax up to bf16 resolution (exact position-by-position agreement
    with plain decoding is not required: a bf16 near-tie may flip between the one-token decode
    kernel and the two-token verification step, after which the sequences part)."""
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.presets import tiny_llama
    from vllm_musa_b200.models.reference import ReferenceDecoder
    from vllm_musa_b200.models.weights import dummy_weights
    cfg = tiny_llama()
    cfg.dtype = torch.bfloat16
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (20, 64, 130)]
    sp = SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True)
    kw = dict(block_size=64, seed=0, num_gpu_blocks=64, max_model_len=512, max_num_seqs=8,
              max_num_batched_tokens=256)
    llm = LLM(cfg, speculative_config={"method": "eagle", "num_speculative_tokens": 1}, **kw)
    got = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert llm.engine.drafter.proposed > 0
    assert llm.engine.scheduler.spec_proposed() > 0
    llm.shutdown()
    ref_cfg = tiny_llama()
    W = {k: v.cpu() for k, v in dummy_weights(ref_cfg, seed=0, std=0.02, device="cuda")}
    ref = ReferenceDecoder(ref_cfg, W)
    for p, toks in zip(prompts, got):
        assert len(toks) == 16
        for k, t in enumerate(toks):
            want = ref.logits(p + toks[:k])[-1]
            gap = float(want.max() - want[t]) / float(want.abs().max())
            assert gap < 0.03, (k, gap)


def test_oracle_tree_drafts_compact_kv_on_gpu():
    """Draft trees whose right continuation is on a non-first branch (nodes 1 -> 3 -> 4): the
    tree-masked verification, the accepted-path KV copies and the next steps keep a greedy
    continuation of the target (teacher-forced against the fp32 reference: every emitted token
    is the argmax up to bf16 resolution; a bf16 near-tie may part the sequence from the plain
    run's, after which its drafts are simply rejected) while cutting the step count."""
    from vllm_musa_b200 import LLM, SamplingParams
    from vllm_musa_b200.models.presets import tiny_llama
    from vllm_musa_b200.models.reference import ReferenceDecoder
    from vllm_musa_b200.models.weights import dummy_weights
    cfg = tiny_llama()
    cfg.dtype = torch.bfloat16
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (20, 64, 100)]
    sp = SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True)
    kw = dict(block_size=64, seed=0, num_gpu_blocks=64, max_model_len=512, max_num_seqs=8,
              max_num_batched_tokens=256, enforce_eager=True)
    plain = [o.outputs[0].token_ids for o in LLM(cfg, **kw).generate(prompts, sp)]
    llm = LLM(cfg, **kw)
    eng = llm.engine
    for i, p in enumerate(prompts):
        eng.add_request(f"r{i}", p, sp)
    iids = {eng._by_name[f"r{i}"]: i for i in range(3)}
    outs = {}
    while eng.has_unfinished_requests():
        for iid in eng.scheduler.decode_request_ids():
            done = len(eng.scheduler.output_tokens(iid))
            right = plain[iids[iid]][done:done + 3]
            if len(right) < 3:
                continue
            wrong = [(t + 1) % 1024 for t in right]
            eng.scheduler.set_draft_tree(iid, [wrong[0], right[0], wrong[1], right[1], right[2],
                                               wrong[2]], [-1, -1, 1, 1, 3, 0])
        for o in eng.step():
            outs[o.request_id] = o.outputs[0].token_ids
    got = [outs[f"r{i}"] for i in range(3)]
    assert eng.num_steps < 25
    assert eng.scheduler.spec_accepted() > 0
    ref_cfg = tiny_llama()
    W = {k: v.cpu() for k, v in dummy_weights(ref_cfg, seed=0, std=0.02, device="cuda")}
    ref = ReferenceDecoder(ref_cfg, W)
    for p, toks in zip(prompts, got):
        assert len(toks) == 30
        for k, t in enumerate(toks):
            want = ref.logits(p + toks[:k])[-1]
            gap = float(want.max() - want[t]) / float(want.abs().max())
            assert gap < 0.03, (k, gap)
