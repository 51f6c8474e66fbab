"""Token-tree speculative decoding on CPU.  A verification step runs the pending token and
every node of a draft tree under ancestor masks (position = pending + 1 + depth, KV slot =
pending + 1 + node index); the scheduler follows the drawn tokens down the tree and the KV of
the accepted path is copied to consecutive slots before the next step.  Outputs must equal
plain decoding (greedy and sampled) while the right continuation sits on a non-first branch,
so the compaction is exercised; the n-gram trie proposer and EAGLE sibling drafts are checked
end to end."""
import pytest
import torch

from vllm_musa_b200 import LLM, SamplingParams
from vllm_musa_b200.models.presets import tiny_llama

V = 1024


def _llm(**kw):
    a = dict(device="cpu", block_size=16, seed=0, num_gpu_blocks=64, max_model_len=128,
             max_num_seqs=4, max_num_batched_tokens=96)
    a.update(kw)
    return LLM(tiny_llama(), **a)


def _prompts():
    g = torch.Generator().manual_seed(5)
    base = torch.randint(0, V, (12,), generator=g).tolist()
    rep = (base * 4)[:40]
    rnd = torch.randint(0, V, (33,), generator=g).tolist()
    return [rep, rnd, rep[:25]]


def _oracle_tree(right):
    """Tree whose right path is nodes 1 -> 3 -> 4 (wrong siblings at 0, 2, 5): accepting it
    moves node 3 and node 4's KV down by one and two slots."""
    w = [(t + 1) % V for t in right] + [0, 0, 0]
    toks, par = [], []
    if len(right) >= 1:
        toks += [w[0], right[0]]
        par += [-1, -1]
    if len(right) >= 2:
        toks += [w[1], right[1]]
        par += [1, 1]
    if len(right) >= 3:
        toks += [right[2], w[2]]
        par += [3, 0]
    return toks, par


def _drive(temperature, max_tokens=20):
    sp = SamplingParams(temperature=temperature, max_tokens=max_tokens, ignore_eos=True,
                        seed=11)
    plain = [o.outputs[0].token_ids for o in _llm().generate(_prompts(), sp)]
    llm = _llm()
    eng = llm.engine
    for i, p in enumerate(_prompts()):
        eng.add_request(f"r{i}", p, sp)
    iids = {eng._by_name[f"r{i}"]: i for i in range(3)}
    outs = {}
    while eng.has_unfinished_requests():
        for iid in eng.scheduler.decode_request_ids():
            done = len(eng.scheduler.output_tokens(iid))
            toks, par = _oracle_tree(plain[iids[iid]][done:done + 3])
            eng.scheduler.set_draft_tree(iid, toks, par)
        for o in eng.step():
            outs[o.request_id] = o.outputs[0].token_ids
    return [outs[f"r{i}"] for i in range(3)], plain, eng


def test_oracle_tree_greedy_matches_plain_with_compaction():
    got, plain, eng = _drive(0.0)
    assert got == plain
    assert eng.scheduler.spec_accepted() > 0
    assert eng.num_steps < 20  # three tokens per verification step


def test_oracle_tree_sampled_matches_plain():
    """Every node row draws with the noise of the output index its token would take, so the
    sampled run equals plain sampling too."""
    got, plain, eng = _drive(0.8)
    assert got == plain
    assert eng.scheduler.spec_accepted() > 0


def test_kv_moves_follow_the_accepted_path():
    llm = _llm()
    eng = llm.engine
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    ref = [o.outputs[0].token_ids for o in _llm().generate([_prompts()[1]], sp)][0]
    eng.add_request("a", _prompts()[1], sp)
    eng.step()  # prefill: first token
    iid = eng._by_name["a"]
    toks, par = _oracle_tree(ref[1:4])
    eng.scheduler.set_draft_tree(iid, toks, par)
    moves = []
    take = eng.scheduler.take_kv_moves

    class _Spy:
        def __getattr__(self, n):
            return getattr(sch, n)

        def take_kv_moves(self):
            m = take()
            moves.extend(m)
            return m

    sch = eng.scheduler
    eng.scheduler = _Spy()
    eng.step()
    eng.scheduler = sch
    assert sch.last_path(iid) == [1, 3, 4]
    n = len(_prompts()[1]) + 1  # first draft's index (the only request: blocks in order)
    assert [(s - d) for s, d in moves] == [1, 2, 2]
    assert [d % 16 for _, d in moves] == [(n + k) % 16 for k in range(3)]
    assert list(sch.output_tokens(iid)) == ref[:5]


def test_ngram_trie_proposer_shapes():
    llm = _llm()
    eng = llm.engine
    sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)
    # the suffix [7, 8] occurs twice before with continuations 1 2 3 and 5 6 ...
    prompt = [7, 8, 1, 2, 3, 9, 7, 8, 5, 6, 4, 9, 7, 8]
    eng.add_request("a", prompt, sp)
    eng.step()
    iid = eng._by_name["a"]
    tok = eng.scheduler.output_tokens(iid)[0]
    L = len(prompt) + 1
    seq = prompt + [tok]
    n = eng.scheduler.propose_ngram_tree(6, 1, 3, 2)
    info = eng.scheduler.request_info(iid)
    d, par = list(info["draft"]), list(info["draft_parent"])
    assert n == len(d) == len(par) <= 6
    assert all(-1 <= p < j for j, p in enumerate(par))
    # every root-to-node path spells a continuation of an earlier occurrence of a suffix
    for j in range(len(d)):
        path, k = [], j
        while k >= 0:
            path.append(d[k])
            k = par[k]
        path.reverse()
        ok = False
        for st in range(L - 1):
            cont = seq[st:st + len(path)]
            if cont == path and st > 0 and seq[st - 1] == seq[-1]:
                ok = True
        assert ok, path
    # a single continuation gives a chain (no parents kept)
    n1 = eng.scheduler.propose_ngram_tree(4, 1, 3, 1)
    info = eng.scheduler.request_info(iid)
    assert n1 == len(info["draft"]) and list(info["draft_parent"]) == []


def test_ngram_tree_spec_end_to_end():
    sp = SamplingParams(temperature=0.0, max_tokens=24, ignore_eos=True)
    plain = [o.outputs[0].token_ids for o in _llm().generate(_prompts(), sp)]
    llm = _llm(speculative_config={"method": "ngram", "num_speculative_tokens": 6,
                                   "tree_width": 3})
    trees = []
    eng = llm.engine
    run = eng.runner.execute

    def spy(plan, extras=None):
        trees.append(plan.tree)
        return run(plan, extras)

    eng.runner.execute = spy
    outs = [o.outputs[0].token_ids for o in llm.generate(_prompts(), sp)]
    assert outs == plain
    assert any(trees) and eng.scheduler.spec_accepted() > 0


def test_eagle_sibling_tree_matches_plain():
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    plain = [o.outputs[0].token_ids for o in _llm().generate(_prompts(), sp)]
    llm = _llm(speculative_config={"method": "eagle", "num_speculative_tokens": 1,
                                   "speculative_token_tree": "[(0,), (1,), (2,)]"})
    assert llm.engine.drafter.tree_width == 3
    trees = []
    run = llm.engine.runner.execute

    def spy(plan, extras=None):
        trees.append(plan.tree)
        return run(plan, extras)

    llm.engine.runner.execute = spy
    outs = [o.outputs[0].token_ids for o in llm.generate(_prompts(), sp)]
    assert outs == plain
    assert any(trees)
    assert llm.engine.drafter.proposed > 0


def test_tree_config_and_contract():
    from vllm_musa_b200.config import SpeculativeConfig
    assert SpeculativeConfig(method="eagle", num_speculative_tokens=1,
                             speculative_token_tree="[(0,), (1,)]").tree_width == 2
    with pytest.raises(ValueError):
        SpeculativeConfig(method="eagle", speculative_token_tree="[(0,), (0, 0)]")
    with pytest.raises(ValueError):
        _llm(speculative_config={"method": "mtp", "num_speculative_tokens": 1,
                                 "tree_width": 2})
    with pytest.raises(ValueError):
        _llm(kv_cache_dtype="fp8",
             speculative_config={"method": "ngram", "num_speculative_tokens": 4,
                                 "tree_width": 2})


def test_set_draft_tree_validates():
    llm = _llm()
    eng = llm.engine
    eng.add_request("a", [1, 2, 3], SamplingParams(max_tokens=4, ignore_eos=True))
    eng.step()
    iid = eng._by_name["a"]
    with pytest.raises(ValueError):
        eng.scheduler.set_draft_tree(iid, [1, 2], [-1, 1])  # parent does not precede
    with pytest.raises(ValueError):
        eng.scheduler.set_draft_tree(iid, [1] * 64, [-1] * 64)  # > 63 nodes
    eng.scheduler.set_draft_tree(iid, [4, 5, 6], [-1, 0, 1])  # a chain: stored without parents
    assert list(eng.scheduler.request_info(iid)["draft_parent"]) == []


def test_mixed_causal_and_tree_rows_cpu():
    """A step batching a prefill chunk (zero mask rows = causal) with a tree request: each
    part equals its own attention computed alone."""
    from vllm_musa_b200 import ops
    from vllm_musa_b200.ops.attention import tree_ancestor_masks
    g = torch.Generator().manual_seed(0)
    Hq, Hkv, D, bs = 4, 2, 64, 16
    kc = torch.randn(8, Hkv, bs, D, generator=g)
    vc = torch.randn(8, Hkv, bs, D, generator=g)
    bt = torch.tensor([[0, 1, 2, 3], [4, 5, 6, 7]], dtype=torch.int32)
    tree = [-1, 0, 0, 1]
    masks = torch.cat([torch.tensor([1]), (tree_ancestor_masks(tree) << 1) | 1])
    q = torch.randn(10 + 5, Hq * D, generator=g)
    lens = torch.tensor([30, 25], dtype=torch.int32)
    cu = torch.tensor([0, 10, 15], dtype=torch.int32)
    tm = torch.cat([torch.zeros(10, dtype=torch.int64), masks])
    both = ops.paged_prefill(q, kc, vc, cu, lens, bt, Hq, Hkv, D ** -0.5, tree_mask=tm)
    causal = ops.paged_prefill(q[:10], kc, vc, cu[:2], lens[:1], bt[:1], Hq, Hkv, D ** -0.5)
    alone = ops.paged_prefill(q[10:], kc, vc, torch.tensor([0, 5], dtype=torch.int32),
                              lens[1:], bt[1:], Hq, Hkv, D ** -0.5, tree_mask=masks)
    torch.testing.assert_close(both[:10], causal)
    torch.testing.assert_close(both[10:], alone)


def test_tree_pruned_by_token_budget_and_max_tokens():
    """Trees cut by the step's token budget (node count) and by the request's remaining tokens
    (depth) still verify exactly: outputs equal plain decoding, max_tokens is never exceeded."""
    for budget, max_tokens in ((8, 7), (12, 5), (40, 3)):
        sp = SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True)
        plain = [o.outputs[0].token_ids for o in _llm().generate(_prompts(), sp)]
        llm = _llm(max_num_batched_tokens=max(budget, 48))
        eng = llm.engine
        for i, p in enumerate(_prompts()):
            eng.add_request(f"r{i}", p, sp)
        iids = {eng._by_name[f"r{i}"]: i for i in range(3)}
        outs = {}
        while eng.has_unfinished_requests():
            for iid in eng.scheduler.decode_request_ids():
                done = len(eng.scheduler.output_tokens(iid))
                right = plain[iids[iid]][done:done + 6] + [0] * 6
                # a deep chain along the right path with a wrong sibling at every level
                toks, par = [], []
                prev = -1
                for d in range(6):
                    toks += [(right[d] + 1) % V, right[d]]
                    par += [prev, prev]
                    prev = len(toks) - 1
                eng.scheduler.set_draft_tree(iid, toks, par)
            for o in eng.step():
                outs[o.request_id] = o.outputs[0].token_ids
        got = [outs[f"r{i}"] for i in range(3)]
        assert got == plain, (budget, max_tokens)
        assert all(len(g) == max_tokens for g in got)


def test_tree_verification_under_preemption():
    """A pool too small for all requests preempts (recomputes) requests while they verify
    trees; the outputs still equal plain decoding."""
    sp = SamplingParams(temperature=0.0, max_tokens=24, ignore_eos=True)
    kw = dict(num_gpu_blocks=9, max_model_len=96)
    plain = [o.outputs[0].token_ids for o in _llm(**kw).generate(_prompts(), sp)]
    llm = _llm(**kw)
    eng = llm.engine
    for i, p in enumerate(_prompts()):
        eng.add_request(f"r{i}", p, sp)
    iids = {eng._by_name[f"r{i}"]: i for i in range(3)}
    outs, preempted = {}, []
    run = eng.runner.execute

    def spy(plan, extras=None):
        preempted.append(plan.num_preempted)
        return run(plan, extras)

    eng.runner.execute = spy
    while eng.has_unfinished_requests():
        for iid in eng.scheduler.decode_request_ids():
            done = len(eng.scheduler.output_tokens(iid))
            toks, par = _oracle_tree(plain[iids[iid]][done:done + 3])
            eng.scheduler.set_draft_tree(iid, toks, par)
        for o in eng.step():
            outs[o.request_id] = o.outputs[0].token_ids
    assert sum(preempted) > 0
    assert [outs[f"r{i}"] for i in range(3)] == plain
