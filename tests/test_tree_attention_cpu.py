"""Tree attention on CPU: ancestor masks, a chain tree equals causal prefill, and each node's
output equals plain attention over the context plus its root-to-node path."""
import math

import torch

from vllm_musa_b200 import ops
from vllm_musa_b200.attention import TreeAttention
from vllm_musa_b200.ops.attention import tree_ancestor_masks


def test_ancestor_masks():
    m = tree_ancestor_masks([-1, 0, 0, 1, -1])
    assert m.tolist() == [0b1, 0b11, 0b101, 0b1011, 0b10000]
    big = tree_ancestor_masks(list(range(-1, 63)))  # a 64-node chain sets the sign bit
    assert int(big[63]) < 0


def _case(ctx, parents, Hq=4, Hkv=2, D=64, bs=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    n = ctx + len(parents)
    nb = (n + bs - 1) // bs
    kc = torch.randn(nb + 2, Hkv, bs, D, generator=g)
    vc = torch.randn(nb + 2, Hkv, bs, D, generator=g)
    bt = torch.randperm(nb + 2, generator=g)[:nb].to(torch.int32).view(1, -1)
    q = torch.randn(len(parents), Hq * D, generator=g)
    cu = torch.tensor([0, len(parents)], dtype=torch.int32)
    sl = torch.tensor([n], dtype=torch.int32)
    return q, kc, vc, bt, cu, sl


def test_chain_tree_is_causal():
    q, kc, vc, bt, cu, sl = _case(20, [-1, 0, 1, 2, 3])
    att = TreeAttention(4, 2, 64)
    tree = att.forward_tree(q, kc, vc, cu, sl, bt, tree_ancestor_masks([-1, 0, 1, 2, 3]))
    causal = ops.paged_prefill(q, kc, vc, cu, sl, bt, 4, 2, 1 / 8)
    torch.testing.assert_close(tree, causal)


def test_node_sees_context_and_its_path():
    parents = [-1, 0, 0, 1, 2, -1, 5]
    ctx = 13
    q, kc, vc, bt, cu, sl = _case(ctx, parents, seed=1)
    out = TreeAttention(4, 2, 64).forward_tree(q, kc, vc, cu, sl, bt,
                                               tree_ancestor_masks(parents))
    n = ctx + len(parents)
    k = ops.attention._gather_kv(kc, bt[0], n)
    v = ops.attention._gather_kv(vc, bt[0], n)
    for i in range(len(parents)):
        path, j = [], i
        while j >= 0:
            path.append(ctx + j)
            j = parents[j]
        idx = torch.tensor(list(range(ctx)) + sorted(path))
        for h in range(4):
            kh = k[idx, h // 2]
            p = torch.softmax(kh @ q[i, h * 64:(h + 1) * 64] / math.sqrt(64), -1)
            torch.testing.assert_close(out[i, h * 64:(h + 1) * 64], p @ v[idx, h // 2],
                                       rtol=1e-4, atol=1e-5)
