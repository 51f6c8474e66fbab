"""Graph fusion passes on CPU: traced graphs with all_reduce -> fused_add_rms_norm and
silu_and_mul -> group_quant_fp8 chains are rewritten to the fused ops, the rewritten module
computes the same values, and chains whose intermediate has other users are left alone."""
import torch
import torch.fx as fx

from vllm_musa_b200.compile import B200PassManager
from vllm_musa_b200.compile import passes as P  # noqa: F401  (registers torch.ops.b200fx)

ops = torch.ops.b200fx


class Block(torch.nn.Module):
    def forward(self, x, residual, w, gu):
        a = ops.all_reduce(x)
        y, r = ops.fused_add_rms_norm(a, residual, w, 1e-6)
        h = ops.silu_and_mul(gu)
        q, s = ops.group_quant_fp8(h)
        return y, r, q, s


class NormQuant(torch.nn.Module):
    """Input norm feeding an fp8 GEMM, then a residual norm feeding another."""
    def forward(self, x, residual, w):
        q0, s0 = ops.group_quant_fp8(ops.rms_norm(x, w, 1e-6))
        y, r = ops.fused_add_rms_norm(x, residual, w, 1e-6)
        q1, s1 = ops.group_quant_fp8(y)
        return q0, s0, q1, s1, r * 2


class Shared(torch.nn.Module):
    def forward(self, x, residual, w):
        a = ops.all_reduce(x)
        y, r = ops.fused_add_rms_norm(a, residual, w, 1e-6)
        return y, r, a * 2  # the all-reduce output has another user: no fusion


def _names(gm):
    return [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]


def test_fusions_rewrite_and_preserve_values():
    g = torch.Generator().manual_seed(0)
    x, res = torch.randn(5, 256, generator=g), torch.randn(5, 256, generator=g)
    w, gu = torch.rand(256, generator=g), torch.randn(5, 512, generator=g)
    gm = fx.symbolic_trace(Block())
    ref = gm(x, res, w, gu)
    pm = B200PassManager()
    assert pm(gm.graph) == 2
    gm.recompile()
    names = " ".join(_names(gm))
    assert "allreduce_add_rms_norm" in names and "silu_mul_fp8_quant" in names
    assert "b200fx.all_reduce" not in names and "group_quant_fp8" not in names
    out = gm(x, res, w, gu)
    torch.testing.assert_close(out[0], ref[0])
    torch.testing.assert_close(out[1], ref[1])
    torch.testing.assert_close(out[2].float(), ref[2].float())
    torch.testing.assert_close(out[3], ref[3])
    assert pm.stats == {"allreduce_rmsnorm": 1, "silu_mul_quant": 1, "rms_norm_quant": 0}


def test_rms_norm_quant_fusion():
    g = torch.Generator().manual_seed(1)
    x, res = torch.randn(6, 256, generator=g), torch.randn(6, 256, generator=g)
    w = torch.rand(256, generator=g) + 0.5
    gm = fx.symbolic_trace(NormQuant())
    ref = gm(x, res, w)
    pm = B200PassManager()
    assert pm(gm.graph) == 2
    gm.graph.lint()
    gm.recompile()
    names = " ".join(_names(gm))
    assert "b200fx.rms_norm_quant_fp8" in names and "add_rms_norm_quant_fp8" in names
    assert "group_quant_fp8" not in names and "b200fx.fused_add_rms_norm" not in names
    out = gm(x, res, w)
    for o, r in zip(out, ref):
        torch.testing.assert_close(o.float(), r.float())
    assert pm.stats["rms_norm_quant"] == 2


def test_rms_norm_quant_not_fused_when_norm_output_shared():
    class M(torch.nn.Module):
        def forward(self, x, residual, w):
            y, r = ops.fused_add_rms_norm(x, residual, w, 1e-6)
            q, s = ops.group_quant_fp8(y)
            return q, s, y + r   # the bf16 normalised row is still needed
    gm = fx.symbolic_trace(M())
    assert B200PassManager([P.RMSNormQuantFusionPass()])(gm.graph) == 0


def test_no_fusion_when_intermediate_is_shared():
    gm = fx.symbolic_trace(Shared())
    pm = B200PassManager().configure(None)
    assert pm(gm.graph) == 0
    assert len(pm.uuid()) == 64


def test_vllm_pass_manager_hook():
    import pytest
    pm_mod = pytest.importorskip("vllm.compilation.passes.pass_manager")
    from vllm_musa_b200.compile.vllm_pass_manager import B200PostGradPassManager, b200_passes
    from vllm_musa_b200.platform import B200Platform
    assert issubclass(B200PostGradPassManager, pm_mod.PostGradPassManager)
    assert B200Platform.get_pass_manager_cls().endswith("B200PostGradPassManager")
    ps = b200_passes()
    assert len(ps) == 3 and all(p.is_applicable_for_range(None) for p in ps)


def test_allreduce_fusion_never_drops_the_reduction(monkeypatch):
    """An all-reduce over a named vLLM group, fused with the add + RMSNorm after it, keeps the
    group name; with no communicator bound to that group the fused op still reduces over it
    (here a stand-in for two ranks holding the same partial sums)."""
    import pytest
    pytest.importorskip("vllm.distributed.parallel_state")

    class M(torch.nn.Module):
        def forward(self, x, residual, w):
            a = torch.ops.vllm.all_reduce(x, "tp:0")
            y, r = ops.fused_add_rms_norm(a, residual, w, 1e-6)
            return y, r

    g = torch.Generator().manual_seed(2)
    x, res = torch.randn(4, 256, generator=g), torch.randn(4, 256, generator=g)
    w = torch.rand(256, generator=g)
    gm = fx.symbolic_trace(M())
    assert B200PassManager([P.AllReduceRMSNormFusionPass()])(gm.graph) == 1
    gm.recompile()
    fused = [n for n in gm.graph.nodes if "allreduce_add_rms_norm" in str(n.target)]
    assert len(fused) == 1 and fused[0].args[4] == "tp:0"
    seen = []

    def fake_all_reduce(t, group_name):
        seen.append(group_name)
        return t * 2

    monkeypatch.setattr(P, "_vllm_all_reduce", fake_all_reduce)
    y, r = gm(x, res, w)
    ry, rr = P._fused_add_rms_norm(x * 2, res, w, 1e-6)
    assert seen == ["tp:0"]
    torch.testing.assert_close(y, ry)
    torch.testing.assert_close(r, rr)


_TLIB = torch.library.Library("b200fxtest", "DEF")
_TLIB.define("fused_add_rms_norm_(Tensor(a!) input, Tensor(b!) residual, Tensor weight, "
             "float epsilon) -> ()")


def _inplace_add_rms(inp, residual, weight, epsilon):
    y, r = P._fused_add_rms_norm(inp, residual, weight, epsilon)
    inp.copy_(y)
    residual.copy_(r)


_TLIB.impl("fused_add_rms_norm_", _inplace_add_rms, "CompositeExplicitAutograd")


def test_allreduce_fusion_matches_inplace_norm_under_auto_functionalized(monkeypatch):
    """vLLM's in-place fused_add_rms_norm appears in post-grad graphs as
    auto_functionalized(op, input=, residual=, weight=, epsilon=) with getitem 1 / 2 users;
    the pass rewrites it (here with a stand-in in-place op of the same schema)."""
    import operator
    monkeypatch.setattr(P, "ADD_RMS_INPLACE", P.ADD_RMS_INPLACE + ("b200fxtest.fused_add_rms_norm_",))
    gr = fx.Graph()
    x, r, w = gr.placeholder("x"), gr.placeholder("r"), gr.placeholder("w")
    ar = gr.call_function(torch.ops.b200fx.all_reduce.default, (x,))
    af = gr.call_function(torch.ops.higher_order.auto_functionalized,
                          (torch.ops.b200fxtest.fused_add_rms_norm_.default,),
                          {"input": ar, "residual": r, "weight": w, "epsilon": 1e-6})
    y = gr.call_function(operator.getitem, (af, 1))
    rr = gr.call_function(operator.getitem, (af, 2))
    gr.output((y, rr))
    gm = fx.GraphModule(torch.nn.Module(), gr)
    g = torch.Generator().manual_seed(3)
    xv, rv = torch.randn(3, 256, generator=g), torch.randn(3, 256, generator=g)
    wv = torch.rand(256, generator=g)
    ref = gm(xv, rv.clone(), wv)
    assert P.AllReduceRMSNormFusionPass()(gm.graph) == 1
    gm.graph.lint()
    gm.recompile()
    names = " ".join(_names(gm))
    assert "auto_functionalized" not in names and "allreduce_add_rms_norm" in names
    out = gm(xv, rv.clone(), wv)
    torch.testing.assert_close(out[0], ref[0])
    torch.testing.assert_close(out[1], ref[1])
