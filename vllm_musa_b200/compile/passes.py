"""Post-grad style graph passes: pattern-match unfused op chains in a torch.fx graph and replace
them with the fused ops of this package.

* ``AllReduceRMSNormFusionPass``  all_reduce(x) -> fused_add_rms_norm(x, residual, w, eps)
  becomes one ``allreduce_add_rms_norm`` (the NVSwitch all-reduce + residual + RMSNorm kernel).
* ``SiluMulQuantFusionPass``      silu_and_mul(x) -> group_quant_fp8(y) becomes one
  ``silu_mul_fp8_quant`` (SwiGLU + 1x128 e4m3 quantisation in one kernel).
* ``RMSNormQuantFusionPass``      rms_norm(x, w, eps) -> group_quant_fp8(y) becomes one
  ``rms_norm_quant_fp8``, and fused_add_rms_norm(x, r, w, eps)[0] -> group_quant_fp8 one
  ``add_rms_norm_quant_fp8`` (residual add + RMSNorm + 1x128 e4m3 quantisation in one pass
  over the row; the updated residual stays an output).

Ops are matched by qualified name, so graphs traced from this package's ``torch.ops.b200fx.*``
ops and graphs holding vLLM's equivalents (``vllm.all_reduce``, ``_C.fused_add_rms_norm``,
``_C.silu_and_mul``, ``_C.per_token_group_fp8_quant``) are both rewritten.  A pass is a callable
on ``torch.fx.Graph`` with a ``uuid()`` (the interface vLLM's pass manager and Inductor's
custom post-grad pass hook expect).

Reference counterparts: vllm_musa/compilation/passes/pass_manager.py:59-83 (pass manager),
vllm_musa/_inductor/musa_allreduce_rms_fusion.py:103-844 (AR + RMSNorm fusion),
vllm_musa/compilation/passes/silu_deepgemm_fusion.py:19-85 (SiLU + quant fusion),
vllm_musa/compilation/passes/rms_deepgemm_fusion.py:18-91 (residual RMSNorm + quant fusion).
"""
from __future__ import annotations

import hashlib
import operator
from typing import Callable, Iterable, List, Optional

import torch
import torch.fx as fx

# --------------------------------------------------------------------------------------------
# Traceable ops (CPU implementations; CUDA tensors dispatch to the package's kernels)
# --------------------------------------------------------------------------------------------
_LIB = torch.library.Library("b200fx", "DEF")
_LIB.define("all_reduce(Tensor x) -> Tensor")
_LIB.define("fused_add_rms_norm(Tensor x, Tensor residual, Tensor w, float eps) -> (Tensor, Tensor)")
_LIB.define("allreduce_add_rms_norm(Tensor x, Tensor residual, Tensor w, float eps, "
            "str? group_name=None) -> (Tensor, Tensor)")
_LIB.define("silu_and_mul(Tensor x) -> Tensor")
_LIB.define("group_quant_fp8(Tensor x) -> (Tensor, Tensor)")
_LIB.define("silu_mul_fp8_quant(Tensor x) -> (Tensor, Tensor)")
_LIB.define("rms_norm(Tensor x, Tensor w, float eps) -> Tensor")
_LIB.define("rms_norm_quant_fp8(Tensor x, Tensor w, float eps) -> (Tensor, Tensor)")
_LIB.define("add_rms_norm_quant_fp8(Tensor x, Tensor residual, Tensor w, float eps) "
            "-> (Tensor, Tensor, Tensor)")

# TP communicators the fused all-reduce op may use, by the name of the process group whose
# all-reduce the pass replaced (None: this package's own b200fx.all_reduce).  A graph whose
# group has no communicator bound keeps the group's own all-reduce (vLLM's, by group name):
# the rewrite never drops a reduction.
_COMMS: dict = {}


def set_communicator(comm, group_name: Optional[str] = None) -> None:
    """Bind ``comm`` (a TPCommunicator) to the all-reduces of ``group_name``."""
    if comm is None:
        _COMMS.pop(group_name, None)
    else:
        _COMMS[group_name] = comm


def _bound(group_name: Optional[str] = None):
    c = _COMMS.get(group_name)
    return c if c is not None and getattr(c, "world", 1) > 1 else None


def _vllm_all_reduce(x, group_name: str):
    """vLLM's own all-reduce over the named group (the op the fusion replaced)."""
    return torch.ops.vllm.all_reduce(x, group_name)


def _all_reduce(x):
    c = _bound(None)
    if c is None:
        return x.clone()
    return c.all_reduce(x.clone())


def _fused_add_rms_norm(x, residual, w, eps):
    from .. import ops
    r = (x.float() + residual.float()).to(x.dtype)
    return ops.rms_norm(r, w, eps), r


def _allreduce_add_rms_norm(x, residual, w, eps, group_name=None):
    c = _bound(group_name)
    if c is not None:
        out, res = c.allreduce_add_rmsnorm(x.clone(), residual.clone(), w, eps)
        return out.clone(), res
    x = _vllm_all_reduce(x, group_name) if group_name is not None else _all_reduce(x)
    return _fused_add_rms_norm(x, residual, w, eps)


def _silu_and_mul(x):
    from .. import ops
    return ops.silu_and_mul(x)


def _group_quant(x):
    from ..ops.activation import group_quant_fp8
    return group_quant_fp8(x)


def _silu_mul_quant(x):
    from ..ops.activation import silu_mul_fp8_quant
    return silu_mul_fp8_quant(x)


def _rms_norm(x, w, eps):
    from .. import ops
    return ops.rms_norm(x, w, eps)


def _rms_norm_quant(x, w, eps):
    from .. import ops
    q, sc, _ = ops.rms_norm_quant_fp8(x, w, eps)
    return q, sc


def _add_rms_norm_quant(x, residual, w, eps):
    from .. import ops
    r = residual.clone()
    q, sc, _ = ops.rms_norm_quant_fp8(x, w, eps, residual=r)
    return q, sc, r


for _name, _fn in (("all_reduce", _all_reduce), ("fused_add_rms_norm", _fused_add_rms_norm),
                   ("rms_norm", _rms_norm), ("rms_norm_quant_fp8", _rms_norm_quant),
                   ("add_rms_norm_quant_fp8", _add_rms_norm_quant),
                   ("allreduce_add_rms_norm", _allreduce_add_rms_norm),
                   ("silu_and_mul", _silu_and_mul), ("group_quant_fp8", _group_quant),
                   ("silu_mul_fp8_quant", _silu_mul_quant)):
    _LIB.impl(_name, _fn, "CompositeExplicitAutograd")

# --------------------------------------------------------------------------------------------
# Matching helpers
# --------------------------------------------------------------------------------------------
ALL_REDUCE = ("b200fx.all_reduce", "vllm.all_reduce")
# functional add + RMSNorm returning (normalised, residual): this package's traceable op and
# vLLM's IR op (vllm.ir.ops.fused_add_rms_norm, default and maybe_inplace overloads)
ADD_RMS = ("b200fx.fused_add_rms_norm", "vllm_ir.fused_add_rms_norm")
# in-place add + RMSNorm (vLLM's _C.fused_add_rms_norm mutates input and residual); in
# post-grad graphs it sits under auto_functionalized, whose output tuple is
# (None, input', residual')
ADD_RMS_INPLACE = ("_C.fused_add_rms_norm",)
SILU_MUL = ("b200fx.silu_and_mul", "_C.silu_and_mul")
GROUP_QUANT = ("b200fx.group_quant_fp8", "_C.per_token_group_fp8_quant")
RMS_NORM = ("b200fx.rms_norm",)


def _qual(target) -> str:
    name = getattr(target, "_qualified_op_name", None) or getattr(target, "__name__", "")
    if hasattr(target, "_schema"):
        name = str(target._schema.name).replace("::", ".")
    elif hasattr(target, "_qualified_op_name"):
        name = target._qualified_op_name.replace("::", ".")
    return name


def _is(node: fx.Node, names: Iterable[str]) -> bool:
    return node.op == "call_function" and any(_qual(node.target).startswith(n) for n in names)


class _Pass:
    name = "pass"

    def uuid(self) -> str:
        src = self.__class__.__name__ + self.name
        return hashlib.sha256(src.encode()).hexdigest()

    def __call__(self, graph: fx.Graph) -> int:
        raise NotImplementedError


def _auto_functionalized_of(node: fx.Node, names: Iterable[str]) -> bool:
    return (node.op == "call_function" and node.args and
            node.target is getattr(torch.ops.higher_order, "auto_functionalized", None) and
            any(_qual(node.args[0]).startswith(n) for n in names))


class AllReduceRMSNormFusionPass(_Pass):
    """all_reduce(x) whose only user is an add + RMSNorm of it (functional
    ``fused_add_rms_norm(ar, residual, w, eps)`` or vLLM's in-place ``_C.fused_add_rms_norm``
    under ``auto_functionalized``).  The fused node carries the all-reduce's process-group
    name, so without a bound communicator it still reduces over that group."""
    name = "allreduce_rmsnorm"

    @staticmethod
    def _source(x) -> Optional[fx.Node]:
        if isinstance(x, fx.Node) and _is(x, ALL_REDUCE) and len(x.users) == 1:
            return x
        return None

    @staticmethod
    def _fused(graph, ar: fx.Node, residual, w, eps) -> fx.Node:
        group = ar.args[1] if len(ar.args) > 1 else ar.kwargs.get("group_name")
        return graph.call_function(torch.ops.b200fx.allreduce_add_rms_norm.default,
                                   (ar.args[0], residual, w, eps, group))

    def __call__(self, graph: fx.Graph) -> int:
        n = 0
        for node in list(graph.nodes):
            if _is(node, ADD_RMS):
                if len(node.args) > 4 and node.args[4] is not None:
                    continue  # variance over a prefix of the row: not this kernel
                src = self._source(node.args[0])
                if src is None:
                    continue
                with graph.inserting_before(node):
                    fused = self._fused(graph, src, *node.args[1:4])
                node.replace_all_uses_with(fused)
                graph.erase_node(node)
                graph.erase_node(src)
                n += 1
            elif _auto_functionalized_of(node, ADD_RMS_INPLACE):
                kw = node.kwargs
                src = self._source(kw.get("input"))
                if src is None or not all(u.target is operator.getitem and u.args[1] in (1, 2)
                                          for u in node.users):
                    continue
                with graph.inserting_before(node):
                    fused = self._fused(graph, src, kw["residual"], kw["weight"], kw["epsilon"])
                for u in list(node.users):
                    with graph.inserting_before(u):
                        g = graph.call_function(operator.getitem, (fused, u.args[1] - 1))
                    u.replace_all_uses_with(g)
                    graph.erase_node(u)
                graph.erase_node(node)
                graph.erase_node(src)
                n += 1
        return n


class SiluMulQuantFusionPass(_Pass):
    """group_quant_fp8(silu_and_mul(x)) with the activation used only by the quantiser."""
    name = "silu_mul_quant"

    def __call__(self, graph: fx.Graph) -> int:
        n = 0
        for node in list(graph.nodes):
            if not _is(node, GROUP_QUANT):
                continue
            act = node.args[0]
            if not isinstance(act, fx.Node) or not _is(act, SILU_MUL) or len(act.users) != 1:
                continue
            with graph.inserting_before(node):
                fused = graph.call_function(torch.ops.b200fx.silu_mul_fp8_quant.default,
                                            (act.args[0],))
            node.replace_all_uses_with(fused)
            graph.erase_node(node)
            graph.erase_node(act)
            n += 1
        return n


class RMSNormQuantFusionPass(_Pass):
    """group_quant_fp8(rms_norm(x, w, eps)) and group_quant_fp8(fused_add_rms_norm(x, r, w,
    eps)[0]), with the normalised row used only by the quantiser (an fp8 GEMM's input)."""
    name = "rms_norm_quant"

    def __call__(self, graph: fx.Graph) -> int:
        n = 0
        for node in list(graph.nodes):
            if not _is(node, GROUP_QUANT):
                continue
            src = node.args[0]
            if not isinstance(src, fx.Node) or len(src.users) != 1:
                continue
            if _is(src, RMS_NORM):
                with graph.inserting_before(node):
                    fused = graph.call_function(torch.ops.b200fx.rms_norm_quant_fp8.default,
                                                tuple(src.args[:3]))
                node.replace_all_uses_with(fused)
                graph.erase_node(node)
                graph.erase_node(src)
                n += 1
            elif self._add_norm_output(src):
                self._rewrite_add(graph, node, src)
                n += 1
        return n

    @staticmethod
    def _add_norm_output(g: fx.Node) -> bool:
        """``g`` is element 0 (the normalised row) of a fused_add_rms_norm whose other users
        are getitem(1) nodes only (the updated residual)."""
        if g.target is not operator.getitem or g.args[1] != 0:
            return False
        fan = g.args[0]
        if not isinstance(fan, fx.Node) or not _is(fan, ADD_RMS):
            return False
        return all(u.target is operator.getitem and u.args[1] in (0, 1) for u in fan.users)

    @staticmethod
    def _rewrite_add(graph: fx.Graph, quant: fx.Node, g0: fx.Node) -> None:
        fan = g0.args[0]
        with graph.inserting_after(fan):
            fused = graph.call_function(torch.ops.b200fx.add_rms_norm_quant_fp8.default,
                                        tuple(fan.args[:4]))
        with graph.inserting_after(fused):
            res = graph.call_function(operator.getitem, (fused, 2))
        # (q, scales) keep their tuple positions 0 and 1; the residual moves to position 2.
        quant.replace_all_uses_with(fused)
        graph.erase_node(quant)
        graph.erase_node(g0)
        for u in list(fan.users):
            u.replace_all_uses_with(res)
            graph.erase_node(u)
        graph.erase_node(fan)


class B200PassManager(_Pass):
    """Runs the fusion passes in order; ``configure`` picks them from a config-like object
    (attributes ``fuse_allreduce_rms`` / ``fuse_act_quant``, default on)."""
    name = "b200_pass_manager"

    def __init__(self, passes: Optional[List[Callable]] = None):
        self.passes = passes if passes is not None else [AllReduceRMSNormFusionPass(),
                                                         SiluMulQuantFusionPass(),
                                                         RMSNormQuantFusionPass()]
        self.stats = {}

    def configure(self, config=None) -> "B200PassManager":
        ps = []
        if getattr(config, "fuse_allreduce_rms", True):
            ps.append(AllReduceRMSNormFusionPass())
        if getattr(config, "fuse_act_quant", True):
            ps.append(SiluMulQuantFusionPass())
        if getattr(config, "fuse_norm_quant", True):
            ps.append(RMSNormQuantFusionPass())
        self.passes = ps
        return self

    def uuid(self) -> str:
        return hashlib.sha256("".join(p.uuid() for p in self.passes).encode()).hexdigest()

    def __call__(self, graph: fx.Graph) -> int:
        total = 0
        for p in self.passes:
            k = p(graph)
            self.stats[p.name] = self.stats.get(p.name, 0) + k
            total += k
        graph.lint()
        return total
