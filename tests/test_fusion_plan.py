"""Host-side tests of the fusion planner (no GPU): which equations form a
group, which values a group writes, and the program limits."""
import pytest

from jax4j_b200 import fusion
from jax4j_b200 import grad as G
from jax4j_b200.core import DType, Primitive as P, Shape
from jax4j_b200.tracing import Tracer, TracedNDArray


class Spec:
    """Shape and dtype only: enough to trace a function."""
    def __init__(self, *dims, dtype=DType.FLOAT32):
        self._s, self._d = Shape(*dims), dtype

    def shape(self):
        return self._s

    def dtype(self):
        return self._d


def test_select_chain_is_one_group_with_two_tails():
    def f(x, y, zero, lo, hi):
        m = x.gt(zero).astype(DType.FLOAT32)
        z = m.mul(x.tanh().mul(y.sigmoid())).add(y.relu().clip(lo, hi))
        return z.sum(-1, True), z.argmax(-1)

    jp = G.make_jaxpr(f, Spec(64, 128), Spec(64, 128), Spec(), Spec(), Spec())
    plan = fusion.plan(jp, keep_for_vjp=False)
    groups = plan.groups
    assert len(groups) == 1
    g = groups[0]
    assert [e.primitive for e in g.tails] == [P.SUM_AXIS, P.ARGMAX]
    assert g.outputs == []                         # z is never written
    assert all(kind == "group" for kind, _ in plan.steps)


def test_keep_for_vjp_writes_values_the_backward_reads():
    def f(x, w):
        return x.mul(w).tanh().relu()

    jp = G.make_jaxpr(f, Spec(8, 16), Spec(8, 16))
    p0 = fusion.plan(jp, keep_for_vjp=False)
    p1 = fusion.plan(jp, keep_for_vjp=True)
    assert len(p0.groups) == len(p1.groups) == 1
    assert [v.id for v in p0.groups[0].outputs] == [jp.outVars[0].id]
    # tanh' reads its output, relu' reads its input (the tanh value)
    assert len(p1.groups[0].outputs) >= 2


def test_dot_splits_groups():
    def f(x, w, b):
        return x.dot(w).mul(b).relu().mul(x.dot(w))

    jp = G.make_jaxpr(f, Spec(8, 16), Spec(16, 16), Spec(16))
    plan = fusion.plan(jp, keep_for_vjp=False)
    kinds = [k for k, _ in plan.steps]
    assert kinds.count("eq") == 2 and kinds.count("group") == 1


def test_dot_bias_relu_runs_in_the_gemm_epilogue():
    def f(x, w1, b1, w2, b2):
        h = x.dot(w1).add(b1).relu()
        return h.dot(w2).add(b2).exp().sum(-1, True)

    jp = G.make_jaxpr(f, Spec(8, 16), Spec(16, 32), Spec(32), Spec(32, 4), Spec(4))
    plan = fusion.plan(jp, keep_for_vjp=True)
    kinds = [k for k, _ in plan.steps]
    assert kinds == ["dot_ep", "dot_ep", "group"]
    first, second = plan.steps[0][1], plan.steps[1][1]
    assert first.relu is not None and second.relu is None
    # the second epilogue's output (the logits) feeds the exp + row-sum group
    assert plan.steps[2][1].inputs[0][0].id == second.add.outputs[0].id


def test_dot_epilogue_needs_a_private_dot_output_and_an_earlier_bias():
    def used_twice(x, w, b):
        z = x.dot(w)
        return z.add(b).relu().add(z)

    def bias_after_dot(x, w, b):
        z = x.dot(w)
        return z.add(b.mul(b)).relu()  # b*b is computed after the DOT

    for f in (used_twice, bias_after_dot):
        jp = G.make_jaxpr(f, Spec(8, 16), Spec(16, 16), Spec(16))
        assert "dot_ep" not in [k for k, _ in fusion.plan(jp, keep_for_vjp=False).steps]


def test_group_limits():
    n = 40

    def f(*xs):
        acc = xs[0]
        for x in xs[1:]:
            acc = acc.add(x)
        return acc

    jp = G.make_jaxpr(f, *[Spec(4, 4) for _ in range(n)])
    plan = fusion.plan(jp, keep_for_vjp=False)
    assert len(plan.groups) >= 3
    for g in plan.groups:
        assert len(g.inputs) <= fusion.MAX_INPUTS and len(g.eqs) <= fusion.MAX_EQS
    # every equation is in exactly one group
    assert sum(len(g.eqs) for g in plan.groups) == n - 1


def test_mismatched_shapes_and_bool_compare_not_fused():
    def f(x, y):
        return x.sum(0).add(y).gt(y).eq(y.gt(y))

    jp = G.make_jaxpr(f, Spec(8, 16), Spec(16))
    plan = fusion.plan(jp, keep_for_vjp=False)
    fused = [e.primitive for g in plan.groups for e in g.eqs]
    assert P.EQ not in fused                      # comparison of two booleans stays unfused
    assert P.SUM_AXIS not in fused


def _compile_all(jp, keep=False):
    plan = fusion.plan(jp, keep_for_vjp=keep)
    srcs = [fusion.group_source(g, compile=True) for g in plan.groups]
    assert srcs
    return srcs


def test_generated_kernels_compile_for_sm100a():
    # sweep-like chain with two tails: row kernels, 1- and 4-wide variants
    def f(x, y, zero, lo, hi):
        m = x.gt(zero).astype(DType.FLOAT32)
        z = m.mul(x.tanh().mul(y.sigmoid())).add(y.relu().clip(lo, hi))
        return z.sum(-1, True), z.argmax(-1), z.mean(-1, False), z.argmin(-1)

    srcs = _compile_all(G.make_jaxpr(f, Spec(16, 64), Spec(16, 64), Spec(), Spec(), Spec()))
    assert "k_rows_block4" in srcs[0] and "float4" in srcs[0]


def test_generated_kernels_compile_for_mixed_dtypes_and_broadcasts():
    def f(x, row, col, d, i):
        t = x.mul(row).sub(col).exp().log()
        b = t.gt(col)
        k = t.astype(DType.INT32).astype(DType.INT64).astype(DType.FLOAT64).add(d)
        return b.astype(DType.FLOAT32).add(t), k.sin().cos(), i.astype(DType.FLOAT32).div(t)

    srcs = _compile_all(G.make_jaxpr(f, Spec(8, 12), Spec(12), Spec(8, 1), Spec(8, 12, dtype=DType.FLOAT64),
                                     Spec(8, 12, dtype=DType.INT32)), keep=True)
    assert any("double" in s for s in srcs)


def test_generated_flat_kernel_compiles():
    def f(x, y):
        return x.mul(y).tanh().max(y).min(x).div(y)

    srcs = _compile_all(G.make_jaxpr(f, Spec(3, 5, 7), Spec(3, 5, 7)))
    assert "k_flat4" in srcs[0] and "k_rows" not in srcs[0]


def test_invalid_program_rejected():
    import ctypes as C
    from jax4j_b200 import _lib
    insn = (fusion._Insn * 1)(fusion._Insn(int(P.ADD), DType.FLOAT32.ordinal, 0, 0, 0.0))  # reads itself
    z = (C.c_int32 * 1)(0)
    prog = fusion._Program(1, insn, 0, z, z, 1, z, 0, z, z)
    rc = _lib.lib().j4c_fused_source(C.cast(C.pointer(prog), C.c_void_p), 0, None, 0, None)
    assert rc == _lib.E_INVALID


def test_program_struct_layout_matches_the_c_abi():
    """j4c_insn is 24 bytes; j4c_program has pointers at 8-byte offsets (the
    layout a Java FFM StructLayout of the header reproduces)."""
    import ctypes as C
    assert C.sizeof(fusion._Insn) == 24
    assert fusion._Insn.value.offset == 16
    P = fusion._Program
    assert [getattr(P, f).offset for f in ("n_insns", "insns", "n_inputs", "input_dtype", "input_bcast",
                                            "n_outputs", "output_insn", "n_tails", "tail_op", "tail_insn")] == \
        [0, 8, 16, 24, 32, 40, 48, 56, 64, 72]


def _leaf(*dims):
    """A host-memory FLOAT32 array standing in for a forward value (planning only)."""
    import torch
    from jax4j_b200.core import ConcreteNDArray
    s = Shape(*dims)
    return ConcreteNDArray._wrap(torch.empty(s.size()), s, DType.FLOAT32, None)


def _softmax_ce_backward(B=64, C=40):
    """The deferred cotangent of the logits for loss = -mean(sum(log(e / sum(e)) * t, -1)),
    built with the rules of Grad.computeVJPs (MEAN, SUM_AXIS, MUL, LOG, DIV, SUM_AXIS, EXP)."""
    from jax4j_b200 import lazy
    g_r = _leaf(B, 1)                     # the mean's cotangent, already spread over the rows
    onehot, p, e = _leaf(B, C), _leaf(B, C), _leaf(B, C)
    s, minus1 = _leaf(B, 1), _leaf(1)
    g_t = lazy.expand(g_r, Shape(B, C))                        # SUM_AXIS VJP
    g_p = lazy.binary(lazy.binary(g_t, onehot, P.MUL), p, P.DIV)  # MUL, then LOG VJP (g / p)
    ga = lazy.binary(g_p, s, P.DIV)                              # DIV VJP w.r.t. e
    t = lazy.binary(lazy.binary(lazy.binary(g_p, e, P.MUL), s, P.DIV), s, P.DIV)
    g_s = lazy.row_sum(lazy.binary(t, minus1, P.MUL), Shape(B, 1))  # DIV VJP w.r.t. s, summed down
    g_e = lazy.binary(ga, lazy.expand(g_s, Shape(B, C)), P.ADD)   # + SUM_AXIS VJP of s = sum(e)
    return lazy.binary(g_e, e, P.MUL)                            # EXP VJP


def test_deferred_softmax_ce_backward_is_two_kernels():
    from jax4j_b200 import lazy
    x = _softmax_ce_backward()
    assert isinstance(x, lazy.Deferred)
    # the planning half of lazy.materialize
    leaves, nodes = [], []
    seen = {}

    def walk(n):
        if not isinstance(n, lazy.Deferred):
            if id(n) not in seen:
                seen[id(n)] = ("in", len(leaves))
                leaves.append(n)
            return seen[id(n)]
        if id(n) not in seen:
            refs = [walk(a) for a in n.args]
            seen[id(n)] = ("eq", len(nodes))
            nodes.append((n, refs))
        return seen[id(n)]

    walk(x)
    jaxpr, plan = lazy._build(leaves, nodes)
    kinds = [k for k, _ in plan.steps]
    assert kinds == ["group", "group"]
    g1, g2 = plan.groups
    assert [e.primitive for e in g1.tails] == [P.SUM_AXIS]
    assert len(g1.outputs) == 1 and len(g2.outputs) == 1   # ga, then the logits' cotangent
    assert g2.outputs[0].id == jaxpr.outVars[0].id
    for g in plan.groups:
        assert "extern \"C\"" in fusion.group_source(g, compile=True)


def test_deferred_values_refuse_what_a_kernel_cannot_broadcast():
    from jax4j_b200 import lazy
    a, b = _leaf(8, 16), _leaf(16, 1)
    assert lazy.binary(a, b, P.ADD) is None              # [16, 1] is no row, column or scalar of [8, 16]
    assert lazy.expand(_leaf(8), Shape(8, 16)) is None    # needs the [8, 1] view first
    assert lazy.row_sum(a, Shape(16)) is None             # a column sum: not a last-axis tail
    assert lazy.row_sum(a, Shape(8)).meta.keepDims is False
    assert lazy.row_sum(a, Shape(8, 1)).meta.keepDims is True


def _host_scalar(v):
    """A one-element constant as ConcreteNDArray.full makes it (value kept on
    the host), without a device."""
    import numpy as np
    import torch
    from jax4j_b200.core import ConcreteNDArray, Device
    a = ConcreteNDArray._wrap(torch.tensor([v], dtype=torch.float32), Shape(1), DType.FLOAT32, Device.host())
    a._scalar = float(np.float32(v))
    return a


def test_scalar_constants_become_literals_and_where_and_clip_specialise():
    zero, lo, hi, one = _host_scalar(0.0), _host_scalar(-1.0), _host_scalar(1.0), _host_scalar(1.0)

    def f(x, y):
        # Numpy.where's equations (api.py Numpy.where; a device scalar there)
        c = x.gt(zero).astype(DType.FLOAT32)
        z = c.mul(x.tanh().mul(y.sigmoid())).add(one.sub(c).mul(y.relu().clip(lo, hi)))
        return z.sum(-1, True), z.argmax(-1)

    jp = G.make_jaxpr(f, Spec(16, 64), Spec(16, 64))
    plan = fusion.plan(jp, keep_for_vjp=False)
    assert len(plan.groups) == 1
    g = plan.groups[0]
    # x and y stay inputs; 0, -1, 1 and the blend's 1 are literals
    assert [v.shape for v, _ in g.inputs] == [Shape(16, 64), Shape(16, 64)]
    assert sorted(g.consts.values()) == [-1.0, 0.0, 1.0, 1.0]
    src = fusion.group_source(g, compile=True)
    assert "= j_where(v" in src                      # the blend as select + one multiply-add pair
    assert "= j_max_nz(v" in src and "= j_min_nz(v" in src  # clip against non-zero literal bounds
    assert "= j_tanh(v" in src and "= j_sigmoid(v" in src


def test_zero_literal_keeps_java_max():
    zero = _host_scalar(0.0)

    def f(x):
        return x.max(zero).min(zero)  # +0 / -0 pairs need Math.max / Math.min's rule

    g = fusion.plan(G.make_jaxpr(f, Spec(4, 8)), keep_for_vjp=False).groups[0]
    src = fusion.group_source(g, compile=True)
    assert "= j_max_nz(v" not in src and "= j_min_nz(v" not in src
    assert "= j_max(v" in src and "= j_min(v" in src
