"""Fused elementwise chains (JAX.jit, the grad interpreter's forward pass and
its deferred backward) against the unfused kernels and the oracle: fused and
unfused results bit for bit (row-reduction tails add in the row reduction
kernel's order), the oracle within the elementwise / reduction tolerances,
argmax exact."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.util import TOL_ELEMENTWISE, TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def _unfused(J, monkeypatch_fn):
    from jax4j_b200 import grad
    old = grad.FUSION
    grad.FUSION = False
    try:
        return monkeypatch_fn()
    finally:
        grad.FUSION = old


@pytest.mark.parametrize("rows,cols", [(4096, 16384), (33, 1000), (3, 7), (1, 5000), (700, 300)])
def test_fused_sweep_matches_oracle(J, rows, cols):
    x = J.Random.normal(J.PRNGKey.key(1), J.Shape(rows, cols))
    y = J.Random.uniform(J.PRNGKey.key(11), J.Shape(rows, cols), -3.0, 3.0)
    zero, lo, hi = (J.ConcreteNDArray.scalar(v) for v in (0.0, -1.0, 1.0))

    def sweep(xx, yy):
        z = J.Numpy.where(xx.gt(zero), xx.tanh().mul(yy.sigmoid()), yy.relu().clip(lo, hi))
        return z, z.sum(-1, True), z.argmax(-1)

    jitted = J.JAX.jit(sweep)
    z, s, am = jitted(x, y)
    groups = [g for g in next(iter(jitted.cache.values())).__dict__["_fusion_plan"].groups]
    assert len(groups) == 1 and len(groups[0].tails) == 2  # one pass: chain + both tails
    rz, rs, ram = orc.sweep(x.numpy(), y.numpy(), want_z=True)
    assert_rel(z.numpy(), rz, TOL_ELEMENTWISE, "z")
    assert_rel(s.numpy(), rs, TOL_REDUCTION, "row sums")
    np.testing.assert_array_equal(am.numpy(), ram)
    # fused values equal the unfused kernels' bit for bit -- the row sums too:
    # the generated tail adds in the row reduction kernel's order
    z2, s2, am2 = _unfused(J, lambda: J.JAX.jit(sweep)(x, y))
    np.testing.assert_array_equal(z.numpy(), z2.numpy())
    np.testing.assert_array_equal(s.numpy(), s2.numpy())
    np.testing.assert_array_equal(am.numpy(), am2.numpy())


def test_fused_broadcast_patterns_and_casts(J):
    r = np.random.default_rng(4)
    a = J.ConcreteNDArray.of(r.standard_normal((64, 96)).astype(np.float32))
    row = J.ConcreteNDArray.of(r.standard_normal(96).astype(np.float32))
    col = J.ConcreteNDArray.of(r.standard_normal((64, 1)).astype(np.float32))
    sc = J.ConcreteNDArray.scalar(0.25)

    def f(x, rv, cv):
        t = x.mul(rv).sub(cv).max(sc).exp().log().sin().cos()
        m = t.gt(cv).astype(J.DType.FLOAT32).add(t.div(rv)).min(x)
        i = m.astype(J.DType.INT32).astype(J.DType.FLOAT32)
        return m.add(i), m.mean(-1, False), m.argmin(-1), t.sum(-1, True)

    got = J.JAX.jit(f)(a, row, col)
    ref = _unfused(J, lambda: f(a, row, col))
    np.testing.assert_array_equal(got[0].numpy(), ref[0].numpy())
    assert_rel(got[1].numpy(), ref[1].numpy(), TOL_REDUCTION)
    np.testing.assert_array_equal(got[2].numpy(), ref[2].numpy())
    assert_rel(got[3].numpy(), ref[3].numpy(), TOL_REDUCTION)


def test_fused_argmax_nan_and_tie_rules(J):
    x = np.float32([[np.nan, 5, 5, 1], [1, 7, 7, np.nan], [-np.inf] * 4, [3, 3, 9, 9],
                    [-np.inf, np.nan, -np.inf, 2], [np.nan] * 4, [-np.inf, -np.inf, np.nan, np.nan],
                    [np.inf, np.inf, -np.inf, np.nan], [0.0, -0.0, 0.0, -0.0], [-0.0, 0.0, -1, -1]])
    a = J.ConcreteNDArray.of(x)
    one = J.ConcreteNDArray.scalar(1.0)
    got = J.JAX.jit(lambda v: (v.mul(one).argmax(-1), v.mul(one).argmin(-1)))(a)
    np.testing.assert_array_equal(got[0].numpy(), orc.argreduce(orc.ARGMAX, x, -1))
    np.testing.assert_array_equal(got[1].numpy(), orc.argreduce(orc.ARGMIN, x, -1))


@pytest.mark.parametrize("cols", [33, 1000, 1001, 4096, 16384])
def test_fused_argmax_ties_across_lanes(J, cols):
    # few distinct values so every row has many ties, spread over lanes and
    # CTA warps; some rows carry NaN / inf; exercises 1- and 4-wide kernels
    r = np.random.default_rng(cols)
    x = r.integers(-3, 4, size=(64, cols)).astype(np.float32)
    x[5, :] = -np.inf
    x[6, 0] = np.nan
    x[7, r.integers(1, cols, 20)] = np.nan
    x[8, :] = np.nan
    x[9, r.integers(0, cols, 5)] = np.inf
    a = J.ConcreteNDArray.of(x)
    one = J.ConcreteNDArray.scalar(1.0)
    got = J.JAX.jit(lambda v: (v.mul(one).argmax(-1), v.mul(one).argmin(-1), v.mul(one).max(one)))(a)
    np.testing.assert_array_equal(got[0].numpy(), orc.argreduce(orc.ARGMAX, x, -1))
    np.testing.assert_array_equal(got[1].numpy(), orc.argreduce(orc.ARGMIN, x, -1))
    np.testing.assert_array_equal(got[2].numpy(), orc.binary(orc.MAX, x, np.float32(1.0)))


def test_fused_max_min_signed_zero_and_nan(J):
    vals = np.float32([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 3.0e38, -1e-45])
    x = np.repeat(vals, len(vals)).reshape(len(vals), len(vals))
    y = np.tile(vals, len(vals)).reshape(len(vals), len(vals))
    a, b = J.ConcreteNDArray.of(x), J.ConcreteNDArray.of(y)
    one = J.ConcreteNDArray.scalar(1.0)
    got = J.JAX.jit(lambda u, v: (u.mul(one).max(v), u.mul(one).min(v), u.mul(one).relu()))(a, b)
    for k, (g, prim) in enumerate([(got[0], orc.MAX), (got[1], orc.MIN)]):
        ref = orc.binary(prim, x, y)
        gb = g.numpy()
        assert np.array_equal(np.isnan(gb), np.isnan(ref))
        ok = ~np.isnan(ref)
        np.testing.assert_array_equal(gb[ok].view(np.uint32), ref[ok].view(np.uint32))
    relu_ref = orc.unary(orc.RELU, x)
    rb = got[2].numpy()
    ok = ~np.isnan(relu_ref)
    np.testing.assert_array_equal(rb[ok].view(np.uint32), relu_ref[ok].view(np.uint32))


def test_fusion_keeps_values_the_backward_reads(J):
    # grad through a fused forward: the relu VJP reads z, the MUL VJP reads both inputs
    r = np.random.default_rng(2)
    x = J.ConcreteNDArray.of(r.standard_normal((32, 48)).astype(np.float32))
    b = J.ConcreteNDArray.of(r.standard_normal(48).astype(np.float32))
    w = J.ConcreteNDArray.of(r.standard_normal((32, 48)).astype(np.float32))
    fn = lambda v: v.add(b).relu().mul(w).tanh().sum(-1).mean()
    g = J.JAX.grad(fn)(x).numpy()
    g_ref = _unfused(J, lambda: J.JAX.grad(fn)(x).numpy())
    assert_rel(g, g_ref, TOL_REDUCTION)


def _eager_backward(fn):
    """fn() with the backward's cotangents computed op by op (no deferral)."""
    from jax4j_b200 import lazy
    old = lazy.ENABLED
    lazy.ENABLED = False
    try:
        return fn()
    finally:
        lazy.ENABLED = old


def test_deferred_backward_softmax_ce_fewer_launches_same_bits(J):
    from jax4j_b200 import _lib
    r = np.random.default_rng(9)
    x = J.ConcreteNDArray.of(r.standard_normal((96, 50)).astype(np.float32))
    w = J.ConcreteNDArray.of((0.1 * r.standard_normal((50, 30))).astype(np.float32))
    b = J.ConcreteNDArray.of((0.1 * r.standard_normal(30)).astype(np.float32))
    t = np.zeros((96, 30), np.float32)
    t[np.arange(96), r.integers(0, 30, 96)] = 1.0
    tt = J.ConcreteNDArray.of(t)
    neg = J.ConcreteNDArray.scalar(-1.0)

    def loss(tree):
        c = tree.children
        logits = x.dot(c["w"].value).add(c["b"].value)
        return J.Nn.softmax(logits).log().mul(tt).sum(-1).mean().mul(neg)

    vg = J.JAX.valueAndGradTree(loss)
    tree = J.PyTree.dictOf({"w": w, "b": b})
    vg(tree)  # plans and kernels compiled once
    n0 = _lib.kernel_launches()
    v1, g1 = vg(tree)
    n1 = _lib.kernel_launches()
    v0, g0 = _eager_backward(lambda: vg(tree))
    n2 = _lib.kernel_launches()
    assert (n1 - n0) + 8 <= (n2 - n1), (n1 - n0, n2 - n1)
    np.testing.assert_array_equal(v1.numpy(), v0.numpy())
    for k in ("w", "b"):
        np.testing.assert_array_equal(g1.children[k].value.numpy(), g0.children[k].value.numpy())


@pytest.mark.parametrize("shape", [(64, 48), (5, 3), (1, 700), (300, 1)])
def test_deferred_backward_rules_match_eager(J, shape):
    """TANH, SIGMOID, EXP, LOG, SIN, COS, DIV with row / column / scalar
    broadcasts, MEAN_AXIS over the last axis and SUM: the deferred VJPs give
    the eager kernels' bits."""
    r = np.random.default_rng(sum(shape))
    x = J.ConcreteNDArray.of(r.standard_normal(shape).astype(np.float32))
    y = J.ConcreteNDArray.of((r.random(shape) + 0.5).astype(np.float32))
    row = J.ConcreteNDArray.of((r.random(shape[-1]) + 0.5).astype(np.float32))
    col = J.ConcreteNDArray.of((r.random((shape[0], 1)) + 0.5).astype(np.float32))
    two = J.ConcreteNDArray.scalar(2.0)

    def f(a, c):
        u = a.tanh().mul(c.sigmoid()).div(row).add(a.exp().div(col))
        v = c.log().mul(a.sin()).sub(a.cos().div(two))
        m = u.mul(v).mean(-1, True)
        return u.div(m.add(two)).sum()

    g = J.JAX.gradBoth(f)
    ga, gc = g(x, y)
    ea, ec = _eager_backward(lambda: g(x, y))
    np.testing.assert_array_equal(ga.numpy(), ea.numpy())
    np.testing.assert_array_equal(gc.numpy(), ec.numpy())
