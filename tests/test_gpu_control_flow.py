"""Lax.cond / whileLoop / foriLoop / scan on the device, eagerly and through
grad: the reference's T/LaxControlFlowTest.java cases, plus a scan over an
RNN-style step checked against a host restatement."""
import numpy as np
import pytest

from tests.util import TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def sc(J, v):
    return J.ConcreteNDArray.of(np.float32([v]))


def first(x):
    return float(x.toFloatArray()[0])


def test_cond_eager_selects_branch(J):  # LaxControlFlowTest.java:30-41
    square = lambda x: x.mul(x)
    negate = lambda x: x.mul(sc(J, -1.0))
    assert first(J.Lax.cond(sc(J, 1.0), square, negate, sc(J, 3.0))) == pytest.approx(9.0, abs=1e-5)
    assert first(J.Lax.cond(sc(J, 0.0), square, negate, sc(J, 3.0))) == pytest.approx(-3.0, abs=1e-5)


def test_cond_grad_follows_taken_branch(J):  # :43-57
    square = lambda x: x.mul(x)
    three = lambda x: x.mul(sc(J, 3.0))
    f_true = lambda x: J.Lax.cond(sc(J, 1.0), square, three, x)
    f_false = lambda x: J.Lax.cond(sc(J, 0.0), square, three, x)
    assert first(J.JAX.grad(f_true)(sc(J, 4.0))) == pytest.approx(8.0, abs=1e-4)
    assert first(J.JAX.grad(f_false)(sc(J, 4.0))) == pytest.approx(3.0, abs=1e-4)


def test_cond_composes_with_surrounding_trace(J):  # :59-71
    fn = lambda x: J.Lax.cond(sc(J, 1.0), lambda y: y.mul(y), lambda y: y, x).add(sc(J, 1.0))
    assert first(fn(sc(J, 5.0))) == pytest.approx(26.0, abs=1e-4)
    assert first(J.JAX.grad(fn)(sc(J, 5.0))) == pytest.approx(10.0, abs=1e-4)


def test_while_loop_eager(J):  # :75-83
    cond = lambda x: sc(J, 1.0 if first(x) < 100.0 else 0.0)
    body = lambda x: x.mul(sc(J, 2.0))
    assert first(J.Lax.whileLoop(cond, body, sc(J, 3.0))) == pytest.approx(192.0, abs=1e-4)


def test_while_loop_is_not_differentiable(J):  # :85-96
    fn = lambda x: J.Lax.whileLoop(lambda s: s.mul(sc(J, 0.0)), lambda s: s.add(sc(J, 1.0)), x)
    with pytest.raises(J.UnsupportedOperationException):
        J.JAX.grad(fn)(sc(J, 5.0))


def test_fori_loop_eager_and_differentiable(J):  # :100-113
    assert first(J.Lax.foriLoop(0, 5, lambda i, acc: acc.add(sc(J, float(i))), sc(J, 0.0))) == pytest.approx(10.0)
    fn = lambda x: J.Lax.foriLoop(0, 5, lambda i, acc: acc.mul(sc(J, 2.0)), x)
    assert first(fn(sc(J, 3.0))) == pytest.approx(96.0, abs=1e-4)
    assert first(J.JAX.grad(fn)(sc(J, 3.0))) == pytest.approx(32.0, abs=1e-4)


def test_scan_eager_running_sum_and_squares(J):  # :117-131
    def step(carry, x):
        c = carry.add(x)
        return [c, c.mul(c)]

    res = J.Lax.scan(step, sc(J, 0.0), J.ConcreteNDArray.of(np.float32([1, 2, 3, 4]).reshape(4, 1)))
    assert first(res.carry()) == pytest.approx(10.0, abs=1e-4)
    np.testing.assert_allclose(res.ys().toFloatArray(), [1, 9, 36, 100], atol=1e-4)


def test_scan_grad_through_carry(J):  # :133-149
    xs = J.ConcreteNDArray.of(np.float32([2, 3, 4]).reshape(3, 1))
    fn = lambda x0: J.Lax.scan(lambda c, x: [c.mul(x), c], x0, xs).carry()
    assert first(fn(sc(J, 5.0))) == pytest.approx(120.0, abs=1e-4)
    assert first(J.JAX.grad(fn)(sc(J, 5.0))) == pytest.approx(24.0, abs=1e-4)


def test_scan_grad_through_stacked_ys(J):  # :151-171
    ts = J.ConcreteNDArray.of(np.float32([1, 2, 3]).reshape(3, 1))

    def step(c, t):
        v = c.add(t)
        return [c, v.mul(v)]

    fn = lambda x0: J.Lax.scan(step, x0, ts).ys().sum()
    x0 = 5.0
    assert first(fn(sc(J, x0))) == pytest.approx((x0 + 1) ** 2 + (x0 + 2) ** 2 + (x0 + 3) ** 2, abs=1e-3)
    assert first(J.JAX.grad(fn)(sc(J, x0))) == pytest.approx(2 * (x0 + 1) + 2 * (x0 + 2) + 2 * (x0 + 3), abs=1e-3)


def test_scan_rnn_step_forward_and_grad_against_host(J):
    """h_t = tanh(h_{t-1} . W + x_t), loss = sum_t sum(h_t): a 12-step scan of
    [16, 32] states with a shared W, forward and d loss / d h_0 checked
    against a float64 host restatement (central differences for the grad)."""
    r = np.random.default_rng(9)
    T, B, H = 12, 16, 32
    W = (r.standard_normal((H, H)) * 0.2).astype(np.float32)
    X = (r.standard_normal((T, B, H)) * 0.5).astype(np.float32)
    h0 = (r.standard_normal((B, H)) * 0.5).astype(np.float32)
    Wd, Xd = J.ConcreteNDArray.of(W), J.ConcreteNDArray.of(X)

    def step(h, x):
        hn = h.dot(Wd).add(x).tanh()
        return [hn, hn]

    loss = lambda h: J.Lax.scan(step, h, Xd).ys().sum()

    def host(h):
        tot = 0.0
        for t in range(T):
            h = np.tanh(h @ W.astype(np.float64) + X[t])
            tot += h.sum()
        return tot

    assert first(loss(J.ConcreteNDArray.of(h0))) == pytest.approx(host(h0.astype(np.float64)), rel=1e-4)
    g = J.JAX.grad(loss)(J.ConcreteNDArray.of(h0)).numpy()
    eps = 1e-3
    num = np.zeros_like(h0, dtype=np.float64)
    base = h0.astype(np.float64)
    for idx in [(0, 0), (3, 7), (15, 31), (8, 16)]:
        e = np.zeros_like(base)
        e[idx] = eps
        num[idx] = (host(base + e) - host(base - e)) / (2 * eps)
        assert g[idx] == pytest.approx(num[idx], rel=5e-3, abs=1e-3)
