"""JAX.jvp (forward mode, Grad.forwardAd): the reference's T/GradTest.java
cases, and forward-mode tangents equal to directional derivatives from
reverse mode on a small MLP, a scan and a cond."""
import numpy as np
import pytest

from tests.util import TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def a(J, v, shape=None):
    v = np.asarray(v, np.float32)
    return J.ConcreteNDArray.of(v.reshape(shape) if shape else v)


def test_polynomial_jvp(J):  # GradTest.java:33-49: f(x) = x*x + x at 3, tangent 1.5
    out = J.JAX.jvp(lambda x: x.mul(x).add(x), a(J, [3.0]), a(J, [1.5]))
    np.testing.assert_allclose(out[0].toFloatArray(), [12.0], atol=1e-5)
    np.testing.assert_allclose(out[1].toFloatArray(), [10.5], atol=1e-5)


def test_sin_jvp(J):  # GradTest.java:51-65
    out = J.JAX.jvp(lambda x: x.sin(), a(J, [0.0]), a(J, [2.0]))
    np.testing.assert_allclose(out[0].toFloatArray(), [0.0], atol=1e-5)
    np.testing.assert_allclose(out[1].toFloatArray(), [2.0], atol=1e-5)


def test_dot_jvp(J):  # GradTest.java:67-83
    out = J.JAX.jvp(lambda x: x.dot(x), a(J, [1, 2, 3, 4], (2, 2)), a(J, [1, 0, 0, 1], (2, 2)))
    np.testing.assert_allclose(out[0].toFloatArray(), [7, 10, 15, 22], atol=1e-5)
    np.testing.assert_allclose(out[1].toFloatArray(), [2, 4, 6, 8], atol=1e-5)


def test_jvp_matches_reverse_mode_directional_derivative(J):
    """<grad f(x), v> (reverse mode) = jvp(f, x, v) (forward mode) for a
    scalar loss built from dot, bias add, tanh, relu, sigmoid, exp/log, div,
    a scan and a cond."""
    r = np.random.default_rng(1)
    W1 = a(J, r.uniform(-0.5, 0.5, (24, 16)))
    W2 = a(J, r.uniform(-0.5, 0.5, (16, 8)))
    b1 = a(J, r.uniform(-0.1, 0.1, 16))
    xs = a(J, r.uniform(-0.5, 0.5, (5, 6, 8)))
    one = a(J, [1.0])

    def f(x):
        h = x.dot(W1).add(b1).tanh()
        g = h.dot(W2).relu().add(h.dot(W2).sigmoid())
        s = J.Lax.scan(lambda c, xt: [c.add(xt).tanh(), c.mul(xt)], g, xs)
        z = J.Lax.cond(one, lambda u: u.exp().add(one).log(), lambda u: u, s.carry())
        return z.div(one.add(z.mul(z))).sum().add(s.ys().sum())

    x = a(J, r.uniform(-1, 1, (6, 24)))
    v = r.uniform(-1, 1, (6, 24)).astype(np.float32)
    grad = J.JAX.grad(f)(x).numpy()
    primal, tangent = J.JAX.jvp(f, x, a(J, v))
    assert_rel(primal.numpy(), f(x).numpy(), 1e-6)
    assert_rel(tangent.numpy(), np.float32([np.sum(grad.astype(np.float64) * v)]), TOL_REDUCTION)


def test_jvp_rejects_max_like_the_reference(J):
    with pytest.raises(J.UnsupportedOperationException):
        J.JAX.jvp(lambda x: x.max(x.mul(a(J, [2.0]))), a(J, [1.0, 2.0]), a(J, [1.0, 1.0]))
