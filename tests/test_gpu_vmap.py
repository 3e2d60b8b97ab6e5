"""JAX.vmap (api/Vmap.java) on the device: the reference's vmap tests
(T/VmapTest.java, T/SelectionOpsTest.java:106-112, T/AxisReduceTest.java:104-119,
T/PmapTest.java:141-152) and per-example parity with the oracle at larger sizes."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.util import TOL_ELEMENTWISE, TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def arr(J, values, shape, dtype=None):
    return J.ConcreteNDArray.of(np.asarray(values, np.float32).reshape(shape))


def test_elementwise_vmap_matches_per_example_loop(J):  # VmapTest.java:23-31
    one = J.ConcreteNDArray.scalar(1.0)
    out = J.JAX.vmap(lambda x: x.mul(x).add(one))(arr(J, [1, 2, 3, 4], (4, 1)))
    assert out.shape().dimensions() == (4, 1)
    np.testing.assert_allclose(out.toFloatArray(), [2, 5, 10, 17], atol=1e-5)


def test_vmap_with_closed_over_constant(J):  # VmapTest.java:33-45
    w = arr(J, [2, 3, 4], (3,))
    out = J.JAX.vmap(lambda x: x.mul(w).sum())(arr(J, [1, 1, 1, 2, 2, 2], (2, 3)))
    assert out.shape().dimensions() == (2,)
    np.testing.assert_allclose(out.toFloatArray(), [9, 18], atol=1e-5)


def test_vmap_mean_per_example(J):  # VmapTest.java:47-55
    out = J.JAX.vmap(lambda x: x.mean())(arr(J, [1, 2, 3, 10, 20, 30], (2, 3)))
    np.testing.assert_allclose(out.toFloatArray(), [2.0, 20.0], atol=1e-5)


def test_vmap_dot_with_shared_matrix(J):  # VmapTest.java:57-68
    eye = arr(J, [1, 0, 0, 1], (2, 2))
    out = J.JAX.vmap(lambda x: x.dot(eye))(arr(J, [1, 2, 3, 4], (2, 1, 2)))
    assert out.shape().dimensions() == (2, 1, 2)
    np.testing.assert_allclose(out.toFloatArray(), [1, 2, 3, 4], atol=1e-5)


def test_vmap_matches_manual_per_example(J):  # VmapTest.java:70-89
    ex = np.float32([[0.1, 0.2], [1.0, -1.0], [0.0, 3.0]])
    out = J.JAX.vmap(lambda x: x.exp().sum())(arr(J, ex, (3, 2)))
    expect = [float(np.exp(np.float64(a)) + np.exp(np.float64(b))) for a, b in ex]
    np.testing.assert_allclose(out.toFloatArray(), expect, atol=1e-4)


def test_vmap_composes_with_argmax(J):  # SelectionOpsTest.java:106-112
    out = J.JAX.vmap(lambda row: row.argmax(0))(arr(J, [1, 5, 3, 9, 2, 4], (2, 3)))
    np.testing.assert_array_equal(out.toIntArray(), [1, 0])


def test_vmap_of_axis_sum_shifts_axis(J):  # AxisReduceTest.java:104-119
    out = J.JAX.vmap(lambda x: x.sum(1))(arr(J, [1, 2, 3, 4, 5, 6, 10, 20, 30, 40, 50, 60], (2, 3, 2)))
    assert out.shape().dimensions() == (2, 3)
    np.testing.assert_allclose(out.toFloatArray(), [3, 7, 11, 30, 70, 110], atol=1e-5)


def test_pmap_composes_with_vmap(J):  # PmapTest.java:141-152
    devices = [J.Device(None), J.Device(None)]
    out = J.JAX.vmap(lambda x: J.JAX.pmap(lambda s: s.mul(s), devices)(x))(arr(J, range(1, 9), (2, 2, 2)))
    assert out.shape().rank() == 3
    np.testing.assert_allclose(out.toFloatArray(), [1, 4, 9, 16, 25, 36, 49, 64], atol=1e-5)


def test_vmap_in_axes_and_out_axis(J):
    """Two arguments: the second unbatched (in_axes -1), the first batched on
    axis 1 of a 2-D array (moved to the front), the result's batch axis moved
    to position 1 (Vmap.java:64-100)."""
    r = np.random.default_rng(3)
    X = r.standard_normal((5, 7)).astype(np.float32)   # batch on axis 1: 7 examples of length 5
    w = r.standard_normal(5).astype(np.float32)
    f = J.JAX.vmap(lambda x, v: x.mul(v).tanh(), in_axes=[1, -1], out_axis=1)
    out = f(J.ConcreteNDArray.of(X), J.ConcreteNDArray.of(w))
    ref = np.tanh((X.T.astype(np.float64) * w).astype(np.float32).astype(np.float64)).astype(np.float32).T
    assert out.shape().dimensions() == (5, 7)
    assert_rel(out.numpy(), ref, TOL_ELEMENTWISE)


@pytest.mark.parametrize("a_b,b_b", [(True, False), (False, True), (True, True)])
def test_batched_dot_per_example_against_oracle(J, a_b, b_b):
    r = np.random.default_rng(11)
    B, M, K, N = 6, 33, 70, 40
    A = r.uniform(-1, 1, (B, M, K) if a_b else (M, K)).astype(np.float32)
    W = r.uniform(-1, 1, (B, K, N) if b_b else (K, N)).astype(np.float32)
    f = J.JAX.vmap(lambda a, w: a.dot(w), in_axes=[0 if a_b else -1, 0 if b_b else -1])
    out = f(J.ConcreteNDArray.of(A), J.ConcreteNDArray.of(W)).numpy()
    assert out.shape == (B, M, N)
    for i in range(B):
        ref = orc.dot(A[i] if a_b else A, W[i] if b_b else W)
        assert_rel(out[i], ref, TOL_REDUCTION, f"example {i}")


def test_vmap_mlp_forward_per_example_against_oracle(J):
    """A per-example 2-layer tanh MLP forward + loss, batched over 256 examples
    (one GEMM per layer for the whole batch), against the oracle per example."""
    r = np.random.default_rng(5)
    dims = [96, 64, 10]
    ws = [r.uniform(-0.2, 0.2, (dims[i], dims[i + 1])).astype(np.float32) for i in range(2)]
    bs = [r.uniform(-0.1, 0.1, dims[i + 1]).astype(np.float32) for i in range(2)]
    X = r.standard_normal((256, 1, 96)).astype(np.float32)
    T = np.zeros((256, 1, 10), np.float32)
    T[np.arange(256), 0, np.arange(256) % 10] = 1
    W1, W2 = (J.ConcreteNDArray.of(w) for w in ws)
    B1, B2 = (J.ConcreteNDArray.of(b) for b in bs)
    neg = J.ConcreteNDArray.scalar(-1.0)

    def per_example(x, t):
        h = x.dot(W1).add(B1).tanh()
        logits = h.dot(W2).add(B2)
        return J.Nn.softmax(logits).log().mul(t).sum(-1).mean().mul(neg)

    out = J.JAX.vmap(per_example)(J.ConcreteNDArray.of(X), J.ConcreteNDArray.of(T)).numpy()
    ref = np.float32([orc.mlp_loss(ws, bs, X[i], T[i], act="tanh") for i in range(256)])
    assert_rel(out, ref, TOL_REDUCTION)


def test_vmap_rejects_unbatched_psum(J):
    with pytest.raises(J.UnsupportedOperationException):
        J.JAX.vmap(lambda x: J.Lax.psum(x))(arr(J, [1, 2, 3, 4], (2, 2)))


@pytest.mark.parametrize("a_b,b_b,B,M,K,N", [(False, True, 5, 130, 200, 70), (True, True, 3, 256, 96, 300),
                                               (True, True, 7, 1, 33, 9)])
def test_strided_batched_gemm_one_launch(J, a_b, b_b, B, M, K, N):
    """j4c_dot_split_batched covers every (example, tile) in one launch."""
    from jax4j_b200 import _lib
    r = np.random.default_rng(B * 100 + M)
    A = r.uniform(-1, 1, (B, M, K) if a_b else (M, K)).astype(np.float32)
    W = r.uniform(-1, 1, (B, K, N) if b_b else (K, N)).astype(np.float32)
    f = J.JAX.vmap(lambda a, w: a.dot(w), in_axes=[0 if a_b else -1, 0 if b_b else -1])
    n0 = _lib.kernel_launches()
    out = f(J.ConcreteNDArray.of(A), J.ConcreteNDArray.of(W))
    launched = _lib.kernel_launches() - n0
    # two operand splits (each a line-max pass and the split) and one GEMM
    assert launched <= 5, launched
    o = out.numpy()
    for i in range(B):
        assert_rel(o[i], orc.dot(A[i] if a_b else A, W[i] if b_b else W), TOL_REDUCTION, f"example {i}")


def _ints(J, v, shape):
    return J.ConcreteNDArray.of(np.asarray(v, np.int32).reshape(shape), dtype=J.DType.INT32)


def test_take_looks_up_rows(J):  # DTypeTest.java:172-181
    table = arr(J, [10, 11, 20, 21, 30, 31, 40, 41], (4, 2))
    out = J.Numpy.take(table, _ints(J, [2, 0, 3], (3,)))
    assert out.shape().dimensions() == (3, 2)
    np.testing.assert_allclose(out.toFloatArray(), [30, 31, 10, 11, 40, 41], atol=1e-6)


def test_take_multi_dim_indices(J):  # DTypeTest.java:183-191
    out = J.Numpy.take(arr(J, [1, 1, 2, 2, 3, 3], (3, 2)), _ints(J, [0, 1, 2, 0], (2, 2)))
    assert out.shape().dimensions() == (2, 2, 2)
    np.testing.assert_allclose(out.toFloatArray(), [1, 1, 2, 2, 3, 3, 1, 1], atol=1e-6)


def test_take_gradient_scatter_adds(J):  # DTypeTest.java:193-204
    idx = _ints(J, [0, 0, 1], (3,))
    g = J.JAX.grad(lambda t: J.Numpy.take(t, idx).sum())(arr(J, [0, 0, 0], (3, 1)))
    np.testing.assert_allclose(g.toFloatArray(), [2, 1, 0], atol=1e-6)


def test_take_composes_with_vmap(J):  # DTypeTest.java:206-214
    table = arr(J, [1, 2, 3, 4], (2, 2))
    out = J.JAX.vmap(lambda idx: J.Numpy.take(table, idx))(_ints(J, [0, 1], (2, 1)))
    assert out.shape().dimensions() == (2, 1, 2)
    np.testing.assert_allclose(out.toFloatArray(), [1, 2, 3, 4], atol=1e-6)


def test_take_embedding_bag_grad_at_size(J):
    """A 50k x 64 embedding table, 20k lookups with many repeats: forward rows
    exact, gradient equal to numpy's scatter-add (within the reduction
    tolerance: repeated rows accumulate in an unspecified order)."""
    r = np.random.default_rng(2)
    T = r.standard_normal((50000, 64)).astype(np.float32)
    I = r.integers(0, 50000, 20000).astype(np.int64)
    I[:5000] = r.integers(0, 100, 5000)
    table, idx = J.ConcreteNDArray.of(T), J.ConcreteNDArray.of(I, dtype=J.DType.INT64)
    np.testing.assert_array_equal(J.Numpy.take(table, idx).numpy(), T[I])
    w = J.ConcreteNDArray.of(r.standard_normal((20000, 64)).astype(np.float32))
    g = J.JAX.grad(lambda t: J.Numpy.take(t, idx).mul(w).sum())(table).numpy()
    ref = np.zeros_like(T, dtype=np.float64)
    np.add.at(ref, I, w.numpy().astype(np.float64))
    assert_rel(g, ref.astype(np.float32), TOL_REDUCTION)


def test_take_rejects_out_of_range(J):
    with pytest.raises(J.IllegalArgumentException):
        J.Numpy.take(arr(J, [1, 2, 3, 4], (2, 2)), _ints(J, [0, 2], (2,)))
