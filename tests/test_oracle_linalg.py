"""The oracle's restatement of api/Linalg.java's LU, solves and Hager estimate
against the reference's own test cases (T/LinalgTest.java), on the CPU."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.util import JavaRandom


def solve(a, b, submatrix=True):
    st, lu, piv, norms, k, p = orc.lu_factor(np.asarray(a, np.float64), submatrix)
    assert st == 0, (st, k, p)
    return orc.lu_solve(lu, piv, np.asarray(b, np.float64))


def cond(a):
    st, lu, piv, norms, _, _ = orc.lu_factor(np.asarray(a, np.float64), False)
    if st:
        return np.inf
    rc = orc.lu_rcond(lu, piv, norms[1])
    return np.inf if rc == 0 or not np.isfinite(rc) else 1.0 / rc


def hilbert(n):
    i = np.arange(n)
    return 1.0 / (i[:, None] + i[None, :] + 1)


def test_known_systems():
    np.testing.assert_allclose(solve(np.eye(3), [3.14, -2.7, 1.0]), [3.14, -2.7, 1.0], atol=1e-15)
    a = [[2, 1, 1], [1, 3, 2], [1, 0, 0]]
    np.testing.assert_allclose(solve(a, [4, 5, 6]), [6, 15, -23], atol=1e-12)
    np.testing.assert_allclose(solve([[0, 1, 2], [3, 4, 5], [6, 7, 9]], [3, 12, 22]), [1, 1, 1], atol=1e-12)


def test_random_dense_residual():
    """LinalgTest.testSolveRandomDenseByResidual: java.util.Random(31), n = 20, diagonal + n."""
    n, r = 20, JavaRandom(31)
    a = r.gaussians(n * n).reshape(n, n) + n * np.eye(n)
    x_true = r.gaussians(n)
    b = np.array([sum(a[i, j] * x_true[j] for j in range(n)) for i in range(n)])
    x = solve(a, b)
    np.testing.assert_allclose(a @ x, b, atol=1e-10)


def test_singular_matrices():
    st, _, _, _, k, p = orc.lu_factor(np.array([[1, 2, 3], [2, 4, 6], [0, 0, 1.0]]))
    assert st == orc.LU_ZERO_PIVOT and k == 1 and p == 0.0
    # a pivot that is not zero but below 1e-14 x max|a|
    st, _, _, norms, k, p = orc.lu_factor(np.array([[1.0, 1.0], [1.0, 1.0 + 1e-15]]))
    assert st == orc.LU_SUBMATRIX and k == 1 and 0 < p <= 1e-14 * norms[0]
    st, *_ = orc.lu_factor(np.array([[1.0, 1.0], [1.0, 1.0 + 1e-15]]), False)
    assert st == 0  # the reciprocal-condition mode only rejects exact zeros in the elimination


def test_transpose_solve():
    r = JavaRandom(1729)
    n = 10
    a = r.gaussians(n * n).reshape(n, n) + n * np.eye(n)
    st, lu, piv, *_ = orc.lu_factor(a)
    b = r.gaussians(n)
    np.testing.assert_allclose(a.T @ orc.lu_solve(lu, piv, b, transpose=True), b, atol=1e-12)
    np.testing.assert_allclose(a @ orc.lu_solve(lu, piv, b), b, atol=1e-12)


def test_condition_estimates():
    assert abs(cond(np.eye(4)) - 1.0) <= 1e-13
    assert abs(cond(np.diag([1.0, 2.0, 4.0])) - 4.0) <= 1e-12
    k5 = cond(hilbert(5))
    assert 3e5 <= k5 <= 3e6  # kappa_inf(H_5) ~ 9.44e5
    assert cond(np.array([[1, 2, 3], [0, 0, 0], [4, 5, 6.0]])) == np.inf
    assert cond(np.array([[1.0, 1.0], [1.0, 1.0 + 1e-12]])) > 1e10
    # Hilbert(15): past the 1e-14 reciprocal-condition gate
    st, lu, piv, norms, _, _ = orc.lu_factor(hilbert(15), False)
    assert st == 0 and orc.lu_rcond(lu, piv, norms[1]) < 1e-14
    # Hilbert(4) is accepted (kappa ~ 2.8e4)
    st, lu, piv, norms, _, _ = orc.lu_factor(hilbert(4), False)
    assert orc.lu_rcond(lu, piv, norms[1]) > 1e-14


@pytest.mark.parametrize("n", [1, 7, 64])
def test_hager_matches_exact_norm_on_small_cases(n):
    """Hager's estimate is a lower bound on ||A^-1||_inf, exact on diagonal and
    typically within a small factor on random matrices."""
    rng = np.random.default_rng(n)
    a = rng.standard_normal((n, n)) + 2 * np.sqrt(n) * np.eye(n)
    st, lu, piv, norms, _, _ = orc.lu_factor(a, False)
    est = 1.0 / (orc.lu_rcond(lu, piv, norms[1]) * norms[1])
    exact = np.abs(np.linalg.inv(a)).sum(axis=1).max()
    assert exact / 3 <= est <= exact * (1 + 1e-12)


# ---- eig / svd: T/LinalgTest.java and T/LinalgSvdTest.java through the oracle --------
def test_eig_reference_cases():
    wr, wi = orc.eig(np.diag([3.0, -1.0, 7.0, 2.0]))
    np.testing.assert_allclose(np.sort(wr), [-1, 2, 3, 7], atol=1e-12)
    np.testing.assert_allclose(wi, 0, atol=1e-12)
    np.testing.assert_allclose(np.sort(orc.eig(np.array([[2.0, 1.0], [1.0, 2.0]]))[0]), [1, 3], atol=1e-13)
    wr, wi = orc.eig(np.array([[0.0, -1.0], [1.0, 0.0]]))
    np.testing.assert_allclose(wr, 0, atol=1e-12)
    np.testing.assert_allclose(np.abs(wi), 1, atol=1e-12)
    assert abs(wi[0] + wi[1]) <= 1e-12
    np.testing.assert_allclose(np.sort(orc.eig(np.array([[0, 0, 0], [1, 0, 1], [0, 1, 0.0]]))[0]), [-1, 0, 1],
                               atol=1e-12)
    a = JavaRandom(41).gaussians(36).reshape(6, 6)
    assert abs(orc.eig(a)[0].sum() - np.trace(a)) <= 1e-10


@pytest.mark.parametrize("n", [1, 2, 7, 40, 150])
def test_eig_matches_lapack(n):
    a = np.random.default_rng(n).standard_normal((n, n))
    wr, wi = orc.eig(a)
    got, want = np.sort_complex(wr + 1j * wi), np.sort_complex(np.linalg.eigvals(a))
    np.testing.assert_allclose(got, want, atol=1e-10 * max(1.0, np.abs(want).max()))
    wr32, _ = orc.eig(a.astype(np.float32))
    assert wr32.dtype == np.float32


def test_svd_reference_cases():
    np.testing.assert_allclose(orc.svd(np.diag([3.0, 1.0, 2.0]))[1], [3, 2, 1], atol=1e-12)
    a = JavaRandom(29).gaussians(12).reshape(4, 3)
    u, s, vt = orc.svd(a)
    np.testing.assert_allclose((u * s) @ vt, a, atol=1e-10)
    for seed, tol in ((31, 1e-9), (37, 1e-11)):
        a = JavaRandom(seed).gaussians(16).reshape(4, 4)
        u, s, vt = orc.svd(a)
        np.testing.assert_allclose(u.T @ u, np.eye(4), atol=tol)
        np.testing.assert_allclose(vt @ vt.T, np.eye(4), atol=tol)
    target = np.array([1.0, 1e-3, 1e-6, 1e-9, 1e-12])
    s = orc.svd(np.diag(target))[1]
    assert np.all(np.abs(s - target) / target <= 1e-13)
    s = orc.svd(JavaRandom(43).gaussians(15).reshape(5, 3))[1]
    assert np.all(s >= 0) and np.all(s[:-1] >= s[1:] - 1e-12)


@pytest.mark.parametrize("m,n", [(1, 1), (3, 2), (30, 30), (120, 45)])
def test_svd_matches_lapack(m, n):
    a = np.random.default_rng(m + n).standard_normal((m, n))
    u, s, vt = orc.svd(a)
    np.testing.assert_allclose(s, np.linalg.svd(a, compute_uv=False), atol=1e-12 * s[0])
    np.testing.assert_allclose((u * s) @ vt, a, atol=1e-12 * s[0])
