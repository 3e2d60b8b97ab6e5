"""Linalg on the device (cuSOLVER through j4c_lu_factor / j4c_lu_solve /
j4c_lu_rcond / j4c_eig / j4c_svd): the reference's own cases
(T/LinalgTest.java, T/LinalgSvdTest.java) with their tolerances, parity with
the oracle's restatement of the LU path (factor checks, solves, Hager's
estimate) on the same inputs, and size-independent properties at larger
sizes (residuals, trace = sum of eigenvalues, A = U diag(sigma) Vt,
orthonormality).  Eigenvalues and singular values are compared, as sets,
with the oracle's restatement of the reference's Francis QR and
Golub-Kahan-Reinsch (and with numpy's LAPACK): the device and the
reference order them differently, and both sets are unique."""
import math

import numpy as np
import pytest

from oracle import oracle as orc
from tests.util import JavaRandom

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def arr(J, a, dt=None):
    a = np.ascontiguousarray(a, dtype=dt or np.asarray(a).dtype)
    if a.dtype not in (np.float32, np.float64):
        a = a.astype(np.float64)
    d = J.DType.FLOAT64 if a.dtype == np.float64 else J.DType.FLOAT32
    return J.ConcreteNDArray.of(a, J.Shape(a.shape), d)


def mat(J, n, *v):
    return arr(J, np.array(v, np.float64).reshape(n, -1))


def vec(J, *v):
    return arr(J, np.array(v, np.float64))


def hilbert(n):
    i = np.arange(n)
    return 1.0 / (i[:, None] + i[None, :] + 1)


RC = "SINGULARITY_CHECK_RECIPROCAL_CONDITION_EST"
SM = "SINGULARITY_CHECK_SUBMATRIX_MAX"


def check(J, name):
    return getattr(J.SingularityCheck, name)


# ---- T/LinalgTest.java --------------------------------------------------------------
def test_solve_identity_known_and_pivoting(J):
    x = J.Linalg.solve(mat(J, 3, 1, 0, 0, 0, 1, 0, 0, 0, 1), vec(J, 3.14, -2.7, 1.0)).toDoubleArray()
    np.testing.assert_allclose(x, [3.14, -2.7, 1.0], atol=1e-15)
    x = J.Linalg.solve(mat(J, 3, 2, 1, 1, 1, 3, 2, 1, 0, 0), vec(J, 4, 5, 6)).toDoubleArray()
    np.testing.assert_allclose(x, [6, 15, -23], atol=1e-12)
    x = J.Linalg.solve(mat(J, 3, 0, 1, 2, 3, 4, 5, 6, 7, 9), vec(J, 3, 12, 22)).toDoubleArray()
    np.testing.assert_allclose(x, [1, 1, 1], atol=1e-12)


def test_solve_random_dense_by_residual(J):
    n, r = 20, JavaRandom(31)
    a = r.gaussians(n * n).reshape(n, n) + n * np.eye(n)
    x_true = r.gaussians(n)
    b = a @ x_true
    x = J.Linalg.solve(arr(J, a), arr(J, b)).toDoubleArray()
    np.testing.assert_allclose(a @ x, b, atol=1e-10)


def test_singular_and_shape_errors(J):
    IAE = J.IllegalArgumentException
    sing = mat(J, 3, 1, 2, 3, 2, 4, 6, 0, 0, 1)
    with pytest.raises(IAE, match=r"column 1 has zero pivot"):
        J.Linalg.solve(sing, vec(J, 1, 2, 3))
    with pytest.raises(IAE):
        J.Linalg.lu(sing)
    with pytest.raises(IAE):
        J.Linalg.lu(sing, check(J, SM))
    with pytest.raises(IAE):
        J.Linalg.solve(mat(J, 2, 1, 2, 3, 4), vec(J, 1, 2, 3))
    lu = J.Linalg.lu(mat(J, 3, 1, 0, 0, 0, 1, 0, 0, 0, 1))
    with pytest.raises(IAE, match="length-3"):
        lu.solve(vec(J, 1, 2))
    with pytest.raises(IAE, match="square"):
        J.Linalg.lu(arr(J, np.arange(6.0).reshape(2, 3)))
    with pytest.raises(IAE, match="matching dtypes"):
        J.Linalg.solve(mat(J, 2, 1, 0, 0, 1), arr(J, np.ones(2, np.float32)))
    with pytest.raises(IAE, match="2-D"):
        J.Linalg.lu(vec(J, 1, 2))
    with pytest.raises(IAE, match="FLOAT32 or FLOAT64"):
        J.Linalg.lu(J.ConcreteNDArray.of(np.eye(2, dtype=np.int32), J.Shape(2, 2), J.DType.INT32))


def test_submatrix_check_matches_oracle_message(J):
    """A nonzero pivot below 1e-14 x max|a_ij| fails the default check at the
    same elimination step as the oracle, with the reference's message; the
    reciprocal-condition mode then rejects it through Hager's estimate."""
    a = np.array([[1.0, 1.0], [1.0, 1.0 + 1e-15]])
    st, _, _, norms, k, p = orc.lu_factor(a)
    assert st == orc.LU_SUBMATRIX and k == 1
    with pytest.raises(J.IllegalArgumentException, match="SUBMATRIX_MAX check"):
        J.Linalg.lu(arr(J, a))
    with pytest.raises(J.IllegalArgumentException, match="ill-conditioned"):
        J.Linalg.lu(arr(J, a), check(J, RC))


def test_eig_reference_cases(J):
    w = J.Linalg.eig(mat(J, 4, 3, 0, 0, 0, 0, -1, 0, 0, 0, 0, 7, 0, 0, 0, 0, 2))
    np.testing.assert_allclose(np.sort(w[0].toDoubleArray()), [-1, 2, 3, 7], atol=1e-12)
    np.testing.assert_allclose(w[1].toDoubleArray(), 0, atol=1e-12)
    wr = np.sort(J.Linalg.eig(mat(J, 2, 2, 1, 1, 2))[0].toDoubleArray())
    np.testing.assert_allclose(wr, [1, 3], atol=1e-13)
    wr, wi = (t.toDoubleArray() for t in J.Linalg.eig(mat(J, 2, 0, -1, 1, 0)))
    np.testing.assert_allclose(wr, 0, atol=1e-12)
    np.testing.assert_allclose(np.abs(wi), 1, atol=1e-12)
    assert abs(wi[0] + wi[1]) <= 1e-12
    wr = np.sort(J.Linalg.eig(mat(J, 3, 0, 0, 0, 1, 0, 1, 0, 1, 0))[0].toDoubleArray())
    np.testing.assert_allclose(wr, [-1, 0, 1], atol=1e-12)
    n, r = 6, JavaRandom(41)
    a = r.gaussians(n * n).reshape(n, n)
    assert abs(J.Linalg.eig(arr(J, a))[0].toDoubleArray().sum() - np.trace(a)) <= 1e-10


def test_generalized_eig_reference_cases(J):
    w = J.Linalg.eig(mat(J, 3, 1, 0, 0, 0, 4, 0, 0, 0, 9), mat(J, 3, 1, 0, 0, 0, 2, 0, 0, 0, 3))
    np.testing.assert_allclose(np.sort(w[0].toDoubleArray()), [1, 2, 3], atol=1e-12)
    np.testing.assert_allclose(w[1].toDoubleArray(), 0, atol=1e-12)
    wr = np.sort(J.Linalg.eig(mat(J, 2, 2, 1, 1, 2), mat(J, 2, 1, 0, 0, 1))[0].toDoubleArray())
    np.testing.assert_allclose(wr, [1, 3], atol=1e-13)
    n, r = 5, JavaRandom(53)
    a = r.gaussians(n * n).reshape(n, n)
    m = r.gaussians(n * n).reshape(n, n)
    b = m @ m.T + n * np.eye(n)
    lam = J.Linalg.eig(arr(J, a), arr(J, b))[0].toDoubleArray()
    tr = sum(J.Linalg.solve(arr(J, b), arr(J, a[:, j].copy())).toDoubleArray()[j] for j in range(n))
    assert abs(lam.sum() - tr) <= 1e-9
    with pytest.raises(J.IllegalArgumentException, match="share shape"):
        J.Linalg.eig(mat(J, 2, 1, 0, 0, 1), mat(J, 3, 1, 0, 0, 0, 1, 0, 0, 0, 1))


def test_lu_reuse_raw_and_float32(J):
    A = mat(J, 3, 2, 1, 1, 1, 3, 2, 1, 0, 0)
    b = vec(J, 4, 5, 6)
    lu = J.Linalg.lu(A)
    np.testing.assert_allclose(lu.solve(b).toDoubleArray(), J.Linalg.solve(A, b).toDoubleArray(), atol=1e-14)
    raw_in = np.array([4.0, 5.0, 6.0])
    raw = lu.solve(raw_in)
    assert isinstance(raw, np.ndarray) and raw.dtype == np.float64
    np.testing.assert_allclose(raw, lu.solve(b).toDoubleArray(), atol=1e-14)
    np.testing.assert_array_equal(raw_in, [4.0, 5.0, 6.0])
    n, r = 10, JavaRandom(1729)
    a = r.gaussians(n * n).reshape(n, n) + n * np.eye(n)
    lu = J.Linalg.lu(arr(J, a))
    assert lu.n() == n
    for _ in range(3):
        bb = arr(J, r.gaussians(n))
        np.testing.assert_allclose(lu.solve(bb).toDoubleArray(), J.Linalg.solve(arr(J, a), bb).toDoubleArray(),
                                   atol=1e-13)
    a32 = arr(J, np.array([[2, 1, 1], [1, 3, 2], [1, 0, 0]], np.float32))
    b32 = arr(J, np.array([4, 5, 6], np.float32))
    x = J.Linalg.lu(a32).solve(b32)
    assert x.dtype() == J.DType.FLOAT32
    np.testing.assert_allclose(x.toFloatArray(), [6, 15, -23], atol=1e-4)
    x = J.Linalg.lu(A).solve(b32)  # FLOAT64 factorisation, FLOAT32 right-hand side
    assert x.dtype() == J.DType.FLOAT32
    np.testing.assert_allclose(x.toFloatArray(), [6, 15, -23], atol=1e-4)


def test_singularity_check_modes_and_cond(J):
    A, b = mat(J, 3, 2, 1, 1, 1, 3, 2, 1, 0, 0), vec(J, 4, 5, 6)
    d = J.Linalg.solve(A, b).toDoubleArray()
    for mode in (SM, RC):
        np.testing.assert_allclose(J.Linalg.solve(A, b, check(J, mode)).toDoubleArray(), d, atol=1e-14)
        np.testing.assert_allclose(J.Linalg.lu(A, check(J, mode)).solve(b).toDoubleArray(), d, atol=1e-14)
    h4 = hilbert(4)
    x = J.Linalg.solve(arr(J, h4), vec(J, 1, 1, 1, 1), check(J, RC)).toDoubleArray()
    np.testing.assert_allclose(h4 @ x, 1, atol=1e-9)
    with pytest.raises(J.IllegalArgumentException, match="ill-conditioned"):
        J.Linalg.lu(arr(J, hilbert(15)), check(J, RC))
    assert abs(J.Linalg.cond(mat(J, 4, *np.eye(4).ravel())) - 1.0) <= 1e-13
    assert abs(J.Linalg.cond(mat(J, 3, 1, 0, 0, 0, 2, 0, 0, 0, 4)) - 4.0) <= 1e-12
    assert 3e5 <= J.Linalg.cond(arr(J, hilbert(5))) <= 3e6
    assert J.Linalg.cond(mat(J, 3, 1, 2, 3, 0, 0, 0, 4, 5, 6)) == math.inf
    assert J.Linalg.cond(mat(J, 2, 1.0, 1.0, 1.0, 1.0 + 1e-12)) > 1e10
    assert J.Linalg.cond(arr(J, np.arange(6.0).reshape(2, 3))) == math.inf  # rejected by the factorisation
    lu = J.Linalg.lu(arr(J, hilbert(5)))
    assert J.Linalg.cond(lu) == J.Linalg.cond(arr(J, hilbert(5)))


# ---- T/LinalgSvdTest.java -----------------------------------------------------------
def test_svd_reference_cases(J):
    s = J.Linalg.svd(mat(J, 3, 3, 0, 0, 0, 1, 0, 0, 0, 2)).sigma().toDoubleArray()
    np.testing.assert_allclose(s, [3, 2, 1], atol=1e-12)
    a = JavaRandom(29).gaussians(12).reshape(4, 3)
    U, s, Vt = (t.numpy() for t in J.Linalg.svd(arr(J, a)))
    assert U.shape == (4, 3) and s.shape == (3,) and Vt.shape == (3, 3)
    np.testing.assert_allclose((U * s) @ Vt, a, atol=1e-10)
    for seed, tol in ((31, 1e-9), (37, 1e-11)):
        a = JavaRandom(seed).gaussians(16).reshape(4, 4)
        U, s, Vt = (t.numpy() for t in J.Linalg.svd(arr(J, a)))
        np.testing.assert_allclose(U.T @ U, np.eye(4), atol=tol)
        np.testing.assert_allclose(Vt @ Vt.T, np.eye(4), atol=tol)
    target = np.array([1.0, 1e-3, 1e-6, 1e-9, 1e-12])
    s = J.Linalg.svd(arr(J, np.diag(target))).sigma().toDoubleArray()
    assert np.all(np.abs(s - target) / target <= 1e-13), s
    a = JavaRandom(43).gaussians(15).reshape(5, 3)
    s = J.Linalg.svd(arr(J, a)).sigma().toDoubleArray()
    assert np.all(s >= 0) and np.all(s[:-1] >= s[1:] - 1e-12)
    with pytest.raises(J.IllegalArgumentException, match="m >= n"):
        J.Linalg.svd(arr(J, np.ones((2, 3))))


def test_svd_float32_returns_float64(J):
    a = np.random.default_rng(3).standard_normal((6, 4)).astype(np.float32)
    svd = J.Linalg.svd(arr(J, a))
    assert svd.U().dtype() == J.DType.FLOAT64 and svd.sigma().dtype() == J.DType.FLOAT64
    U, s, Vt = (t.numpy() for t in svd)
    np.testing.assert_allclose((U * s) @ Vt, a.astype(np.float64), atol=1e-12)


# ---- parity with the oracle, and scale ----------------------------------------------------
@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("n", [1, 2, 3, 17, 64, 255, 1024])
def test_lu_solve_and_cond_match_oracle(J, n, dt):
    rng = np.random.default_rng(n)
    a = (rng.standard_normal((n, n)) + 2 * np.sqrt(n) * np.eye(n)).astype(dt)
    b = rng.standard_normal(n).astype(dt)
    st, lu, piv, norms, _, _ = orc.lu_factor(a.astype(np.float64))
    assert st == 0
    want = orc.lu_solve(lu, piv, b.astype(np.float64))
    f = J.Linalg.lu(arr(J, a))
    x = f.solve(arr(J, b))
    assert x.dtype() == (J.DType.FLOAT64 if dt == np.float64 else J.DType.FLOAT32)
    tol = 1e-12 if dt == np.float64 else 1e-6
    np.testing.assert_allclose(x.numpy().astype(np.float64), want, rtol=tol, atol=tol * np.abs(want).max())
    np.testing.assert_allclose(f.solveTranspose(b.astype(np.float64)), orc.lu_solve(lu, piv, b, transpose=True),
                               rtol=1e-12, atol=1e-12 * np.abs(want).max())
    kappa = 1.0 / orc.lu_rcond(lu, piv, norms[1])
    assert abs(J.Linalg.cond(arr(J, a)) - kappa) <= 1e-9 * kappa


@pytest.mark.parametrize("n", [4, 40, 200])
def test_ill_conditioned_matches_oracle_decision(J, n):
    """Matrices with a prescribed condition number on either side of the
    1e14 gate: the device accepts or rejects exactly where the oracle does."""
    rng = np.random.default_rng(100 + n)
    q1, _ = np.linalg.qr(rng.standard_normal((n, n)))
    q2, _ = np.linalg.qr(rng.standard_normal((n, n)))
    for kappa in (1e8, 1e17):
        a = (q1 * np.geomspace(1.0, 1.0 / kappa, n)) @ q2
        st, lu, piv, norms, _, _ = orc.lu_factor(a, False)
        rejected_ref = st != 0 or orc.lu_rcond(lu, piv, norms[1]) < 1e-14
        try:
            J.Linalg.lu(arr(J, a), check(J, RC))
            rejected = False
        except J.IllegalArgumentException:
            rejected = True
        assert rejected == rejected_ref == (kappa > 1e14)


@pytest.mark.parametrize("n", [1, 5, 64, 300])
def test_eig_matches_oracle_and_trace(J, n):
    rng = np.random.default_rng(n)
    a = rng.standard_normal((n, n))
    wr, wi = (t.toDoubleArray() for t in J.Linalg.eig(arr(J, a)))
    got = np.sort_complex(wr + 1j * wi)
    owr, owi = orc.eig(a)
    want = np.sort_complex(owr + 1j * owi)
    lapack = np.sort_complex(np.linalg.eigvals(a))
    np.testing.assert_allclose(want, lapack, atol=1e-9 * max(1.0, np.abs(lapack).max()))
    scale = max(1.0, np.abs(want).max())
    np.testing.assert_allclose(np.sort(got.real), np.sort(want.real), atol=1e-9 * scale)
    np.testing.assert_allclose(np.sort(np.abs(got.imag)), np.sort(np.abs(want.imag)), atol=1e-9 * scale)
    assert abs(wr.sum() - np.trace(a)) <= 1e-9 * scale * n
    assert abs(wi.sum()) <= 1e-9 * scale * n  # conjugate pairs
    w32 = J.Linalg.eig(arr(J, a.astype(np.float32)))
    assert w32[0].dtype() == J.DType.FLOAT32


@pytest.mark.parametrize("m,n", [(1, 1), (4, 3), (64, 64), (500, 200), (1024, 512)])
def test_svd_matches_oracle_and_reconstructs(J, m, n):
    rng = np.random.default_rng(m * 7 + n)
    a = rng.standard_normal((m, n))
    U, s, Vt = (t.numpy() for t in J.Linalg.svd(arr(J, a)))
    s_ref = orc.svd(a)[1] if m * n <= 100_000 else np.linalg.svd(a, compute_uv=False)
    np.testing.assert_allclose(s, s_ref, rtol=1e-11, atol=1e-11 * s[0])
    np.testing.assert_allclose((U * s) @ Vt, a, atol=1e-10 * s[0])
    np.testing.assert_allclose(U.T @ U, np.eye(n), atol=1e-10)
    np.testing.assert_allclose(Vt @ Vt.T, np.eye(n), atol=1e-10)


def test_large_solve_residual(J):
    """n = 4096 through the device path: relative residual at FP64 level."""
    n = 4096
    rng = np.random.default_rng(7)
    a = rng.standard_normal((n, n))
    b = rng.standard_normal(n)
    x = J.Linalg.solve(arr(J, a), arr(J, b)).toDoubleArray()
    r = np.abs(a @ x - b).max() / (np.abs(a).sum(axis=1).max() * np.abs(x).max())
    assert r < 1e-13, r
