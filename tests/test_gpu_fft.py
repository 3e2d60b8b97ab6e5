"""Fft on the device (cuFFT through j4c_fft / j4c_rfft / j4c_irfft / j4c_dct1)
against the oracle's restatement of the reference's radix-2 transform, and
the reference's own test cases (T/FftTest.java, T/FftGpuTest.java,
T/FftGpu3DTest.java).  Tolerances are the reference's: FP64 1e-9 (1e-8 for
3-D grids), FP32 1e-4 (1e-3 for 3-D grids), relative to the tensor's scale
(tests/util.assert_rel)."""
import numpy as np
import pytest

from oracle import oracle as orc
from tests.util import assert_rel

pytestmark = pytest.mark.gpu

TOL = {np.float64: 1e-9, np.float32: 1e-4}
TOL3 = {np.float64: 1e-8, np.float32: 1e-3}


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def arr(J, a):
    a = np.ascontiguousarray(a)
    dt = J.DType.FLOAT64 if a.dtype == np.float64 else J.DType.FLOAT32
    return J.ConcreteNDArray.of(a, J.Shape(a.shape), dt)


@pytest.mark.parametrize("dt", [np.float32, np.float64])
@pytest.mark.parametrize("n", [1, 2, 16, 256, 4096, 1 << 16])
def test_fft_ifft_rfft_irfft_match_oracle(J, n, dt):
    r = np.random.default_rng(n)
    re, im = r.standard_normal(n).astype(dt), r.standard_normal(n).astype(dt)
    for inverse in (False, True):
        got = (J.Fft.ifft if inverse else J.Fft.fft)(arr(J, re), arr(J, im))
        want = orc.fft(re, im, inverse)
        assert got[0].dtype() == got[1].dtype() and got[0].numpy().dtype == dt
        assert_rel(got[0].numpy(), want[0], TOL[dt], f"re n={n} inverse={inverse}")
        assert_rel(got[1].numpy(), want[1], TOL[dt], f"im n={n} inverse={inverse}")
    hr, hi = J.Fft.rfft(arr(J, re))
    wr, wi = orc.rfft(re)
    assert hr.shape().dimensions() == (n // 2 + 1,)
    assert_rel(hr.numpy(), wr, TOL[dt])
    assert_rel(hi.numpy(), wi, TOL[dt])
    if n >= 2:
        # an arbitrary (non-Hermitian) half spectrum: the real part of the mirrored inverse
        h = n // 2 + 1
        sr, si = r.standard_normal(h).astype(dt), r.standard_normal(h).astype(dt)
        got = J.Fft.irfft(arr(J, sr), arr(J, si))
        assert got.shape().dimensions() == (n,)
        assert_rel(got.numpy(), orc.irfft(sr, si), TOL[dt])


@pytest.mark.parametrize("dt", [np.float32, np.float64])
@pytest.mark.parametrize("shape", [(16, 8, 32), (16, 16, 32), (8, 8, 16), (64, 64, 64), (1, 8, 16), (8, 1, 4),
                                   (2, 2, 2), (4, 4, 1)])
def test_3d_transforms_match_oracle(J, shape, dt):
    r = np.random.default_rng(sum(shape))
    re, im = r.standard_normal(shape).astype(dt), r.standard_normal(shape).astype(dt)
    for inverse in (False, True):
        got = (J.Fft.ifft3 if inverse else J.Fft.fft3)(arr(J, re), arr(J, im))
        want = orc.fft(re, im, inverse)
        assert_rel(got[0].numpy(), want[0], TOL3[dt])
        assert_rel(got[1].numpy(), want[1], TOL3[dt])
    hr, hi = J.Fft.rfft3(arr(J, re))
    wr, wi = orc.rfft(re)
    assert hr.shape().dimensions() == shape[:2] + (shape[2] // 2 + 1,)
    assert_rel(hr.numpy(), wr, TOL3[dt])
    assert_rel(hi.numpy(), wi, TOL3[dt])
    if shape[2] >= 2:
        sshape = shape[:2] + (shape[2] // 2 + 1,)
        sr, si = r.standard_normal(sshape).astype(dt), r.standard_normal(sshape).astype(dt)
        got = J.Fft.irfft3(arr(J, sr), arr(J, si))
        assert got.shape().dimensions() == shape
        assert_rel(got.numpy(), orc.irfft(sr, si), TOL3[dt])
        same = J.Fft.irfft3OnDevice(arr(J, sr), arr(J, si), shape[2])
        np.testing.assert_array_equal(same.numpy(), got.numpy())


@pytest.mark.parametrize("dt", [np.float32, np.float64])
@pytest.mark.parametrize("n", [1, 2, 3, 5, 17, 33, 257, 4097])
def test_dct1_matches_oracle(J, n, dt):
    x = np.random.default_rng(n).standard_normal(n).astype(dt)
    got = J.Fft.dctI(arr(J, x)).numpy()
    assert_rel(got, orc.dct1(x), TOL[dt] if n < 1000 else 10 * TOL[dt])


# ---- T/FftTest.java, through the device ---------------------------------------------
def test_reference_fft_closed_forms(J):
    got = J.Fft.fft(arr(J, np.array([1.0, 2, 3, 4])), arr(J, np.zeros(4)))
    np.testing.assert_allclose(got[0].numpy(), [10, -2, -2, -2], atol=1e-12)
    np.testing.assert_allclose(got[1].numpy(), [0, 2, 0, -2], atol=1e-12)
    got = J.Fft.fft(arr(J, np.ones(16)), arr(J, np.zeros(16)))
    np.testing.assert_allclose(got[0].numpy(), np.r_[16.0, np.zeros(15)], atol=1e-10)
    np.testing.assert_allclose(got[1].numpy(), np.zeros(16), atol=1e-10)


def test_reference_round_trips(J):
    r = np.random.default_rng(42)
    a, b = r.standard_normal(64), r.standard_normal(64)
    back = J.Fft.ifft(*J.Fft.fft(arr(J, a), arr(J, b)))
    np.testing.assert_allclose(back[0].numpy(), a, atol=1e-12)
    np.testing.assert_allclose(back[1].numpy(), b, atol=1e-12)
    a32, b32 = (r.standard_normal(32).astype(np.float32) for _ in range(2))
    back = J.Fft.ifft(*J.Fft.fft(arr(J, a32), arr(J, b32)))
    np.testing.assert_allclose(back[0].numpy(), a32, atol=1e-4)
    np.testing.assert_allclose(back[1].numpy(), b32, atol=1e-4)
    x = r.standard_normal(64)
    fr, fi = J.Fft.fft(arr(J, x), arr(J, np.zeros(64)))
    hr, hi = J.Fft.rfft(arr(J, x))
    np.testing.assert_allclose(hr.numpy(), fr.numpy()[:33], atol=1e-12)
    np.testing.assert_allclose(hi.numpy(), fi.numpy()[:33], atol=1e-12)
    np.testing.assert_allclose(J.Fft.irfft(hr, hi).numpy(), x, atol=1e-12)
    x32 = r.standard_normal(128).astype(np.float32)
    np.testing.assert_allclose(J.Fft.irfft(*J.Fft.rfft(arr(J, x32))).numpy(), x32, atol=1e-4)
    g = r.standard_normal((8, 4, 16))
    h = r.standard_normal((8, 4, 16))
    back = J.Fft.ifft3(*J.Fft.fft3(arr(J, g), arr(J, h)))
    np.testing.assert_allclose(back[0].numpy(), g, atol=1e-10)
    np.testing.assert_allclose(back[1].numpy(), h, atol=1e-10)
    np.testing.assert_allclose(J.Fft.irfft3(*J.Fft.rfft3(arr(J, g))).numpy(), g, atol=1e-10)
    g32 = g.astype(np.float32)
    np.testing.assert_allclose(J.Fft.irfft3(*J.Fft.rfft3(arr(J, g32))).numpy(), g32, atol=1e-3)


def test_reference_dct1(J):
    r = np.random.default_rng(11)
    n = 17
    x = r.standard_normal(n)
    j = np.arange(1, n - 1)
    want = [x[0] + (1 if k % 2 == 0 else -1) * x[-1] + 2 * np.sum(x[1:-1] * np.cos(np.pi * j * k / (n - 1)))
            for k in range(n)]
    np.testing.assert_allclose(J.Fft.dctI(arr(J, x)).numpy(), want, atol=1e-9)
    x = r.standard_normal(33)
    np.testing.assert_allclose(J.Fft.dctI(J.Fft.dctI(arr(J, x))).numpy(), 64.0 * x, atol=1e-9)
    one = arr(J, np.array([3.14]))
    assert J.Fft.dctI(one) is one  # length 1: the input itself (FftTest.java:223-229)
    raw_in = np.array(x)
    raw = J.Fft.dctIRaw(raw_in)
    np.testing.assert_allclose(raw, J.Fft.dctI(arr(J, x)).numpy(), atol=1e-15)
    np.testing.assert_array_equal(raw_in, x)  # not mutated (FftTest.java:256-271)
    y = J.Fft.dctIRaw([3.14])
    assert y.shape == (1,) and y[0] == 3.14


def test_reference_invalid_lengths(J):
    IAE = J.IllegalArgumentException
    with pytest.raises(IAE):
        J.Fft.fft(arr(J, np.array([1.0, 2, 3])), arr(J, np.zeros(3)))
    with pytest.raises(IAE):
        J.Fft.rfft(arr(J, np.ones(6)))
    with pytest.raises(IAE):
        J.Fft.dctI(arr(J, np.ones(6)))
    with pytest.raises(IAE):
        J.Fft.dctIRaw(np.ones(6))
    with pytest.raises(IAE):
        J.Fft.dctIRaw([])
    with pytest.raises(IAE):
        J.Fft.fft3(arr(J, np.ones((4, 3, 4))), arr(J, np.ones((4, 3, 4))))
    with pytest.raises(IAE):
        J.Fft.fft(arr(J, np.ones(4)), arr(J, np.ones(4, np.float32)))
    with pytest.raises(IAE):
        J.Fft.irfft(arr(J, np.ones(4)), arr(J, np.ones(4)))  # implies N = 6
    with pytest.raises(IAE):
        J.Fft.rfft(arr(J, np.ones((4, 4))))
