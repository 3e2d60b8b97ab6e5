"""Shared test helpers."""
import numpy as np

# Tolerances of the north-star contract: bit-exact for BOOL/INT32/index
# outputs; FP32 elementwise 1e-5 and reductions/dot/gradients 1e-4, relative
# in the per-tensor sense |g - r| <= tol * max(|r|, rms(r)).
TOL_ELEMENTWISE = 1e-5
TOL_REDUCTION = 1e-4


def assert_rel(got, ref, tol, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    if ref.size == 0:
        return
    both_nan = np.isnan(got) & np.isnan(ref)
    assert not np.any(np.isnan(got) ^ np.isnan(ref)), f"{what}: NaN pattern differs"
    g = np.where(both_nan, 0, got)
    r = np.where(both_nan, 0, ref)
    rms = float(np.sqrt(np.mean(r * r)))
    bound = tol * np.maximum(np.abs(r), rms)
    err = np.abs(g - r)
    bad = err > bound + 1e-30
    if np.any(bad):
        i = int(np.argmax(err - bound))
        raise AssertionError(f"{what}: {int(bad.sum())} of {ref.size} elements beyond tol {tol}; "
                             f"worst at flat {i}: got {g.flat[i]!r} ref {r.flat[i]!r} (rms {rms:.3g})")


class JavaRandom:
    """java.util.Random as the Java SE API specifies it (a 48-bit linear
    congruential generator; nextDouble from 53 bits; nextGaussian by the
    polar method with the second deviate cached), so the reference's tests
    that seed `new java.util.Random(seed)` get the same input matrices."""
    _MULT, _ADD, _MASK = 0x5DEECE66D, 0xB, (1 << 48) - 1

    def __init__(self, seed: int):
        self._seed = (seed ^ self._MULT) & self._MASK
        self._next_gaussian = None

    def _next(self, bits: int) -> int:
        self._seed = (self._seed * self._MULT + self._ADD) & self._MASK
        v = self._seed >> (48 - bits)
        return v - (1 << 32) if v >= 1 << 31 else v  # Java's (int) narrowing

    def nextDouble(self) -> float:
        return ((self._next(26) << 27) + self._next(27)) * 2.0 ** -53

    def nextGaussian(self) -> float:
        if self._next_gaussian is not None:
            v, self._next_gaussian = self._next_gaussian, None
            return v
        while True:
            v1 = 2.0 * self.nextDouble() - 1.0
            v2 = 2.0 * self.nextDouble() - 1.0
            s = v1 * v1 + v2 * v2
            if 0.0 < s < 1.0:
                break
        mul = np.sqrt(-2.0 * np.log(s) / s)
        self._next_gaussian = float(v2 * mul)
        return float(v1 * mul)

    def gaussians(self, n: int) -> np.ndarray:
        return np.array([self.nextGaussian() for _ in range(n)])
