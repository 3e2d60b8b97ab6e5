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
