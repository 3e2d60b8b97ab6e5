"""The algebraic identities the generated kernels rely on, checked on the host
with IEEE FP32 arithmetic (numpy float32), over every special value:

- Numpy.where's arithmetic blend c*x + (1-c)*y with c in {0, 1} equals
  s + (+0 * t) with s the selected operand and t the other (the kernels'
  j_where: two selects, one multiply, one add);
- a zero dividend over a non-zero, non-NaN divisor is the signed zero whose
  sign is the XOR of the operands' signs (r_div / j_div answer it directly);
- Java's Math.max / Math.min equal max.NaN / min.NaN whenever one operand is
  a non-zero constant (j_max_nz / j_min_nz), i.e. the +0 / -0 rule never
  applies."""
import itertools

import numpy as np

F = np.float32
SPECIAL = [F(0.0), F(-0.0), F(1.0), F(-1.0), F(2.5), F(-3e38), F(3e38), F(1e-45), F(-1e-45),
           F(np.inf), F(-np.inf), F(np.nan)]


def bits(x):
    return np.array([x], dtype=np.float32).view(np.uint32)[0]


def same(a, b):
    a, b = F(a), F(b)
    if np.isnan(a) or np.isnan(b):
        return bool(np.isnan(a) and np.isnan(b))
    return bits(a) == bits(b)


def test_where_blend_equals_select_plus_signed_zero():
    with np.errstate(all="ignore"):
        for c, x, y in itertools.product([F(0.0), F(1.0)], SPECIAL, SPECIAL):
            blend = F(F(c * x) + F(F(F(1.0) - c) * y))
            s, t = (x, y) if c == 1.0 else (y, x)
            fused = F(s + F(F(0.0) * t))
            assert same(blend, fused), (c, x, y, blend, fused)


def test_zero_dividend_shortcut_is_ieee_division():
    with np.errstate(all="ignore"):
        for a, b in itertools.product([F(0.0), F(-0.0)], SPECIAL):
            ref = F(a / b)
            if b == b and b != 0.0:
                sign = (bits(a) ^ bits(b)) & np.uint32(0x80000000)
                short = np.array([sign], dtype=np.uint32).view(np.float32)[0]
                assert same(ref, short), (a, b, ref, short)


def java_max(a, b):
    if np.isnan(a) or np.isnan(b):
        return F(np.nan)
    if a == 0.0 and b == 0.0:
        return a if not np.signbit(a) else b
    return a if a >= b else b


def java_min(a, b):
    if np.isnan(a) or np.isnan(b):
        return F(np.nan)
    if a == 0.0 and b == 0.0:
        return a if np.signbit(a) else b
    return a if a <= b else b


def max_nan(a, b):  # PTX max.NaN.f32 on operands that are not both zeros
    if np.isnan(a) or np.isnan(b):
        return F(np.nan)
    return a if a >= b else b


def min_nan(a, b):
    if np.isnan(a) or np.isnan(b):
        return F(np.nan)
    return a if a <= b else b


def test_max_min_against_a_non_zero_constant():
    consts = [c for c in SPECIAL if not (c == 0.0)]
    for a, k in itertools.product(SPECIAL, consts):
        for x, y in ((a, k), (k, a)):
            assert same(java_max(x, y), max_nan(x, y)), (x, y)
            assert same(java_min(x, y), min_nan(x, y)), (x, y)
