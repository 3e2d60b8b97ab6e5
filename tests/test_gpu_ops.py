"""Parity of every device op with the CPU oracle on seeded inputs.

Bit-exact for BOOL/INT32/index results, the RNG streams and the IEEE
add/sub/mul/div/max/min; FP32 transcendental unary ops within 1e-5 and
reductions/dot within 1e-4 (relative per tensor, tests/util.py).
"""
import numpy as np
import pytest

from jax4j_b200 import _lib
from oracle import oracle as orc
from tests.util import TOL_ELEMENTWISE, TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def dev(J, a, dtype=None):
    a = np.asarray(a)
    dt = dtype or {np.dtype(np.float32): J.DType.FLOAT32, np.dtype(np.int32): J.DType.INT32,
                   np.dtype(np.bool_): J.DType.BOOL, np.dtype(np.float64): J.DType.FLOAT64,
                   np.dtype(np.int64): J.DType.INT64}[a.dtype]
    shape = list(a.shape) if a.ndim else [1]
    return J.ConcreteNDArray.of(a.reshape(shape), J.Shape(shape), dt)


def rng(seed=0):
    return np.random.default_rng(seed)


BIN = ["add", "sub", "mul", "div", "max", "min"]
SHAPES = [((4097,), (4097,)), ((3,), (1,)), ((64, 130), (130,)), ((64, 130), (64, 1)),
          ((5, 1, 7), (1, 6, 1)), ((2, 3, 4, 5), (3, 1, 5)), ((1,), (33, 17)), ((256, 1024), (256, 1024))]


@pytest.mark.parametrize("op", BIN)
@pytest.mark.parametrize("sa,sb", SHAPES)
def test_binary_bit_exact(J, op, sa, sb):
    r = rng(hash((op, sa, sb)) % 2**32)
    a = r.standard_normal(sa).astype(np.float32)
    b = r.standard_normal(sb).astype(np.float32)
    if op == "div":
        b[np.abs(b) < 1e-3] = 0.5
    got = getattr(dev(J, a), op)(dev(J, b)).numpy()
    ref = orc.binary(getattr(orc, op.upper()), a, b)
    np.testing.assert_array_equal(got, ref)


def test_binary_java_special_values(J):
    # zero dividends over every kind of divisor (division answers them directly)
    a = np.float32([np.nan, 1, -0.0, 0.0, np.inf, -np.inf, 3, 0,
                    0.0, -0.0, 0.0, -0.0, 0.0, -0.0, 0.0, -0.0, 0.0, -0.0])
    b = np.float32([1, np.nan, 0.0, -0.0, np.inf, 2, 0, 0,
                    3, 3, -3, -3, np.inf, -np.inf, 1e-45, -1e-45, np.nan, 3e38])
    for op in BIN:
        got = getattr(dev(J, a), op)(dev(J, b)).numpy()
        ref = orc.binary(getattr(orc, op.upper()), a, b)
        assert np.array_equal(got, ref, equal_nan=True), op
        real = ~np.isnan(ref)  # a NaN's sign is not observable in Java
        assert np.array_equal(np.signbit(got[real]), np.signbit(ref[real])), op


@pytest.mark.parametrize("op", ["gt", "ge", "lt", "le", "eq", "ne"])
def test_compare_bit_exact(J, op):
    r = rng(1)
    a = r.integers(-3, 4, (64, 129)).astype(np.float32)
    b = r.integers(-3, 4, (129,)).astype(np.float32)
    a[0, :4] = [np.nan, 0.0, -0.0, np.inf]
    got = getattr(dev(J, a), op)(dev(J, b)).toBoolArray().reshape(a.shape)
    ref = orc.compare(getattr(orc, op.upper()), orc.F32, a, b).astype(bool)
    np.testing.assert_array_equal(got, ref)
    ai = a[1:].astype(np.int32)
    bi = b.astype(np.int32)
    got = getattr(dev(J, ai), op)(dev(J, bi)).toBoolArray().reshape(ai.shape)
    np.testing.assert_array_equal(got, orc.compare(getattr(orc, op.upper()), orc.I32, ai, bi).astype(bool))


@pytest.mark.parametrize("op", ["exp", "log", "sin", "cos", "tanh", "relu", "sigmoid"])
@pytest.mark.parametrize("n", [1, 3, 4097, 1 << 20])
def test_unary(J, op, n):
    r = rng(n)
    x = (r.standard_normal(n) * 3).astype(np.float32)
    if op == "log":
        x = np.abs(x) + 1e-3
    got = getattr(dev(J, x), op)().toFloatArray()
    ref = orc.unary(getattr(orc, op.upper()), x)
    if op == "relu":
        np.testing.assert_array_equal(got, ref)
    else:
        assert_rel(got, ref, TOL_ELEMENTWISE, op)


def test_tanh_sigmoid_per_element_error_bounds(J):
    """The one-exponential tanh and sigmoid (jmath.cuh) against FP64, per
    element, with the bounds derived beside them: tanh within 13 units of
    2^-23 relative (1.6e-6) everywhere; sigmoid within (3.5 + 1.2|x|)
    units while its value is normal, below 1.2e-38 in absolute terms past
    x < -87.3; special values and signed zeros as the reference's
    (float) Math.tanh / 1 / (1 + Math.exp(-x))."""
    u = 2.0 ** -23
    r = rng(9)
    x = np.concatenate([np.linspace(-30, 30, 400001), r.standard_normal(200000) * 4,
                        np.linspace(-0.3, 0.3, 100001), np.geomspace(1e-38, 1e-2, 4000),
                        -np.geomspace(1e-38, 1e-2, 4000), np.linspace(-100, 100, 20001)]).astype(np.float32)
    xd = x.astype(np.float64)
    th = np.asarray(dev(J, x).tanh().toFloatArray(), np.float64)
    ref_t = np.tanh(xd)
    err_t = np.abs(th - ref_t) / np.maximum(np.abs(ref_t), 1e-300)
    assert err_t.max() <= 13 * u, f"tanh: worst {err_t.max() / u:.2f} u at x = {x[np.argmax(err_t)]!r}"
    sg = np.asarray(dev(J, x).sigmoid().toFloatArray(), np.float64)
    with np.errstate(over="ignore"):
        ref_s = 1.0 / (1.0 + np.exp(-xd))
    normal = ref_s >= 2.0 ** -126
    bound = (3.5 + 1.2 * np.abs(xd)) * u
    err_s = np.abs(sg - ref_s) / np.maximum(ref_s, 1e-300)
    assert np.all(err_s[normal] <= bound[normal]), \
        f"sigmoid: worst {np.max(err_s[normal] / bound[normal]):.3f} of the bound at x = {x[normal][np.argmax(err_s[normal] / bound[normal])]!r}"
    assert np.all(np.abs(sg - ref_s)[~normal] <= 2.0 ** -126)
    sp = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-45, -1e-45, 44.5, -44.5, 88.0, -88.0], np.float32)
    t = np.asarray(dev(J, sp).tanh().toFloatArray())
    s_ = np.asarray(dev(J, sp).sigmoid().toFloatArray())
    assert np.isnan(t[0]) and np.isnan(s_[0])
    assert t[1] == 1.0 and t[2] == -1.0 and s_[1] == 1.0 and s_[2] == 0.0
    assert t[3] == 0.0 and not np.signbit(t[3]) and t[4] == 0.0 and np.signbit(t[4])
    assert s_[3] == 0.5 and s_[4] == 0.5
    assert t[5] == np.float32(1e-45) and t[6] == np.float32(-1e-45)
    assert t[7] == 1.0 and t[8] == -1.0 and t[9] == 1.0 and t[10] == -1.0
    assert s_[9] == 1.0 and 0.0 <= s_[10] <= 2.0 ** -126


CASTS = [("float32", "int32"), ("float32", "bool"), ("float32", "float64"), ("float32", "int64"),
         ("int32", "float32"), ("int32", "bool"), ("bool", "float32"), ("bool", "int32"),
         ("float64", "float32"), ("float64", "int32"), ("int64", "int32"), ("int64", "float32")]


@pytest.mark.parametrize("src,dst", CASTS)
def test_cast_bit_exact(J, src, dst):
    r = rng(7)
    base = np.concatenate([r.standard_normal(1000) * 1e3,
                           [np.nan, np.inf, -np.inf, 3e10, -3e10, -0.0, 0.0, 2.5, -2.5, 1.0]])
    np_src = {"float32": np.float32, "float64": np.float64, "int32": np.int32, "int64": np.int64,
              "bool": np.bool_}[src]
    if src in ("int32", "int64", "bool"):
        base = np.nan_to_num(base, nan=0, posinf=0, neginf=0)
        if src == "int64":
            base = np.concatenate([base, [2**40 + 3, -(2**40) - 7]])
        elif src == "int32":
            base = np.clip(base, -2**31, 2**31 - 1)
    x = base.astype(np_src)
    D = {"float32": J.DType.FLOAT32, "float64": J.DType.FLOAT64, "int32": J.DType.INT32,
         "int64": J.DType.INT64, "bool": J.DType.BOOL}
    got = dev(J, x, D[src]).astype(D[dst]).numpy()
    O = {"float32": orc.F32, "float64": orc.F64, "int32": orc.I32, "int64": orc.I64, "bool": orc.BOOL}
    ref = orc.cast(O[src], O[dst], x.astype(np.uint8) if src == "bool" else x)
    if dst == "bool":
        ref = ref.astype(bool)
    assert np.array_equal(got, ref, equal_nan=True), (src, dst)


@pytest.mark.parametrize("n", [1, 5, 4096, 1 << 20, 3 * 1048576 + 7])
@pytest.mark.parametrize("mean", [False, True])
def test_reduce_all(J, n, mean):
    x = rng(n).standard_normal(n).astype(np.float32)
    a = dev(J, x)
    got = (a.mean() if mean else a.sum()).toFloatArray()
    ref = orc.reduce_all(orc.MEAN if mean else orc.SUM, x)
    # relative to the sum of magnitudes: the order of a float sum is free
    scale = float(np.abs(x).sum()) / (n if mean else 1)
    assert abs(float(got[0]) - float(ref[0])) <= TOL_REDUCTION * max(scale, 1e-30)


@pytest.mark.parametrize("shape,axis", [((4, 16384), -1), ((7, 33), 1), ((4096, 10), 1), ((8192, 64), 0),
                                        ((3, 1000, 5), 1), ((2, 3), 0), ((1, 1), 0), ((600, 2048), 1)])
@pytest.mark.parametrize("keep", [False, True])
@pytest.mark.parametrize("mean", [False, True])
def test_reduce_axis(J, shape, axis, keep, mean):
    x = rng(sum(shape)).standard_normal(shape).astype(np.float32)
    a = dev(J, x)
    got = (a.mean(axis, keep) if mean else a.sum(axis, keep)).numpy()
    ref = orc.reduce_axis(orc.MEAN_AXIS if mean else orc.SUM_AXIS, x, axis, keep)
    assert got.shape == ref.shape
    n = shape[axis]
    scale = np.abs(x).sum(axis=axis, keepdims=keep) / (n if mean else 1)
    assert np.all(np.abs(got - ref) <= TOL_REDUCTION * np.maximum(scale, 1e-30))


@pytest.mark.parametrize("shape,axis", [((4, 16384), -1), ((100, 7), 1), ((9, 3000), 1), ((64, 5), 0),
                                        ((3, 50, 4), 1)])
@pytest.mark.parametrize("op", ["argmax", "argmin"])
def test_argreduce_bit_exact(J, shape, axis, op):
    r = rng(3)
    x = r.integers(-5, 6, shape).astype(np.float32)  # many ties: the first must win
    if len(shape) == 2 and shape[1] > 3:
        x[0, 0] = np.nan          # NaN first: index 0 wins
        x[1, 2] = np.nan          # NaN later: skipped
        x[2, :] = -np.inf         # all equal: index 0
    got = getattr(dev(J, x), op)(axis).numpy()
    ref = orc.argreduce(getattr(orc, op.upper()), x, axis)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("gshape,tshape", [((64, 130), (130,)), ((64, 130), (64, 1)), ((64, 130), (1,)),
                                            ((4, 5, 6), (5, 1)), ((4, 5, 6), (4, 1, 6)),
                                            ((8192, 16), (16,)), ((3,), (2, 3)), ((6,), (2, 3)),
                                            ((2, 3, 4, 5), (3, 1, 5))])
def test_broadcast_like(J, gshape, tshape):
    from jax4j_b200 import grad as G
    g = rng(5).standard_normal(gshape).astype(np.float32)
    got = G.broadcast_like(dev(J, g), J.Shape(tshape)).numpy()
    ref = orc.broadcast_like(g, tshape)
    assert_rel(got, ref, TOL_REDUCTION, f"{gshape}->{tshape}")


def test_relu_and_maxmin_grad(J):
    from jax4j_b200 import grad as G
    r = rng(9)
    g = r.standard_normal((40, 50)).astype(np.float32)
    x = r.integers(-2, 3, (40, 50)).astype(np.float32)
    np.testing.assert_array_equal(G.relu_grad(dev(J, g), dev(J, x)).numpy(), orc.relu_grad(g, x))
    b = r.integers(-2, 3, (50,)).astype(np.float32)
    for is_max in (True, False):
        ga, gb = G.maxmin_grad(dev(J, g), dev(J, x), dev(J, b), is_max)
        ra, rb = orc.maxmin_grad(is_max, g, x, b)
        np.testing.assert_array_equal(ga.numpy(), ra)
        assert_rel(gb.numpy(), rb, TOL_REDUCTION)


@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (2, 3, 4), (37, 53, 29), (128, 128, 128), (256, 784, 512),
                                   (256, 512, 10), (300, 1000, 257), (1024, 1024, 1024)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_dot(J, M, K, N, ta, tb):
    from jax4j_b200.core import _dot_raw
    r = rng(M * 7 + K * 3 + N)
    A = r.uniform(-1, 1, (M, K)).astype(np.float32)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    a = dev(J, A.T.copy() if ta else A)
    b = dev(J, B.T.copy() if tb else B)
    got = _dot_raw(a, b, bool(ta), bool(tb), a.device()).numpy()
    ref = orc.dot(A, B, threads=8)
    assert_rel(got, ref, TOL_REDUCTION, f"dot {M}x{K}x{N} ta={ta} tb={tb}")


def test_dot_public_api_and_f64(J):
    r = rng(11)
    A = r.uniform(-1, 1, (65, 33)).astype(np.float32)
    B = r.uniform(-1, 1, (33, 17)).astype(np.float32)
    got = dev(J, A).dot(dev(J, B)).toFloatArray().reshape(65, 17)
    assert_rel(got, orc.dot(A, B), TOL_REDUCTION)
    got64 = dev(J, A.astype(np.float64)).dot(dev(J, B.astype(np.float64))).numpy()
    np.testing.assert_allclose(got64, A.astype(np.float64) @ B.astype(np.float64), rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (65, 33, 17), (130, 257, 200), (64, 8, 128)])
def test_dot_f64_tensor_path(J, ta, tb, M, K, N):
    """FLOAT64 dot on the FP64 tensor path (DMMA, k-groups of 4 per
    instruction): within 1e-12 of numpy's FP64 product, every layout, ragged
    tiles included."""
    r = rng(M * 7 + K)
    A = r.uniform(-1, 1, (K, M) if ta else (M, K))
    B = r.uniform(-1, 1, (N, K) if tb else (K, N))
    a, b = dev(J, A), dev(J, B)
    from jax4j_b200 import _lib
    import torch
    out = torch.empty(M * N, dtype=torch.float64, device="cuda")
    _lib.call("j4c_dot", 1, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, K, N, int(ta), int(tb),
              torch.cuda.current_stream().cuda_stream)
    ref = (A.T if ta else A) @ (B.T if tb else B)
    np.testing.assert_allclose(out.cpu().numpy().reshape(M, N), ref, rtol=1e-12, atol=1e-12 * max(1.0, np.sqrt(K)))


@pytest.mark.parametrize("rows,cols,special", [(300, 1000, False), (517, 130, True), (64, 4097, False)])
def test_sgd_update_lines_equals_update_then_max_pass(J, rows, cols, special):
    """j4c_sgd_update_lines (psumSgdTree's update of a 2-D weight) gives the
    elementwise chain's bits and the line words a max pass over the result
    would, NaN/Inf flag included."""
    import torch
    from jax4j_b200 import api as A, _lib
    r = rng(rows + cols)
    w = r.standard_normal((rows, cols)).astype(np.float32)
    g = (r.standard_normal((rows, cols)) * 10).astype(np.float32)
    if special:
        g[3, 5] = np.inf
        w[7, 1] = np.nan
    W, G = dev(J, w), dev(J, g)
    old = A.SGD_LINES_MIN
    try:
        A.SGD_LINES_MIN = 1
        got = A._sgd_leaf(W, G, 0.125, 0.01, A._sgd_update(0.125, 0.01))
    finally:
        A.SGD_LINES_MIN = old
    ref = A._sgd_update(0.125, 0.01)(W, G)
    np.testing.assert_array_equal(got.numpy().view(np.uint32), ref.numpy().view(np.uint32))
    assert got._lines is not None
    lines = torch.empty(rows + cols + 1, dtype=torch.int32, device="cuda")
    _lib.call("j4c_split_lines", ref.data_ptr(), rows, cols, lines.data_ptr(), torch.cuda.current_stream().cuda_stream)
    np.testing.assert_array_equal(got._lines.cpu().numpy(), lines.cpu().numpy())
    assert bool(got._lines[-1].item()) == special


def test_transpose(J):
    from jax4j_b200 import _lib
    import torch
    x = rng(1).standard_normal((37, 70)).astype(np.float32)
    a = dev(J, x)
    out = torch.empty(x.size, dtype=torch.float32, device="cuda")
    _lib.call("j4c_transpose", 0, a.data_ptr(), 37, 70, out.data_ptr(), a._stream())
    np.testing.assert_array_equal(out.cpu().numpy().reshape(70, 37), orc.transpose(x))


@pytest.mark.parametrize("n", [1, 17, 100003])
def test_random_streams_bit_exact(J, n):
    key = J.PRNGKey.key(12345)
    u = J.Random.uniform(key, J.Shape(n), -3.0, 3.0).toFloatArray()
    np.testing.assert_array_equal(u, orc.uniform(key.state(), (n,), -3.0, 3.0))
    g = J.Random.glorotUniform(key, J.Shape(n), 1024, 4096).toFloatArray()
    np.testing.assert_array_equal(g, orc.glorot_uniform(key.state(), (n,), 1024, 4096))
    z = J.Random.normal(key, J.Shape(n)).toFloatArray()
    # Box-Muller runs in double: libm and CUDA's double log/cos may differ in
    # the last double ulp, which can move the float by one ulp
    assert_rel(z, orc.normal(key.state(), (n,)), 1e-6)
    # a shard of the stream equals the same slice of the whole array
    part = J.Random.uniform(key, J.Shape(n), -3.0, 3.0, offset=n // 3, count=n - n // 3).toFloatArray()
    np.testing.assert_array_equal(part, u[n // 3:])
    assert [k.state() for k in J.Random.split(key, 5)] == orc.split(key.state(), 5)


def test_psum_slots_order(J):
    import ctypes as C
    from jax4j_b200 import _lib
    r = rng(2)
    slots = [r.standard_normal(10001).astype(np.float32) * 10 ** i for i in range(5)]
    arrs = [dev(J, s) for s in slots]
    import torch
    out = torch.empty(10001, dtype=torch.float32, device="cuda")
    ptrs = (C.c_void_p * 5)(*[a.data_ptr() for a in arrs])
    _lib.call("j4c_psum_slots", 0, ptrs, 5, out.data_ptr(), 10001, arrs[0]._stream())
    np.testing.assert_array_equal(out.cpu().numpy(), orc.psum(slots))


def test_device_placement_rules(J):
    # DevicePlacementTest.java:28-111
    g0, g1 = J.Device(None), J.Device(None)
    a = dev(J, np.float32([1, 2, 3])).to(g0)
    b = dev(J, np.float32([4, 5, 6])).to(g1)
    with pytest.raises(J.IllegalStateException, match="different devices"):
        a.add(b)
    c = dev(J, np.float32([4, 5, 6])).to(g0)
    r = a.mul(c)
    assert r.device() is g0
    np.testing.assert_allclose(r.toFloatArray(), [4, 10, 18])
    row = dev(J, np.float32([[1, 2, 3], [4, 5, 6]])).to(g0)
    assert row.add(dev(J, np.float32([10, 20, 30])).to(g0)).device() is g0
    h = J.Device.host()
    assert dev(J, np.float32([1, 2])).to(h).add(dev(J, np.float32([1, 1])).to(h)).device() is h


def test_empty_and_single_element(J):
    x = dev(J, np.float32([2.0]))
    assert x.sum().toFloatArray()[0] == 2.0
    assert x.argmax(0).toIntArray()[0] == 0
    e = J.ConcreteNDArray(np.zeros(0, np.float32), J.Shape(0, 3), J.DType.FLOAT32)
    assert e.add(e).shape() == J.Shape(0, 3)
    assert e.exp().shape() == J.Shape(0, 3)


def _split_alloc(J, x_dev, rd, cd, fill):
    """hi and lo arrays for a split whose data is [rd, cd], pre-filled."""
    import torch
    n = _lib.lib().j4c_split_floats(rd, cd)
    return [torch.full((n,), fill, dtype=torch.float32, device=x_dev) for _ in range(2)]


def _split_parts(hi, lo, rd, cd, axis):
    """Decode split arrays whose data is [rd, cd] in the library's format:
    (hi, lo) as float64 [rd, cd] in x's units, their padding columns, the
    per-element quantum below which an element's split is exact to an
    absolute error (3xFP16: the FP16 subnormal step of its line in x's
    units; 3xTF32: 0), and the line words (3xFP16; `axis` "rows" or "cols")."""
    from jax4j_b200.core import split_kind
    hb = hi.cpu().numpy().view(np.uint8)
    lb = lo.cpu().numpy().view(np.uint8)
    f16 = split_kind() == 1
    p = (cd + 7) // 8 * 8 if f16 else (cd + 3) // 4 * 4
    nb = rd * p * (2 if f16 else 4)
    n_lines = rd if axis == "rows" else cd
    words = hb[nb + 32:nb + 32 + 4 * n_lines].view(np.uint32)
    mx = words.view(np.float32).astype(np.float64)
    e = np.where(words == 0, 0, np.minimum(14 - (np.frexp(mx)[1] - 1), 126))
    sc = 2.0 ** -e.astype(np.float64)
    sc = sc[:, None] if axis == "rows" else sc[None, :]
    if f16:
        h = hb[:nb].view(np.float16).reshape(rd, p).astype(np.float64)
        l = lb[:nb].view(np.float16).reshape(rd, p).astype(np.float64)
        return h[:, :cd] * sc, l[:, :cd] * sc, (h[:, cd:], l[:, cd:]), 2.0 ** -24 * sc, words
    h = hb[:nb].view(np.float32).reshape(rd, p)
    l = lb[:nb].view(np.float32).reshape(rd, p)
    assert np.all(h[:, :cd].view(np.uint32) & 0x1FFF == 0) and np.all(l[:, :cd].view(np.uint32) & 0x1FFF == 0)
    return (h[:, :cd].astype(np.float64) * sc, l[:, :cd].astype(np.float64) * sc, (h[:, cd:], l[:, cd:]),
            2.0 ** -149 * sc, words)


def _split_written_bytes(rd, cd, n_lines):
    """Bytes of a hi array that a split writes (data, header, line words) and of a lo array."""
    from jax4j_b200.core import split_kind
    n = rd * ((cd + 7) // 8 * 8) * 2 if split_kind() == 1 else rd * ((cd + 3) // 4 * 4) * 4
    return n + 32 + 4 * n_lines, n


def _line_max_bits(x, axis):
    a = np.abs(np.where(np.isfinite(x), x, 0)).astype(np.float32)
    return a.max(axis=1 if axis == "rows" else 0).view(np.uint32)


@pytest.mark.parametrize("entry,axis", [("j4c_split_f32", "rows"), ("j4c_split_f32_cols", "cols")])
@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (37, 53), (64, 1000), (129, 4097)])
def test_split_f32_layout(J, rows, cols, entry, axis):
    """j4c_split_f32 (a line per row) and j4c_split_f32_cols (a line per
    column) in the library's format (3xFP16: each line scaled by 2^e with its
    max |x| 2^e in [2^14, 2^15), hi = fp16(x 2^e), lo = fp16(x 2^e - hi), the
    line maxima after the header; 3xTF32: hi = tf32(x), lo = tf32(x - hi)):
    hi + lo = x to 2^-21 relative (plus the FP16 subnormal step of the line
    for elements far below its max), padding zero.  The values span 2^+-29
    around 1, so lines differ in magnitude by many powers of two."""
    r = rng(rows * 31 + cols)
    x = (r.standard_normal((rows, cols)) * np.exp(r.uniform(-20, 20, (rows, cols)))).astype(np.float32)
    a = dev(J, x)
    hi, lo = _split_alloc(J, a.tensor().device, rows, cols, 7.0)
    _lib.call(entry, a.data_ptr(), rows, cols, hi.data_ptr(), lo.data_ptr(), a._stream())
    h, l, pads, quantum, words = _split_parts(hi, lo, rows, cols, axis)
    assert all(np.all(pd == 0) for pd in pads)
    np.testing.assert_array_equal(words, _line_max_bits(x, axis))
    err = np.abs(h + l - x)
    assert np.all(err <= np.abs(x) * 2.0 ** -21 + quantum)


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_dot_ws_and_split_reuse(J, ta, tb):
    """j4c_dot_ws (splits inside) and j4c_dot_split reusing the split of A
    that its layout takes in a second product with another operand."""
    import torch
    from jax4j_b200.core import _split_of
    M, K, N = 200, 300, 150
    r = rng(ta * 2 + tb + 5)
    A = r.uniform(-1, 1, (M, K)).astype(np.float32)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    a = dev(J, A.T.copy() if ta else A)
    b = dev(J, B.T.copy() if tb else B)
    ws_bytes = _lib.lib().j4c_dot_workspace_size(0, M, K, N)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=a.tensor().device)
    out = torch.empty(M * N, dtype=torch.float32, device=a.tensor().device)
    _lib.call("j4c_dot_ws", 0, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, K, N, ta, tb, ws.data_ptr(),
              ws_bytes, a._stream())
    ref = orc.dot(A, B, threads=8)
    assert_rel(out.cpu().numpy().reshape(M, N), ref, TOL_REDUCTION, "dot_ws")
    # op(A) . C2 twice with A's one split of the kind its layout needs
    ah, al = _split_of(a, "c" if ta else "r")
    for n2 in (70, 33):
        C2 = r.uniform(-1, 1, (K, n2)).astype(np.float32)
        c2 = dev(J, C2)
        ch, cl = _split_of(c2, "c")
        out2 = torch.empty(M * n2, dtype=torch.float32, device=a.tensor().device)
        _lib.call("j4c_dot_split", ah.data_ptr(), al.data_ptr(), ch.data_ptr(), cl.data_ptr(), out2.data_ptr(),
                  M, K, n2, ta, 0, a._stream())
        assert_rel(out2.cpu().numpy().reshape(M, n2), orc.dot(A, C2, threads=8), TOL_REDUCTION, "split reuse")


def test_dot_rejects_a_split_of_the_wrong_kind(J):
    """A K-major operand needs a split with row lines and an MN-major one
    column lines; a GEMM given the other kind computes nothing and records
    device status 0x7C06, and the library keeps working afterwards."""
    import ctypes as C
    import torch
    from jax4j_b200.core import _split_of
    M, K, N = 64, 96, 80
    r = rng(99)
    A = r.uniform(-1, 1, (M, K)).astype(np.float32)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    a, b = dev(J, A), dev(J, B)
    out = torch.full((M * N,), 5.0, dtype=torch.float32, device=a.tensor().device)
    (ah, al), (bh, bl) = _split_of(a, "c"), _split_of(b, "c")  # A wants row lines here
    _lib.call("j4c_dot_split", ah.data_ptr(), al.data_ptr(), bh.data_ptr(), bl.data_ptr(), out.data_ptr(),
              M, K, N, 0, 0, a._stream())
    torch.cuda.synchronize()
    code = C.c_int(0)
    assert _lib.lib().j4c_device_status(C.byref(code)) == 0
    assert code.value == 0x7C06
    assert torch.all(out == 5.0)  # nothing written
    ah, al = _split_of(a, "r")
    _lib.call("j4c_dot_split", ah.data_ptr(), al.data_ptr(), bh.data_ptr(), bl.data_ptr(), out.data_ptr(),
              M, K, N, 0, 0, a._stream())
    assert_rel(out.cpu().numpy().reshape(M, N), orc.dot(A, B), TOL_REDUCTION, "after the rejected call")
    assert _lib.lib().j4c_device_status(C.byref(code)) == 0 and code.value == 0


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (37, 53), (64, 1000), (130, 67)])
def test_split_f32_transposed_layout(J, rows, cols):
    """j4c_split_f32_transposed: the split of x^T as [cols, pitch(rows)],
    padding zero, a line per data row (x's columns)."""
    r = rng(rows * 17 + cols)
    x = (r.standard_normal((rows, cols)) * np.exp(r.uniform(-10, 10, (1, cols)))).astype(np.float32)
    a = dev(J, x)
    hi, lo = _split_alloc(J, a.tensor().device, cols, rows, 7.0)
    _lib.call("j4c_split_f32_transposed", a.data_ptr(), rows, cols, hi.data_ptr(), lo.data_ptr(), a._stream())
    h, l, pads, quantum, words = _split_parts(hi, lo, cols, rows, "rows")
    assert all(np.all(pd == 0) for pd in pads)
    np.testing.assert_array_equal(words, _line_max_bits(x, "cols"))
    err = np.abs(h + l - x.T)
    assert np.all(err <= np.abs(x.T) * 2.0 ** -21 + quantum)


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("M,K,N", [(200, 96, 130), (37, 53, 29)])
def test_dot_epilogue_equals_unfused_sequence(J, ta, tb, M, K, N):
    """j4c_dot_split_ep: bias add, relu output and relu' mask in the GEMM's
    store give exactly what the separate kernels give."""
    from jax4j_b200 import grad as G
    from jax4j_b200.core import _dot_raw
    r = rng(M + 3 * N + 7 * ta + 11 * tb)
    A = r.uniform(-1, 1, (M, K)).astype(np.float32)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    a = dev(J, A.T.copy() if ta else A)
    b = dev(J, B.T.copy() if tb else B)
    bias = dev(J, r.uniform(-1, 1, N).astype(np.float32))
    mask = dev(J, r.integers(-1, 2, (M, N)).astype(np.float32))
    plain = _dot_raw(a, b, bool(ta), bool(tb), a.device())
    z, h = _dot_raw(a, b, bool(ta), bool(tb), a.device(), bias=bias, act=True)
    np.testing.assert_array_equal(z.numpy(), plain.add(bias).numpy())
    np.testing.assert_array_equal(h.numpy(), plain.add(bias).relu().numpy())
    masked = _dot_raw(a, b, bool(ta), bool(tb), a.device(), mask=mask)
    np.testing.assert_array_equal(masked.numpy(), G.relu_grad(plain, mask).numpy())


def test_mlp_grads_with_gemm_epilogues_equal_the_unfused_interpreter(J):
    """The forward's DOT+bias+relu epilogues and the backward's relu'-masked
    input gradients change no bit of the loss or of any gradient."""
    from jax4j_b200 import grad as G
    r = rng(5)
    dims = [64, 96, 96, 10]
    ws = [dev(J, r.uniform(-0.3, 0.3, (dims[i], dims[i + 1])).astype(np.float32)) for i in range(3)]
    bs = [dev(J, r.uniform(-0.1, 0.1, dims[i + 1]).astype(np.float32)) for i in range(3)]
    x = dev(J, r.standard_normal((48, 64)).astype(np.float32))
    t = np.zeros((48, 10), np.float32)
    t[np.arange(48), np.arange(48) % 10] = 1
    tt = dev(J, t)
    neg = J.ConcreteNDArray.scalar(-1.0)
    names = ["w1", "b1", "w2", "b2", "w3", "b3"]
    params = dict(zip(names, [ws[0], bs[0], ws[1], bs[1], ws[2], bs[2]]))

    def loss(tr):
        c = tr.children
        a = x
        for i in (1, 2):
            a = a.dot(c[f"w{i}"].value).add(c[f"b{i}"].value).relu()
        logits = a.dot(c["w3"].value).add(c["b3"].value)
        return J.Nn.softmax(logits).log().mul(tt).sum(-1).mean().mul(neg)

    v1, g1 = J.JAX.valueAndGradTree(loss)(J.PyTree.dictOf(params))
    old = G.FUSION
    G.FUSION = False
    try:
        v0, g0 = J.JAX.valueAndGradTree(loss)(J.PyTree.dictOf(params))
    finally:
        G.FUSION = old
    np.testing.assert_array_equal(v1.numpy(), v0.numpy())
    for k in names:
        np.testing.assert_array_equal(g1.children[k].value.numpy(), g0.children[k].value.numpy())


@pytest.mark.parametrize("n", [1, 2, 17, 1000, 100000])
def test_random_permutation_bit_exact(J, n):
    from oracle import oracle as orc
    key = J.Random.split(J.PRNGKey.key(42), 3)[1]
    got = J.Random.permutation(key, n)
    assert got.dtype() == J.DType.INT32
    np.testing.assert_array_equal(got.numpy(), orc.permutation(key.state(), n))


def test_he_normal_and_dropout(J):
    from oracle import oracle as orc
    key = J.PRNGKey.key(3)
    h = J.Random.heNormal(key, J.Shape(64, 32), 64).numpy()
    std = np.float32(np.sqrt(2.0 / 64))
    assert_rel(h, (orc.normal(key.state(), (64, 32)).astype(np.float64) * std).astype(np.float32), TOL_ELEMENTWISE)
    x = J.ConcreteNDArray.of(np.arange(1, 2049, dtype=np.float32).reshape(32, 64))
    d = J.Nn.dropout(x, key, 0.25, True).numpy()
    keep = orc.uniform(key.state(), (32, 64)) < np.float32(0.75)
    ref = (x.numpy() * keep.astype(np.float32)).astype(np.float64) / np.float64(np.float32(0.75))
    np.testing.assert_array_equal(d, ref.astype(np.float32))
    np.testing.assert_array_equal(J.Nn.dropout(x, key, 0.25, False).numpy(), x.numpy())


# ---- RandomTest.java:104-183: permutation, heNormal and dropout, as the reference tests them ----
def test_reference_permutation_is_a_valid_permutation(J):
    perm = J.Random.permutation(J.PRNGKey.key(4), 200)
    assert perm.dtype() == J.DType.INT32
    assert sorted(perm.numpy().tolist()) == list(range(200))


def test_reference_he_normal_scales_by_expected_std(J):
    fan_in, n = 256, 20000
    expected = float(np.float32(np.sqrt(2.0 / fan_in)))
    w = J.Random.heNormal(J.PRNGKey.key(6), J.Shape(n), fan_in).numpy().astype(np.float64)
    assert abs(np.sqrt((w * w).sum() / n) - expected) <= expected * 0.15


def test_reference_dropout_modes(J):
    x = J.ConcreteNDArray.of(np.array([1, 2, 3, 4], np.float32))
    np.testing.assert_array_equal(J.Nn.dropout(x, J.PRNGKey.key(1), 0.5, False).numpy(), [1, 2, 3, 4])
    ones = J.ConcreteNDArray.of(np.ones(20000, np.float32))
    out = J.Nn.dropout(ones, J.PRNGKey.key(8), 0.4, True).numpy()
    kept = out[out != 0]
    np.testing.assert_allclose(kept, np.float32(1.0) / np.float32(0.6), atol=1e-4)
    assert abs((out == 0).mean() - 0.4) <= 0.02


def test_reference_dropout_gradient(J):
    """Zero at dropped positions, 1 / (1 - rate) at kept ones, through JAX.grad."""
    x = J.ConcreteNDArray.of(np.ones(8, np.float32))
    key, rate = J.PRNGKey.key(123), 0.5
    m = J.Random.bernoulli(key, 1.0 - rate, x.shape()).numpy().astype(bool)
    g = J.JAX.grad(lambda v: J.Nn.dropout(v, key, rate, True).sum())(x).numpy()
    np.testing.assert_array_equal(g[~m], 0.0)
    np.testing.assert_allclose(g[m], 1.0 / (1.0 - rate), atol=1e-4)


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("M,K,N", [(512, 1024, 1024), (4096, 1024, 4096), (300, 1100, 257)])
def test_dot_tail_split_shapes(J, ta, tb, M, K, N):
    """Products whose last wave of output tiles is cut along K (16 tiles into
    4 parts, 512 tiles' last 68 into 2, a ragged 6-tile product into 4):
    within the dot tolerance of the float64 product, and the bias / relu /
    relu' epilogues, applied once the parts are added, equal the unfused
    sequence bit for bit."""
    from jax4j_b200 import grad as G
    from jax4j_b200.core import _dot_raw
    r = rng(M + K + N + 5 * ta + 7 * tb)
    A = r.uniform(-1, 1, (M, K)).astype(np.float32)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    a = dev(J, A.T.copy() if ta else A)
    b = dev(J, B.T.copy() if tb else B)
    bias = dev(J, r.uniform(-1, 1, N).astype(np.float32))
    mask = dev(J, r.integers(-1, 2, (M, N)).astype(np.float32))
    plain = _dot_raw(a, b, bool(ta), bool(tb), a.device())
    assert_rel(plain.numpy(), (A.astype(np.float64) @ B.astype(np.float64)).astype(np.float32), TOL_REDUCTION)
    again = _dot_raw(a, b, bool(ta), bool(tb), a.device())
    np.testing.assert_array_equal(again.numpy(), plain.numpy())  # deterministic
    z, h = _dot_raw(a, b, bool(ta), bool(tb), a.device(), bias=bias, act=True)
    np.testing.assert_array_equal(z.numpy(), plain.add(bias).numpy())
    np.testing.assert_array_equal(h.numpy(), plain.add(bias).relu().numpy())
    _, h_only = _dot_raw(a, b, bool(ta), bool(tb), a.device(), bias=bias, act=True, store_c=False)
    np.testing.assert_array_equal(h_only.numpy(), h.numpy())
    masked = _dot_raw(a, b, bool(ta), bool(tb), a.device(), mask=mask)
    np.testing.assert_array_equal(masked.numpy(), G.relu_grad(plain, mask).numpy())


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (64, 64), (130, 257), (8192, 1000), (1000, 4096)])
def test_split_f32_both_equals_the_two_passes(J, rows, cols):
    """j4c_split_f32_both writes exactly what j4c_split_f32 and
    j4c_split_f32_transposed write (data, padding, header, line words), and
    j4c_split_f32_ex with row and column lines exactly what j4c_split_f32
    and j4c_split_f32_cols write."""
    r = rng(rows * 5 + cols)
    a = dev(J, r.standard_normal((rows, cols)).astype(np.float32))
    d = a.tensor().device
    out = _split_alloc(J, d, rows, cols, 7.0) + _split_alloc(J, d, cols, rows, 7.0)
    ref = _split_alloc(J, d, rows, cols, 9.0) + _split_alloc(J, d, cols, rows, 9.0)
    _lib.call("j4c_split_f32_both", a.data_ptr(), rows, cols, *[t.data_ptr() for t in out], a._stream())
    _lib.call("j4c_split_f32", a.data_ptr(), rows, cols, ref[0].data_ptr(), ref[1].data_ptr(), a._stream())
    _lib.call("j4c_split_f32_transposed", a.data_ptr(), rows, cols, ref[2].data_ptr(), ref[3].data_ptr(),
              a._stream())
    (hb, lb), (hbt, lbt) = _split_written_bytes(rows, cols, rows), _split_written_bytes(cols, rows, cols)
    for o, e, nb in zip(out, ref, (hb, lb, hbt, lbt)):
        assert torch_equal_bytes(o, e, nb)
    rc = _split_alloc(J, d, rows, cols, 7.0) + _split_alloc(J, d, rows, cols, 7.0)
    _lib.call("j4c_split_f32_ex", a.data_ptr(), rows, cols, *[t.data_ptr() for t in rc], None, None, None,
              a._stream())
    cref = _split_alloc(J, d, rows, cols, 9.0)
    _lib.call("j4c_split_f32_cols", a.data_ptr(), rows, cols, cref[0].data_ptr(), cref[1].data_ptr(), a._stream())
    hbc, lbc = _split_written_bytes(rows, cols, cols)
    for o, e, nb in zip(rc, ref[:2] + cref, (hb, lb, hbc, lbc)):
        assert torch_equal_bytes(o, e, nb)


def torch_equal_bytes(a, b, nbytes):
    import torch
    return torch.equal(a.view(torch.uint8)[:nbytes], b.view(torch.uint8)[:nbytes])


@pytest.mark.parametrize("ta,tb,act,masked", [(0, 0, True, False), (1, 0, True, False), (0, 1, False, True),
                                              (0, 0, False, True), (1, 1, True, False)])
def test_epilogue_line_maxima_and_split_from_them(J, ta, tb, act, masked):
    """An epilogue GEMM leaves the line maxima (rows, then columns) of the
    output a later split reads (the relu output, or the masked C); the splits
    that take them are byte-identical to ones that scan the output
    themselves, for every kind and in one pass."""
    from jax4j_b200.core import _dot_raw
    r = rng(ta * 8 + tb * 4 + act * 2 + masked)
    M, K, N = 333, 257, 1030  # ragged edges, several tiles, the transposed store for (0, 0)
    A = (r.standard_normal((M, K)) * 3).astype(np.float32)
    A[5] *= np.float32(2.0 ** -40)  # a row far below the others
    B = r.standard_normal((K, N)).astype(np.float32)
    a = dev(J, A.T.copy() if ta else A)
    b = dev(J, B.T.copy() if tb else B)
    bias = dev(J, r.standard_normal(N).astype(np.float32) * 1e-12) if act else None
    mask = dev(J, r.standard_normal((M, N)).astype(np.float32)) if masked else None
    res = _dot_raw(a, b, bool(ta), bool(tb), a.device(), bias=bias, mask=mask, act=act)
    out = res[1] if act else res
    assert out._lines is not None
    got = out._lines.cpu().numpy().view(np.uint32)
    o = out.numpy()
    assert got.size == M + N + 1
    np.testing.assert_array_equal(got[:M], _line_max_bits(o, "rows"))
    np.testing.assert_array_equal(got[M:M + N], _line_max_bits(o, "cols"))
    assert got[M + N] == 0  # no NaN or infinity written
    d = out.tensor().device
    for pair in (("r", "t"), ("r", "c"), ("c",)):
        given, scan = [], []
        for k in ("r", "c", "t"):
            if k in pair:
                rd, cd = (N, M) if k == "t" else (M, N)
                given += _split_alloc(J, d, rd, cd, 7.0)
                scan += _split_alloc(J, d, rd, cd, 9.0)
            else:
                given += [None, None]
                scan += [None, None]
        ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        _lib.call("j4c_split_f32_ex", out.data_ptr(), M, N, *[ptr(t) for t in given], out._lines.data_ptr(),
                  out._stream())
        _lib.call("j4c_split_f32_ex", out.data_ptr(), M, N, *[ptr(t) for t in scan], None, out._stream())
        for i, k in enumerate(("r", "c", "t")):
            if k in pair:
                rd, cd, nl = (N, M, N) if k == "t" else (M, N, M if k == "r" else N)
                hb, lb = _split_written_bytes(rd, cd, nl)
                assert torch_equal_bytes(given[2 * i], scan[2 * i], hb), (pair, k)
                assert torch_equal_bytes(given[2 * i + 1], scan[2 * i + 1], lb), (pair, k)


def _rel_err_vs_fp64(got, A, B):
    """Per-element error of a product against an FP64 one, relative to
    sum_k |a_ik b_kj| (the scale of a dot's own rounding), and numpy's FP32
    product's error measured the same way."""
    exact = A.astype(np.float64) @ B.astype(np.float64)
    scale = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64)
    scale = np.where(scale == 0, 1.0, scale)
    fp32 = np.abs((A @ B).astype(np.float64) - exact) / scale
    return np.abs(got.astype(np.float64) - exact) / scale, fp32


@pytest.mark.parametrize("K", [256, 4096])
def test_dot_accuracy_against_fp64(J, K):
    """The split GEMM's error per element, relative to sum_k |a_ik b_kj|,
    against an FP64 product: within a few times numpy's FP32 product on
    N(0, 1) rows and on rows 2^-20 and 2^-30 below the tensor's max (each
    line of a 3xFP16 operand carries its own scale), in every operand layout."""
    from jax4j_b200.core import _dot_raw
    r = rng(K)
    M, N = 256, 384
    A = r.standard_normal((M, K)).astype(np.float32)
    A[::7] *= np.float32(2.0 ** -20)   # rows far below the tensor's max
    A[3::11] *= np.float32(2.0 ** -30)
    B = r.standard_normal((K, N)).astype(np.float32)
    B[:, ::5] *= np.float32(2.0 ** -25)  # columns far below the max
    for ta, tb in ((0, 0), (1, 0), (0, 1), (1, 1)):
        a, b = dev(J, A.T.copy() if ta else A), dev(J, B.T.copy() if tb else B)
        got = _dot_raw(a, b, bool(ta), bool(tb), a.device()).numpy()
        err, fp32 = _rel_err_vs_fp64(got, A, B)
        assert err.max() <= max(4 * fp32.max(), 1e-6), ((ta, tb), err.max(), fp32.max())


@pytest.mark.parametrize("a_max,b_max", [(1e-30, 1e30), (1e-20, 1e20), (1e30, 1e-30), (3e38, 3e-39),
                                         (1e-38, 1e-3), (2e-40, 1e35)])
def test_dot_extreme_magnitudes(J, a_max, b_max):
    """Operands whose whole range sits at either end of FP32's exponent range
    (down to FP32 subnormals, up to 3e38), paired so that the products stay
    finite and normal: per element within a few times numpy's FP32 error
    against FP64 (every line is scaled into the split format's range, which
    also keeps FP32 subnormals exact)."""
    from jax4j_b200.core import _dot_raw
    r = rng(int(abs(np.log10(a_max))) + 3)
    M, K, N = 192, 512, 160
    A = (r.uniform(-1, 1, (M, K)) * a_max).astype(np.float32)
    B = (r.uniform(-1, 1, (K, N)) * b_max).astype(np.float32)
    a, b = dev(J, A), dev(J, B)
    got = _dot_raw(a, b, False, False, a.device()).numpy()
    assert np.all(np.isfinite(got))
    err, fp32 = _rel_err_vs_fp64(got, A, B)
    assert err.max() <= max(4 * fp32.max(), 2e-6), (err.max(), fp32.max())


def _with_specials(r, shape, kinds):
    x = r.uniform(-1, 1, shape).astype(np.float32)
    x[r.uniform(size=shape) < 0.05] = 0.0  # exact zeros: 0 * inf = NaN
    flat = x.reshape(-1)
    for k in kinds:
        idx = r.choice(flat.size, size=3, replace=False)
        flat[idx] = {"inf": np.inf, "-inf": -np.inf, "nan": np.nan}[k]
    return x


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("where", ["a", "b", "both"])
@pytest.mark.parametrize("M,K,N", [(150, 200, 170), (300, 96, 280)])  # single CTAs; CTA pairs (>= 256 rows)
def test_dot_special_values_equal_the_reference(J, ta, tb, where, M, K, N):
    """An operand holding +-Inf or NaN: the product is the reference's
    sequential FP32 sum (core/ConcreteNDArray.java:452-459) bit for bit --
    Inf rows and columns, 0 * Inf = NaN, +Inf + -Inf = NaN, NaN spreading --
    in every layout, as the oracle computes it."""
    from jax4j_b200.core import _dot_raw
    r = rng(ta * 4 + tb * 2 + len(where) + M)
    A = _with_specials(r, (M, K), ["inf", "-inf", "nan"] if where in ("a", "both") else [])
    B = _with_specials(r, (K, N), ["-inf", "inf"] if where in ("b", "both") else [])
    a, b = dev(J, A.T.copy() if ta else A), dev(J, B.T.copy() if tb else B)
    got = _dot_raw(a, b, bool(ta), bool(tb), a.device()).numpy()
    ref = orc.dot(A, B)
    assert np.any(~np.isfinite(ref))
    assert np.array_equal(got, ref, equal_nan=True), int(np.sum(~((got == ref) | (np.isnan(got) & np.isnan(ref)))))


def test_dot_special_values_through_the_epilogue_and_vmap(J):
    """The exact path under a bias + relu epilogue (the relu output stored),
    with its line maxima for the next split, and in the strided-batched
    GEMM of vmap."""
    from jax4j_b200.core import _dot_raw
    r = rng(1234)
    M, K, N = 130, 96, 140
    A = _with_specials(r, (M, K), ["inf", "nan"])
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = r.uniform(-1, 1, N).astype(np.float32)
    a, b, bi = dev(J, A), dev(J, B), dev(J, bias)
    _, h = _dot_raw(a, b, False, False, a.device(), bias=bi, act=True, store_c=False)
    z = (orc.dot(A, B) + bias).astype(np.float32)
    want = np.where(np.isnan(z), z, np.maximum(z, np.float32(0)))
    assert np.array_equal(h.numpy(), want, equal_nan=True)
    lines = h._lines.cpu().numpy().view(np.uint32)
    np.testing.assert_array_equal(lines[:M], _line_max_bits(want, "rows"))
    np.testing.assert_array_equal(lines[M:M + N], _line_max_bits(want, "cols"))
    assert lines[M + N] != 0  # the relu output holds NaN and infinity
    # ... and a product taking it as an operand runs the exact path too
    from jax4j_b200.core import _dot_raw as dr
    C2 = r.uniform(-1, 1, (N, 20)).astype(np.float32)
    got2 = dr(h, dev(J, C2), False, False, a.device()).numpy()
    assert np.array_equal(got2, orc.dot(h.numpy(), C2), equal_nan=True)
    # vmap's strided-batched dot: [3, M, K] . [3, K, N] with a special in one entry
    A3 = np.stack([r.uniform(-1, 1, (M, K)).astype(np.float32) for _ in range(3)])
    B3 = np.stack([r.uniform(-1, 1, (K, N)).astype(np.float32) for _ in range(3)])
    A3[1, 7, 9] = np.inf
    B3[2, 4, 11] = np.nan
    got = J.JAX.vmap(lambda x, w: x.dot(w), in_axes=[0, 0])(dev(J, A3), dev(J, B3)).numpy()
    for i in range(3):
        assert np.array_equal(got[i], orc.dot(A3[i], B3[i]), equal_nan=True), i


def _pack_bits(m):
    """x > 0 of a [rows, cols] array as rows of ceil(cols / 32) uint32 words."""
    rows, cols = m.shape
    w = (cols + 31) // 32
    padded = np.zeros((rows, w * 32), dtype=bool)
    padded[:, :cols] = m
    return np.packbits(padded.reshape(rows, w, 4, 8)[:, :, ::-1, ::-1].reshape(rows, w * 32),
                       axis=1).view(">u4").astype(np.uint32).reshape(rows, w)


@pytest.mark.parametrize("M,K,N,special", [(333, 257, 1030, False), (256, 512, 4096, False), (130, 96, 70, True)])
def test_relu_bits_equal_the_float_mask(J, M, K, N, special):
    """A forward epilogue (bias + relu) leaves h > 0 as bits; an input
    gradient masked by those bits equals the one masked by the float relu
    output bit for bit -- in the tensor-core path and in the exact path of
    operands holding NaN/Inf."""
    from jax4j_b200 import core
    from jax4j_b200.core import _dot_raw
    r = rng(M + N)
    A = r.standard_normal((M, K)).astype(np.float32)
    if special:
        A[3, 5], A[7, 1] = np.inf, np.nan
    W = (r.standard_normal((K, N)) * 0.05).astype(np.float32)
    bias = r.standard_normal(N).astype(np.float32) * 0.1
    a, w, b = dev(J, A), dev(J, W), dev(J, bias)
    _, h = _dot_raw(a, w, False, False, a.device(), bias=b, act=True, store_c=False)
    assert h._relu_bits is not None
    hh = h.numpy()
    np.testing.assert_array_equal(h._relu_bits.cpu().numpy().view(np.uint32).reshape(M, -1), _pack_bits(hh > 0))
    G = r.standard_normal((M, 64)).astype(np.float32)
    W2 = r.standard_normal((N, 64)).astype(np.float32)  # dX = G . W2^T, masked by h > 0
    g, w2 = dev(J, G), dev(J, W2)
    with_bits = _dot_raw(g, w2, False, True, a.device(), mask=h).numpy()
    bits, h._relu_bits = h._relu_bits, None
    with_floats = _dot_raw(g, w2, False, True, a.device(), mask=h).numpy()
    h._relu_bits = bits
    assert np.array_equal(with_bits, with_floats, equal_nan=True)


def test_relu_bits_rejected_where_c_is_stored_transposed(J):
    """The K-major A . MN-major B form stores C transposed, so it cannot
    take relu bits: j4c_dot_split_ep_bits rejects them there."""
    import torch
    from jax4j_b200.core import _split_of
    M, K, N = 64, 32, 96
    r = rng(3)
    a, b = dev(J, r.standard_normal((M, K)).astype(np.float32)), dev(J, r.standard_normal((K, N)).astype(np.float32))
    (ah, al), (bh, bl) = _split_of(a, "r"), _split_of(b, "c")
    act = torch.empty(M * N, dtype=torch.float32, device=a.tensor().device)
    bits = torch.empty(M * 3, dtype=torch.int32, device=a.tensor().device)
    rc = _lib.lib().j4c_dot_split_ep_bits(ah.data_ptr(), al.data_ptr(), bh.data_ptr(), bl.data_ptr(), None, M, K, N,
                                          0, 0, None, None, None, act.data_ptr(), bits.data_ptr(), None,
                                          a._stream())
    assert rc == _lib.E_INVALID
    assert "transposed split" in _lib.lib().j4c_last_error().decode()
