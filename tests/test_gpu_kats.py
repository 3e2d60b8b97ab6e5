"""The reference's known-answer tests (tests/golden/kats.json), run through
the public API on the GPU -- the same cases that pin the CPU oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def J():
    import jax4j_b200 as j
    return j


def _arr(J, values, shape=None, dtype="float32"):
    dt = {"float32": J.DType.FLOAT32, "int32": J.DType.INT32, "bool": J.DType.BOOL}[dtype]
    v = np.asarray(values)
    shape = shape if shape is not None else [len(values)]
    return J.ConcreteNDArray.of(v.reshape(shape), J.Shape(shape), dt)


def _scalar(J, v):
    return J.ConcreteNDArray.of(np.float32([v]))


def test_gpu_kats(J, kats):
    ran = 0
    for k in kats:
        kind = k["kind"]
        tol = k.get("tol") or 0
        if kind == "compare":
            a, b = _arr(J, k["a"], dtype=k["dtype"]), _arr(J, k["b"], dtype=k["dtype"])
            r = getattr(a, k["op"])(b)
            assert r.dtype() == J.DType.BOOL
            assert r.toBoolArray().tolist() == k["expected"], k["id"]
        elif kind == "binary":
            a, b = _arr(J, k["a"], k["a_shape"]), _arr(J, k["b"], k["b_shape"])
            r = getattr(a, k["op"])(b)
            assert list(r.shape().dimensions()) == k["shape"], k["id"]
            np.testing.assert_allclose(r.toFloatArray(), k["expected"], atol=tol, err_msg=k["id"])
        elif kind == "binary_error":
            a, b = _arr(J, k["a"], k["a_shape"]), _arr(J, k["b"], k["b_shape"])
            with pytest.raises(J.IllegalArgumentException):
                getattr(a, k["op"])(b)
        elif kind == "clip":
            r = _arr(J, k["x"]).clip(_scalar(J, k["lo"]), _scalar(J, k["hi"]))
            np.testing.assert_allclose(r.toFloatArray(), k["expected"], atol=tol, err_msg=k["id"])
        elif kind == "argreduce":
            x = _arr(J, k["x"], k["shape"])
            r = getattr(x, k["op"])(k["axis"])
            assert r.dtype() == J.DType.INT32 and r.toIntArray().tolist() == k["expected"], k["id"]
        elif kind == "reduce_axis":
            x = _arr(J, k["x"], k["shape"])
            r = getattr(x, k["op"])(k["axis"], k["keep_dims"])
            assert list(r.shape().dimensions()) == k["out_shape"], k["id"]
            np.testing.assert_allclose(r.toFloatArray(), k["expected"], atol=tol, err_msg=k["id"])
        elif kind == "cast":
            x = _arr(J, k["x"], dtype=k["src"])
            dst = {"float32": J.DType.FLOAT32, "int32": J.DType.INT32, "bool": J.DType.BOOL}[k["dst"]]
            r = x.astype(dst)
            assert r.numpy().tolist() == np.asarray(k["expected"]).astype(dst.numpy).tolist(), k["id"]
        elif kind == "promote_add":
            r = _arr(J, k["a"], dtype=k["a_dtype"]).add(_arr(J, k["b"], dtype=k["b_dtype"]))
            assert str(r.dtype()) == k["expected_dtype"]
            np.testing.assert_allclose(r.toFloatArray(), k["expected"], atol=1e-6)
        elif kind == "int_add_error":
            with pytest.raises(J.IllegalArgumentException, match=k["message"]):
                _arr(J, k["a"], dtype="int32").add(_arr(J, k["b"], dtype="int32"))
        elif kind == "promote_compare":
            r = getattr(_arr(J, k["a"], dtype=k["a_dtype"]), k["op"])(_arr(J, k["b"], dtype=k["b_dtype"]))
            assert r.dtype() == J.DType.BOOL and r.toBoolArray().tolist() == k["expected"]
        elif kind == "softmax":
            p = J.Nn.softmax(_arr(J, k["x"], k["shape"])).toFloatArray()
            np.testing.assert_allclose(p.reshape(k["shape"]).sum(-1), k["row_sums"], atol=tol)
            for i, v in k["check"].items():
                assert abs(p[int(i)] - v) <= tol, k["id"]
        elif kind == "where_square_neg":
            fn = lambda x: J.Numpy.where(x.gt(_scalar(J, 0)), x.mul(x), x.mul(_scalar(J, -1)))
            x = _scalar(J, k["x"])
            assert abs(fn(x).toFloatArray()[0] - k["expected"]) <= 1e-5
            assert abs(J.JAX.grad(fn)(x).toFloatArray()[0] - k["grad"]) <= tol
        elif kind in ("psum", "psum_mean", "all_gather_sum", "pmap_square", "grad_pmap_square",
                      "grad_pmap_psum"):
            _pmap_kat(J, k)
        elif kind == "psum_identity":
            x = _arr(J, k["x"])
            np.testing.assert_allclose(J.Lax.psum(x).toFloatArray(), k["expected"], atol=tol)
        elif kind == "all_gather_identity":
            r = J.Lax.allGather(_arr(J, k["x"]), 1)
            assert list(r.shape().dimensions()) == k["expected_shape"]
            np.testing.assert_allclose(r.toFloatArray(), k["expected"], atol=tol)
        elif kind == "grad_scalar":
            fns = {"div10": lambda x: _scalar(J, 10).div(x), "exp": lambda x: x.exp(),
                   "log": lambda x: x.log(), "sin": lambda x: x.sin(), "cos": lambda x: x.cos(),
                   "tanh": lambda x: x.tanh(), "relu": lambda x: x.relu(), "sigmoid": lambda x: x.sigmoid()}
            g = J.JAX.grad(fns[k["fn"]])(_scalar(J, k["x"])).toFloatArray()[0]
            assert abs(g - k["expected"]) <= tol, (k["id"], g)
        elif kind == "grad_dot":
            b = _arr(J, k["b"], k["b_shape"])
            g = J.JAX.grad(lambda a: a.dot(b).sum())(_arr(J, k["a"], k["a_shape"])).toFloatArray()
            np.testing.assert_allclose(g, k["expected"], atol=tol)
        elif kind == "grad_max2":
            g = J.JAX.grad(lambda a: a.max(_scalar(J, 2)).sum())(_scalar(J, k["x"])).toFloatArray()[0]
            assert abs(g - k["expected"]) <= tol, k["id"]
        elif kind == "grad_axis":
            fn = (lambda x: x.sum(k["axis"], k["keep_dims"]).sum()) if k["op"] == "sum" else \
                 (lambda x: x.mean(k["axis"], k["keep_dims"]).sum())
            g = J.JAX.grad(fn)(_arr(J, k["x"], k["shape"])).toFloatArray()
            np.testing.assert_allclose(g, k["expected"], atol=tol, err_msg=k["id"])
        elif kind == "grad_softmax_sum":
            g = J.JAX.grad(lambda x: J.Nn.softmax(x).sum())(_arr(J, k["x"], k["shape"])).toFloatArray()
            np.testing.assert_allclose(g, k["expected"], atol=tol)
        elif kind == "grad_compare":
            g = J.JAX.grad(lambda x: x.gt(_scalar(J, 0)))(_scalar(J, k["x"])).toFloatArray()
            np.testing.assert_allclose(g, [k["expected"]], atol=tol)
        elif kind == "grad_argmax":
            g = J.JAX.grad(lambda x: x.argmax(0))(_arr(J, k["x"])).toFloatArray()
            np.testing.assert_allclose(g, k["expected"], atol=tol)
        elif kind == "grad_identity_cast":
            g = J.JAX.grad(lambda x: x.astype(J.DType.FLOAT32).mul(x).sum())(_scalar(J, k["x"]))
            assert abs(g.toFloatArray()[0] - k["expected"]) <= tol
        elif kind == "grad_nonfloat_cast":
            g = J.JAX.grad(lambda x: x.astype(J.DType.BOOL).astype(J.DType.FLOAT32).sum())(_arr(J, k["x"]))
            np.testing.assert_allclose(g.toFloatArray(), k["expected"], atol=tol)
        else:
            raise AssertionError(f"unhandled KAT kind {kind}")
        ran += 1
    assert ran == len(kats)


def _pmap_kat(J, k):
    devices = [J.Device(None), J.Device(None)]
    tol = k["tol"]
    kind = k["kind"]
    if kind == "psum":
        x = J.ConcreteNDArray.of(np.float32(k["shards"]))
        r = J.JAX.pmap(lambda s: J.Lax.psum(s), devices)(x)
        np.testing.assert_allclose(r.toFloatArray(), np.ravel(k["expected"]), atol=tol)
    elif kind == "psum_mean":
        x = J.ConcreteNDArray.of(np.float32(k["shards"]))
        total = _scalar(J, k["total"])
        r = J.JAX.pmap(lambda s: J.Lax.psum(s.sum()).div(total), devices)(x)
        np.testing.assert_allclose(r.toFloatArray(), k["expected"], atol=tol)
    elif kind == "all_gather_sum":
        x = J.ConcreteNDArray.of(np.float32(k["shards"]))
        r = J.JAX.pmap(lambda s: J.Lax.allGather(s, 2).sum(), devices)(x)
        np.testing.assert_allclose(r.toFloatArray(), k["expected"], atol=tol)
    elif kind == "pmap_square":
        x = _arr(J, k["x"], k["shape"])
        r = J.JAX.pmap(lambda s: s.mul(s), devices)(x)
        assert list(r.shape().dimensions()) == k["shape"]
        np.testing.assert_allclose(r.toFloatArray(), k["expected"], atol=tol)
    elif kind == "grad_pmap_square":
        fn = lambda x: J.JAX.pmap(lambda s: s.mul(s), devices)(x).sum()
        x = _arr(J, k["x"], k["shape"])
        assert abs(fn(x).toFloatArray()[0] - k["forward"]) <= tol
        np.testing.assert_allclose(J.JAX.grad(fn)(x).toFloatArray(), k["expected"], atol=tol)
    elif kind == "grad_pmap_psum":
        two = _scalar(J, 2)
        fn = lambda x: J.JAX.pmap(lambda s: J.Lax.psum(s.mul(s).sum()).div(two), devices)(x).sum()
        x = _arr(J, k["x"], k["shape"])
        assert abs(fn(x).toFloatArray()[0] - k["forward"]) <= tol
        np.testing.assert_allclose(J.JAX.grad(fn)(x).toFloatArray(), k["expected"], atol=tol)
