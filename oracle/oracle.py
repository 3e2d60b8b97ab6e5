"""numpy/ctypes front end of the CPU oracle (test infrastructure only).

Loads oracle/_build/libj4c_oracle.so (built by oracle/build.py) and exposes
each restated reference function on numpy arrays.  The product never imports
this module: only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg do, and only as the checker or the timed CPU baseline.

Parity of the restatement is pinned against the known-answer tests of the
reference's JUnit suite (tests/golden/kats.json); the reference itself needs
a JDK and the TornadoVM jars and cannot run here.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

# Primitive ordinals (ir/Primitive.java:6-42) and DType ordinals (core/DType.java:7-11).
ADD, SUB, MUL, DIV, DOT = 0, 1, 2, 3, 4
EXP, LOG, SIN, COS = 5, 6, 7, 8
SUM, MEAN, SUM_AXIS, MEAN_AXIS = 9, 10, 11, 12
TANH, RELU, SIGMOID = 13, 14, 15
GT, GE, LT, LE, EQ, NE = 19, 20, 21, 22, 23, 24
MAX, MIN, ARGMAX, ARGMIN = 25, 26, 27, 28
F32, F64, I32, I64, BOOL = 0, 1, 2, 3, 4

_NP = {F32: np.float32, F64: np.float64, I32: np.int32, I64: np.int64, BOOL: np.uint8}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        _lib = C.CDLL(path)
        _declare(_lib)
    return _lib


P = C.c_void_p
CI64 = C.c_int64


def _declare(L):
    L.orc_mix64.restype = C.c_uint64
    L.orc_mix64.argtypes = [C.c_uint64]
    L.orc_split.argtypes = [C.c_uint64, C.c_int, P]
    L.orc_uniform.argtypes = [C.c_uint64, CI64, C.c_float, C.c_float, P]
    L.orc_permutation.argtypes = [C.c_uint64, CI64, P]
    L.orc_fft.argtypes = [C.c_int, C.c_int, P, P, P, C.c_int]
    L.orc_rfft.argtypes = [C.c_int, C.c_int, P, P, P, P]
    L.orc_irfft.argtypes = [C.c_int, C.c_int, P, P, P, P]
    L.orc_dct1.argtypes = [C.c_int, CI64, P, P]
    L.orc_lu_factor.argtypes = [P, CI64, C.c_int, P, P, P, P]
    L.orc_lu_solve.argtypes = [P, P, CI64, P, P]
    L.orc_lu_solve_t.argtypes = [P, P, CI64, P, P]
    L.orc_lu_rcond.restype = C.c_double
    L.orc_lu_rcond.argtypes = [P, P, CI64, C.c_double]
    L.orc_eig.argtypes = [C.c_int, CI64, P, P, P]
    L.orc_svd.argtypes = [C.c_int, CI64, CI64, P, P, P, P]
    L.orc_normal.argtypes = [C.c_uint64, CI64, P]
    L.orc_glorot_uniform.argtypes = [C.c_uint64, CI64, C.c_int, C.c_int, P]
    L.orc_broadcast_index.restype = CI64
    L.orc_broadcast_index.argtypes = [P, C.c_int, P, C.c_int, CI64]
    L.orc_binary_f32.argtypes = [C.c_int, P, P, C.c_int, P, P, C.c_int, P, P, C.c_int]
    L.orc_compare.argtypes = [C.c_int, C.c_int, P, P, C.c_int, P, P, C.c_int, P, P, C.c_int]
    L.orc_unary_f32.argtypes = [C.c_int, P, CI64, P]
    L.orc_cast.argtypes = [C.c_int, C.c_int, P, CI64, P]
    L.orc_reduce_all_f32.argtypes = [C.c_int, P, CI64, P]
    L.orc_reduce_axis_f32.argtypes = [C.c_int, P, CI64, CI64, CI64, P]
    L.orc_argreduce_f32.argtypes = [C.c_int, P, CI64, CI64, CI64, P]
    L.orc_dot_f32.argtypes = [P, P, P, CI64, CI64, CI64, CI64, CI64, C.c_int]
    L.orc_broadcast_like_f32.argtypes = [P, P, C.c_int, P, P, C.c_int]
    L.orc_relu_grad_f32.argtypes = [P, P, CI64, P]
    L.orc_axis_broadcast_like_f32.argtypes = [P, P, C.c_int, C.c_int, P]
    L.orc_transpose_f32.argtypes = [P, CI64, CI64, P]
    L.orc_maxmin_grad_f32.argtypes = [C.c_int, P, P, C.c_int, P, P, C.c_int, P, P, C.c_int, P, P]
    L.orc_psum_f32.argtypes = [P, C.c_int, CI64, P]
    L.orc_mlp_loss_grad_f32.argtypes = [C.c_int, P, C.c_int, P, P, P, P, CI64, P, P, P, P, P, C.c_int]
    L.orc_mlp_loss_f32.argtypes = [C.c_int, P, C.c_int, P, P, P, P, CI64, P, C.c_int]
    L.orc_sweep_f32.argtypes = [P, P, CI64, CI64, P, P, P]


def _p(a: np.ndarray):
    return a.ctypes.data_as(P)


def _dims(shape):
    d = np.asarray(list(shape) if len(shape) else [], dtype=np.int64)
    return d, len(shape)


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


def broadcast_shape(a, b):
    """core/Shape.java:37-49."""
    rank = max(len(a), len(b))
    out = []
    for i in range(rank):
        da = 1 if i < rank - len(a) else a[i - (rank - len(a))]
        db = 1 if i < rank - len(b) else b[i - (rank - len(b))]
        if da != db and da != 1 and db != 1:
            raise ValueError(f"Shapes {list(a)} and {list(b)} are not broadcast-compatible")
        out.append(max(da, db))
    return tuple(out)


# ---- Random.java ----
def mix64(z: int) -> int:
    return int(lib().orc_mix64(z & 0xFFFFFFFFFFFFFFFF))


def split(state: int, num: int = 2):
    out = np.zeros(num, dtype=np.uint64)
    lib().orc_split(state & 0xFFFFFFFFFFFFFFFF, num, _p(out))
    return [int(v) for v in out]


def uniform(state: int, shape, lo=0.0, hi=1.0):
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.float32)
    lib().orc_uniform(state & 0xFFFFFFFFFFFFFFFF, n, lo, hi, _p(out))
    return out.reshape(shape)


def permutation(state: int, n: int):
    """Random.permutation (Random.java:130-140)."""
    out = np.empty(max(n, 1), dtype=np.int32)
    lib().orc_permutation(state & 0xFFFFFFFFFFFFFFFF, n, _p(out))
    return out[:n]


def normal(state: int, shape):
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.float32)
    lib().orc_normal(state & 0xFFFFFFFFFFFFFFFF, n, _p(out))
    return out.reshape(shape)


def glorot_uniform(state: int, shape, fan_in: int, fan_out: int):
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    lib().orc_glorot_uniform(state & 0xFFFFFFFFFFFFFFFF, n, fan_in, fan_out, _p(out))
    return out.reshape(shape)


# ---- ConcreteNDArray.java ----
def binary(prim: int, a, b):
    a = _c(a)
    b = _c(b)
    oshape = broadcast_shape(a.shape, b.shape)
    out = np.empty(oshape, dtype=np.float32)
    ad, ar = _dims(a.shape)
    bd, br = _dims(b.shape)
    od, orank = _dims(oshape)
    rc = lib().orc_binary_f32(prim, _p(a), _p(ad), ar, _p(b), _p(bd), br, _p(out), _p(od), orank)
    if rc != 0:
        raise ValueError(f"not a binary primitive: {prim}")
    return out


def compare(prim: int, dtype: int, a, b):
    a = _c(a, _NP[dtype])
    b = _c(b, _NP[dtype])
    oshape = broadcast_shape(a.shape, b.shape)
    out = np.empty(oshape, dtype=np.uint8)
    ad, ar = _dims(a.shape)
    bd, br = _dims(b.shape)
    od, orank = _dims(oshape)
    rc = lib().orc_compare(prim, dtype, _p(a), _p(ad), ar, _p(b), _p(bd), br, _p(out), _p(od), orank)
    if rc != 0:
        raise ValueError("unsupported compare")
    return out


def unary(prim: int, a):
    a = _c(a)
    out = np.empty_like(a)
    if lib().orc_unary_f32(prim, _p(a), a.size, _p(out)) != 0:
        raise ValueError(f"not a unary primitive: {prim}")
    return out


def cast(src: int, dst: int, a):
    a = _c(a, _NP[src])
    out = np.empty(a.shape, dtype=_NP[dst])
    if lib().orc_cast(src, dst, _p(a), a.size, _p(out)) != 0:
        raise ValueError("unsupported cast")
    return out


def reduce_all(prim: int, a):
    a = _c(a)
    out = np.empty(1, dtype=np.float32)
    lib().orc_reduce_all_f32(prim, _p(a), a.size, _p(out))
    return out


def _axis_split(shape, axis):
    axis = axis + len(shape) if axis < 0 else axis
    outer = int(np.prod(shape[:axis])) if axis > 0 else 1
    inner = int(np.prod(shape[axis + 1:])) if axis + 1 < len(shape) else 1
    return axis, outer, shape[axis], inner


def reduce_axis(prim: int, a, axis: int, keep_dims: bool):
    a = _c(a)
    ax, outer, size, inner = _axis_split(a.shape, axis)
    out = np.empty(outer * inner, dtype=np.float32)
    lib().orc_reduce_axis_f32(prim, _p(a), outer, size, inner, _p(out))
    shape = list(a.shape)
    if keep_dims:
        shape[ax] = 1
    else:
        shape.pop(ax)
    return out.reshape(shape)


def argreduce(prim: int, a, axis: int):
    a = _c(a)
    ax, outer, size, inner = _axis_split(a.shape, axis)
    out = np.empty(outer * inner, dtype=np.int32)
    lib().orc_argreduce_f32(prim, _p(a), outer, size, inner, _p(out))
    shape = list(a.shape)
    shape.pop(ax)
    return out.reshape(shape)


def dot(a, b, rows=None, threads: int = 1):
    """C = A.B with the reference's sequential float k-sum.  rows=(r0, r1)
    computes only that row range (returned as a [r1-r0, N] array)."""
    a = _c(a)
    b = _c(b)
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    r0, r1 = (0, M) if rows is None else rows
    out = np.empty((M, N), dtype=np.float32) if rows is None else np.empty((r1 - r0, N), np.float32)
    base = out.ctypes.data - r0 * N * 4
    lib().orc_dot_f32(_p(a), _p(b), C.c_void_p(base), M, K, N, r0, r1, threads)
    return out


# ---- Grad.java helpers ----
def broadcast_like(g, target_shape):
    g = _c(g)
    out = np.empty(target_shape, dtype=np.float32)
    gd, gr = _dims(g.shape)
    td, tr = _dims(tuple(target_shape))
    lib().orc_broadcast_like_f32(_p(g), _p(gd), gr, _p(out), _p(td), tr)
    return out


def relu_grad(g, x):
    g = _c(g)
    x = _c(x)
    out = np.empty_like(x)
    lib().orc_relu_grad_f32(_p(g), _p(x), x.size, _p(out))
    return out


def axis_broadcast_like(g, shape, axis: int):
    g = _c(g)
    out = np.empty(shape, dtype=np.float32)
    d, r = _dims(tuple(shape))
    lib().orc_axis_broadcast_like_f32(_p(g), _p(d), r, axis, _p(out))
    return out


def transpose(a):
    a = _c(a)
    rows, cols = a.shape
    out = np.empty((cols, rows), dtype=np.float32)
    lib().orc_transpose_f32(_p(a), rows, cols, _p(out))
    return out


def maxmin_grad(is_max: bool, g, a, b):
    g = _c(g)
    a = _c(a)
    b = _c(b)
    od, orank = _dims(g.shape)
    ad, ar = _dims(a.shape)
    bd, br = _dims(b.shape)
    ga = np.empty(g.shape, np.float32)
    gb = np.empty(g.shape, np.float32)
    lib().orc_maxmin_grad_f32(int(is_max), _p(g), _p(od), orank, _p(a), _p(ad), ar, _p(b),
                              _p(bd), br, _p(ga), _p(gb))
    return broadcast_like(ga, a.shape), broadcast_like(gb, b.shape)


def psum(slots):
    slots = [_c(s) for s in slots]
    n = slots[0].size
    ptrs = (C.c_void_p * len(slots))(*[s.ctypes.data for s in slots])
    out = np.empty_like(slots[0])
    lib().orc_psum_f32(ptrs, len(slots), n, _p(out))
    return out


# ---- MLP cross-entropy (examples/MNISTFromScratch.java:103-125) ----
def mlp_hidden_preacts(ws, bs, x, act: str = "relu", threads: int = 1):
    """Pre-activations z_l = a_l.W_l + b_l of the hidden layers, computed with
    the same restated ops (dot, broadcast add, activation) as the MLP oracle."""
    a = _c(x)
    zs = []
    for l in range(len(ws) - 1):
        z = binary(ADD, dot(a, ws[l], threads=threads), bs[l])
        zs.append(z)
        a = unary(TANH if act == "tanh" else RELU, z)
    return zs


def mlp_loss_grad(ws, bs, x, onehot, act: str = "tanh", want_gx: bool = False, threads: int = 1,
                  relu_masks=None):
    L = len(ws)
    ws = [_c(w) for w in ws]
    bs = [_c(b) for b in bs]
    x = _c(x)
    onehot = _c(onehot)
    dims = np.array([ws[0].shape[0]] + [w.shape[1] for w in ws], dtype=np.int64)
    wp = (C.c_void_p * L)(*[w.ctypes.data for w in ws])
    bp = (C.c_void_p * L)(*[b.ctypes.data for b in bs])
    gws = [np.empty_like(w) for w in ws]
    gbs = [np.empty_like(b) for b in bs]
    gwp = (C.c_void_p * L)(*[g.ctypes.data for g in gws])
    gbp = (C.c_void_p * L)(*[g.ctypes.data for g in gbs])
    gx = np.empty_like(x) if want_gx else None
    loss = np.zeros(1, np.float32)
    mp = None
    if relu_masks is not None:
        masks = [np.ascontiguousarray(m, dtype=np.uint8) for m in relu_masks]
        mp = (C.c_void_p * len(masks))(*[m.ctypes.data for m in masks])
    lib().orc_mlp_loss_grad_f32(L, _p(dims), 0 if act == "tanh" else 1, wp, bp, _p(x), _p(onehot),
                                x.shape[0], _p(loss), gwp, gbp,
                                _p(gx) if gx is not None else None, mp, threads)
    return float(loss[0]), gws, gbs, gx


def mlp_loss(ws, bs, x, onehot, act: str = "tanh", threads: int = 1):
    L = len(ws)
    ws = [_c(w) for w in ws]
    bs = [_c(b) for b in bs]
    x = _c(x)
    onehot = _c(onehot)
    dims = np.array([ws[0].shape[0]] + [w.shape[1] for w in ws], dtype=np.int64)
    wp = (C.c_void_p * L)(*[w.ctypes.data for w in ws])
    bp = (C.c_void_p * L)(*[b.ctypes.data for b in bs])
    loss = np.zeros(1, np.float32)
    lib().orc_mlp_loss_f32(L, _p(dims), 0 if act == "tanh" else 1, wp, bp, _p(x), _p(onehot),
                           x.shape[0], _p(loss), threads)
    return float(loss[0])


def sweep(x, y, want_z: bool = False):
    """where(x.gt(0), tanh(x)*sigmoid(y), relu(y).clip(-1,1)) + sum(-1,keep) + argmax(-1)."""
    x = _c(x)
    y = _c(y)
    rows, cols = x.shape
    z = np.empty_like(x) if want_z else None
    s = np.empty((rows, 1), np.float32)
    am = np.empty(rows, np.int32)
    lib().orc_sweep_f32(_p(x), _p(y), rows, cols, _p(z) if z is not None else None, _p(s), _p(am))
    return z, s, am


def nproc() -> int:
    return len(os.sched_getaffinity(0))


# ---- Fft (api/Fft.java) -------------------------------------------------------
def _fft_dtype(a: np.ndarray) -> int:
    if a.dtype == np.float64:
        return F64
    if a.dtype == np.float32:
        return F32
    raise TypeError(f"fft oracle: float32 or float64, got {a.dtype}")


def _fft_dims(shape):
    return np.asarray(shape, dtype=np.int64)


def fft(re, im, inverse=False):
    """Fft.fft / ifft / fft3 / ifft3 (Fft.java:64-80, 292-371, 405-418, 571-612)."""
    re = np.ascontiguousarray(re).copy()
    im = np.ascontiguousarray(im, dtype=re.dtype).copy()
    d = _fft_dims(re.shape)
    lib().orc_fft(_fft_dtype(re), re.ndim, _p(d), _p(re), _p(im), int(bool(inverse)))
    return re, im


def rfft(x):
    """Fft.rfft / rfft3 (Fft.java:93-127, 423-492): the half spectrum along the last axis."""
    x = np.ascontiguousarray(x)
    out_shape = x.shape[:-1] + (x.shape[-1] // 2 + 1,)
    ore, oim = np.empty(out_shape, x.dtype), np.empty(out_shape, x.dtype)
    d = _fft_dims(x.shape)
    lib().orc_rfft(_fft_dtype(x), x.ndim, _p(d), _p(x), _p(ore), _p(oim))
    return ore, oim


def irfft(re, im):
    """Fft.irfft / irfft3 (Fft.java:130-186, 494-568): the real signal of length 2 (h - 1) on the last axis."""
    re = np.ascontiguousarray(re)
    im = np.ascontiguousarray(im, dtype=re.dtype)
    shape = re.shape[:-1] + (2 * (re.shape[-1] - 1),)
    out = np.empty(shape, re.dtype)
    d = _fft_dims(shape)
    lib().orc_irfft(_fft_dtype(re), re.ndim, _p(d), _p(re), _p(im), _p(out))
    return out


def dct1(x):
    """Fft.dctI (Fft.java:200-227, 373-398)."""
    x = np.ascontiguousarray(x)
    out = np.empty_like(x)
    lib().orc_dct1(_fft_dtype(x), x.shape[0], _p(x), _p(out))
    return out


# ---- Linalg (api/Linalg.java) ----------------------------------------------------
LU_ZERO_PIVOT, LU_SUBMATRIX = 1, 2


def lu_factor(a, submatrix_check: bool = True):
    """Linalg.luFactorInPlace (Linalg.java:1021-1085) on a copy of the n x n
    matrix `a` (computed in FP64).  Returns (status, lu, piv, norms, fail_k,
    fail_pivot): status 0, LU_ZERO_PIVOT or LU_SUBMATRIX; lu the packed
    row-major factors; piv[i] the original row of factored row i; norms =
    (max |a_ij|, max row sum)."""
    lu = np.array(a, dtype=np.float64, copy=True, order="C")
    n = lu.shape[0]
    piv = np.empty(n, np.int64)
    norms = np.zeros(2, np.float64)
    fk = np.zeros(1, np.int64)
    fp = np.zeros(1, np.float64)
    st = lib().orc_lu_factor(_p(lu), n, int(bool(submatrix_check)), _p(piv), _p(norms), _p(fk), _p(fp))
    return st, lu, piv, norms, int(fk[0]), float(fp[0])


def lu_solve(lu, piv, b, transpose: bool = False):
    """LU.substitute / LU.solveTranspose (Linalg.java:178-232)."""
    b = np.ascontiguousarray(b, dtype=np.float64)
    x = np.empty_like(b)
    f = lib().orc_lu_solve_t if transpose else lib().orc_lu_solve
    f(_p(lu), _p(piv), lu.shape[0], _p(b), _p(x))
    return x


def lu_rcond(lu, piv, inf_norm: float) -> float:
    """Linalg.reciprocalConditionNumber (Linalg.java:1102-1153): Hager's estimate."""
    return float(lib().orc_lu_rcond(_p(lu), _p(piv), lu.shape[0], float(inf_norm)))


def eig(a):
    """Linalg.eig(A) (Linalg.java:768-800, 815-1005): Householder reduction to
    Hessenberg form, then Francis double-shift QR; (wr, wi) in the order the
    eigenvalues deflate, in a's dtype.  Raises if the iteration does not
    converge (the reference's IllegalStateException)."""
    a = np.ascontiguousarray(a)
    n = a.shape[0]
    wr, wi = np.empty(n, a.dtype), np.empty(n, a.dtype)
    if lib().orc_eig(_fft_dtype(a), n, _p(a), _p(wr), _p(wi)):
        raise RuntimeError("eig: Francis QR failed to converge")
    return wr, wi


def svd(a):
    """Linalg.svd (Linalg.java:411-460, 485-749): Golub-Kahan bidiagonalisation
    and Golub-Reinsch QR sweeps; (U [m, n], sigma [n], Vt [n, n]) in FP64."""
    a = np.ascontiguousarray(a)
    m, n = a.shape
    u, s, vt = np.empty((m, n)), np.empty(n), np.empty((n, n))
    if lib().orc_svd(_fft_dtype(a), m, n, _p(a), _p(u), _p(s), _p(vt)):
        raise RuntimeError("svd: QR sweep failed to converge")
    return u, s, vt
