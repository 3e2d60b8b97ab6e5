"""Array core: DType, Shape, Device, PRNGKey and the device-resident NDArray.

Mirrors the reference's core package (core/NDArray.java, core/ConcreteNDArray.java,
core/Shape.java, core/DType.java, core/Device.java, core/PRNGKey.java; paths
relative to src/main/java/com/marmanis/jax4j/) with the same method names,
argument meaning and exceptions.  The difference is storage: a
ConcreteNDArray holds a resident HBM buffer (a torch tensor used only as the
allocation) and every operation runs a libjax4j_cuda kernel on the array's
GPU stream.  There is no host compute path.
"""
from __future__ import annotations

import enum
import threading
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import call, dims as _dims


# ---------------------------------------------------------------------------
# Exceptions named like the Java ones the reference throws.
# ---------------------------------------------------------------------------
class IllegalArgumentException(ValueError):
    pass


class IllegalStateException(RuntimeError):
    pass


class UnsupportedOperationException(NotImplementedError):
    pass


# ---------------------------------------------------------------------------
# Primitive ordinals (ir/Primitive.java:6-42); the C ABI takes them as-is.
# ---------------------------------------------------------------------------
class Primitive(enum.IntEnum):
    ADD = 0
    SUB = 1
    MUL = 2
    DIV = 3
    DOT = 4
    EXP = 5
    LOG = 6
    SIN = 7
    COS = 8
    SUM = 9
    MEAN = 10
    SUM_AXIS = 11
    MEAN_AXIS = 12
    TANH = 13
    RELU = 14
    SIGMOID = 15
    COND = 16
    WHILE = 17
    SCAN = 18
    GT = 19
    GE = 20
    LT = 21
    LE = 22
    EQ = 23
    NE = 24
    MAX = 25
    MIN = 26
    ARGMAX = 27
    ARGMIN = 28
    PMAP = 29
    PSUM = 30
    ALL_GATHER = 31
    CAST = 32
    GATHER = 33
    FFI_CALL = 34
    CHECKPOINT = 35

    def __str__(self):
        return self.name.lower()


# ---------------------------------------------------------------------------
# DType (core/DType.java)
# ---------------------------------------------------------------------------
class DType(enum.Enum):
    FLOAT32 = (0, 4, "float32")
    FLOAT64 = (1, 8, "float64")
    INT32 = (2, 4, "int32")
    INT64 = (3, 8, "int64")
    BOOL = (4, 1, "bool")

    @property
    def ordinal(self) -> int:
        return self.value[0]

    def byteSize(self) -> int:
        return self.value[1]

    def __str__(self):
        return self.value[2]

    @property
    def torch(self) -> torch.dtype:
        return _TORCH[self]

    @property
    def numpy(self):
        return _NUMPY[self]

    def is_floating(self) -> bool:
        return self in (DType.FLOAT32, DType.FLOAT64)

    @staticmethod
    def promote(d1: "DType", d2: "DType") -> "DType":
        """core/DType.java:25-40."""
        if d1 == d2:
            return d1
        if d1 == DType.BOOL:
            return d2
        if d2 == DType.BOOL:
            return d1
        if d1 == DType.FLOAT64 or d2 == DType.FLOAT64:
            return DType.FLOAT64
        if (d1 == DType.INT64 and d2 == DType.FLOAT32) or (d1 == DType.FLOAT32 and d2 == DType.INT64):
            return DType.FLOAT64
        if d1 == DType.FLOAT32 or d2 == DType.FLOAT32:
            return DType.FLOAT32
        if d1 == DType.INT64 or d2 == DType.INT64:
            return DType.INT64
        return DType.INT32


_TORCH = {DType.FLOAT32: torch.float32, DType.FLOAT64: torch.float64, DType.INT32: torch.int32,
          DType.INT64: torch.int64, DType.BOOL: torch.uint8}
_NUMPY = {DType.FLOAT32: np.float32, DType.FLOAT64: np.float64, DType.INT32: np.int32,
          DType.INT64: np.int64, DType.BOOL: np.bool_}


# ---------------------------------------------------------------------------
# Shape (core/Shape.java)
# ---------------------------------------------------------------------------
class Shape:
    __slots__ = ("_d",)

    def __init__(self, *dims):
        if len(dims) == 1 and isinstance(dims[0], (list, tuple)):
            dims = tuple(dims[0])
        self._d = tuple(int(d) for d in dims)

    def dimensions(self) -> tuple:
        return self._d

    def rank(self) -> int:
        return len(self._d)

    def size(self) -> int:
        s = 1
        for d in self._d:
            s *= d
        return s

    @staticmethod
    def broadcast(a: "Shape", b: "Shape") -> "Shape":
        """core/Shape.java:37-49."""
        rank = max(a.rank(), b.rank())
        out = []
        for i in range(rank):
            da = 1 if i < rank - a.rank() else a._d[i - (rank - a.rank())]
            db = 1 if i < rank - b.rank() else b._d[i - (rank - b.rank())]
            if da != db and da != 1 and db != 1:
                raise IllegalArgumentException(f"Shapes {a} and {b} are not broadcast-compatible")
            out.append(max(da, db))
        return Shape(out)

    def normalizeAxis(self, axis: int) -> int:
        """core/Shape.java:52-58."""
        norm = self.rank() + axis if axis < 0 else axis
        if norm < 0 or norm >= self.rank():
            raise IllegalArgumentException(f"axis {axis} out of bounds for shape {self}")
        return norm

    def reduceAxis(self, axis: int, keepDims: bool) -> "Shape":
        """core/Shape.java:65-77."""
        norm = self.normalizeAxis(axis)
        if keepDims:
            d = list(self._d)
            d[norm] = 1
            return Shape(d)
        return Shape([d for i, d in enumerate(self._d) if i != norm])

    def axis_split(self, axis: int):
        """(outer, axis_len, inner) of the block decomposition used by reductions."""
        outer = 1
        for d in self._d[:axis]:
            outer *= d
        inner = 1
        for d in self._d[axis + 1:]:
            inner *= d
        return outer, self._d[axis], inner

    def __eq__(self, other):
        return isinstance(other, Shape) and self._d == other._d

    def __hash__(self):
        return hash(self._d)

    def __repr__(self):
        return "[" + ", ".join(str(d) for d in self._d) + "]"

    def __iter__(self):
        return iter(self._d)

    def __len__(self):
        return len(self._d)

    def __getitem__(self, i):
        return self._d[i]


# ---------------------------------------------------------------------------
# Device (core/Device.java): identity equality, host() singleton.
# ---------------------------------------------------------------------------
class Device:
    """A logical execution target.

    Device(None) is a synthetic device (the reference's `new Device(null)`):
    distinct by identity, physically the process's default GPU.  Device.cuda(i)
    is GPU i.  Device.host() is the reference's host singleton; there is no
    host compute, so it too resolves to the default GPU and only keeps the
    reference's device-tag rules (core/ConcreteNDArray.java:261-267).
    """

    _host: Optional["Device"] = None
    _cuda: dict = {}
    _default: Optional["Device"] = None
    _default_ordinal: int = 0
    _lock = threading.Lock()

    __slots__ = ("_ordinal", "_name", "__weakref__")

    def __init__(self, ordinal: Optional[int] = None, name: Optional[str] = None):
        self._ordinal = ordinal
        self._name = name

    @classmethod
    def host(cls) -> "Device":
        with cls._lock:
            if cls._host is None:
                cls._host = Device(None, "Host-CPU")
            return cls._host

    @classmethod
    def cuda(cls, ordinal: int) -> "Device":
        with cls._lock:
            d = cls._cuda.get(ordinal)
            if d is None:
                d = Device(ordinal, f"cuda:{ordinal}")
                cls._cuda[ordinal] = d
            return d

    @classmethod
    def getDevices(cls) -> list:
        """core/Device.java:53-77: one Device per visible GPU."""
        n = torch.cuda.device_count()
        return [cls.cuda(i) for i in range(n)]

    @classmethod
    def defaultDevice(cls) -> "Device":
        """core/Device.java:82-99: prefers a GPU; here a GPU is required."""
        with cls._lock:
            if cls._default is not None:
                return cls._default
        d = cls.cuda(cls._default_ordinal)
        with cls._lock:
            cls._default = d
        return d

    @classmethod
    def setDefault(cls, device: "Device") -> None:
        """Selects the process's default device (one process per GPU binds its own)."""
        with cls._lock:
            cls._default = device
            if device._ordinal is not None:
                cls._default_ordinal = device._ordinal

    def ordinal(self) -> int:
        """Physical CUDA ordinal backing this device."""
        return self._ordinal if self._ordinal is not None else Device._default_ordinal

    def is_synthetic(self) -> bool:
        return self._ordinal is None

    def getName(self) -> str:
        if self._name:
            return self._name
        return "synthetic"

    def torch_device(self) -> torch.device:
        return torch.device("cuda", self.ordinal())

    def __repr__(self):
        return f"Device[{self.getName()}#{id(self):x}]"


# ---------------------------------------------------------------------------
# PRNGKey (core/PRNGKey.java)
# ---------------------------------------------------------------------------
class PRNGKey:
    __slots__ = ("_state",)

    def __init__(self, state: int):
        self._state = int(state) & 0xFFFFFFFFFFFFFFFF

    @staticmethod
    def key(seed: int) -> "PRNGKey":
        return PRNGKey(seed)

    def state(self) -> int:
        return self._state

    def __eq__(self, other):
        return isinstance(other, PRNGKey) and other._state == self._state

    def __hash__(self):
        return hash(self._state)

    def __repr__(self):
        return f"PRNGKey[state={self._state}]"


# ---------------------------------------------------------------------------
# Streams: one per (thread, GPU) via torch's thread-local current stream.
# ---------------------------------------------------------------------------
def stream_of(ordinal: int) -> int:
    """Handle of the device's current torch stream, with that device made the
    calling thread's current device first: the library launches on the current
    device, and the default stream's handle (0) does not name one, so an op on
    another GPU's array must not run with a different device current."""
    if torch.cuda.current_device() != ordinal:
        torch.cuda.set_device(ordinal)
    return torch.cuda.current_stream(ordinal).cuda_stream


# ---------------------------------------------------------------------------
# NDArray (core/NDArray.java)
# ---------------------------------------------------------------------------
class NDArray:
    """The public array interface (core/NDArray.java:7-132)."""

    def shape(self) -> Shape: raise NotImplementedError
    def dtype(self) -> DType: raise NotImplementedError
    def device(self) -> Device: raise NotImplementedError

    def sum(self, axis=None, keepDims=False):  # noqa: D401
        raise NotImplementedError

    def clip(self, lo, hi):
        """core/NDArray.java:82: max(lo).min(hi)."""
        return self.max(lo).min(hi)

    # numpy-ish conveniences for Python callers
    def __add__(self, o): return self.add(_as_array(o, self))
    def __sub__(self, o): return self.sub(_as_array(o, self))
    def __mul__(self, o): return self.mul(_as_array(o, self))
    def __truediv__(self, o): return self.div(_as_array(o, self))
    def __matmul__(self, o): return self.dot(o)


def _as_array(v, like: Optional[NDArray] = None) -> NDArray:
    if isinstance(v, NDArray):
        return v
    if isinstance(v, (int, float)):
        return ConcreteNDArray.scalar(float(v))
    return ConcreteNDArray.of(v)


class ConcreteNDArray(NDArray):
    """A device-resident array (core/ConcreteNDArray.java).

    Storage is a flat, contiguous HBM buffer of shape.size() elements of the
    dtype (BOOL as one byte 0/1).  Instances are immutable, which is what
    lets a FLOAT32 array keep the hi/lo splits of its values (`_split`, by
    kind) once it has been a dot operand, for the other dots it takes part in.
    """

    __slots__ = ("_t", "_shape", "_dtype", "_device", "_split", "_ready", "_lines", "_relu_bits", "_scalar")

    def __init__(self, data, shape=None, dtype: DType = None, device: Device = None):
        if device is None:
            device = Device.defaultDevice()
        if isinstance(data, torch.Tensor):
            t = data
            if dtype is None:
                dtype = _from_torch(t.dtype)
            if t.dtype != dtype.torch or t.device.type != "cuda" or t.device.index != device.ordinal():
                t = t.to(device=device.torch_device(), dtype=dtype.torch)
            t = t.reshape(-1)
            if not t.is_contiguous():
                t = t.contiguous()
        else:
            arr = np.asarray(data)
            if dtype is None:
                dtype = _dtype_of_numpy(arr)
            if dtype == DType.BOOL:
                arr = arr.astype(np.bool_).astype(np.uint8)
            else:
                arr = arr.astype(dtype.numpy)
            t = torch.from_numpy(np.ascontiguousarray(arr).reshape(-1)).to(
                device=device.torch_device(), non_blocking=False)
        if shape is None:
            shape = Shape(t.numel())
        elif not isinstance(shape, Shape):
            shape = Shape(shape)
        if t.numel() != shape.size():
            raise IllegalArgumentException(f"data has {t.numel()} elements but shape {shape} needs {shape.size()}")
        self._t = t
        self._shape = shape
        self._dtype = dtype
        self._device = device
        self._split = None  # {kind: (hi, lo)}: "r" row lines, "c" column lines, "t" transposed
        self._ready = None  # CUDA event recorded once the value was produced, when tracked
        self._lines = None  # device words [rows + cols + 1]: line maxima (bits of max finite |x|), NaN/Inf flag
        self._relu_bits = None  # a relu output's x > 0 as bits (rows of ceil(cols / 32) words), from its GEMM
        self._scalar = None  # host copy of a one-element floating array made by full() / scalar()

    # ---- construction helpers ----
    @staticmethod
    def of(values, shape=None, dtype: DType = DType.FLOAT32, device: Device = None) -> "ConcreteNDArray":
        arr = np.asarray(values)
        if shape is None:
            shape = Shape(arr.shape) if arr.ndim > 0 else Shape(1)
        return ConcreteNDArray(arr, shape, dtype, device)

    @staticmethod
    def scalar(v: float, dtype: DType = DType.FLOAT32, device: Device = None) -> "ConcreteNDArray":
        return ConcreteNDArray.full(Shape(1), v, dtype, device)

    @staticmethod
    def full(shape, value: float, dtype: DType = DType.FLOAT32, device: Device = None) -> "ConcreteNDArray":
        shape = shape if isinstance(shape, Shape) else Shape(shape)
        device = device or Device.defaultDevice()
        t = torch.empty(shape.size(), dtype=dtype.torch, device=device.torch_device())
        call("j4c_fill", dtype.ordinal, t.data_ptr(), t.numel(), float(value), stream_of(device.ordinal()))
        out = ConcreteNDArray._wrap(t, shape, dtype, device)
        if shape.size() == 1 and dtype in (DType.FLOAT32, DType.FLOAT64):
            # the value the fill kernel stored ((float) value for FLOAT32), so
            # a fused program can take it as a literal
            out._scalar = float(np.float32(value)) if dtype == DType.FLOAT32 else float(value)
        return out

    @staticmethod
    def _wrap(t: torch.Tensor, shape: Shape, dtype: DType, device: Device) -> "ConcreteNDArray":
        obj = ConcreteNDArray.__new__(ConcreteNDArray)
        obj._t = t
        obj._shape = shape
        obj._dtype = dtype
        obj._device = device
        obj._split = None
        obj._ready = None
        obj._lines = None
        obj._relu_bits = None
        obj._scalar = None
        return obj

    def _new(self, shape: Shape, dtype: DType) -> torch.Tensor:
        return torch.empty(shape.size(), dtype=dtype.torch, device=self._t.device)

    def _stream(self) -> int:
        return stream_of(self._t.device.index)

    # ---- accessors ----
    def shape(self) -> Shape:
        return self._shape

    def dtype(self) -> DType:
        return self._dtype

    def device(self) -> Device:
        return self._device

    def tensor(self) -> torch.Tensor:
        """The backing HBM buffer (flat).  Arrays are immutable: a caller that
        refills this buffer in place (an input slot reused across steps) wraps
        it in a new array afterwards, since this one may keep a split of its
        old values for dot."""
        return self._t

    def data_ptr(self) -> int:
        return self._t.data_ptr()

    def to(self, device: Device) -> "ConcreteNDArray":
        """core/ConcreteNDArray.java:148-151: re-tags; moves the buffer only if the
        target is another physical GPU."""
        t = self._t
        if t.device.type == "cuda" and t.device.index != device.ordinal():
            t = t.to(device.torch_device())
        return ConcreteNDArray._wrap(t, self._shape, self._dtype, device)

    def reshape(self, shape) -> "ConcreteNDArray":
        shape = shape if isinstance(shape, Shape) else Shape(shape)
        if shape.size() != self._shape.size():
            raise IllegalArgumentException(f"cannot reshape {self._shape} to {shape}")
        return ConcreteNDArray._wrap(self._t, shape, self._dtype, self._device)

    # ---- tracing ----
    def _to_traced(self):
        return TracedNDArray(Tracer.current().nextConstant(self))

    # ---- dtype guards (core/ConcreteNDArray.java:169-188) ----
    def _require_floating(self, op: str):
        if not self._dtype.is_floating():
            raise IllegalArgumentException(
                f"{op} requires FLOAT32 or FLOAT64 operands, got {self._dtype} — use .astype() to convert.")

    def _require_same_floating(self, other: NDArray, op: str):
        self._require_floating(op)
        if other.dtype() != self._dtype:
            raise IllegalArgumentException(
                f"{op} requires both operands to share the same floating dtype, got {self._dtype} "
                f"and {other.dtype()} — use .astype() to convert.")

    def _check_devices(self, other: "ConcreteNDArray") -> Device:
        """core/ConcreteNDArray.java:261-267 / :442-447: arrays on different
        devices do not combine.  Returns the result's device.  One relaxation:
        an array on the process's default device combines with an array on
        any device backed by the same GPU (it acts as a constant replicated to
        the pmap shards that share the GPU); the result takes the other
        device.  Combinations the reference accepts behave identically."""
        a, b = self._device, other._device
        if a is b:
            return a
        dflt = Device.defaultDevice()
        if (a is dflt or b is dflt) and a.ordinal() == b.ordinal():
            return b if a is dflt else a
        raise IllegalStateException(f"Cannot combine arrays on different devices: {a} vs {b}")

    def _promote_or_trace(self, other: NDArray, traced_op, eager):
        """The shared prologue of elementwise/compare/dot
        (core/ConcreteNDArray.java:221-231, 331-341, 408-418)."""
        target = DType.promote(self._dtype, other.dtype())
        left = self if self._dtype == target else self.astype(target)
        right = other if other.dtype() == target else other.astype(target)
        if isinstance(left, TracedNDArray) or isinstance(right, TracedNDArray) or Tracer.current() is not None:
            lt = left if isinstance(left, TracedNDArray) else left._to_traced()
            rt = right if isinstance(right, TracedNDArray) else right._to_traced()
            return traced_op(lt, rt)
        return eager(left, right)

    # ---- elementwise binary (core/ConcreteNDArray.java:219-316) ----
    def _elementwise(self, other: NDArray, prim: Primitive, traced_op):
        other = _as_array(other)
        if self._dtype != other.dtype() or isinstance(other, TracedNDArray) or Tracer.current() is not None:
            return self._promote_or_trace(other, traced_op,
                                          lambda l, r: l._elementwise(r, prim, traced_op))
        self._require_same_floating(other, str(prim))
        dev = self._check_devices(other)
        out_shape = Shape.broadcast(self._shape, other._shape)
        out = self._new(out_shape, self._dtype)
        call("j4c_binary", int(prim), self._dtype.ordinal, self._t.data_ptr(), _dims(self._shape),
             self._shape.rank(), other._t.data_ptr(), _dims(other._shape), other._shape.rank(),
             out.data_ptr(), self._stream())
        return ConcreteNDArray._wrap(out, out_shape, self._dtype, dev)

    def add(self, other): return self._elementwise(other, Primitive.ADD, lambda a, b: a.add(b))
    def sub(self, other): return self._elementwise(other, Primitive.SUB, lambda a, b: a.sub(b))
    def mul(self, other): return self._elementwise(other, Primitive.MUL, lambda a, b: a.mul(b))
    def div(self, other): return self._elementwise(other, Primitive.DIV, lambda a, b: a.div(b))
    def max(self, other): return self._elementwise(other, Primitive.MAX, lambda a, b: a.max(b))
    def min(self, other): return self._elementwise(other, Primitive.MIN, lambda a, b: a.min(b))

    # ---- comparisons (core/ConcreteNDArray.java:328-404) ----
    def _compare(self, other: NDArray, prim: Primitive, traced_op):
        other = _as_array(other)
        if self._dtype != other.dtype() or isinstance(other, TracedNDArray) or Tracer.current() is not None:
            return self._promote_or_trace(other, traced_op, lambda l, r: l._compare(r, prim, traced_op))
        if self._dtype == DType.BOOL:
            raise IllegalArgumentException(
                f"{prim} requires FLOAT32, INT32, FLOAT64, or INT64 operands, got {self._dtype}")
        # the reference's comparison applies no device-tag rule (its result
        # keeps the receiver's device); both buffers must share a GPU here
        if self._device.ordinal() != other._device.ordinal():
            raise IllegalStateException(
                f"Cannot combine arrays on different devices: {self._device} vs {other._device}")
        dev = self._device
        out_shape = Shape.broadcast(self._shape, other._shape)
        out = self._new(out_shape, DType.BOOL)
        call("j4c_compare", int(prim), self._dtype.ordinal, self._t.data_ptr(), _dims(self._shape),
             self._shape.rank(), other._t.data_ptr(), _dims(other._shape), other._shape.rank(),
             out.data_ptr(), self._stream())
        return ConcreteNDArray._wrap(out, out_shape, DType.BOOL, dev)

    def gt(self, other): return self._compare(other, Primitive.GT, lambda a, b: a.gt(b))
    def ge(self, other): return self._compare(other, Primitive.GE, lambda a, b: a.ge(b))
    def lt(self, other): return self._compare(other, Primitive.LT, lambda a, b: a.lt(b))
    def le(self, other): return self._compare(other, Primitive.LE, lambda a, b: a.le(b))
    def eq(self, other): return self._compare(other, Primitive.EQ, lambda a, b: a.eq(b))
    def ne(self, other): return self._compare(other, Primitive.NE, lambda a, b: a.ne(b))

    # ---- dot (core/ConcreteNDArray.java:406-461) ----
    def dot(self, other: NDArray, trans_a: bool = False, trans_b: bool = False):
        if self._dtype != other.dtype() or isinstance(other, TracedNDArray) or Tracer.current() is not None:
            return self._promote_or_trace(other, lambda a, b: a.dot(b), lambda l, r: l.dot(r))
        self._require_same_floating(other, "dot")
        dev = self._check_devices(other)
        return _dot_raw(self, other, trans_a, trans_b, dev)

    # ---- reductions (core/ConcreteNDArray.java:463-618) ----
    def sum(self, axis: Optional[int] = None, keepDims: bool = False):
        if Tracer.current() is not None:
            return self._to_traced().sum(axis, keepDims) if axis is not None else self._to_traced().sum()
        self._require_floating("sum")
        if axis is None:
            return self._reduce_all(Primitive.SUM)
        return self._reduce_axis(axis, keepDims, Primitive.SUM_AXIS)

    def mean(self, axis: Optional[int] = None, keepDims: bool = False):
        if Tracer.current() is not None:
            return self._to_traced().mean(axis, keepDims) if axis is not None else self._to_traced().mean()
        self._require_floating("mean")
        if axis is None:
            return self._reduce_all(Primitive.MEAN)
        return self._reduce_axis(axis, keepDims, Primitive.MEAN_AXIS)

    def _reduce_all(self, prim: Primitive):
        out = self._new(Shape(1), self._dtype)
        call("j4c_reduce_all", int(prim), self._dtype.ordinal, self._t.data_ptr(), self._shape.size(),
             out.data_ptr(), self._stream())
        return ConcreteNDArray._wrap(out, Shape(1), self._dtype, self._device)

    def _reduce_axis(self, axis: int, keepDims: bool, prim: Primitive):
        norm = self._shape.normalizeAxis(axis)
        outer, n, inner = self._shape.axis_split(norm)
        out_shape = self._shape.reduceAxis(norm, keepDims)
        out = self._new(out_shape, self._dtype)
        call("j4c_reduce_axis", int(prim), self._dtype.ordinal, self._t.data_ptr(), outer, n, inner,
             out.data_ptr(), self._stream())
        return ConcreteNDArray._wrap(out, out_shape, self._dtype, self._device)

    def argmax(self, axis: int):
        if Tracer.current() is not None:
            return self._to_traced().argmax(axis)
        self._require_floating("argmax")
        return self._argreduce(axis, Primitive.ARGMAX)

    def argmin(self, axis: int):
        if Tracer.current() is not None:
            return self._to_traced().argmin(axis)
        self._require_floating("argmin")
        return self._argreduce(axis, Primitive.ARGMIN)

    def _argreduce(self, axis: int, prim: Primitive):
        norm = self._shape.normalizeAxis(axis)
        outer, n, inner = self._shape.axis_split(norm)
        out_shape = self._shape.reduceAxis(norm, False)
        out = self._new(out_shape, DType.INT32)
        call("j4c_argreduce", int(prim), self._dtype.ordinal, self._t.data_ptr(), outer, n, inner,
             out.data_ptr(), self._stream())
        return ConcreteNDArray._wrap(out, out_shape, DType.INT32, self._device)

    # ---- unary (core/ConcreteNDArray.java:627-664) ----
    def _unary(self, prim: Primitive, traced_op):
        if Tracer.current() is not None:
            return traced_op(self._to_traced())
        self._require_floating(str(prim))
        out = self._new(self._shape, self._dtype)
        call("j4c_unary", int(prim), self._dtype.ordinal, self._t.data_ptr(), self._shape.size(),
             out.data_ptr(), self._stream())
        return ConcreteNDArray._wrap(out, self._shape, self._dtype, self._device)

    def exp(self): return self._unary(Primitive.EXP, lambda a: a.exp())
    def log(self): return self._unary(Primitive.LOG, lambda a: a.log())
    def sin(self): return self._unary(Primitive.SIN, lambda a: a.sin())
    def cos(self): return self._unary(Primitive.COS, lambda a: a.cos())
    def tanh(self): return self._unary(Primitive.TANH, lambda a: a.tanh())
    def relu(self): return self._unary(Primitive.RELU, lambda a: a.relu())
    def sigmoid(self): return self._unary(Primitive.SIGMOID, lambda a: a.sigmoid())

    # ---- astype (core/ConcreteNDArray.java:666-730) ----
    def astype(self, target: DType):
        if Tracer.current() is not None:
            return self._to_traced().astype(target)
        if target == self._dtype:
            return self
        out = self._new(self._shape, target)
        call("j4c_cast", self._dtype.ordinal, target.ordinal, self._t.data_ptr(), self._shape.size(),
             out.data_ptr(), self._stream())
        return ConcreteNDArray._wrap(out, self._shape, target, self._device)

    # ---- host transfer (core/ConcreteNDArray.java:732-760) ----
    def _host(self, dtype: DType, accessor: str) -> np.ndarray:
        if self._dtype != dtype:
            raise IllegalStateException(
                f"{accessor}() requires dtype {dtype}, but this array is {self._dtype}")
        arr = self._t.cpu().numpy()
        return arr.astype(np.bool_) if dtype == DType.BOOL else arr

    def toFloatArray(self) -> np.ndarray: return self._host(DType.FLOAT32, "toFloatArray")
    def toIntArray(self) -> np.ndarray: return self._host(DType.INT32, "toIntArray")
    def toBoolArray(self) -> np.ndarray: return self._host(DType.BOOL, "toBoolArray")
    def toDoubleArray(self) -> np.ndarray: return self._host(DType.FLOAT64, "toDoubleArray")
    def toLongArray(self) -> np.ndarray: return self._host(DType.INT64, "toLongArray")

    def numpy(self) -> np.ndarray:
        """The data as a numpy array of this array's shape (any dtype)."""
        arr = self._t.cpu().numpy()
        if self._dtype == DType.BOOL:
            arr = arr.astype(np.bool_)
        return arr.reshape(self._shape.dimensions())

    def __repr__(self):
        return f"Array({self.numpy().tolist()}, shape={self._shape}, dtype={self._dtype})"

    def __eq__(self, other):
        if self is other:
            return True
        if not isinstance(other, ConcreteNDArray):
            return False
        if self._shape != other._shape or self._dtype != other._dtype:
            return False
        return bool(torch.equal(self._t.cpu(), other._t.cpu()))

    def __hash__(self):
        return hash((self._shape, self._dtype))


def _from_torch(dt: torch.dtype) -> DType:
    for k, v in _TORCH.items():
        if v == dt:
            return k
    if dt == torch.bool:
        return DType.BOOL
    raise IllegalArgumentException(f"unsupported tensor dtype {dt}")


def _dtype_of_numpy(arr: np.ndarray) -> DType:
    if arr.dtype == np.bool_:
        return DType.BOOL
    if arr.dtype == np.float64:
        return DType.FLOAT64
    if arr.dtype == np.int32:
        return DType.INT32
    if arr.dtype == np.int64:
        return DType.INT64
    return DType.FLOAT32


# When a list, every dot launch appends (start_event, end_event, flops, bytes):
# CUDA events recorded on the launching stream around the kernel (used by the
# benchmark to time the GEMM kernels inside its timed region) and the launch's
# algorithmic HBM bytes: each FP32 operand read once as its hi/lo split (4 B per
# element for 3xFP16, 8 B for 3xTF32), every output written once, the
# epilogue's bias and mask read once.
DOT_TIMING = None

# The relu' mask of an input gradient read as the bits the forward GEMM left
# (1/32 of the bytes of the float relu output).
RELU_BITS = True


_SPLIT_KIND = None


def split_kind() -> int:
    """The library's FLOAT32 dot split: 1 = 3xFP16 (power-of-two scaled FP16
    hi/lo), 0 = 3xTF32 (J4C_GEMM_SPLIT=tf32); fixed for the process."""
    global _SPLIT_KIND
    if _SPLIT_KIND is None:
        _SPLIT_KIND = int(_lib.lib().j4c_dot_split_kind())
    return _SPLIT_KIND


def split_bytes_per_element() -> int:
    """HBM bytes of one operand element's hi + lo split (read once by a GEMM)."""
    return 4 if split_kind() == 1 else 8


# Split kinds of a 2-D FLOAT32 array x [rows, cols] (j4c_split_f32_ex):
#   "r": x's layout, one line per row -- read K-major (x is A [M, K] or B^T [N, K])
#   "c": x's layout, one line per column -- read MN-major (x is A^T [K, M] or B [K, N])
#   "t": x^T, its rows (x's columns) as lines -- read K-major with the trans flag flipped
def _kind(kind: str) -> str:
    return kind


def _split_lines(x: "ConcreteNDArray"):
    """x's line maxima (rows then columns), from the GEMM that wrote x or one
    max pass, kept on the array for every split of it."""
    if x._lines is None:
        rows, cols = x._shape.dimensions()
        lines = torch.empty(rows + cols + 1, dtype=torch.int32, device=x._t.device)
        call("j4c_split_lines", x._t.data_ptr(), rows, cols, lines.data_ptr(), x._stream())
        x._lines = lines
    return x._lines


def _make_splits(x: "ConcreteNDArray", kinds) -> None:
    """The splits of x of the given kinds that it lacks, in one pass ("c" and
    "t" are alternatives: not both in one pass)."""
    kinds = [k for k in dict.fromkeys(_kind(k) for k in kinds) if not (x._split and k in x._split)]
    if not kinds:
        return
    if "c" in kinds and "t" in kinds:
        _make_splits(x, ["t"])
        kinds.remove("t")
    rows, cols = x._shape.dimensions()
    L = _lib.lib()
    out = {}
    for k in kinds:
        n = L.j4c_split_floats(cols, rows) if k == "t" else L.j4c_split_floats(rows, cols)
        out[k] = (torch.empty(n, dtype=torch.float32, device=x._t.device),
                  torch.empty(n, dtype=torch.float32, device=x._t.device))
    ptrs = []
    for k in ("r", "c", "t"):
        ptrs += [out[k][0].data_ptr(), out[k][1].data_ptr()] if k in out else [None, None]
    lines = _split_lines(x)
    call("j4c_split_f32_ex", x._t.data_ptr(), rows, cols, *ptrs,
         lines.data_ptr() if lines is not None else None, x._stream())
    if x._split is None:
        x._split = {}
    x._split.update(out)


def _split_of(x: "ConcreteNDArray", kind: str):
    """The (hi, lo) split of a 2-D FLOAT32 array of the given kind, made on
    first use and kept on the (immutable) array."""
    kind = _kind(kind)
    if x._split is None or kind not in x._split:
        _make_splits(x, [kind])
    return x._split[kind]


def dot_supports_epilogue(a: "ConcreteNDArray") -> bool:
    """Whether _dot_raw can fuse a bias / relu' / relu into the product's store."""
    return a._dtype == DType.FLOAT32


def _dot_raw(a: "ConcreteNDArray", b: "ConcreteNDArray", trans_a: bool, trans_b: bool,
             device: Device, bias: "ConcreteNDArray" = None, mask: "ConcreteNDArray" = None,
             act: bool = False, store_c: bool = True):
    """C = op(A) . op(B) on the tensor cores; op = transpose when flagged.

    FLOAT32 only, optional epilogue (j4c_dot_split_ep): C += bias (a [N]
    vector), C = mask > 0 ? C : 0 (mask [M, N]), and with act=True also
    returns relu(C); the result is then (C, relu(C)), or (None, relu(C)) with
    store_c=False (C itself is not written)."""
    ad, bd = a._shape.dimensions(), b._shape.dimensions()
    if len(ad) != 2 or len(bd) != 2:
        raise IllegalArgumentException(f"dot requires 2-D operands, got {a._shape} and {b._shape}")
    M, K = (ad[1], ad[0]) if trans_a else (ad[0], ad[1])
    K2, N = (bd[1], bd[0]) if trans_b else (bd[0], bd[1])
    if K != K2:
        raise IllegalArgumentException(f"dot: inner dimensions differ ({a._shape} . {b._shape})")
    epilogue = bias is not None or mask is not None or act
    if epilogue:
        if a._dtype != DType.FLOAT32 or not (M and N and K):
            raise IllegalArgumentException("dot epilogue needs a non-empty FLOAT32 product")
        if bias is not None and (bias._dtype != DType.FLOAT32 or bias._shape.size() != N):
            raise IllegalArgumentException(f"dot epilogue: bias {bias._shape} does not match N = {N}")
        if mask is not None and (mask._dtype != DType.FLOAT32 or mask._shape.size() != M * N):
            raise IllegalArgumentException(f"dot epilogue: mask {mask._shape} does not match [{M}, {N}]")
    if not store_c and not (act and a._dtype == DType.FLOAT32 and M and N and K):
        raise IllegalArgumentException("dot: C may only be skipped when the relu output is written")
    out = torch.empty(M * N if store_c else 0, dtype=a._dtype.torch, device=a._t.device)
    act_out = torch.empty(M * N, dtype=a._dtype.torch, device=a._t.device) if act else None
    timing = DOT_TIMING
    out_max = None
    act_bits = None
    if a._dtype == DType.FLOAT32 and M and N and K:
        # tensor-core path: each operand's 3xTF32 split is made once per array.
        # With K the leading dimension of both stored operands (A^T . B, the
        # weight gradient) one of them goes in transposed (K-major) form: the
        # smaller one, so the extra split pass is as short as possible.
        # The split kind follows how the GEMM reads an operand: op(A) = A and
        # op(B) = B^T K-major (row lines), op(A) = A^T and op(B) = B MN-major
        # (column lines), or a transposed split read K-major.  Both operands
        # K-major is the fastest form, so B [K, N] goes in transposed for
        # A . B; with K leading in both stored operands (A^T . B, the weight
        # gradient) the smaller one goes in transposed.
        ta, tb = trans_a, trans_b
        if ta and not tb:
            if a._shape.size() < b._shape.size():
                (ah, al), ta = _split_of(a, "t"), False
                bh, bl = _split_of(b, "c")
            else:
                ah, al = _split_of(a, "c")
                (bh, bl), tb = _split_of(b, "t"), True
        elif not ta and not tb:
            ah, al = _split_of(a, "r")
            (bh, bl), tb = _split_of(b, "t"), True
        else:
            ah, al = _split_of(a, "c" if ta else "r")
            bh, bl = _split_of(b, "r" if tb else "c")
        if timing is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        if epilogue:
            # the epilogue also takes the line maxima of the output a later split
            # will read (the relu output, or C), sparing it a max pass; a relu
            # output leaves its x > 0 bits, and a mask that has them is read as
            # bits (C stored untransposed: not the K-major A . MN-major B form)
            out_max = torch.empty(M + N + 1, dtype=torch.int32, device=a._t.device)
            bits_ok = bool(ta or tb) and RELU_BITS
            mask_bits = mask._relu_bits if (mask is not None and bits_ok) else None
            act_bits = (torch.empty(M * ((N + 31) // 32), dtype=torch.int32, device=a._t.device)
                        if act and bits_ok else None)
            call("j4c_dot_split_ep_bits", ah.data_ptr(), al.data_ptr(), bh.data_ptr(), bl.data_ptr(),
                 out.data_ptr() if store_c else None,
                 M, K, N, int(ta), int(tb), bias.data_ptr() if bias is not None else None,
                 mask.data_ptr() if (mask is not None and mask_bits is None) else None,
                 mask_bits.data_ptr() if mask_bits is not None else None,
                 act_out.data_ptr() if act_out is not None else None,
                 act_bits.data_ptr() if act_bits is not None else None,
                 out_max.data_ptr(), a._stream())
        else:
            call("j4c_dot_split", ah.data_ptr(), al.data_ptr(), bh.data_ptr(), bl.data_ptr(), out.data_ptr(),
                 M, K, N, int(ta), int(tb), a._stream())
    else:
        ws_bytes = _lib.lib().j4c_dot_workspace_size(a._dtype.ordinal, M, K, N)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=a._t.device) if ws_bytes else None
        if timing is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        call("j4c_dot_ws", a._dtype.ordinal, a._t.data_ptr(), b._t.data_ptr(), out.data_ptr(), M, K, N,
             int(trans_a), int(trans_b), ws.data_ptr() if ws is not None else None, ws_bytes,
             a._stream())
    if timing is not None:
        ev1.record()
        if a._dtype == DType.FLOAT32:
            nbytes = split_bytes_per_element() * (M * K + K * N) \
                + 4 * M * N * (int(store_c) + int(act) + int(mask is not None)) + (4 * N if bias is not None else 0)
        else:
            nbytes = a._dtype.byteSize() * (M * K + K * N + M * N)
        timing.append((ev0, ev1, 2.0 * M * N * K, nbytes))
    c = ConcreteNDArray._wrap(out, Shape(M, N), a._dtype, device) if store_c else None
    if act:
        h = ConcreteNDArray._wrap(act_out, Shape(M, N), a._dtype, device)
        if out_max is not None:
            h._lines = out_max
        if act_bits is not None:
            h._relu_bits = act_bits
        return c, h
    if out_max is not None:
        c._lines = out_max
    return c


from .tracing import TracedNDArray, Tracer  # noqa: E402  (late import: tracing imports core)
