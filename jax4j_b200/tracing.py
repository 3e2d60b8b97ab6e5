"""Tracing and IR: Var, Equation, Jaxpr, metadata records, Tracer, TracedNDArray.

Mirrors ir/*.java and tracing/*.java of the reference (paths relative to
src/main/java/com/marmanis/jax4j/): a per-thread stack of tracers records
equations with shape/dtype inference, so pmap shard threads never share
trace state (tracing/Tracer.java:16-33).
"""
from __future__ import annotations

import itertools
import threading
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

from .core import DType, NDArray, Primitive, Shape, UnsupportedOperationException


# ---------------------------------------------------------------------------
# IR records (ir/Var.java, ir/Equation.java, ir/Jaxpr.java, ir/*Meta.java)
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class Var:
    id: int
    shape: Shape
    dtype: DType

    def __repr__(self):
        return f"v{self.id}{self.shape}"


@dataclass(frozen=True)
class AxisMeta:
    axis: int
    keepDims: bool


@dataclass(frozen=True)
class PmapMeta:
    bodyJaxpr: "Jaxpr"
    devices: tuple

    def numDevices(self) -> int:
        return len(self.devices)


@dataclass(frozen=True)
class CheckpointMeta:
    subJaxpr: "Jaxpr"


@dataclass(frozen=True)
class CondMeta:
    """ir/CondMeta: the two branches of a COND, each one operand -> one result."""
    trueBranch: "Jaxpr"
    falseBranch: "Jaxpr"


@dataclass(frozen=True)
class WhileMeta:
    """ir/WhileMeta: condition (state -> BOOL/number [1]) and body (state -> state)."""
    condFn: "Jaxpr"
    bodyFn: "Jaxpr"


@dataclass(frozen=True)
class ScanMeta:
    """ir/ScanMeta: the step (carry, x_t) -> (new carry, y_t)."""
    stepFn: "Jaxpr"


@dataclass
class Equation:
    inputs: List[Var]
    outputs: List[Var]
    primitive: Primitive
    metadata: Any = None

    def __repr__(self):
        m = f" [{self.metadata}]" if self.metadata is not None and not isinstance(self.metadata, PmapMeta) else ""
        return (", ".join(map(repr, self.outputs)) + f" = {self.primitive}{m} "
                + ", ".join(map(repr, self.inputs)))


@dataclass
class Jaxpr:
    inVars: List[Var]
    outVars: List[Var]
    equations: List[Equation]
    consts: Dict[int, NDArray] = field(default_factory=dict)

    def __repr__(self):
        s = "{ lambda " + ", ".join(map(repr, self.inVars)) + " ; "
        if self.consts:
            s += f"consts: {sorted(self.consts)} ; "
        s += "\n  let\n"
        for e in self.equations:
            s += f"    {e!r}\n"
        return s + "  in (" + ", ".join(map(repr, self.outVars)) + ") }"


# ---------------------------------------------------------------------------
# Tracer (tracing/Tracer.java)
# ---------------------------------------------------------------------------
class _Stack(threading.local):
    def __init__(self):
        self.stack: List["Tracer"] = []


_stack = _Stack()


class Tracer:
    def __init__(self):
        self.equations: List[Equation] = []
        self._counter = itertools.count()
        self.consts: Dict[int, NDArray] = {}

    @staticmethod
    def start() -> None:
        _stack.stack.append(Tracer())

    @staticmethod
    def current() -> Optional["Tracer"]:
        s = _stack.stack
        return s[-1] if s else None

    @staticmethod
    def stop(inVars: List[Var], outVars: List[Var]) -> Jaxpr:
        t = _stack.stack.pop()
        return Jaxpr(list(inVars), list(outVars), t.equations, t.consts)

    @staticmethod
    def abort() -> None:
        """tracing/Tracer.java:59-63: pop without building a Jaxpr."""
        _stack.stack.pop()

    def nextVar(self, shape: Shape, dtype: DType) -> Var:
        return Var(next(self._counter), shape, dtype)

    def nextConstant(self, value: NDArray) -> Var:
        v = self.nextVar(value.shape(), value.dtype())
        self.consts[v.id] = value
        return v

    def addEquation(self, eq: Equation) -> None:
        self.equations.append(eq)


def to_var(a: NDArray) -> Var:
    if isinstance(a, TracedNDArray):
        return a.getVar()
    return Tracer.current().nextConstant(a)


# ---------------------------------------------------------------------------
# TracedNDArray (tracing/TracedNDArray.java)
# ---------------------------------------------------------------------------
class TracedNDArray(NDArray):
    __slots__ = ("_var",)

    def __init__(self, var: Var):
        self._var = var

    def getVar(self) -> Var:
        return self._var

    def shape(self) -> Shape:
        return self._var.shape

    def dtype(self) -> DType:
        return self._var.dtype

    def device(self):
        from .core import Device
        return Device.defaultDevice()

    def to(self, device):
        return self

    def _apply(self, prim: Primitive, inputs, out_shape: Shape, out_dtype: DType = None, meta=None):
        tracer = Tracer.current()
        in_vars = [to_var(i) for i in inputs]
        out = tracer.nextVar(out_shape, out_dtype if out_dtype is not None else self.dtype())
        tracer.addEquation(Equation(in_vars, [out], prim, meta))
        return TracedNDArray(out)

    def _elementwise(self, other, prim: Primitive, traced_op):
        from .core import _as_array
        other = _as_array(other)
        if self.dtype() != other.dtype():
            target = DType.promote(self.dtype(), other.dtype())
            left = self if self.dtype() == target else self.astype(target)
            right = other if other.dtype() == target else other.astype(target)
            return traced_op(left, right)
        return self._apply(prim, [self, other], Shape.broadcast(self.shape(), other.shape()))

    def _compare(self, other, prim: Primitive, traced_op):
        from .core import _as_array
        other = _as_array(other)
        if self.dtype() != other.dtype():
            target = DType.promote(self.dtype(), other.dtype())
            left = self if self.dtype() == target else self.astype(target)
            right = other if other.dtype() == target else other.astype(target)
            return traced_op(left, right)
        return self._apply(prim, [self, other], Shape.broadcast(self.shape(), other.shape()), DType.BOOL)

    def add(self, o): return self._elementwise(o, Primitive.ADD, lambda a, b: a.add(b))
    def sub(self, o): return self._elementwise(o, Primitive.SUB, lambda a, b: a.sub(b))
    def mul(self, o): return self._elementwise(o, Primitive.MUL, lambda a, b: a.mul(b))
    def div(self, o): return self._elementwise(o, Primitive.DIV, lambda a, b: a.div(b))
    def max(self, o): return self._elementwise(o, Primitive.MAX, lambda a, b: a.max(b))
    def min(self, o): return self._elementwise(o, Primitive.MIN, lambda a, b: a.min(b))

    def gt(self, o): return self._compare(o, Primitive.GT, lambda a, b: a.gt(b))
    def ge(self, o): return self._compare(o, Primitive.GE, lambda a, b: a.ge(b))
    def lt(self, o): return self._compare(o, Primitive.LT, lambda a, b: a.lt(b))
    def le(self, o): return self._compare(o, Primitive.LE, lambda a, b: a.le(b))
    def eq(self, o): return self._compare(o, Primitive.EQ, lambda a, b: a.eq(b))
    def ne(self, o): return self._compare(o, Primitive.NE, lambda a, b: a.ne(b))

    def dot(self, other):
        if self.dtype() != other.dtype():
            target = DType.promote(self.dtype(), other.dtype())
            left = self if self.dtype() == target else self.astype(target)
            right = other if other.dtype() == target else other.astype(target)
            return left.dot(right)
        out = Shape(self.shape()[0], other.shape()[1])
        return self._apply(Primitive.DOT, [self, other], out)

    def exp(self): return self._apply(Primitive.EXP, [self], self.shape())
    def log(self): return self._apply(Primitive.LOG, [self], self.shape())
    def sin(self): return self._apply(Primitive.SIN, [self], self.shape())
    def cos(self): return self._apply(Primitive.COS, [self], self.shape())
    def tanh(self): return self._apply(Primitive.TANH, [self], self.shape())
    def relu(self): return self._apply(Primitive.RELU, [self], self.shape())
    def sigmoid(self): return self._apply(Primitive.SIGMOID, [self], self.shape())

    def sum(self, axis: Optional[int] = None, keepDims: bool = False):
        if axis is None:
            return self._apply(Primitive.SUM, [self], Shape(1))
        norm = self.shape().normalizeAxis(axis)
        return self._apply(Primitive.SUM_AXIS, [self], self.shape().reduceAxis(norm, keepDims),
                           meta=AxisMeta(norm, keepDims))

    def mean(self, axis: Optional[int] = None, keepDims: bool = False):
        if axis is None:
            return self._apply(Primitive.MEAN, [self], Shape(1))
        norm = self.shape().normalizeAxis(axis)
        return self._apply(Primitive.MEAN_AXIS, [self], self.shape().reduceAxis(norm, keepDims),
                           meta=AxisMeta(norm, keepDims))

    def argmax(self, axis: int):
        norm = self.shape().normalizeAxis(axis)
        return self._apply(Primitive.ARGMAX, [self], self.shape().reduceAxis(norm, False), DType.INT32,
                           AxisMeta(norm, False))

    def argmin(self, axis: int):
        norm = self.shape().normalizeAxis(axis)
        return self._apply(Primitive.ARGMIN, [self], self.shape().reduceAxis(norm, False), DType.INT32,
                           AxisMeta(norm, False))

    def astype(self, target: DType):
        return self._apply(Primitive.CAST, [self], self.shape(), target, target)

    def _no_data(self, *a, **k):
        raise UnsupportedOperationException(
            "Cannot get data from a traced array. You must JIT compile it first.")

    toFloatArray = toIntArray = toBoolArray = toDoubleArray = toLongArray = numpy = _no_data

    def __repr__(self):
        return f"Traced({self._var!r}, {self.dtype()})"
