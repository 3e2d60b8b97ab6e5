"""Deferred elementwise cotangents for the backward pass.

The VJP rules (Grad.computeVJPs, api/Grad.java:341-472) are chains of small
elementwise operations -- the softmax cross-entropy backward alone is a dozen
passes over [batch, classes], each a kernel launch that reads and writes the
whole array.  With fusion on, the grad interpreter builds these operations as
a DAG of `Deferred` values over concrete arrays instead; the first consumer
that needs memory (a DOT, a sum down to a shape other than a row sum, a
collective, a recorded gradient) evaluates the DAG through the planner and
generated kernels a traced forward uses (`fusion.plan`): one kernel per
shape, with sums over the last axis as reduction tails.  Plans, and with
them the compiled kernels, are cached by the DAG's structure, so a training
loop compiles each distinct backward once.

Every operation is the same IEEE operation the eager kernels perform, in the
same order per element; only sums over the last axis are added in the
generated kernel's order instead of the eager reduction's.
"""
from __future__ import annotations

import itertools
import os
from typing import Dict, List, Optional, Tuple

from .core import ConcreteNDArray, DType, NDArray, Primitive as P, Shape
from .tracing import AxisMeta, Equation, Jaxpr, Var

ENABLED = os.environ.get("J4C_LAZY_BACKWARD", "1") != "0"
FLOAT_TYPES = (DType.FLOAT32, DType.FLOAT64)
_ids = itertools.count(1 << 40)  # synthetic var ids, apart from the tracer's
_PLANS: Dict[tuple, Tuple[Jaxpr, object]] = {}
_MAX_PLANS = 512


class Deferred(NDArray):
    """A value not yet computed: `prim` applied to `args` (Deferred or
    concrete), broadcast to `shp`.  CAST with the same dtype is a broadcast
    copy; SUM_AXIS (AxisMeta on the last axis) is a row sum."""

    __slots__ = ("prim", "args", "shp", "dt", "dev", "meta", "value")

    def __init__(self, prim: P, args: list, shape: Shape, dtype: DType, device, meta=None):
        self.prim, self.args, self.shp, self.dt, self.dev, self.meta = prim, args, shape, dtype, device, meta
        self.value: Optional[ConcreteNDArray] = None

    def shape(self) -> Shape:
        return self.shp

    def dtype(self) -> DType:
        return self.dt

    def device(self):
        return self.dev

    def add(self, other):  # gradient accumulation (Grad.java:157, 180)
        return binary(self, other, P.ADD)

    def __repr__(self):
        return f"Deferred({self.prim.name}, {self.shp}, {self.dt})"


def _kind(x: NDArray, shape: Shape) -> Optional[int]:
    from .fusion import bcast_kind
    return bcast_kind(x.shape(), shape)


def _fusible(*xs) -> bool:
    dt = xs[0].dtype()
    return ENABLED and dt in FLOAT_TYPES and all(x.dtype() == dt for x in xs) and \
        all(isinstance(x, (Deferred, ConcreteNDArray)) for x in xs)


def binary(a: NDArray, b: NDArray, prim: P) -> Optional[Deferred]:
    """a `prim` b as a deferred value, or None when the pair does not fit a
    generated kernel (the caller then computes it eagerly)."""
    if not _fusible(a, b):
        return None
    try:
        out = Shape.broadcast(a.shape(), b.shape())
    except Exception:  # noqa: BLE001 - shape errors are reported by the eager path
        return None
    if out.rank() < 1 or _kind(a, out) is None or _kind(b, out) is None:
        return None
    return Deferred(prim, [a, b], out, a.dtype(), a.device())


def expand(x: NDArray, shape: Shape) -> Optional[Deferred]:
    """x broadcast to `shape` (a scalar, a row vector or a [rows, 1] column)."""
    if not _fusible(x) or shape.rank() < 1 or _kind(x, shape) is None:
        return None
    return Deferred(P.CAST, [x], shape, x.dtype(), x.device(), x.dtype())


def row_sum(x: NDArray, target: Shape) -> Optional[Deferred]:
    """x [..., n] summed over its last axis to `target` ([..., 1] or [...])."""
    if not _fusible(x):
        return None
    d = x.shape().dimensions()
    if len(d) < 2:
        return None
    keep = target.dimensions() == d[:-1] + (1,)
    if not keep and target.dimensions() != d[:-1]:
        return None
    return Deferred(P.SUM_AXIS, [x], target, x.dtype(), x.device(), AxisMeta(len(d) - 1, keep))


def materialize(x):
    """The concrete value of x (evaluating its DAG once; x itself if concrete)."""
    if not isinstance(x, Deferred):
        return x
    if x.value is not None:
        return x.value
    leaves: List[ConcreteNDArray] = []
    leaf_index: Dict[int, int] = {}
    nodes: List[tuple] = []          # (Deferred, refs) in evaluation order
    node_index: Dict[int, int] = {}

    def ref(n) -> tuple:
        if isinstance(n, Deferred) and n.value is not None:
            n = n.value
        if isinstance(n, Deferred):
            return ("eq", node_index[id(n)])
        k = id(n)
        if k not in leaf_index:
            leaf_index[k] = len(leaves)
            leaves.append(n)
        return ("in", leaf_index[k])

    # post-order walk without recursion (chains can be long)
    stack = [(x, False)]
    while stack:
        n, expanded = stack.pop()
        if id(n) in node_index:
            continue
        if expanded:
            node_index[id(n)] = len(nodes)
            nodes.append((n, [ref(a) for a in n.args]))
            continue
        stack.append((n, True))
        for a in reversed(n.args):
            if isinstance(a, Deferred) and a.value is None and id(a) not in node_index:
                stack.append((a, False))
    sig = (tuple((l.shape(), l.dtype()) for l in leaves),
           tuple((n.prim, tuple(refs), n.shp, n.dt, n.meta) for n, refs in nodes))
    cached = _PLANS.get(sig)
    if cached is None:
        cached = _build(leaves, nodes)
        if len(_PLANS) >= _MAX_PLANS:
            _PLANS.pop(next(iter(_PLANS)))
        _PLANS[sig] = cached
    jaxpr, plan = cached
    values: Dict[int, NDArray] = {v.id: leaf for v, leaf in zip(jaxpr.inVars, leaves)}
    from . import fusion
    from .grad import _run_equation
    for kind, item in plan.steps:
        if kind == "group":
            fusion.run_group(item, values)
        else:
            _run_equation(item, values)
    x.value = values[jaxpr.outVars[0].id]
    x.args = []  # the DAG below is no longer needed
    return x.value


def _build(leaves, nodes) -> Tuple[Jaxpr, object]:
    """A Jaxpr of the DAG (leaves as inputs, the last node as output) and its plan."""
    from . import fusion
    in_vars = [Var(next(_ids), l.shape(), l.dtype()) for l in leaves]
    out_vars: List[Var] = []
    eqs: List[Equation] = []
    for n, refs in nodes:
        ins = [in_vars[i] if k == "in" else out_vars[i] for k, i in refs]
        o = Var(next(_ids), n.shp, n.dt)
        out_vars.append(o)
        eqs.append(Equation(ins, [o], n.prim, n.meta))
    jaxpr = Jaxpr(in_vars, [out_vars[-1]], eqs)
    return jaxpr, fusion.plan(jaxpr, False)


def cached_plans() -> int:
    return len(_PLANS)
