"""JAX.vmap: automatic batching (api/Vmap.java).

`fn` is traced once against per-example placeholders; the Jaxpr is then
replayed on the batched arguments, each equation through its batching rule
(Vmap.applyBatchingRule, Vmap.java:176-245).  Elementwise, comparison and cast
equations need no rule: a batched [B, ...] operand broadcasts against an
unbatched one through the ordinary kernels.  Reductions shift their axis past
the batch axis, a whole-array SUM/MEAN of a batched value becomes one
reduction per example, DOT multiplies per example, and a PMAP with a batched
input runs once per example.  As in the reference: in_axes 0 (or -1 for an
unbatched argument; axis 1 of a 2-D argument is moved to the front), the
batch axis leads the output (out_axis 1 moves it back for 2-D outputs), and
eager execution -- vmap does not compose with further tracing.

Device mapping: a DOT with only its left operand batched is one GEMM over
[B*M, K]; other batched FLOAT32 DOTs are one strided-batched GEMM launch
(j4c_dot_split_batched); per-example SUM/MEAN is one row reduction over
[B, rest].
"""
from __future__ import annotations

from typing import Callable, Dict, List, Sequence

from . import pmap as _pm
from ._lib import call
from .core import (ConcreteNDArray, DType, IllegalArgumentException, NDArray, Primitive as P, Shape,
                   UnsupportedOperationException)
from .grad import broadcast_like, make_jaxpr


class _Spec:
    """Shape and dtype of a per-example placeholder."""

    def __init__(self, shape: Shape, dtype: DType):
        self._s, self._d = shape, dtype

    def shape(self) -> Shape:
        return self._s

    def dtype(self) -> DType:
        return self._d


def move_axis_to_front(a: NDArray, axis: int) -> NDArray:
    """Vmap.moveAxisToFront (Vmap.java:150-164): axis 0 of any rank, or axis 1
    of a 2-D array (a transpose)."""
    if axis == 0:
        return a
    d = a.shape().dimensions()
    if len(d) == 2 and axis == 1:
        import torch
        rows, cols = d
        out = torch.empty(rows * cols, dtype=a.dtype().torch, device=a.tensor().device)
        call("j4c_transpose", a.dtype().ordinal, a.data_ptr(), rows, cols, out.data_ptr(), a._stream())
        return ConcreteNDArray._wrap(out, Shape(cols, rows), a.dtype(), a.device())
    raise UnsupportedOperationException(
        f"moveAxisToFront: only axis=0 (any rank) or axis=1 on 2-D arrays is supported; got axis={axis} "
        f"rank={len(d)}")


def _leading(x: ConcreteNDArray, b: int) -> ConcreteNDArray:
    """Example b of a batched array (a view)."""
    d = x.shape().dimensions()
    per = Shape(d[1:])
    n = per.size()
    return ConcreteNDArray._wrap(x.tensor()[b * n:(b + 1) * n], per, x.dtype(), x.device())


def batched_reduce(x: ConcreteNDArray, batch: int, mean: bool) -> ConcreteNDArray:
    """Vmap.batchedReduce (Vmap.java:252-262): one sum (mean) per example."""
    rows = x.reshape(Shape(batch, x.shape().size() // batch))
    return rows.mean(1) if mean else rows.sum(1)


def batched_dot(a: ConcreteNDArray, a_batched: bool, b: ConcreteNDArray, b_batched: bool,
                batch: int) -> ConcreteNDArray:
    """Vmap.batchedDot (Vmap.java:269-297): per-example [M,K] . [K,N]."""
    if not a_batched and not b_batched:
        return a.dot(b)
    ad = a.shape().dimensions()[1:] if a_batched else a.shape().dimensions()
    bd = b.shape().dimensions()[1:] if b_batched else b.shape().dimensions()
    if len(ad) != 2 or len(bd) != 2:
        raise IllegalArgumentException(f"vmap dot needs 2-D examples, got {Shape(ad)} . {Shape(bd)}")
    M, K = ad
    N = bd[1]
    if a_batched and not b_batched:
        # every example shares B: one product over the stacked rows
        return a.reshape(Shape(batch * M, K)).dot(b).reshape(Shape(batch, M, N))
    if a.dtype() == b.dtype() == DType.FLOAT32 and M and K and N:
        return _strided_batched_dot(a, a_batched, b, b_batched, batch, M, K, N)
    outs = [(_leading(a, i) if a_batched else a).dot(_leading(b, i) if b_batched else b) for i in range(batch)]
    return _pm.stack(outs).reshape(Shape(batch, M, N))


def _strided_batched_dot(a, a_batched, b, b_batched, batch, M, K, N) -> ConcreteNDArray:
    """One launch of the strided-batched tcgen05 GEMM (j4c_dot_split_batched):
    each operand is split once as its [entries * rows, cols] storage."""
    import torch
    from .core import _split_of
    dev = a._check_devices(b)
    a2 = a.reshape(Shape(batch * M, K)) if a_batched else a
    b2 = b.reshape(Shape(batch * K, N)) if b_batched else b
    ah, al = _split_of(a2, "r")  # read K-major: one line per row (per entry)
    bh, bl = _split_of(b2, "c")  # read MN-major: one line per column, shared by the entries
    out = torch.empty(batch * M * N, dtype=torch.float32, device=a.tensor().device)
    call("j4c_dot_split_batched", ah.data_ptr(), al.data_ptr(), bh.data_ptr(), bl.data_ptr(), out.data_ptr(),
         batch, M, K, N, 0, 0, int(a_batched), int(b_batched), a._stream())
    return ConcreteNDArray._wrap(out, Shape(batch, M, N), DType.FLOAT32, dev)


def broadcast_to_batch(x: NDArray, batch: int) -> ConcreteNDArray:
    """Vmap.broadcastToBatch (Vmap.java:299-309)."""
    return broadcast_like(x, Shape((batch,) + x.shape().dimensions()))


def _rule(eq, inputs: List[NDArray], batched: List[bool], batch: int) -> NDArray:
    """Vmap.applyBatchingRule (Vmap.java:176-245)."""
    p = eq.primitive
    m = eq.metadata
    if p == P.ADD: return inputs[0].add(inputs[1])
    if p == P.SUB: return inputs[0].sub(inputs[1])
    if p == P.MUL: return inputs[0].mul(inputs[1])
    if p == P.DIV: return inputs[0].div(inputs[1])
    if p == P.EXP: return inputs[0].exp()
    if p == P.LOG: return inputs[0].log()
    if p == P.SIN: return inputs[0].sin()
    if p == P.COS: return inputs[0].cos()
    if p == P.TANH: return inputs[0].tanh()
    if p == P.RELU: return inputs[0].relu()
    if p == P.SIGMOID: return inputs[0].sigmoid()
    if p == P.SUM: return batched_reduce(inputs[0], batch, False) if batched[0] else inputs[0].sum()
    if p == P.MEAN: return batched_reduce(inputs[0], batch, True) if batched[0] else inputs[0].mean()
    if p in (P.SUM_AXIS, P.MEAN_AXIS):
        axis = m.axis + 1 if batched[0] else m.axis  # the batch axis was inserted at 0
        return inputs[0].sum(axis, m.keepDims) if p == P.SUM_AXIS else inputs[0].mean(axis, m.keepDims)
    if p == P.DOT: return batched_dot(inputs[0], batched[0], inputs[1], batched[1], batch)
    if p == P.GT: return inputs[0].gt(inputs[1])
    if p == P.GE: return inputs[0].ge(inputs[1])
    if p == P.LT: return inputs[0].lt(inputs[1])
    if p == P.LE: return inputs[0].le(inputs[1])
    if p == P.EQ: return inputs[0].eq(inputs[1])
    if p == P.NE: return inputs[0].ne(inputs[1])
    if p == P.MAX: return inputs[0].max(inputs[1])
    if p == P.MIN: return inputs[0].min(inputs[1])
    if p in (P.ARGMAX, P.ARGMIN):
        axis = m.axis + 1 if batched[0] else m.axis
        return inputs[0].argmax(axis) if p == P.ARGMAX else inputs[0].argmin(axis)
    if p == P.CAST: return inputs[0].astype(m)
    if p == P.GATHER:
        # batched indices already carry the batch axis in their shape
        from .grad import take_eager
        return take_eager(inputs[0], inputs[1])
    if p == P.CHECKPOINT:
        # the rematerialisation hint is a no-op under vmap: batch the body inline
        return run(m.subJaxpr, [inputs[0]], [batched[0]], batch)
    if p == P.PMAP:
        if not batched[0]:
            return _pm.run_forward_jaxpr(m.bodyJaxpr, m.devices, [_pm.split(x, m.numDevices()) for x in inputs])
        # one pmap per example; collectives stay scoped to the D shards of that example
        outs = []
        for i in range(batch):
            ex = [_leading(x, i) if bt else x for x, bt in zip(inputs, batched)]
            outs.append(_pm.run_forward_jaxpr(m.bodyJaxpr, m.devices, [_pm.split(x, m.numDevices()) for x in ex]))
        return _pm.stack(outs)
    raise UnsupportedOperationException(f"vmap has no batching rule for primitive: {p.name}")


def run(jaxpr, args: Sequence[NDArray], is_batched: Sequence[bool], batch: int) -> NDArray:
    """Vmap.runMulti (Vmap.java:113-144)."""
    values: Dict[int, NDArray] = dict(jaxpr.consts)  # closed-over constants are never batched
    batched = set()
    for v, a, bt in zip(jaxpr.inVars, args, is_batched):
        values[v.id] = a
        if bt:
            batched.add(v.id)
    for eq in jaxpr.equations:
        inputs = [values[v.id] for v in eq.inputs]
        flags = [v.id in batched for v in eq.inputs]
        values[eq.outputs[0].id] = _rule(eq, inputs, flags, batch)
        if any(flags):
            batched.add(eq.outputs[0].id)
    out_var = jaxpr.outVars[0]
    out = values[out_var.id]
    if out_var.id not in batched:
        out = broadcast_to_batch(out, batch)
    return out


def vmap(fn: Callable, in_axes: Sequence[int] = None, out_axis: int = 0) -> Callable:
    """Vmap.vmap (Vmap.java:41-100) for one or two arguments."""

    def mapped(*args: NDArray) -> NDArray:
        if not 1 <= len(args) <= 2:
            raise IllegalArgumentException("vmap maps functions of one or two arrays")
        axes = list(in_axes) if in_axes is not None else [0] * len(args)
        if len(axes) != len(args):
            raise IllegalArgumentException("vmap: in_axes needs one entry per argument")
        norm = [move_axis_to_front(a, ax) if ax > 0 else a for a, ax in zip(args, axes)]
        flags = [ax >= 0 for ax in axes]
        if not any(flags):
            raise IllegalArgumentException("vmap: at least one argument must be batched")
        for a, bt in zip(norm, flags):
            if bt and a.shape().rank() == 0:
                raise IllegalArgumentException("vmap requires at least a 1-D array with a leading batch dimension")
        batch = next(a.shape().dimensions()[0] for a, bt in zip(norm, flags) if bt)
        specs = [_Spec(Shape(a.shape().dimensions()[1:]) if bt else a.shape(), a.dtype())
                 for a, bt in zip(norm, flags)]
        jaxpr = make_jaxpr(fn, *specs)
        out = run(jaxpr, norm, flags, batch)
        return move_axis_to_front(out, out_axis) if out_axis > 0 else out

    return mapped
