"""Public transform and library API: JAX, Lax, Nn, Numpy, Random.

Same entry points, argument meaning and error behaviour as the reference's
api/JAX.java, api/Lax.java, api/Nn.java, api/Numpy.java and api/Random.java
(paths relative to src/main/java/com/marmanis/jax4j/).  Python methods keep
the Java names; where Java overloads on arity, the Python function accepts
the extra argument (pmap of several sharded inputs, grad with argnum).
"""
from __future__ import annotations

import ctypes as C
import decimal
import enum
import math
import os
from typing import Callable, List, Optional, Sequence

import numpy as np
import torch

from . import grad as _grad
from . import pmap as _pm
from ._lib import call, dims as _dims
from .core import (ConcreteNDArray, Device, DType, IllegalArgumentException, NDArray, PRNGKey,
                   Primitive, Shape, stream_of)
from .pytree import PyTree, PyTrees
from .tracing import (CheckpointMeta, CondMeta, Equation, PmapMeta, ScanMeta, Tracer, TracedNDArray, WhileMeta,
                      to_var)


# ---------------------------------------------------------------------------
# JAX (api/JAX.java)
# ---------------------------------------------------------------------------
class JAX:
    @staticmethod
    def make_jaxpr(fn: Callable, *args: NDArray):
        """JAX.make_jaxpr (JAX.java:30-55)."""
        return _grad.make_jaxpr(fn, *args)

    @staticmethod
    def jvp(fn: Callable, arg: NDArray, tangent: NDArray) -> List[NDArray]:
        """JAX.jvp (JAX.java:62-66): forward mode; returns [primal out, tangent out]."""
        jaxpr = _grad.make_jaxpr(fn, arg)
        primals, tangents = _grad.forward_ad(jaxpr, [arg], [tangent])
        return [primals[0], tangents[0]]

    @staticmethod
    def grad(fn: Callable, argnum: int = None) -> Callable:
        """JAX.grad (JAX.java:279-289)."""
        return _grad.grad(fn, argnum)

    @staticmethod
    def gradBoth(fn: Callable) -> Callable:
        return _grad.grad_both(fn)

    @staticmethod
    def gradTree(fn: Callable) -> Callable:
        """JAX.gradTree (JAX.java:303-305)."""
        return _grad.grad_tree(fn)

    @staticmethod
    def value_and_grad(fn: Callable) -> Callable:
        """JAX.value_and_grad (JAX.java:243-245)."""
        return _grad.value_and_grad(fn)

    @staticmethod
    def valueAndGradTree(fn: Callable) -> Callable:
        """value_and_grad over a PyTree of parameters (one forward + backward)."""
        return _grad.value_and_grad_tree(fn)

    @staticmethod
    def jit(fn: Callable) -> Callable:
        """JAX.jit (JAX.java:92-125): traced once per input signature, then the
        cached Jaxpr is executed -- its elementwise chains as fused generated
        kernels (jax4j_b200/fusion.py) -- and transparent inside another
        trace.  A function may return a tuple of arrays."""
        cache = {}

        def jitted(*args):
            if Tracer.current() is not None:
                return fn(*args)
            key = tuple((a.shape(), a.dtype()) for a in args)
            jaxpr = cache.get(key)
            if jaxpr is None:
                jaxpr = _grad.make_jaxpr(fn, *args)
                cache[key] = jaxpr
            outs = _grad.forward_interpret(jaxpr, list(args))
            return tuple(outs) if jaxpr.__dict__.get("_tuple_out") else outs[0]

        jitted.cache = cache
        return jitted

    @staticmethod
    def jitGrad(fn: Callable) -> Callable:
        """JAX.jitGrad (JAX.java:137-151)."""
        cache = {}

        def g(arg):
            if Tracer.current() is not None:
                return _grad.grad(fn)(arg)
            key = (arg.shape(), arg.dtype())
            jaxpr = cache.get(key)
            if jaxpr is None:
                jaxpr = _grad.make_jaxpr(fn, arg)
                cache[key] = jaxpr
            return _grad._backward(jaxpr, [arg])[0]

        g.cache = cache
        return g

    @staticmethod
    def jitGradTree(fn: Callable) -> Callable:
        """JAX.jitGradTree (JAX.java:168-183)."""
        cache = {}

        def g(tree):
            if Tracer.current() is not None:
                return _grad.grad_tree(fn)(tree)
            leaves = PyTrees.flatten(tree)
            key = tuple((l.shape(), l.dtype()) for l in leaves)
            jaxpr = cache.get(key)
            if jaxpr is None:
                jaxpr = _grad._trace_tree(fn, tree, leaves)
                cache[key] = jaxpr
            return PyTrees.unflatten(tree, _grad._backward(jaxpr, leaves))

        g.cache = cache
        return g

    @staticmethod
    def vmap(fn: Callable, in_axes: Sequence[int] = None, out_axis: int = 0) -> Callable:
        """JAX.vmap (JAX.java:311-337, api/Vmap.java): batches fn over the
        leading axis of its one or two arguments.  in_axes[i] = -1 leaves
        argument i unbatched; axis 1 of a 2-D argument (and out_axis 1 of a
        2-D result) is moved by a transpose."""
        from .vmap import vmap as _vmap
        return _vmap(fn, in_axes, out_axis)

    @staticmethod
    def checkpoint(fn: Callable) -> Callable:
        """JAX.checkpoint (JAX.java:258-274): a CHECKPOINT equation under a trace."""
        def c(arg):
            if Tracer.current() is not None:
                sub = _trace_body(fn, [(arg.shape(), arg.dtype())])
                tracer = Tracer.current()
                in_var = to_var(arg)
                ov = sub.outVars[0]
                out = tracer.nextVar(ov.shape, ov.dtype)
                tracer.addEquation(Equation([in_var], [out], Primitive.CHECKPOINT, CheckpointMeta(sub)))
                return TracedNDArray(out)
            return fn(arg)
        return c

    @staticmethod
    def pmap(fn: Callable, devices: Sequence[Device]) -> Callable:
        """JAX.pmap (JAX.java:356-377): every argument is sharded along axis 0
        (its leading dim must equal len(devices)); results are stacked to
        [D, *out].  Under a trace a PMAP equation is emitted so grad composes
        with the collectives in the body."""
        devices = tuple(devices)
        D = len(devices)

        def mapped(*inputs: NDArray):
            if not inputs:
                raise IllegalArgumentException("pmap needs at least one input")
            if Tracer.current() is not None:
                specs = []
                for x in inputs:
                    d = x.shape().dimensions()
                    if not d or d[0] != D:
                        raise IllegalArgumentException(
                            f"pmap: input leading dim {d[0] if d else 0} must equal numDevices {D}")
                    specs.append((Shape(d[1:]), x.dtype()))
                body = _trace_body(fn, specs)
                tracer = Tracer.current()
                in_vars = [to_var(x) for x in inputs]
                ov = body.outVars[0]
                out = tracer.nextVar(Shape((D,) + ov.shape.dimensions()), ov.dtype)
                tracer.addEquation(Equation(in_vars, [out], Primitive.PMAP, PmapMeta(body, devices)))
                return TracedNDArray(out)
            return _pm.run_forward(fn, inputs, devices)

        return mapped


class ScanResult:
    """Lax.ScanResult (Lax.java:127): the final carry and the stacked ys
    (record accessors carry() and ys(); also unpacks as (carry, ys))."""

    def __init__(self, carry: NDArray, ys: NDArray):
        self._carry, self._ys = carry, ys

    def carry(self) -> NDArray:
        return self._carry

    def ys(self) -> NDArray:
        return self._ys

    def __iter__(self):
        return iter((self._carry, self._ys))


def _trace_step(step_fn: Callable, carry_shape, carry_dtype, x_shape, x_dtype):
    """Lax.traceStep (Lax.java:219-233)."""
    Tracer.start()
    try:
        t = Tracer.current()
        cv = t.nextVar(carry_shape, carry_dtype)
        xv = t.nextVar(x_shape, x_dtype)
        outs = step_fn(TracedNDArray(cv), TracedNDArray(xv))
        return Tracer.stop([cv, xv], [to_var(outs[0]), to_var(outs[1])])
    except BaseException:
        Tracer.abort()
        raise


def _trace_body(fn: Callable, specs) -> "Jaxpr":
    """JAX.traceBody (JAX.java:379-391) for any number of inputs."""
    Tracer.start()
    try:
        t = Tracer.current()
        in_vars = [t.nextVar(s, d) for s, d in specs]
        result = fn(*[TracedNDArray(v) for v in in_vars])
        if not isinstance(result, TracedNDArray):
            result = TracedNDArray(t.nextConstant(result))
        return Tracer.stop(in_vars, [result.getVar()])
    except BaseException:
        Tracer.abort()
        raise


# ---------------------------------------------------------------------------
# Lax collectives (api/Lax.java:166-217)
# ---------------------------------------------------------------------------
class Lax:
    @staticmethod
    def psum(x: NDArray) -> NDArray:
        """Lax.psum (Lax.java:176-187): PSUM equation under a trace, all-reduce
        sum inside pmap, identity outside."""
        if Tracer.current() is not None:
            tracer = Tracer.current()
            v = to_var(x)
            out = tracer.nextVar(x.shape(), x.dtype())
            tracer.addEquation(Equation([v], [out], Primitive.PSUM, None))
            return TracedNDArray(out)
        return _pm.psum_value(x)

    @staticmethod
    def allGather(x: NDArray, numDevices: int) -> NDArray:
        """Lax.allGather (Lax.java:202-217)."""
        if Tracer.current() is not None:
            tracer = Tracer.current()
            v = to_var(x)
            out = tracer.nextVar(Shape((numDevices,) + x.shape().dimensions()), x.dtype())
            tracer.addEquation(Equation([v], [out], Primitive.ALL_GATHER, numDevices))
            return TracedNDArray(out)
        return _pm.all_gather_value(x)

    # ---- control flow (Lax.java:69-217) ----
    @staticmethod
    def cond(pred: NDArray, trueFn: Callable, falseFn: Callable, operand: NDArray) -> NDArray:
        """Lax.cond (Lax.java:72-88): eager -> the taken branch; traced -> one
        COND equation holding both branches (its VJP flows through the taken
        branch, pred gets zero)."""
        if Tracer.current() is None:
            return trueFn(operand) if _grad.is_true(pred) else falseFn(operand)
        t_br = _grad.make_jaxpr(trueFn, operand)
        f_br = _grad.make_jaxpr(falseFn, operand)
        tracer = Tracer.current()
        pv, ov = to_var(pred), to_var(operand)
        out = tracer.nextVar(t_br.outVars[0].shape, operand.dtype())
        tracer.addEquation(Equation([pv, ov], [out], Primitive.COND, CondMeta(t_br, f_br)))
        return TracedNDArray(out)

    @staticmethod
    def whileLoop(condFn: Callable, bodyFn: Callable, init: NDArray) -> NDArray:
        """Lax.whileLoop (Lax.java:92-110): not reverse-mode differentiable."""
        if Tracer.current() is None:
            state = init
            while _grad.is_true(condFn(state)):
                state = bodyFn(state)
            return state
        c = _grad.make_jaxpr(condFn, init)
        b = _grad.make_jaxpr(bodyFn, init)
        tracer = Tracer.current()
        iv = to_var(init)
        out = tracer.nextVar(b.outVars[0].shape, init.dtype())
        tracer.addEquation(Equation([iv], [out], Primitive.WHILE, WhileMeta(c, b)))
        return TracedNDArray(out)

    @staticmethod
    def foriLoop(lower: int, upper: int, bodyFn: Callable, init: NDArray) -> NDArray:
        """Lax.foriLoop (Lax.java:119-125): a host loop; under a trace each call
        appends its equations, so it is differentiable with no new primitive."""
        state = init
        for i in range(lower, upper):
            state = bodyFn(i, state)
        return state

    @staticmethod
    def scan(stepFn: Callable, initCarry: NDArray, xs: NDArray) -> "ScanResult":
        """Lax.scan (Lax.java:135-163): stepFn(carry, x_t) -> [new carry, y_t]
        for each leading slice of xs; returns (final carry, stacked ys)."""
        d = xs.shape().dimensions()
        steps = d[0]
        x_step = Shape(d[1:])
        if Tracer.current() is None:
            carry, ys = initCarry, []
            for t in range(steps):
                carry, y = stepFn(carry, _grad.slice_leading(xs, t))
                ys.append(y)
            return ScanResult(carry, _grad.stack_leading(ys))
        step = _trace_step(stepFn, initCarry.shape(), initCarry.dtype(), x_step, xs.dtype())
        tracer = Tracer.current()
        cv, xv = to_var(initCarry), to_var(xs)
        y_shape = step.outVars[1].shape
        c_out = tracer.nextVar(step.outVars[0].shape, initCarry.dtype())
        ys_out = tracer.nextVar(Shape((steps,) + y_shape.dimensions()), xs.dtype())
        tracer.addEquation(Equation([cv, xv], [c_out, ys_out], Primitive.SCAN, ScanMeta(step)))
        return ScanResult(TracedNDArray(c_out), TracedNDArray(ys_out))

    @staticmethod
    def setAllGatherVjp(mode: str) -> None:
        """'slice' (default, the reference's ALL_GATHER VJP: the local slice of
        the cotangent) or 'reduce_scatter' (the transpose of all-gather: the
        cotangents' slices for this shard summed over shards)."""
        _pm.set_all_gather_vjp(mode)

    @staticmethod
    def psumTree(tree: PyTree) -> PyTree:
        """PyTrees.map(Lax::psum, tree) with few collectives: over NCCL the
        leaves go in buckets of ~J4C_PSUM_BUCKET_MB, each all-reduced on a side
        stream as soon as the backward pass has produced its gradients
        (overlapping communication with the rest of the backward); shards
        sharing a GPU pack every leaf into one slot sum.  Each element's sum is
        the same as a leaf-by-leaf psum."""
        ctx = _pm.PmapContext.current()
        leaves = PyTrees.flatten(tree)
        if ctx is None or Tracer.current() is not None or not leaves:
            return PyTrees.map(Lax.psum, tree)
        if ctx.numDevices == 1:
            return tree  # the sum over one shard is the shard (arrays are immutable)
        first = leaves[0]
        if any(l.dtype() != first.dtype() or l.tensor().device != first.tensor().device for l in leaves):
            return PyTrees.map(Lax.psum, tree)
        _pm.verify_signature(ctx, "psumTree", first.dtype(), [l.shape().size() for l in leaves])
        if isinstance(ctx.collective, _pm.NcclCollective) and PSUM_BUCKET_BYTES > 0:
            return PyTrees.unflatten(tree, _psum_overlapped(ctx, leaves))
        total = sum(l.shape().size() for l in leaves)
        flat = torch.empty(total, dtype=first.dtype().torch, device=first.tensor().device)
        s = first._stream()
        off = 0
        es = first.dtype().byteSize()
        for l in leaves:
            n = l.shape().size()
            call("j4c_memcpy_d2d", flat.data_ptr() + off * es, l.data_ptr(), n * es, s)
            off += n
        packed = ConcreteNDArray._wrap(flat, Shape(total), first.dtype(), first.device())
        summed = ctx.collective.psum(ctx.deviceIndex, packed)
        out, off = [], 0
        for l in leaves:
            n = l.shape().size()
            out.append(ConcreteNDArray._wrap(summed.tensor()[off:off + n], l.shape(), l.dtype(),
                                             summed.device()))
            off += n
        return PyTrees.unflatten(tree, out)


    @staticmethod
    def psumSgdTree(params: PyTree, grads: PyTree, scale: float, lr: float) -> PyTree:
        """The SGD update of a data-parallel step with its gradient all-reduce:
        every leaf w of `params` becomes w - ((psum(g) * scale) * lr) for the
        matching leaf g of `grads` -- the reference's psum of the gradients
        (api/Lax.java:184-186) followed by the elementwise update
        w.sub(g.mul(scale).mul(lr)), e.g. scale = 1/D for the mean gradient.

        With J4C_PSUM_SGD=1, in one-process-per-GPU runs with FLOAT32 leaves,
        the all-reduce and the update are one j4c_psum_sgd call per bucket
        over peer memory, overlapped with the rest of the backward like
        psumTree's buckets; the sum over ranks is taken in rank order, so every
        rank holds the same bits.  Otherwise (the default: NCCL measured as
        fast or faster; one shard; shards sharing a process; other dtypes) it
        is psumTree followed by the elementwise update.  The new parameters
        are fresh arrays."""
        pl, gl = PyTrees.flatten(params), PyTrees.flatten(grads)
        if len(pl) != len(gl):
            raise IllegalArgumentException(f"psumSgdTree: {len(pl)} parameters but {len(gl)} gradients")
        for w, g in zip(pl, gl):
            if w.shape() != g.shape() or w.dtype() != g.dtype():
                raise IllegalArgumentException(f"psumSgdTree: parameter {w.shape()} {w.dtype()} does not match "
                                               f"gradient {g.shape()} {g.dtype()}")
        ctx = _pm.PmapContext.current()
        from . import distributed, psum_sgd
        st = distributed.state()
        if (ctx is not None and ctx.numDevices > 1 and Tracer.current() is None and st is not None
                and ctx.collective is st.collective and isinstance(st.collective, _pm.NcclCollective)
                and all(isinstance(x, ConcreteNDArray) for x in pl + gl)
                and psum_sgd.eligible(pl, gl, st.world_size)):
            _pm.verify_signature(ctx, "psumSgdTree", pl[0].dtype(), [w.shape().size() for w in pl])
            dev = pl[0].tensor().device
            bucket = max(4, PSUM_BUCKET_BYTES // 4) if PSUM_BUCKET_BYTES > 0 else 1 << 62
            return PyTrees.unflatten(params, psum_sgd.fused(ctx, st, pl, gl, float(scale), float(lr),
                                                            _comm_stream(dev), bucket))
        summed = PyTrees.flatten(Lax.psumTree(grads))
        update = _sgd_update(float(scale), float(lr))
        return PyTrees.unflatten(params, [_sgd_leaf(w, g, float(scale), float(lr), update)
                                          for w, g in zip(pl, summed)])


# Gradient all-reduce overlapped with the backward pass.  The backward records
# a CUDA event on each gradient when it is complete; psumTree groups the leaves
# into buckets (last leaves first, the order the backward completes them) and
# all-reduces each bucket on a side stream as soon as its gradients exist, so
# the NCCL traffic of the last layers runs while the first layers' backward is
# still computing.  J4C_PSUM_BUCKET_MB=0 restores the single packed all-reduce.
PSUM_BUCKET_BYTES = int(float(os.environ.get("J4C_PSUM_BUCKET_MB", "32")) * (1 << 20))
_comm_streams = {}


def _comm_stream(device) -> "torch.cuda.Stream":
    s = _comm_streams.get(device)
    if s is None:
        s = _comm_streams[device] = torch.cuda.Stream(device=device)
    return s


_sgd_updates = {}

# Weights at least this large are updated by j4c_sgd_update_lines, which also
# leaves the new weight's line maxima for its next splits (no max pass).
SGD_LINES_MIN = 1 << 16


def _sgd_leaf(w, g, scale: float, lr: float, update):
    """One leaf's w - ((g * scale) * lr): a 2-D FLOAT32 weight on the GPU
    through j4c_sgd_update_lines (the same bits as the elementwise chain, plus
    the result's line maxima kept on it), anything else through `update`."""
    if (isinstance(w, ConcreteNDArray) and isinstance(g, ConcreteNDArray) and Tracer.current() is None
            and w.dtype() == DType.FLOAT32 and g.dtype() == DType.FLOAT32 and w.shape() == g.shape()
            and w.shape().rank() == 2 and w.shape().size() >= SGD_LINES_MIN
            and w.tensor().device.type == "cuda" and g.tensor().device == w.tensor().device):
        rows, cols = w.shape().dimensions()
        t = torch.empty(rows * cols, dtype=torch.float32, device=w.tensor().device)
        lines = torch.empty(rows + cols + 1, dtype=torch.int32, device=t.device)
        wt, gt = w.tensor().contiguous(), g.tensor().contiguous()
        call("j4c_sgd_update_lines", wt.data_ptr(), gt.data_ptr(), rows, cols, C.c_float(scale), C.c_float(lr),
             t.data_ptr(), lines.data_ptr(), w._stream())
        out = ConcreteNDArray._wrap(t, w.shape(), DType.FLOAT32, w.device())
        out._lines = lines
        return out
    return update(w, g)


def _sgd_update(scale: float, lr: float):
    """w - ((g * scale) * lr) as one jitted elementwise chain (cached per
    scale and lr, which become literals of the generated kernel)."""
    f = _sgd_updates.get((scale, lr))
    if f is None:
        s_arr, lr_arr = ConcreteNDArray.scalar(scale), ConcreteNDArray.scalar(lr)
        f = _sgd_updates[(scale, lr)] = JAX.jit(lambda w, g: w.sub(g.mul(s_arr).mul(lr_arr)))
    return f


def _psum_overlapped(ctx, leaves: List[ConcreteNDArray]) -> List[ConcreteNDArray]:
    dev = leaves[0].tensor().device
    dt = leaves[0].dtype()
    es = dt.byteSize()
    compute = torch.cuda.current_stream(dev)
    comm = _comm_stream(dev)
    capturing = torch.cuda.is_current_stream_capturing()
    # buckets of consecutive leaves, walked from the last leaf (ready first)
    buckets, cur, size = [], [], 0
    for i in reversed(range(len(leaves))):
        cur.append(i)
        size += leaves[i].shape().size() * es
        if size >= PSUM_BUCKET_BYTES:
            buckets.append(cur)
            cur, size = [], 0
    if cur:
        buckets.append(cur)
    out: List[Optional[ConcreteNDArray]] = [None] * len(leaves)
    done = []
    entry = torch.cuda.Event()
    entry.record(compute)  # work before psumTree (for leaves without a ready event)
    for b in buckets:
        with torch.cuda.stream(comm):
            for i in b:
                comm.wait_event(leaves[i]._ready if leaves[i]._ready is not None else entry)
            total = sum(leaves[i].shape().size() for i in b)
            buf = torch.empty(total, dtype=dt.torch, device=dev)  # allocated on the side stream
            off = 0
            for i in b:
                n = leaves[i].shape().size()
                call("j4c_memcpy_d2d", buf.data_ptr() + off * es, leaves[i].data_ptr(), n * es, comm.cuda_stream)
                out[i] = ConcreteNDArray._wrap(buf[off:off + n], leaves[i].shape(), dt, _pm._result_device(leaves[i]))
                off += n
            call("j4c_psum", ctx.collective.comms[ctx.deviceIndex], dt.ordinal, buf.data_ptr(), buf.data_ptr(),
                 total, comm.cuda_stream)
            ev = torch.cuda.Event()
            ev.record(comm)
            done.append(ev)
        if not capturing:
            buf.record_stream(compute)  # read on the compute stream after the wait below
    for ev in done:
        compute.wait_event(ev)
    return out


# ---------------------------------------------------------------------------
# Nn / Numpy (api/Nn.java:21-25, api/Numpy.java:39-44)
# ---------------------------------------------------------------------------
class Nn:
    @staticmethod
    def softmax(x: NDArray) -> NDArray:
        """Nn.softmax: exp(x) / sum(exp(x), -1, keepDims) -- no max subtraction,
        as in the reference."""
        e = x.exp()
        return e.div(e.sum(-1, True))


def _dropout(x: NDArray, key: PRNGKey, rate: float, training: bool) -> NDArray:
    """Nn.dropout (Nn.java:42-47): keep with probability 1 - rate, rescale by
    1 / (1 - rate); a pass-through when not training."""
    if not training:
        return x
    p = float(np.float32(1.0) - np.float32(rate))  # 1f - rate in float, as the reference
    keep = Random.bernoulli(key, p, x.shape()).astype(DType.FLOAT32)
    return x.mul(keep).div(ConcreteNDArray.scalar(p))


Nn.dropout = staticmethod(_dropout)


class Numpy:
    @staticmethod
    def take(table: NDArray, indices: NDArray) -> NDArray:
        """Numpy.take (Numpy.java:54-66): embedding lookup, rows of a
        [rows, dim] table -> [*indices.shape, dim]; a GATHER equation under a
        trace (its VJP scatter-adds into the table)."""
        if Tracer.current() is not None:
            tracer = Tracer.current()
            tv, iv = to_var(table), to_var(indices)
            out = tracer.nextVar(Shape(indices.shape().dimensions() + (table.shape().dimensions()[1],)),
                                 table.dtype())
            tracer.addEquation(Equation([tv, iv], [out], Primitive.GATHER, None))
            return TracedNDArray(out)
        return _grad.take_eager(table, indices)

    @staticmethod
    def where(cond: NDArray, x: NDArray, y: NDArray) -> NDArray:
        """Numpy.where: c*x + (1-c)*y with c = cond as FLOAT32 (an arithmetic
        blend, not a select, exactly as the reference computes it)."""
        c = cond.astype(DType.FLOAT32) if cond.dtype() == DType.BOOL else cond
        one = ConcreteNDArray.scalar(1.0, DType.FLOAT32, _dev_of(c))
        inv = one.sub(c)
        return c.mul(x).add(inv.mul(y))


def _dev_of(x: NDArray):
    return x.device() if isinstance(x, ConcreteNDArray) else None


# ---------------------------------------------------------------------------
# Random (api/Random.java): SplitMix64 streams, generated on the device
# ---------------------------------------------------------------------------
_GAMMA = 0x9E3779B97F4A7C15
_SPLIT = 0xD1B54A32D192ED03
_M64 = 0xFFFFFFFFFFFFFFFF


def _mix64(z: int) -> int:
    z &= _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


class Random:
    @staticmethod
    def split(key: PRNGKey, num: int = 2) -> List[PRNGKey]:
        """Random.split (Random.java:70-81)."""
        return [PRNGKey(_mix64(key.state() ^ _SPLIT ^ ((_GAMMA * (i + 1)) & _M64))) for i in range(num)]

    @staticmethod
    def uniform(key: PRNGKey, shape, lo: float = 0.0, hi: float = 1.0, device: Device = None,
                offset: int = 0, count: int = None) -> ConcreteNDArray:
        """Random.uniform (Random.java:86-98).  offset/count select elements
        [offset, offset+count) of the full array (a shard's rows)."""
        shape = shape if isinstance(shape, Shape) else Shape(shape)
        n = shape.size() if count is None else count
        device = device or Device.defaultDevice()
        t = torch.empty(n, dtype=torch.float32, device=device.torch_device())
        call("j4c_random_uniform", key.state(), offset, n, float(np.float32(lo)), float(np.float32(hi)),
             t.data_ptr(), stream_of(device.ordinal()))
        out_shape = shape if count is None else Shape(n)
        return ConcreteNDArray._wrap(t, out_shape, DType.FLOAT32, device)

    @staticmethod
    def normal(key: PRNGKey, shape, device: Device = None, offset: int = 0,
               count: int = None) -> ConcreteNDArray:
        """Random.normal (Random.java:104-113): Box-Muller."""
        shape = shape if isinstance(shape, Shape) else Shape(shape)
        n = shape.size() if count is None else count
        device = device or Device.defaultDevice()
        t = torch.empty(n, dtype=torch.float32, device=device.torch_device())
        call("j4c_random_normal", key.state(), offset, n, t.data_ptr(), stream_of(device.ordinal()))
        out_shape = shape if count is None else Shape(n)
        return ConcreteNDArray._wrap(t, out_shape, DType.FLOAT32, device)

    @staticmethod
    def bernoulli(key: PRNGKey, p: float, shape, device: Device = None) -> ConcreteNDArray:
        """Random.bernoulli (Random.java:116-123): uniform < p."""
        u = Random.uniform(key, shape, 0.0, 1.0, device)
        return u.lt(ConcreteNDArray.scalar(float(np.float32(p)), DType.FLOAT32, u.device()))

    @staticmethod
    def permutation(key: PRNGKey, n: int, device: Device = None) -> ConcreteNDArray:
        """Random.permutation (Random.java:130-140): INT32 permutation of 0..n-1."""
        device = device or Device.defaultDevice()
        t = torch.empty(max(n, 1), dtype=torch.int32, device=device.torch_device())
        call("j4c_random_permutation", key.state(), n, t.data_ptr(), stream_of(device.ordinal()))
        return ConcreteNDArray._wrap(t[:n], Shape(n), DType.INT32, device)

    @staticmethod
    def heNormal(key: PRNGKey, shape, fanIn: int, device: Device = None) -> ConcreteNDArray:
        """Random.heNormal (Random.java:153-157): N(0, 1) * sqrt(2 / fanIn)."""
        std = float(np.float32(math.sqrt(2.0 / fanIn)))
        x = Random.normal(key, shape, device)
        return x.mul(ConcreteNDArray.scalar(std, DType.FLOAT32, x.device()))

    @staticmethod
    def glorotUniform(key: PRNGKey, shape, fanIn: int, fanOut: int, device: Device = None,
                      offset: int = 0, count: int = None) -> ConcreteNDArray:
        """Random.glorotUniform (Random.java:147-150)."""
        limit = float(np.float32(math.sqrt(6.0 / (fanIn + fanOut))))
        return Random.uniform(key, shape, -limit, limit, device, offset, count)


# ---------------------------------------------------------------------------
# Fft (api/Fft.java)
# ---------------------------------------------------------------------------
def _pow2(n: int) -> bool:
    return n >= 1 and (n & (n - 1)) == 0


def _fft_operand(x, who: str) -> ConcreteNDArray:
    if not isinstance(x, ConcreteNDArray):
        raise IllegalArgumentException(f"{who}: a concrete array is required (FFTs are not traced primitives)")
    if x.dtype() not in (DType.FLOAT32, DType.FLOAT64):
        raise IllegalArgumentException(f"{who} requires FLOAT32 or FLOAT64 input, got {x.dtype()}")
    return x


def _fft_pair(re, im, rank: int, who: str):
    re, im = _fft_operand(re, who), _fft_operand(im, who)
    if re.shape().rank() != rank or im.shape().rank() != rank:
        kind = "1-D vectors" if rank == 1 else "3-D inputs"
        raise IllegalArgumentException(f"{who} require {kind}, got shapes {re.shape()}, {im.shape()}")
    if re.shape() != im.shape():
        raise IllegalArgumentException(f"{who} real and imaginary parts must have the same shape: "
                                       f"{re.shape()} vs {im.shape()}")
    if re.dtype() != im.dtype():
        raise IllegalArgumentException(f"{who} real and imaginary parts must share dtype: "
                                       f"{re.dtype()} vs {im.dtype()}")
    re._check_devices(im)
    return re, im


def _fft_new(like: ConcreteNDArray, shape: Shape) -> ConcreteNDArray:
    t = torch.empty(shape.size(), dtype=like.dtype().torch, device=like.tensor().device)
    return ConcreteNDArray._wrap(t, shape, like.dtype(), like.device())


def _fft_complex(re, im, inverse: bool, rank: int) -> List[ConcreteNDArray]:
    who = "fft/ifft" if rank == 1 else "fft3/ifft3"
    re, im = _fft_pair(re, im, rank, who)
    d = re.shape().dimensions()
    if not all(_pow2(n) for n in d):
        what = "length" if rank == 1 else "dimensions"
        raise IllegalArgumentException(f"{who} {what} must be {'a power' if rank == 1 else 'powers'} of two, "
                                       f"got {re.shape()}")
    ore, oim = _fft_new(re, re.shape()), _fft_new(re, re.shape())
    call("j4c_fft", re.dtype().ordinal, rank, _dims(d), re.data_ptr(), im.data_ptr(), ore.data_ptr(),
         oim.data_ptr(), int(inverse), re._stream())
    return [ore, oim]


def _rfft(x, rank: int) -> List[ConcreteNDArray]:
    who = "rfft" if rank == 1 else "rfft3"
    x = _fft_operand(x, who)
    if x.shape().rank() != rank:
        raise IllegalArgumentException(f"{who} requires a {rank}-D input, got shape {x.shape()}")
    d = x.shape().dimensions()
    if not all(_pow2(n) for n in d):
        what = "length must be a power" if rank == 1 else "dimensions must be powers"
        raise IllegalArgumentException(f"{who} {what} of two, got {d[0] if rank == 1 else x.shape()}")
    out_shape = Shape(d[:-1] + (d[-1] // 2 + 1,))
    ore, oim = _fft_new(x, out_shape), _fft_new(x, out_shape)
    call("j4c_rfft", x.dtype().ordinal, rank, _dims(d), x.data_ptr(), ore.data_ptr(), oim.data_ptr(), x._stream())
    return [ore, oim]


def _irfft(re, im, rank: int, n_last: Optional[int] = None) -> ConcreteNDArray:
    who = "irfft" if rank == 1 else "irfft3"
    re, im = _fft_pair(re, im, rank, who)
    d = re.shape().dimensions()
    n = 2 * (d[-1] - 1) if n_last is None else n_last
    if n < 2 or not _pow2(n) or n // 2 + 1 != d[-1]:
        last = "N" if rank == 1 else "N3"
        raise IllegalArgumentException(f"{who} input length implies {last} = {n}, which must be a power of two >= 2")
    if not all(_pow2(k) for k in d[:-1]):
        raise IllegalArgumentException(f"{who} leading dimensions must be powers of two, got {re.shape()}")
    out_shape = Shape(d[:-1] + (n,))
    out = _fft_new(re, out_shape)
    call("j4c_irfft", re.dtype().ordinal, rank, _dims(out_shape.dimensions()), re.data_ptr(), im.data_ptr(),
         out.data_ptr(), re._stream())
    return out


class Fft:
    """api/Fft.java: discrete Fourier transforms, resident on the device
    (cuFFT through j4c_fft / j4c_rfft / j4c_irfft / j4c_dct1).  A complex
    signal is a pair (real, imaginary) of equal-shape arrays; 1-D vectors or
    3-D grids with power-of-two extents; FLOAT32 or FLOAT64, outputs of the
    input's dtype.  As in the reference, FFTs are numerical primitives with
    no VJP or vmap rule.  The reference's *OnDevice entry points are the same
    calls here (every array already lives on a GPU)."""

    @staticmethod
    def fft(re: NDArray, im: NDArray) -> List[ConcreteNDArray]:
        """Fft.fft (Fft.java:64-67): y_k = sum_j (re_j + i im_j) exp(-2 pi i j k / N)."""
        return _fft_complex(re, im, False, 1)

    @staticmethod
    def ifft(re: NDArray, im: NDArray) -> List[ConcreteNDArray]:
        """Fft.ifft (Fft.java:75-78): the inverse, scaled by 1/N."""
        return _fft_complex(re, im, True, 1)

    @staticmethod
    def rfft(x: NDArray) -> List[ConcreteNDArray]:
        """Fft.rfft (Fft.java:93-127): the N/2 + 1 independent bins of a real signal."""
        return _rfft(x, 1)

    @staticmethod
    def irfft(re: NDArray, im: NDArray) -> ConcreteNDArray:
        """Fft.irfft (Fft.java:130-186): the real signal of length 2 (len(re) - 1)."""
        return _irfft(re, im, 1)

    @staticmethod
    def dctI(x: NDArray) -> NDArray:
        """Fft.dctI (Fft.java:200-227): unnormalised DCT-I, n = 1 or n - 1 a power of two."""
        x = _fft_operand(x, "dctI")
        if x.shape().rank() != 1:
            raise IllegalArgumentException(f"dctI requires a 1-D input, got shape {x.shape()}")
        n = x.shape().dimensions()[0]
        if n == 1:
            return x
        if n < 2 or not _pow2(n - 1):
            raise IllegalArgumentException(f"dctI requires (N - 1) to be a power of two, got N = {n}")
        out = _fft_new(x, x.shape())
        call("j4c_dct1", x.dtype().ordinal, n, x.data_ptr(), out.data_ptr(), x._stream())
        return out

    @staticmethod
    def dctIRaw(x) -> np.ndarray:
        """Fft.dctIRaw (Fft.java:237-247): host doubles in, a fresh host array
        out (the input is never aliased nor changed)."""
        a = np.array(x, dtype=np.float64, copy=True).reshape(-1)
        n = a.shape[0]
        if n == 0:
            raise IllegalArgumentException("dctIRaw: input must be non-empty")
        if n == 1:
            return a
        if not _pow2(n - 1):
            raise IllegalArgumentException(f"dctIRaw requires (N - 1) to be a power of two, got N = {n}")
        arr = ConcreteNDArray.of(a, Shape(n), DType.FLOAT64)
        return Fft.dctI(arr).numpy().astype(np.float64).copy()

    @staticmethod
    def fft3(re: NDArray, im: NDArray) -> List[ConcreteNDArray]:
        """Fft.fft3 (Fft.java:405-408): every axis of an (N1, N2, N3) grid."""
        return _fft_complex(re, im, False, 3)

    @staticmethod
    def ifft3(re: NDArray, im: NDArray) -> List[ConcreteNDArray]:
        """Fft.ifft3 (Fft.java:414-417)."""
        return _fft_complex(re, im, True, 3)

    @staticmethod
    def rfft3(x: NDArray) -> List[ConcreteNDArray]:
        """Fft.rfft3 (Fft.java:423-492): (N1, N2, N3) real -> (N1, N2, N3/2 + 1) complex."""
        return _rfft(x, 3)

    @staticmethod
    def irfft3(re: NDArray, im: NDArray) -> ConcreteNDArray:
        """Fft.irfft3 (Fft.java:494-568)."""
        return _irfft(re, im, 3)

    @staticmethod
    def fftOnDevice(re: NDArray, im: NDArray, inverse: bool) -> List[ConcreteNDArray]:
        """Fft.fftOnDevice (Fft.java:812-835)."""
        return _fft_complex(re, im, inverse, 1)

    @staticmethod
    def fft3OnDevice(re: NDArray, im: NDArray, inverse: bool) -> List[ConcreteNDArray]:
        """Fft.fft3OnDevice (Fft.java:1018-1036)."""
        return _fft_complex(re, im, inverse, 3)

    @staticmethod
    def rfft3OnDevice(x: NDArray) -> List[ConcreteNDArray]:
        """Fft.rfft3OnDevice (Fft.java:1045-1063)."""
        return _rfft(x, 3)

    @staticmethod
    def irfft3OnDevice(re: NDArray, im: NDArray, fullN2: int) -> ConcreteNDArray:
        """Fft.irfft3OnDevice (Fft.java:1072-1100): fullN2 is the last extent of the signal."""
        return _irfft(re, im, 3, fullN2)


# ---- Linalg ---------------------------------------------------------------------------
def _jdouble(x: float) -> str:
    """java.lang.Double.toString of x (shortest digits; E notation outside
    [1e-3, 1e7)), for the reference's exception messages."""
    x = float(x)
    if x != x:
        return "NaN"
    if math.isinf(x):
        return "Infinity" if x > 0 else "-Infinity"
    if x == 0.0:
        return "-0.0" if math.copysign(1.0, x) < 0 else "0.0"
    if 1e-3 <= abs(x) < 1e7:
        r = repr(x)
        return r if "e" not in r else format(x, "f")
    _, digits, exponent = decimal.Decimal(repr(abs(x))).normalize().as_tuple()
    ds = "".join(map(str, digits))
    sign = "-" if x < 0 else ""
    return f"{sign}{ds[0]}.{ds[1:] or '0'}E{len(ds) - 1 + exponent}"


class SingularityCheck(enum.Enum):
    """Linalg.SingularityCheck (Linalg.java:28-70): when lu / solve reject A.

    SINGULARITY_CHECK_SUBMATRIX_MAX (the default): a pivot at or below
    1e-14 x max|a_ij| of the original matrix.
    SINGULARITY_CHECK_RECIPROCAL_CONDITION_EST: only exact-zero pivots in
    the elimination, then Hager's estimate of 1 / kappa_inf below 1e-14."""
    SINGULARITY_CHECK_SUBMATRIX_MAX = 0
    SINGULARITY_CHECK_RECIPROCAL_CONDITION_EST = 1


_RCOND_TOL = 1e-14  # Linalg.java:1096


class LU:
    """Linalg.LU (Linalg.java:116-233): P A = L U of a square matrix, held on
    the device in FP64 (column-major packed factors and the row swaps), for
    any number of O(n^2) solves.  solve(b) of an array returns an array of
    b's dtype; solve of host doubles returns fresh host doubles."""

    def __init__(self, lu: Optional[torch.Tensor], ipiv: Optional[torch.Tensor], n: int, inf_norm: float,
                 device: Device):
        self._lu, self._ipiv, self._n, self._inf_norm, self._device = lu, ipiv, n, inf_norm, device

    def n(self) -> int:
        """Order of the factored matrix (Linalg.java:133)."""
        return self._n

    def _stream(self) -> int:
        return stream_of(self._lu.device.index) if self._lu is not None else 0

    def _solve_tensor(self, b: torch.Tensor, dtype: DType, nrhs: int, transpose: bool) -> torch.Tensor:
        """X = A^-1 B (or A^-T B) for B row-major [n, nrhs] of dtype on the device."""
        x = torch.empty_like(b)
        if self._n:
            call("j4c_lu_solve", self._n, nrhs, self._lu.data_ptr(), self._ipiv.data_ptr(), int(transpose),
                 dtype.ordinal, b.data_ptr(), x.data_ptr(), self._stream())
        return x

    def solve(self, b):
        """LU.solve (Linalg.java:141-176): A x = b."""
        if isinstance(b, NDArray):
            if b.shape().rank() != 1 or b.shape().dimensions()[0] != self._n:
                raise IllegalArgumentException(
                    f"LU.solve: b must be length-{self._n} vector, got shape {b.shape()}")
            if b.dtype() not in (DType.FLOAT32, DType.FLOAT64):
                raise IllegalArgumentException(f"LU.solve requires FLOAT32 or FLOAT64 RHS, got {b.dtype()}")
            if not isinstance(b, ConcreteNDArray):
                raise IllegalArgumentException("LU.solve: a concrete right-hand side is required")
            t = b.tensor()
            if self._lu is not None and t.device != self._lu.device:
                t = t.to(self._lu.device)
            x = self._solve_tensor(t, b.dtype(), 1, False)
            return ConcreteNDArray._wrap(x, Shape(self._n), b.dtype(), self._device)
        return self._solve_host(b, False)

    def _solve_host(self, b, transpose: bool) -> np.ndarray:
        a = np.array(b, dtype=np.float64, copy=True).reshape(-1)
        if a.shape[0] != self._n:
            who = "LU.solveTranspose" if transpose else "LU.solve"
            raise IllegalArgumentException(f"{who}: b length must be {self._n}, got {a.shape[0]}")
        if not self._n:
            return a
        t = torch.from_numpy(a).to(self._lu.device)
        return self._solve_tensor(t, DType.FLOAT64, 1, transpose).cpu().numpy()

    def solveTranspose(self, b) -> np.ndarray:
        """LU.solveTranspose (Linalg.java:206-233): A^T x = b on host doubles."""
        return self._solve_host(b, True)

    def _rcond(self) -> float:
        """Linalg.reciprocalConditionNumber (Linalg.java:1102-1107)."""
        if self._inf_norm == 0.0 or not self._n:
            return 0.0
        out = C.c_double(0.0)
        call("j4c_lu_rcond", self._n, self._lu.data_ptr(), self._ipiv.data_ptr(), float(self._inf_norm),
             C.addressof(out), self._stream())
        return out.value


def _la_concrete(A, who: str) -> ConcreteNDArray:
    if not isinstance(A, ConcreteNDArray):
        raise IllegalArgumentException(f"{who}: a concrete array is required (linear algebra is not traced)")
    return A


def _la_square(A, who: str) -> int:
    if A.shape().rank() != 2:
        raise IllegalArgumentException(f"{who}: A must be 2-D, got shape {A.shape()}")
    n = A.shape().dimensions()[0]
    if A.shape().dimensions()[1] != n:
        raise IllegalArgumentException(f"{who}: A must be square, got shape {A.shape()}")
    if A.dtype() not in (DType.FLOAT32, DType.FLOAT64):
        raise IllegalArgumentException(f"{who} requires FLOAT32 or FLOAT64, got {A.dtype()}")
    return n


def _lu_factor(A, check: SingularityCheck) -> LU:
    """Linalg.factorFromNDArray + luFactorInPlace (Linalg.java:313-333,
    1021-1085): the factorisation on the device (j4c_lu_factor), then the
    reference's per-step checks applied to the pivots in elimination order."""
    n = _la_square(A, "lu")
    A = _la_concrete(A, "lu")
    if n == 0:
        return LU(None, None, 0, 0.0, A.device())
    dev = A.tensor().device
    lu = torch.empty(n * n, dtype=torch.float64, device=dev)
    ipiv = torch.empty(n, dtype=torch.int64, device=dev)
    pivots = np.empty(n, np.float64)
    norms = np.zeros(2, np.float64)
    call("j4c_lu_factor", A.dtype().ordinal, n, A.data_ptr(), lu.data_ptr(), ipiv.data_ptr(),
         pivots.ctypes.data, norms.ctypes.data, A._stream())
    tol = 1e-14 * norms[0] if check is SingularityCheck.SINGULARITY_CHECK_SUBMATRIX_MAX else 0.0
    bad = np.flatnonzero((pivots == 0.0) | (pivots <= tol))
    if bad.size:
        k = int(bad[0])
        if pivots[k] == 0.0:
            raise IllegalArgumentException(f"lu: matrix is singular (column {k} has zero pivot)")
        raise IllegalArgumentException(
            f"lu: matrix is singular under SUBMATRIX_MAX check (pivot {_jdouble(pivots[k])} \u2264 "
            f"{_jdouble(tol)} = 1e-14 \u00d7 \u2016A\u2016_max)")
    return LU(lu, ipiv, n, float(norms[1]), A.device())


class Linalg:
    """api/Linalg.java: dense real linear algebra on the device.  cuSOLVER
    does the O(n^3) work in FP64 for both input dtypes (the reference's own
    precision); the reference's argument checks, singularity rules and
    exception messages are kept.  Linear algebra is not traced: inputs are
    concrete arrays."""

    SingularityCheck = SingularityCheck
    LU = LU

    @staticmethod
    def solve(A: NDArray, b: NDArray,
              check: SingularityCheck = SingularityCheck.SINGULARITY_CHECK_SUBMATRIX_MAX) -> ConcreteNDArray:
        """Linalg.solve (Linalg.java:83-98): x with A x = b, in b's dtype."""
        if A.dtype() != b.dtype():
            raise IllegalArgumentException(f"solve requires matching dtypes: {A.dtype()} vs {b.dtype()}")
        return Linalg.lu(A, check).solve(b)

    @staticmethod
    def lu(A: NDArray, check: SingularityCheck = SingularityCheck.SINGULARITY_CHECK_SUBMATRIX_MAX) -> LU:
        """Linalg.lu (Linalg.java:244-265)."""
        f = _lu_factor(A, check)
        if check is SingularityCheck.SINGULARITY_CHECK_RECIPROCAL_CONDITION_EST:
            rcond = f._rcond()
            if rcond < _RCOND_TOL:
                raise IllegalArgumentException(
                    f"lu: matrix is ill-conditioned (rcond \u2248 {_jdouble(rcond)} < {_jdouble(_RCOND_TOL)}, "
                    f"so \u03ba_\u221e \u2273 {_jdouble(1.0 / _RCOND_TOL)})")
        return f

    @staticmethod
    def cond(A) -> float:
        """Linalg.cond (Linalg.java:279-305): Hager's estimate of
        kappa_inf = ||A||_inf ||A^-1||_inf; +inf for a matrix the
        factorisation rejects.  Accepts an array or an LU."""
        if not isinstance(A, LU):
            try:
                A = _lu_factor(A, SingularityCheck.SINGULARITY_CHECK_RECIPROCAL_CONDITION_EST)
            except IllegalArgumentException:
                return math.inf
        rcond = A._rcond()
        if rcond == 0.0 or not math.isfinite(rcond):
            return math.inf
        return 1.0 / rcond

    @staticmethod
    def eig(A: NDArray, B: Optional[NDArray] = None) -> List[ConcreteNDArray]:
        """Linalg.eig(A) (Linalg.java:768-800): [real, imag] of the n
        eigenvalues (input dtype), complex ones in adjacent conjugate pairs.
        Linalg.eig(A, B) (Linalg.java:345-366): the generalized eigenvalues
        of A x = lambda B x as the eigenvalues of C = B^-1 A, formed with
        one factorisation of B (default check) and one multi-column solve;
        FLOAT64 results, as the reference's."""
        if B is not None:
            return _eig_pair(A, B)
        if A.shape().rank() != 2:
            raise IllegalArgumentException(f"eig: A must be 2-D, got shape {A.shape()}")
        n = A.shape().dimensions()[0]
        if A.shape().dimensions()[1] != n:
            raise IllegalArgumentException(f"eig: A must be square, got shape {A.shape()}")
        if A.dtype() not in (DType.FLOAT32, DType.FLOAT64):
            raise IllegalArgumentException(f"eig requires FLOAT32 or FLOAT64, got {A.dtype()}")
        A = _la_concrete(A, "eig")
        wr, wi = _fft_new(A, Shape(n)), _fft_new(A, Shape(n))
        if n:
            call("j4c_eig", A.dtype().ordinal, n, A.data_ptr(), wr.data_ptr(), wi.data_ptr(), A._stream())
        return [wr, wi]

    @staticmethod
    def svd(A: NDArray) -> "Svd":
        """Linalg.svd (Linalg.java:411-460): thin SVD A = U diag(sigma) Vt of
        an m x n matrix, m >= n; U [m, n], sigma [n] descending and
        non-negative, Vt [n, n]; FLOAT64 results for both input dtypes."""
        if A.shape().rank() != 2:
            raise IllegalArgumentException(f"svd: A must be 2-D, got shape {A.shape()}")
        m, n = A.shape().dimensions()
        if m < n:
            raise IllegalArgumentException(f"svd currently requires m >= n (thin SVD), got shape {A.shape()}")
        if A.dtype() not in (DType.FLOAT32, DType.FLOAT64):
            raise IllegalArgumentException(f"svd requires FLOAT32 or FLOAT64, got {A.dtype()}")
        A = _la_concrete(A, "svd")
        dev = A.tensor().device

        def new(*shape):
            return ConcreteNDArray._wrap(torch.empty(math.prod(shape), dtype=torch.float64, device=dev),
                                         Shape(shape), DType.FLOAT64, A.device())

        U, sigma, Vt = new(m, n), new(n), new(n, n)
        if n:
            call("j4c_svd", A.dtype().ordinal, m, n, A.data_ptr(), U.data_ptr(), sigma.data_ptr(), Vt.data_ptr(),
                 A._stream())
        return Svd(U, sigma, Vt)


class Svd:
    """Linalg.Svd (Linalg.java:396): the record (U, sigma, Vt)."""
    __slots__ = ("_U", "_sigma", "_Vt")

    def __init__(self, U, sigma, Vt):
        self._U, self._sigma, self._Vt = U, sigma, Vt

    def U(self) -> ConcreteNDArray:
        return self._U

    def sigma(self) -> ConcreteNDArray:
        return self._sigma

    def Vt(self) -> ConcreteNDArray:
        return self._Vt

    def __iter__(self):
        return iter((self._U, self._sigma, self._Vt))


Linalg.Svd = Svd


def _eig_pair(A, B) -> List[ConcreteNDArray]:
    """Linalg.eig(A, B) (Linalg.java:345-381)."""
    label = "eig(A, B)"
    if A.shape().rank() != 2 or B.shape().rank() != 2:
        raise IllegalArgumentException(f"{label}: inputs must be 2-D")
    n = A.shape().dimensions()[0]
    if A.shape().dimensions()[1] != n:
        raise IllegalArgumentException(f"{label}: A must be square")
    if B.shape().dimensions()[0] != n or B.shape().dimensions()[1] != n:
        raise IllegalArgumentException(f"{label}: A and B must share shape")
    if A.dtype() != B.dtype():
        raise IllegalArgumentException(f"eig(A, B) requires matching dtypes: {A.dtype()} vs {B.dtype()}")
    A = _la_concrete(A, label)
    f = Linalg.lu(B)
    if n == 0:
        return Linalg.eig(ConcreteNDArray.of(np.zeros((0, 0)), Shape(0, 0), DType.FLOAT64, A.device()))
    a = A.tensor()
    if a.device != f._lu.device:
        a = a.to(f._lu.device)
    c = f._solve_tensor(a.to(torch.float64), DType.FLOAT64, n, False)  # C = B^-1 A, all n columns at once
    return Linalg.eig(ConcreteNDArray._wrap(c, Shape(n, n), DType.FLOAT64, A.device()))
