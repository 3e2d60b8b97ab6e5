"""Fusion of a traced Jaxpr's elementwise chains into generated kernels.

Replaces the reference's TornadoJitCompiler (backend/TornadoJitCompiler.java:82-246),
which compiles every Jaxpr equation to its own task, with a planner that groups
elementwise equations of one shape into a single kernel (j4c_fused_compile /
j4c_fused_launch), with reductions over the last axis (SUM_AXIS, MEAN_AXIS,
ARGMAX, ARGMIN) computed in the same pass.

Plan rules:
  * a group has one shape S, viewed as [rows, cols] (cols = last dimension);
  * an equation joins a group if it is elementwise with output shape S and
    each input is either produced by the group or is an outside value that
    already exists when the group runs and broadcasts to S as a full array,
    a [cols] row vector, a [rows, 1] column or a single value;
  * a last-axis reduction of a group value becomes a tail of the group; its
    result is only available after the group, so consumers of it start a
    new group;
  * a group value is written to memory only if something outside the group
    needs it: a later equation, a Jaxpr output, or (for the grad interpreter)
    a VJP rule that reads it.
Everything else runs equation by equation, as before.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Dict, List, Optional

import torch

from . import _lib
from ._lib import call
from .core import ConcreteNDArray, DType, NDArray, Primitive as P, Shape, stream_of
from .tracing import AxisMeta, Jaxpr

ELEMENTWISE = {P.ADD, P.SUB, P.MUL, P.DIV, P.MAX, P.MIN, P.EXP, P.LOG, P.SIN, P.COS, P.TANH,
               P.RELU, P.SIGMOID, P.GT, P.GE, P.LT, P.LE, P.EQ, P.NE, P.CAST}
TAILS = {P.SUM_AXIS, P.MEAN_AXIS, P.ARGMAX, P.ARGMIN}
FUSED_DTYPES = {DType.FLOAT32, DType.FLOAT64, DType.INT32, DType.BOOL}
BCAST_FULL, BCAST_ROW, BCAST_COL, BCAST_SCALAR = 0, 1, 2, 3
OP_INPUT = -1
OP_CONST = -2

# which operands each primitive's VJP rule reads (api/Grad.java:341-472);
# "out" = the equation's own output
_VJP_READS = {
    P.MUL: ("in",), P.DIV: ("in",), P.EXP: ("out",), P.LOG: ("in",), P.SIN: ("in",),
    P.COS: ("in",), P.TANH: ("out",), P.RELU: ("out",), P.SIGMOID: ("out",), P.DOT: ("in",),
    P.MAX: ("in",), P.MIN: ("in",), P.COND: ("in",), P.SCAN: ("in",),
}


class _Insn(C.Structure):
    _fields_ = [("op", C.c_int32), ("dtype", C.c_int32), ("a", C.c_int32), ("b", C.c_int32),
                ("value", C.c_double)]


class _Program(C.Structure):
    _fields_ = [("n_insns", C.c_int32), ("insns", C.POINTER(_Insn)),
                ("n_inputs", C.c_int32), ("input_dtype", C.POINTER(C.c_int32)),
                ("input_bcast", C.POINTER(C.c_int32)),
                ("n_outputs", C.c_int32), ("output_insn", C.POINTER(C.c_int32)),
                ("n_tails", C.c_int32), ("tail_op", C.POINTER(C.c_int32)),
                ("tail_insn", C.POINTER(C.c_int32))]


# Program limits of j4c_fused_compile (16 inputs, 16 outputs, 8 tails); a group
# holds at most 16 equations, so it never has more than 16 outputs.
MAX_INPUTS, MAX_EQS, MAX_TAILS = 16, 16, 8


def _rc(shape: Shape):
    d = shape.dimensions()
    if not d:
        return 1, 1
    rows = 1
    for x in d[:-1]:
        rows *= x
    return rows, d[-1]


def bcast_kind(inp: Shape, group: Shape) -> Optional[int]:
    """How an input of shape `inp` broadcasts over a group of shape `group`."""
    if inp == group:
        return BCAST_FULL
    if inp.size() == 1:
        return BCAST_SCALAR
    gd, idn = group.dimensions(), inp.dimensions()
    if len(idn) > len(gd):
        return None
    pad = (1,) * (len(gd) - len(idn)) + idn
    if pad[-1] == gd[-1] and all(x == 1 for x in pad[:-1]):
        return BCAST_ROW
    if pad[-1] == 1 and pad[:-1] == gd[:-1]:
        return BCAST_COL
    return None


class Group:
    def __init__(self, shape: Shape, step: int):
        self.shape = shape
        self.step = step
        self.eqs = []
        self.values = set()        # var ids produced by the group's elementwise equations
        self.tails = []            # (eq) last-axis reductions of group values
        self.tail_values = set()   # var ids produced by the tails
        self.input_ids = set()     # var ids read from outside the group
        self.inputs: List[tuple] = []  # (var, kind) in slot order
        self.consts: Dict[int, float] = {}  # var id -> value of a one-element constant taken as a literal
        self.outputs: List = []        # vars written to memory
        self.handle = None


class Plan:
    def __init__(self, steps, groups):
        self.steps = steps    # list of ("eq", eq) | ("group", Group)
        self.groups = groups


def _is_fusible(eq) -> bool:
    if eq.primitive not in ELEMENTWISE:
        return False
    if eq.outputs[0].dtype not in FUSED_DTYPES or any(v.dtype not in FUSED_DTYPES for v in eq.inputs):
        return False
    if eq.primitive in (P.GT, P.GE, P.LT, P.LE, P.EQ, P.NE) and eq.inputs[0].dtype == DType.BOOL:
        return False
    if eq.primitive not in (P.GT, P.GE, P.LT, P.LE, P.EQ, P.NE, P.CAST) and \
            not eq.outputs[0].dtype.is_floating():
        return False
    return eq.outputs[0].shape.rank() >= 1


class DotEpilogue:
    """DOT -> ADD(bias [N]) [-> RELU]: the bias add and the relu run in the
    GEMM's store (j4c_dot_split_ep); the DOT's own output is never written."""

    def __init__(self, dot, add, relu, bias, store_sum=True):
        self.dot, self.add, self.relu, self.bias = dot, add, relu, bias
        self.inputs = [dot.inputs[0], dot.inputs[1], bias]
        # with a relu whose input z = dot + bias is read by nothing else (relu's
        # VJP reads its output), only the relu output is written
        self.store_sum = store_sum


def _dot_epilogues(jaxpr: Jaxpr) -> Dict[int, DotEpilogue]:
    """Finds DOT -> ADD(bias) [-> RELU] chains whose DOT output feeds only the
    ADD and whose bias exists before the DOT.  Keyed by id(dot equation)."""
    eqs = jaxpr.equations
    uses: Dict[int, list] = {}
    pos: Dict[int, int] = {}
    for i, eq in enumerate(eqs):
        for v in eq.inputs:
            uses.setdefault(v.id, []).append(eq)
        for o in eq.outputs:
            pos[o.id] = i
    outs = {v.id for v in jaxpr.outVars}
    found: Dict[int, DotEpilogue] = {}
    for i, eq in enumerate(eqs):
        if eq.primitive != P.DOT:
            continue
        z0 = eq.outputs[0]
        if z0.dtype != DType.FLOAT32 or z0.shape.rank() != 2 or z0.id in outs or len(uses.get(z0.id, [])) != 1:
            continue
        add = uses[z0.id][0]
        if add.primitive != P.ADD or add.inputs[0].id == add.inputs[1].id:
            continue
        bias = add.inputs[1] if add.inputs[0].id == z0.id else add.inputs[0]
        if (bias.dtype != DType.FLOAT32 or bcast_kind(bias.shape, z0.shape) != BCAST_ROW
                or add.outputs[0].shape != z0.shape or pos.get(bias.id, -1) >= i):
            continue
        relu = next((e for e in uses.get(add.outputs[0].id, []) if e.primitive == P.RELU), None)
        z = add.outputs[0]
        store_sum = relu is None or z.id in outs or len(uses.get(z.id, [])) != 1
        found[id(eq)] = DotEpilogue(eq, add, relu, bias, store_sum)
    return found


def plan(jaxpr: Jaxpr, keep_for_vjp: bool) -> Plan:
    """Groups the Jaxpr's equations.  keep_for_vjp: also write every value a
    VJP rule will read (the grad interpreter's forward pass)."""
    eqs = jaxpr.equations
    # A group is launched when something outside it first needs one of its
    # values (or at the end), so an equation can join an open group whenever
    # its other inputs already exist.  Open groups never read one another:
    # reading an open group's value from elsewhere closes (launches) it first.
    producer: Dict[int, Group] = {}   # var id -> group computing it (values and tails)
    steps: list = []
    groups: List[Group] = []
    open_groups: List[Group] = []

    def close(g: Group) -> None:
        if g in open_groups:
            open_groups.remove(g)
            g.step = len(steps)
            steps.append(("group", g))

    def close_producers(e, keep: Group = None) -> None:
        for v in e.inputs:
            g = producer.get(v.id)
            if g is not None and g is not keep:
                close(g)

    def fits(g: Group, eq) -> bool:
        S = g.shape
        if len(g.eqs) >= MAX_EQS:
            return False
        new_inputs = {v.id for v in eq.inputs if v.id not in g.values} - g.input_ids
        if len(g.input_ids) + len(new_inputs) > MAX_INPUTS:
            return False
        return all(v.id in g.values or (v.id not in g.tail_values and bcast_kind(v.shape, S) is not None)
                   for v in eq.inputs)

    epilogues = _dot_epilogues(jaxpr)
    folded = {id(e.add) for e in epilogues.values()} | {id(e.relu) for e in epilogues.values() if e.relu}

    for eq in eqs:
        if id(eq) in folded:
            continue  # computed by its DOT's epilogue step
        ep = epilogues.get(id(eq))
        if ep is not None:
            close_producers(ep)
            steps.append(("dot_ep", ep))
            continue
        if _is_fusible(eq):
            S = eq.outputs[0].shape
            target = None
            for g in reversed(open_groups):
                if g.shape == S and fits(g, eq):
                    target = g
                    break
            if target is None and all(bcast_kind(v.shape, S) is not None for v in eq.inputs):
                target = Group(S, -1)
                groups.append(target)
                open_groups.append(target)
            if target is not None:
                close_producers(eq, keep=target)
                target.input_ids.update(v.id for v in eq.inputs if v.id not in target.values)
                target.eqs.append(eq)
                target.values.add(eq.outputs[0].id)
                producer[eq.outputs[0].id] = target
                continue
        elif eq.primitive in TAILS:
            g = producer.get(eq.inputs[0].id)
            m: AxisMeta = eq.metadata
            if (g is not None and g in open_groups and eq.inputs[0].id in g.values
                    and len(g.tails) < MAX_TAILS
                    and m.axis == g.shape.rank() - 1 and eq.inputs[0].dtype.is_floating()):
                g.tails.append(eq)
                g.tail_values.add(eq.outputs[0].id)
                producer[eq.outputs[0].id] = g
                continue
        # a regular equation: the groups it reads from are launched before it
        close_producers(eq)
        steps.append(("eq", eq))
    for g in list(open_groups):
        close(g)
    groups.sort(key=lambda g: g.step)

    # which group values must be written
    used_outside: set = set(v.id for v in jaxpr.outVars)
    group_of_eq = {}
    for g in groups:
        for e in g.eqs:
            group_of_eq[id(e)] = g
        for e in g.tails:
            group_of_eq[id(e)] = g
    for eq in eqs:
        g_eq = group_of_eq.get(id(eq))
        for v in eq.inputs:
            g_v = producer.get(v.id)
            if g_v is not None and g_v is not g_eq:
                used_outside.add(v.id)
        if keep_for_vjp:
            reads = _VJP_READS.get(eq.primitive, ())
            if "in" in reads:
                used_outside.update(v.id for v in eq.inputs)
            if "out" in reads:
                used_outside.update(v.id for v in eq.outputs)
    for g in groups:
        g.outputs = [e.outputs[0] for e in g.eqs if e.outputs[0].id in used_outside]
        # inputs in slot order
        seen = {}
        for e in g.eqs:
            for v in e.inputs:
                if v.id not in g.values and v.id not in seen:
                    seen[v.id] = (v, bcast_kind(v.shape, g.shape))
        g.inputs = list(seen.values())
        # one-element floating constants of the Jaxpr (Numpy.where's 1, clip's
        # bounds, ...) become literals of the generated kernel, as long as the
        # group keeps an input to read
        lit = {}
        for v, k in g.inputs:
            c = jaxpr.consts.get(v.id)
            val = getattr(c, "_scalar", None) if isinstance(c, ConcreteNDArray) else None
            if k == BCAST_SCALAR and val is not None and c.dtype() == v.dtype:
                lit[v.id] = val
        if lit and len(lit) < len(g.inputs):
            g.consts = lit
            g.inputs = [(v, k) for v, k in g.inputs if v.id not in lit]
    # drop groups that write nothing (all dead) by turning them into no-ops
    return Plan(steps, groups)


def _program(g: Group):
    insns = []
    index: Dict[int, int] = {}
    slot = {v.id: i for i, (v, _) in enumerate(g.inputs)}

    def operand(v):
        if v.id in index:
            return index[v.id]
        if v.id in g.consts:
            insns.append((OP_CONST, v.dtype.ordinal, -1, -1, g.consts[v.id]))
        else:
            insns.append((OP_INPUT, v.dtype.ordinal, slot[v.id], -1, 0.0))
        index[v.id] = len(insns) - 1
        return index[v.id]

    for e in g.eqs:
        a = operand(e.inputs[0])
        b = operand(e.inputs[1]) if len(e.inputs) > 1 else -1
        insns.append((int(e.primitive), e.outputs[0].dtype.ordinal, a, b, 0.0))
        index[e.outputs[0].id] = len(insns) - 1
    outs = [index[v.id] for v in g.outputs]
    tail_ops = [int(e.primitive) for e in g.tails]
    tail_insn = [index[e.inputs[0].id] for e in g.tails]
    return insns, outs, tail_ops, tail_insn


def _c_program(g: Group):
    """The group as a j4c_program struct (with the arrays it points to)."""
    insns, outs, tail_ops, tail_insn = _program(g)
    arr = (_Insn * len(insns))(*[_Insn(*t) for t in insns])
    in_dt = (C.c_int32 * max(1, len(g.inputs)))(*[v.dtype.ordinal for v, _ in g.inputs])
    in_bc = (C.c_int32 * max(1, len(g.inputs)))(*[k for _, k in g.inputs])
    out_i = (C.c_int32 * max(1, len(outs)))(*outs)
    t_op = (C.c_int32 * max(1, len(tail_ops)))(*tail_ops)
    t_in = (C.c_int32 * max(1, len(tail_insn)))(*tail_insn)
    prog = _Program(len(insns), arr, len(g.inputs), in_dt, in_bc, len(outs), out_i, len(tail_ops), t_op, t_in)
    return prog, (arr, in_dt, in_bc, out_i, t_op, t_in)


# J4C_FUSED_LOG=1 prints each group's program to stderr when it is compiled:
# shape, inputs (broadcast kind), instructions, outputs and tails.
FUSED_LOG = os.environ.get("J4C_FUSED_LOG", "0") == "1"
_KINDS = {BCAST_FULL: "full", BCAST_ROW: "row", BCAST_COL: "col", BCAST_SCALAR: "scalar"}


def describe(g: Group) -> str:
    insns, outs, tail_ops, tail_insn = _program(g)
    names = {int(p): p.name for p in P}
    body = []
    for i, (op, dt, a, b, val) in enumerate(insns):
        if op == OP_INPUT:
            v, k = g.inputs[a]
            body.append(f"v{i}=in{a}[{_KINDS.get(k, k)}]")
        elif op == OP_CONST:
            body.append(f"v{i}={val:g}")
        else:
            body.append(f"v{i}={names.get(op, op)}(v{a}{', v%d' % b if b >= 0 else ''})")
    tails = [f"{names.get(o, o)}(v{t})" for o, t in zip(tail_ops, tail_insn)]
    return (f"fused group {g.shape}: {'; '.join(body)} | out {['v%d' % o for o in outs]} | tails {tails}")


def compile_group(g: Group) -> None:
    if FUSED_LOG:
        import sys
        print(describe(g), file=sys.stderr, flush=True)
    prog, _keep = _c_program(g)
    handle = C.c_void_p()
    _lib.check(_lib.lib().j4c_fused_compile(C.cast(C.pointer(prog), C.c_void_p), C.byref(handle)),
               "j4c_fused_compile")
    g.handle = handle.value


def group_source(g: Group, compile: bool = False) -> str:
    """The CUDA source generated for a group; with compile=True it is also
    compiled by NVRTC for sm_100a (no GPU needed)."""
    prog, _keep = _c_program(g)
    n = C.c_size_t()
    pp = C.cast(C.pointer(prog), C.c_void_p)
    _lib.check(_lib.lib().j4c_fused_source(pp, 0, None, 0, C.byref(n)), "j4c_fused_source")
    buf = C.create_string_buffer(n.value)
    _lib.check(_lib.lib().j4c_fused_source(pp, 1 if compile else 0, buf, n.value, C.byref(n)),
               "j4c_fused_source")
    return buf.value.decode()


def run_group(g: Group, values: Dict[int, NDArray]) -> None:
    """Launches one group, writing its outputs and tails into `values`."""
    if not g.outputs and not g.tails:
        return
    if g.handle is None:
        compile_group(g)
    ins = [values[v.id] for v, _ in g.inputs]
    dev_arr = next((x for x in ins if isinstance(x, ConcreteNDArray) and x.shape().size() > 1), None)
    if dev_arr is None:
        dev_arr = next(x for x in ins if isinstance(x, ConcreteNDArray))
    device = dev_arr.device()
    tdev = dev_arr.tensor().device
    for (v, _), x in zip(g.inputs, ins):
        t = x.tensor()
        if t.device != tdev or t.dtype != v.dtype.torch or t.numel() != v.shape.size():
            raise RuntimeError(f"fused group: input {v} is {t.dtype}[{t.numel()}] on {t.device}, "
                               f"expected {v.dtype.torch}[{v.shape.size()}] on {tdev}")
    R, Cc = _rc(g.shape)
    outs = []
    for v in g.outputs:
        t = torch.empty(g.shape.size(), dtype=v.dtype.torch, device=tdev)
        outs.append(t)
        values[v.id] = ConcreteNDArray._wrap(t, g.shape, v.dtype, device)
    tails = []
    for e in g.tails:
        o = e.outputs[0]
        t = torch.empty(o.shape.size(), dtype=o.dtype.torch, device=tdev)
        tails.append(t)
        values[o.id] = ConcreteNDArray._wrap(t, o.shape, o.dtype, device)
    pin = (C.c_void_p * max(1, len(ins)))(*[x.data_ptr() for x in ins])
    pout = (C.c_void_p * max(1, len(outs)))(*[t.data_ptr() for t in outs])
    ptail = (C.c_void_p * max(1, len(tails)))(*[t.data_ptr() for t in tails])
    stream = stream_of(tdev.index)
    call("j4c_fused_launch", g.handle, R, Cc, pin, pout, ptail, stream)


def run_dot_epilogue(ep: DotEpilogue, values: Dict[int, NDArray]) -> None:
    """One GEMM for DOT + bias add (+ relu); falls back to the three
    equations when the operands do not take the fused path."""
    from .core import _dot_raw, dot_supports_epilogue
    from .grad import execute_primitive
    a, w, b = (values[v.id] for v in ep.inputs)
    if (all(isinstance(x, ConcreteNDArray) for x in (a, w, b)) and dot_supports_epilogue(a)
            and a.dtype() == w.dtype() == b.dtype() and b.tensor().device == a.tensor().device):
        dev = a._check_devices(w)
        res = _dot_raw(a, w, False, False, dev, bias=b, act=ep.relu is not None, store_c=ep.store_sum)
        if ep.relu is not None:
            z, h = res
            if ep.store_sum:
                values[ep.add.outputs[0].id] = z
            values[ep.relu.outputs[0].id] = h
        else:
            values[ep.add.outputs[0].id] = res
        return
    z0 = execute_primitive(P.DOT, ep.dot, [a, w])
    z = execute_primitive(P.ADD, ep.add, [z0, b] if ep.add.inputs[0].id == ep.dot.outputs[0].id else [b, z0])
    values[ep.dot.outputs[0].id] = z0
    values[ep.add.outputs[0].id] = z
    if ep.relu is not None:
        values[ep.relu.outputs[0].id] = execute_primitive(P.RELU, ep.relu, [z])


def plan_for(jaxpr: Jaxpr, keep_for_vjp: bool) -> Plan:
    key = "_fusion_plan_vjp" if keep_for_vjp else "_fusion_plan"
    p = jaxpr.__dict__.get(key)
    if p is None:
        p = plan(jaxpr, keep_for_vjp)
        jaxpr.__dict__[key] = p
    return p
