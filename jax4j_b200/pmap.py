"""pmap executor and collectives (api/Pmap.java, api/PmapContext.java,
api/SharedCollective.java of the reference).

Three placements share one executor:

* shards on one GPU (the reference's synthetic `new Device(null)` devices):
  one host thread per shard on the GPU's shared stream; psum deposits each
  shard's buffer in a slot and one kernel per shard sums the slots in slot
  order -- the reference's own summation order, so results are bit-identical
  across shards (api/SharedCollective.java:44-54);
* one shard per GPU in one process (Device.cuda(i)): one thread per GPU on
  that GPU's stream, psum/allGather are NCCL collectives on communicators
  created once per device set;
* one process per GPU (torchrun; jax4j_b200.distributed.initialize()): each
  process runs only its own shard; psum/allGather are NCCL collectives over
  NVLink/NVSwitch and the stacked pmap output is an all-gather.

Every barrier and collective wait has a deadline; a shard that raises aborts
the barrier so its peers fail at once instead of waiting forever (the
reference's CyclicBarrier.await has no timeout, SharedCollective.java:78-85).
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from concurrent.futures import ThreadPoolExecutor
from concurrent.futures import wait as wait_futures
from typing import Callable, List, Optional, Sequence

import torch

from . import _lib
from ._lib import call
from .core import (ConcreteNDArray, Device, DType, IllegalArgumentException,
                   IllegalStateException, NDArray, Shape, stream_of)

BARRIER_TIMEOUT_S = float(os.environ.get("J4C_BARRIER_TIMEOUT_S", "120"))
COMM_TIMEOUT_MS = int(os.environ.get("J4C_COMM_TIMEOUT_MS", "120000"))


class CollectiveError(RuntimeError):
    """A collective could not complete (a peer failed, or a deadline passed)."""


# ---------------------------------------------------------------------------
# PmapContext (api/PmapContext.java)
# ---------------------------------------------------------------------------
class PmapContext:
    _tls = threading.local()

    def __init__(self, deviceIndex: int, numDevices: int, collective):
        self.deviceIndex = deviceIndex
        self.numDevices = numDevices
        self.collective = collective

    @classmethod
    def current(cls) -> Optional["PmapContext"]:
        return getattr(cls._tls, "ctx", None)

    @classmethod
    def set(cls, ctx: Optional["PmapContext"]) -> None:
        cls._tls.ctx = ctx


# ---------------------------------------------------------------------------
# split / stack (Pmap.java:42-73)
# ---------------------------------------------------------------------------
def split(x: NDArray, num_devices: int) -> List[ConcreteNDArray]:
    """Pmap.split: [D, *rest] -> D shards of *rest (views, no copy)."""
    if isinstance(x, LocalShard):
        raise IllegalArgumentException("a LocalShard holds one rank's shard and cannot be split")
    d = x.shape().dimensions()
    if len(d) == 0 or d[0] != num_devices:
        raise IllegalArgumentException(
            f"pmap: input leading dim {d[0] if d else 0} must equal numDevices {num_devices}")
    shard_shape = Shape(d[1:])
    n = shard_shape.size()
    t = x.tensor()
    tag = _result_device(x)
    return [ConcreteNDArray._wrap(t[i * n:(i + 1) * n], shard_shape, x.dtype(), tag)
            for i in range(num_devices)]


def stack(shards: Sequence[NDArray]) -> ConcreteNDArray:
    """Pmap.stack: D equal shards -> [D, *shard] on the default device."""
    shard_shape = shards[0].shape()
    dev = Device.defaultDevice()
    tgt = dev.torch_device()
    parts = [s.tensor() if s.tensor().device == tgt else s.tensor().to(tgt) for s in shards]
    out = torch.cat(parts) if len(parts) > 1 else parts[0].clone()
    return ConcreteNDArray._wrap(out, Shape((len(shards),) + shard_shape.dimensions()),
                                 shards[0].dtype(), dev)


class LocalShard(NDArray):
    """This process's shard of a pmap input in one-process-per-GPU runs: the
    leading [D] axis is implicit, so no rank materialises the global array."""

    def __init__(self, local: ConcreteNDArray, num_devices: int):
        self.local = local
        self.num_devices = num_devices

    def shape(self) -> Shape:
        return Shape((self.num_devices,) + self.local.shape().dimensions())

    def dtype(self) -> DType:
        return self.local.dtype()

    def device(self) -> Device:
        return self.local.device()


# ---------------------------------------------------------------------------
# Collectives
# ---------------------------------------------------------------------------
def _result_device(x: ConcreteNDArray) -> Device:
    """The reference wraps collective results as default-device arrays
    (Lax.java:186, SharedCollective.java:73); keep that tag whenever the data
    already lives on the default device's GPU."""
    dflt = Device.defaultDevice()
    return dflt if dflt.ordinal() == x.device().ordinal() else x.device()


class SlotCollective:
    """Shards sharing one GPU (and its stream): SharedCollective's two-phase
    deposit/barrier/read protocol with the sum done on the device."""

    def __init__(self, num_devices: int, timeout_s: float = BARRIER_TIMEOUT_S):
        self.num_devices = num_devices
        self.barrier = threading.Barrier(num_devices, timeout=timeout_s)
        self.slots: List[Optional[ConcreteNDArray]] = [None] * num_devices

    def _await(self):
        try:
            self.barrier.wait()
        except threading.BrokenBarrierError as e:
            raise CollectiveError("Collective barrier broken: a shard failed or timed out") from e

    def abort(self):
        self.barrier.abort()

    def psum(self, index: int, x: ConcreteNDArray) -> ConcreteNDArray:
        self.slots[index] = x
        self._await()
        n = x.shape().size()
        for s in self.slots:
            if s.shape().size() != n or s.dtype() != x.dtype():
                raise CollectiveError("psum: shards deposited different sizes or dtypes")
        out = torch.empty_like(x.tensor())
        ptrs = (C.c_void_p * self.num_devices)(*[s.data_ptr() for s in self.slots])
        call("j4c_psum_slots", x.dtype().ordinal, ptrs, self.num_devices, out.data_ptr(), n, x._stream())
        self._await()
        return ConcreteNDArray._wrap(out, x.shape(), x.dtype(), _result_device(x))

    def reduceScatter(self, index: int, x: ConcreteNDArray) -> ConcreteNDArray:
        """Sum over shards of slice `index` of every shard's [D, *shard] value."""
        self.slots[index] = x
        self._await()
        n = x.shape().size() // self.num_devices
        for s in self.slots:
            if s.shape().size() != x.shape().size() or s.dtype() != x.dtype():
                raise CollectiveError("reduceScatter: shards deposited different sizes or dtypes")
        es = x.dtype().byteSize()
        out = torch.empty(n, dtype=x.dtype().torch, device=x.tensor().device)
        ptrs = (C.c_void_p * self.num_devices)(*[s.data_ptr() + index * n * es for s in self.slots])
        call("j4c_psum_slots", x.dtype().ordinal, ptrs, self.num_devices, out.data_ptr(), n, x._stream())
        self._await()
        return ConcreteNDArray._wrap(out, Shape(x.shape().dimensions()[1:]), x.dtype(), _result_device(x))

    def allGather(self, index: int, x: ConcreteNDArray) -> ConcreteNDArray:
        self.slots[index] = x
        self._await()
        parts = [s.tensor() for s in self.slots]
        for p in parts:
            if p.numel() != x.tensor().numel():
                raise CollectiveError("allGather: shards deposited different sizes")
        out = torch.cat(parts)
        self._await()
        shape = Shape((self.num_devices,) + x.shape().dimensions())
        return ConcreteNDArray._wrap(out, shape, x.dtype(), _result_device(x))


class NcclCollective:
    """One shard per GPU: each rank is an NCCL communicator (j4c_comm)."""

    def __init__(self, comms: List[int]):
        self.comms = comms
        self.num_devices = len(comms)
        self.aborted = False

    def abort(self):
        """Aborts every rank's communicator, which ends NCCL kernels waiting on
        a peer; the communicators cannot be used afterwards."""
        for c in self.comms:
            _lib.lib().j4c_comm_abort(c)
        self.aborted = True
        with _comm_lock:
            for k, v in list(_comm_cache.items()):
                if v is self:
                    del _comm_cache[k]

    def psum(self, index: int, x: ConcreteNDArray) -> ConcreteNDArray:
        out = torch.empty_like(x.tensor())
        s = x._stream()
        call("j4c_psum", self.comms[index], x.dtype().ordinal, x.data_ptr(), out.data_ptr(),
             x.shape().size(), s)
        return ConcreteNDArray._wrap(out, x.shape(), x.dtype(), _result_device(x))

    def psum_inplace(self, index: int, t: torch.Tensor, dtype: DType) -> None:
        call("j4c_psum", self.comms[index], dtype.ordinal, t.data_ptr(), t.data_ptr(), t.numel(),
             stream_of(t.device.index))

    def allGather(self, index: int, x: ConcreteNDArray) -> ConcreteNDArray:
        out = torch.empty(self.num_devices * x.shape().size(), dtype=x.dtype().torch,
                          device=x.tensor().device)
        call("j4c_all_gather", self.comms[index], x.dtype().ordinal, x.data_ptr(), out.data_ptr(),
             x.shape().size(), x._stream())
        shape = Shape((self.num_devices,) + x.shape().dimensions())
        return ConcreteNDArray._wrap(out, shape, x.dtype(), _result_device(x))

    def reduceScatter(self, index: int, x: ConcreteNDArray) -> ConcreteNDArray:
        """Sum over ranks of slice `index` of every rank's [D, *shard] value."""
        n = x.shape().size() // self.num_devices
        out = torch.empty(n, dtype=x.dtype().torch, device=x.tensor().device)
        call("j4c_reduce_scatter", self.comms[index], x.dtype().ordinal, x.data_ptr(), out.data_ptr(), n,
             x._stream())
        return ConcreteNDArray._wrap(out, Shape(x.shape().dimensions()[1:]), x.dtype(), _result_device(x))

    def wait(self, index: int, stream: int) -> None:
        call("j4c_comm_wait", self.comms[index], stream)


_comm_cache = {}
_comm_lock = threading.Lock()


def _nccl_for(ordinals: tuple) -> NcclCollective:
    with _comm_lock:
        c = _comm_cache.get(ordinals)
        if c is None:
            arr = (C.c_int * len(ordinals))(*ordinals)
            out = (C.c_void_p * len(ordinals))()
            call("j4c_comm_init_all", arr, len(ordinals), COMM_TIMEOUT_MS, out)
            c = NcclCollective([out[i] for i in range(len(ordinals))])
            _comm_cache[ordinals] = c
        return c


# ---------------------------------------------------------------------------
# eager collective entry points used by Lax and the Grad interpreter
# ---------------------------------------------------------------------------
def verify_signature(ctx: "PmapContext", kind: str, dtype: DType, counts) -> None:
    """One-process-per-GPU runs: checks that every rank issues this collective
    with the same dtype and element counts before any rank enqueues it
    (distributed.verify_collective).  Shards sharing a process compare their
    deposits in the collective itself."""
    from . import distributed
    st = distributed.state()
    if st is not None and ctx.collective is st.collective:
        distributed.verify_collective(kind, dtype.name, counts)


def psum_value(x: NDArray) -> NDArray:
    """Lax.psum eager branch (Lax.java:184-186): identity outside pmap."""
    ctx = PmapContext.current()
    if ctx is None or ctx.numDevices == 1:
        return x  # a sum over one shard is the shard itself (arrays are immutable)
    verify_signature(ctx, "psum", x.dtype(), (x.shape().size(),))
    return ctx.collective.psum(ctx.deviceIndex, x)


def all_gather_value(x: NDArray) -> NDArray:
    """Lax.allGather eager branch (Lax.java:211-216)."""
    ctx = PmapContext.current()
    if ctx is None:
        return stack([x])
    verify_signature(ctx, "allGather", x.dtype(), (x.shape().size(),))
    return ctx.collective.allGather(ctx.deviceIndex, x)


# The ALL_GATHER VJP.  "slice" (default): the reference's rule
# (Grad.java:437-441), the local slice of gOut with no communication.
# "reduce_scatter": the transpose of all-gather -- every shard's gOut slice
# for this shard, summed over shards -- which is what a loss that each shard
# computes from the gathered value needs.
ALLGATHER_VJP = os.environ.get("J4C_ALLGATHER_VJP", "slice")


def set_all_gather_vjp(mode: str) -> None:
    global ALLGATHER_VJP
    if mode not in ("slice", "reduce_scatter"):
        raise IllegalArgumentException(f"allGather VJP must be 'slice' or 'reduce_scatter', got {mode!r}")
    ALLGATHER_VJP = mode


def all_gather_vjp(g: ConcreteNDArray) -> ConcreteNDArray:
    """ALL_GATHER VJP: see ALLGATHER_VJP."""
    ctx = PmapContext.current()
    if ctx is None:
        return g
    if ALLGATHER_VJP == "reduce_scatter" and ctx.numDevices > 1:
        verify_signature(ctx, "reduceScatter", g.dtype(), (g.shape().size(),))
        return ctx.collective.reduceScatter(ctx.deviceIndex, g)
    return split(g, ctx.numDevices)[ctx.deviceIndex]


# ---------------------------------------------------------------------------
# placement and execution (Pmap.java:76-166)
# ---------------------------------------------------------------------------
def _spmd():
    from . import distributed
    return distributed.state()


def _placement(devices: Sequence[Device]):
    """('spmd', state) | ('slots', None) | ('nccl', NcclCollective)."""
    st = _spmd()
    D = len(devices)
    if st is not None and st.world_size == D:
        return "spmd", st
    ordinals = tuple(d.ordinal() for d in devices)
    if len(set(ordinals)) == 1:
        return "slots", None
    if len(set(ordinals)) == D:
        return "nccl", _nccl_for(ordinals)
    raise IllegalArgumentException(
        "pmap: shards must all share one GPU or each have their own GPU, got ordinals "
        f"{list(ordinals)}")


RUN_TIMEOUT_S = float(os.environ.get("J4C_PMAP_TIMEOUT_S", "600"))


def run_parallel(D: int, task: Callable[[int], object], collective) -> list:
    """Pmap.runParallel (Pmap.java:135-166): one thread per shard; the first
    failure aborts the collective so no peer blocks, and is re-raised.  The
    wait for the shards is bounded: past RUN_TIMEOUT_S the collective is
    aborted (which also ends device-side waits) and CollectiveError raised."""
    results = [None] * D
    errors: List[Optional[BaseException]] = [None] * D

    def run(i):
        try:
            results[i] = task(i)
        except BaseException as e:  # noqa: BLE001 - re-raised below
            errors[i] = e
            if collective is not None:
                collective.abort()

    if D == 1:
        run(0)
    else:
        ex = ThreadPoolExecutor(max_workers=D)
        futs = [ex.submit(run, i) for i in range(D)]
        done, pending = wait_futures(futs, timeout=RUN_TIMEOUT_S)
        if pending:
            if collective is not None:
                collective.abort()
            wait_futures(pending, timeout=30)
            ex.shutdown(wait=False, cancel_futures=True)
            raise CollectiveError(f"pmap: shards did not finish within {RUN_TIMEOUT_S} s; "
                                  "the collective was aborted")
        ex.shutdown(wait=True)
    first = next((e for e in errors if e is not None and not isinstance(e, CollectiveError)), None)
    if first is None:
        first = next((e for e in errors if e is not None), None)
    if first is not None:
        raise first
    return results


def _heartbeat():
    from . import distributed
    distributed.heartbeat()


class _Bound:
    """Makes a shard thread use its device and the stream the pmap caller had
    current on that device (so shards sharing a GPU stay ordered with the
    caller's work, and a CUDA-graph capture on the caller's stream sees them)."""

    def __init__(self, ordinal: int, stream):
        self.ordinal, self.stream = ordinal, stream

    def __enter__(self):
        self._dev = torch.cuda.device(self.ordinal)
        self._dev.__enter__()
        self._st = torch.cuda.stream(self.stream)
        self._st.__enter__()

    def __exit__(self, *exc):
        self._st.__exit__(*exc)
        self._dev.__exit__(*exc)
        return False


def _binder(devices: Sequence[Device]):
    """Called on the pmap caller's thread: records each device's current stream."""
    streams = {o: torch.cuda.current_stream(o) for o in {d.ordinal() for d in devices}}
    return lambda device: _Bound(device.ordinal(), streams[device.ordinal()])


def shards_of(x: NDArray, D: int) -> List[Optional[ConcreteNDArray]]:
    """split(x, D), except that a LocalShard yields only this rank's shard
    (the other slots are None; one-process-per-GPU runs read only their own)."""
    if isinstance(x, LocalShard):
        st = _spmd()
        if st is None:
            raise IllegalArgumentException("a LocalShard input needs a one-process-per-GPU run "
                                           "(distributed.initialize)")
        if x.num_devices != D:
            raise IllegalArgumentException("LocalShard built for a different device count")
        out: List[Optional[ConcreteNDArray]] = [None] * D
        out[st.rank] = x.local
        return out
    return split(x, D)


def _local_inputs(inputs: Sequence[NDArray], D: int, rank: int) -> List[ConcreteNDArray]:
    out = []
    for x in inputs:
        if isinstance(x, LocalShard):
            if x.num_devices != D:
                raise IllegalArgumentException("LocalShard built for a different device count")
            out.append(x.local)
        else:
            out.append(split(x, D)[rank])
    return out


def _gather_stack(st, local: ConcreteNDArray) -> ConcreteNDArray:
    """Stacks every rank's result: an all-gather across the processes."""
    from . import distributed
    distributed.verify_collective("pmap output allGather", local.dtype().name, (local.shape().size(),))
    return st.collective.allGather(0, local)


def run_forward(fn: Callable, inputs: Sequence[NDArray], devices: Sequence[Device]) -> ConcreteNDArray:
    """Pmap.runForward (Pmap.java:76-90)."""
    D = len(devices)
    mode, obj = _placement(devices)
    if mode == "spmd":
        st = obj
        _heartbeat()
        shards = _local_inputs(inputs, D, st.rank)
        PmapContext.set(PmapContext(st.rank, D, st.collective))
        try:
            res = fn(*[s.to(devices[st.rank]) for s in shards])
        finally:
            PmapContext.set(None)
        return _gather_stack(st, res)
    shards = [split(x, D) for x in inputs]
    coll = SlotCollective(D) if mode == "slots" else obj
    bind = _binder(devices)
    # Every shard reaches its device before any shard thread starts: a copy
    # issued from a shard thread could queue behind a peer's collective
    # kernel on the source GPU and wait for itself.
    placed = [[s[i].to(devices[i]) for s in shards] for i in range(D)]

    def task(i):
        with bind(devices[i]):
            PmapContext.set(PmapContext(i, D, coll))
            try:
                return fn(*placed[i])
            finally:
                PmapContext.set(None)

    return stack(run_parallel(D, task, coll))


def _body_on(jaxpr, device: Device):
    """The body with its closed-over constants placed on `device` (pmap
    replicates closed-over values to every shard's device).  Cached on the
    Jaxpr itself, so the copies live exactly as long as the trace."""
    from .tracing import Jaxpr
    if all(v.device() is device for v in jaxpr.consts.values()):
        return jaxpr
    placed = jaxpr.__dict__.setdefault("_placed", {})
    hit = placed.get(id(device))
    if hit is not None and hit[0] is device:
        return hit[1]
    moved = Jaxpr(jaxpr.inVars, jaxpr.outVars, jaxpr.equations,
                  {k: v.to(device) for k, v in jaxpr.consts.items()})
    placed[id(device)] = (device, moved)
    return moved


def run_forward_jaxpr(body, devices: Sequence[Device], shards: List[List[ConcreteNDArray]]):
    """Pmap.runForwardJaxpr (Pmap.java:97-110); shards[k][i] is input k of shard i."""
    from .grad import forward_interpret
    D = len(devices)
    mode, obj = _placement(devices)
    if mode == "spmd":
        st = obj
        _heartbeat()
        PmapContext.set(PmapContext(st.rank, D, st.collective))
        try:
            res = forward_interpret(_body_on(body, devices[st.rank]),
                                    [s[st.rank].to(devices[st.rank]) for s in shards])[0]
        finally:
            PmapContext.set(None)
        return _gather_stack(st, res)
    coll = SlotCollective(D) if mode == "slots" else obj
    bind = _binder(devices)
    bodies = [_body_on(body, devices[i]) for i in range(D)]  # placed before any thread starts
    placed = [[s[i].to(devices[i]) for s in shards] for i in range(D)]

    def task(i):
        with bind(devices[i]):
            PmapContext.set(PmapContext(i, D, coll))
            try:
                return forward_interpret(bodies[i], placed[i])[0]
            finally:
                PmapContext.set(None)

    return stack(run_parallel(D, task, coll))


def run_backward_jaxpr(body, devices: Sequence[Device], in_shards: List[List[ConcreteNDArray]],
                       g_shards: List[ConcreteNDArray]) -> List[List[ConcreteNDArray]]:
    """Pmap.runBackwardJaxpr (Pmap.java:118-133): returns g_in[i][k], the
    cotangent of input k on shard i (for spmd runs, every rank's slot holds
    the all-gathered stack split back into shards)."""
    from .grad import backward_interpret
    D = len(devices)
    mode, obj = _placement(devices)
    if mode == "spmd":
        st = obj
        _heartbeat()
        r = st.rank
        PmapContext.set(PmapContext(r, D, st.collective))
        try:
            g_local = backward_interpret(_body_on(body, devices[r]),
                                         [s[r].to(devices[r]) for s in in_shards],
                                         [g_shards[r].to(devices[r])])
        finally:
            PmapContext.set(None)
        stacked = [split(_gather_stack(st, g), D) for g in g_local]
        return [[stacked[k][i] for k in range(len(g_local))] for i in range(D)]
    coll = SlotCollective(D) if mode == "slots" else obj
    bind = _binder(devices)
    bodies = [_body_on(body, devices[i]) for i in range(D)]  # placed before any thread starts
    placed = [[s[i].to(devices[i]) for s in in_shards] for i in range(D)]
    seeds = [g_shards[i].to(devices[i]) for i in range(D)]

    def task(i):
        with bind(devices[i]):
            PmapContext.set(PmapContext(i, D, coll))
            try:
                return backward_interpret(bodies[i], placed[i], [seeds[i]])
            finally:
                PmapContext.set(None)

    return run_parallel(D, task, coll)
