"""Lax.psumSgdTree: the data-parallel gradient all-reduce fused with the SGD
update, for one-process-per-GPU runs.

The reference's training step sums each gradient over the shards with
Lax.psum (api/Lax.java:184-186, SharedCollective.java:44-54) and updates
every parameter with elementwise ops.  Here the gradients go in buckets (the
last leaves first, the order the backward completes them) over a side
stream as soon as they exist, like Lax.psumTree's overlapped buckets, but
each bucket is one call of j4c_psum_sgd (psum_sgd.cu): the peers'
gradients of rank r's slice come over NVLink on the copy engines, rank r sums
and updates its slice locally, and every rank copies the other updated
slices out of the peers' exchange buffers -- no NCCL call, no separate update
kernels, and no SM time for the NVLink traffic.

Peer memory: each rank allocates one buffer (j4c_peer_alloc) holding the flag
block, every bucket's packed gradients and every bucket's exchange area, at
offsets that are the same on all ranks; the CUDA IPC handles go to every rank
over the host process group and are mapped once (j4c_peer_open).  A group is
made per tree signature (leaf sizes), on first use, outside any graph
capture.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import call
from .core import ConcreteNDArray, DType

HANDLE_BYTES = 64          # J4C_PEER_HANDLE_BYTES
MAX_RANKS, MAX_SEGS = 8, 16
FLAG_AREA = 256            # bytes reserved for the flag block at the start of the buffer
# Off unless J4C_PSUM_SGD=1: measured on B200s, NCCL's all-reduce (NVLS from
# 4 MB at 8 GPUs) plus one update kernel per parameter is as fast at 2 GPUs
# and faster at 8, where the copy engines pull from 7 peers per bucket.
ENABLED = os.environ.get("J4C_PSUM_SGD", "0") == "1"


def plan_buckets(sizes: Sequence[int], bucket_floats: int, max_segs: int = MAX_SEGS) -> List[List[int]]:
    """Leaf indices per bucket, walked from the last leaf: a bucket closes
    once it holds bucket_floats floats or max_segs leaves."""
    buckets, cur, n = [], [], 0
    for i in reversed(range(len(sizes))):
        cur.append(i)
        n += sizes[i]
        if n >= bucket_floats or len(cur) == max_segs:
            buckets.append(cur)
            cur, n = [], 0
    if cur:
        buckets.append(cur)
    return buckets


def layout(sizes: Sequence[int], buckets: Sequence[Sequence[int]]) -> Tuple[List[int], List[int], int]:
    """Byte offsets of each bucket's gradient and exchange areas in the peer
    buffer, and the buffer's size: [flags | G_0 .. G_k | U_0 .. U_k]."""
    lens = [sum(sizes[i] for i in b) for b in buckets]
    g_off, off = [], FLAG_AREA
    for n in lens:
        g_off.append(off)
        off += 4 * n
    u_off = []
    for n in lens:
        u_off.append(off)
        off += 4 * n
    return g_off, u_off, off


def eligible(leaves_w: Sequence[ConcreteNDArray], leaves_g: Sequence[ConcreteNDArray], world: int) -> bool:
    """The fused path takes FLOAT32 leaves on one GPU whose sizes are
    multiples of 4 floats and whose parameters are 16-byte aligned, with
    every bucket holding at least 4 floats per rank."""
    if not ENABLED or world < 2 or world > MAX_RANKS or not leaves_w:
        return False
    dev = leaves_w[0].tensor().device
    if dev.type != "cuda":
        return False
    for w, g in zip(leaves_w, leaves_g):
        if w.dtype() != DType.FLOAT32 or g.dtype() != DType.FLOAT32:
            return False
        if w.tensor().device != dev or g.tensor().device != dev:
            return False
        n = w.shape().size()
        if n != g.shape().size() or n % 4 or w.data_ptr() % 16:
            return False
    return True


class PeerGroup:
    """One rank's peer buffer and its mappings of every other rank's."""

    def __init__(self, rank: int, world: int, nbytes: int):
        self.rank, self.world, self.nbytes = rank, world, nbytes
        own = C.c_void_p()
        handle = (C.c_char * HANDLE_BYTES)()
        call("j4c_peer_alloc", nbytes, C.byref(own), C.cast(handle, C.c_void_p), HANDLE_BYTES)
        self.own = own.value
        import torch.distributed as dist
        handles: list = [None] * world
        dist.all_gather_object(handles, bytes(handle.raw))
        self.base: List[int] = []
        self.opened: List[int] = []
        for p in range(world):
            if p == rank:
                self.base.append(self.own)
                continue
            raw = (C.c_char * HANDLE_BYTES).from_buffer_copy(handles[p])
            ptr = C.c_void_p()
            call("j4c_peer_open", C.cast(raw, C.c_void_p), HANDLE_BYTES, C.byref(ptr))
            self.base.append(ptr.value)
            self.opened.append(ptr.value)

    def pointers(self, offset: int):
        return (C.c_void_p * self.world)(*[b + offset for b in self.base])

    def close(self) -> None:
        for p in self.opened:
            _lib.lib().j4c_peer_close(p)
        self.opened = []
        if self.own:
            _lib.lib().j4c_peer_free(self.own)
            self.own = None


class FusedPlan:
    def __init__(self, sizes: Tuple[int, ...], rank: int, world: int, bucket_floats: int):
        self.sizes = sizes
        self.buckets = plan_buckets(sizes, bucket_floats)
        self.lens = [sum(sizes[i] for i in b) for b in self.buckets]
        g_off, u_off, nbytes = layout(sizes, self.buckets)
        self.group = PeerGroup(rank, world, nbytes)
        self.flags = self.group.pointers(0)
        self.g_ptrs = [self.group.pointers(o) for o in g_off]
        self.u_ptrs = [self.group.pointers(o) for o in u_off]
        self.g_own = [self.group.own + o for o in g_off]


_plans: Dict[tuple, FusedPlan] = {}
_plans_lock = threading.Lock()


def _plan_for(st, sizes: Tuple[int, ...], bucket_floats: int) -> FusedPlan:
    key = (sizes, bucket_floats)
    with _plans_lock:
        p = _plans.get(key)
        if p is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("psumSgdTree: the peer buffers of a new tree are set up by an eager "
                                   "call before a graph capture")
            p = FusedPlan(sizes, st.rank, st.world_size, bucket_floats)
            _plans[key] = p
        return p


def close_all() -> None:
    """Unmaps and frees every peer buffer (distributed.shutdown)."""
    with _plans_lock:
        for p in _plans.values():
            p.group.close()
        _plans.clear()


def fused(ctx, st, leaves_w: List[ConcreteNDArray], leaves_g: List[ConcreteNDArray], scale: float, lr: float,
          comm: "torch.cuda.Stream", bucket_floats: int) -> List[ConcreteNDArray]:
    """The fused path: per bucket, on `comm`, pack the gradients into this
    rank's peer buffer and run j4c_psum_sgd; the updated parameters are
    views of one fresh tensor per bucket.  The compute stream waits for every
    bucket before it returns."""
    dev = leaves_w[0].tensor().device
    compute = torch.cuda.current_stream(dev)
    capturing = torch.cuda.is_current_stream_capturing()
    sizes = tuple(w.shape().size() for w in leaves_w)
    plan = _plan_for(st, sizes, bucket_floats)
    # A gradient's ready event (recorded by the backward when it produced the
    # gradient) is all a bucket waits for, so the exchange overlaps the rest
    # of the backward; the parameters were read by the forward before any
    # gradient existed.  A gradient without an event waits for everything
    # enqueued before this call.
    entry = torch.cuda.Event()
    entry.record(compute)
    out: List[Optional[ConcreteNDArray]] = [None] * len(leaves_w)
    done = []
    L = _lib.lib()
    for b, idxs in enumerate(plan.buckets):
        n = plan.lens[b]
        with torch.cuda.stream(comm):
            for i in idxs:
                comm.wait_event(leaves_g[i]._ready if leaves_g[i]._ready is not None else entry)
            s = comm.cuda_stream
            off = 0
            for i in idxs:
                m = sizes[i]
                call("j4c_memcpy_d2d", plan.g_own[b] + 4 * off, leaves_g[i].data_ptr(), 4 * m, s)
                off += m
            res = torch.empty(n, dtype=torch.float32, device=dev)  # allocated on the side stream
            stage = torch.empty(n + 4 * st.world_size, dtype=torch.float32, device=dev)
            seg_len = (C.c_int64 * len(idxs))(*[sizes[i] for i in idxs])
            seg_ptr = (C.c_void_p * len(idxs))(*[leaves_w[i].data_ptr() for i in idxs])
            _lib.check(L.j4c_psum_sgd(plan.g_ptrs[b], plan.u_ptrs[b], plan.flags, st.world_size, st.rank, n,
                                      len(idxs), seg_len, seg_ptr, C.c_float(scale), C.c_float(lr),
                                      stage.data_ptr(), res.data_ptr(), s), "j4c_psum_sgd")
            off = 0
            for i in idxs:
                m = sizes[i]
                w = leaves_w[i]
                out[i] = ConcreteNDArray._wrap(res[off:off + m], w.shape(), w.dtype(), w.device())
                off += m
            ev = torch.cuda.Event()
            ev.record(comm)
            done.append(ev)
        if not capturing:
            # read on the compute stream after the waits below; the inputs
            # stay allocated until the side stream has used them
            res.record_stream(compute)
            stage.record_stream(comm)
            for i in idxs:
                leaves_g[i].tensor().record_stream(comm)
                leaves_w[i].tensor().record_stream(comm)
    for ev in done:
        compute.wait_event(ev)
    return out
