"""One process per GPU (torchrun): binds this process to its GPU and joins the
NCCL group that pmap's collectives run on.

torch.distributed supplies only the plumbing -- the rendezvous store that
carries the NCCL group id from rank 0 to the others, and a host barrier.  The
collectives themselves are libjax4j_cuda's j4c_psum / j4c_all_gather on a
communicator created by j4c_comm_init_rank with a deadline.

    from jax4j_b200 import distributed
    st = distributed.initialize()          # reads RANK / WORLD_SIZE / LOCAL_RANK
    devices = distributed.global_devices() # len == world size; this rank's is local
    out = JAX.pmap(body, devices)(LocalShard(x_local, st.world_size))
"""
from __future__ import annotations

import ctypes as C
import datetime
import os
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from ._lib import call
from .core import Device
from .pmap import COMM_TIMEOUT_MS, NcclCollective


@dataclass
class SpmdState:
    rank: int
    world_size: int
    local_rank: int
    comm: int
    collective: NcclCollective
    devices: List[Device]
    verified: set = field(default_factory=set)


_state: Optional[SpmdState] = None


def state() -> Optional[SpmdState]:
    return _state


def initialize(timeout_s: float = 120.0, collective_factory=None) -> SpmdState:
    """Joins the job described by RANK/WORLD_SIZE/LOCAL_RANK/MASTER_ADDR/MASTER_PORT.

    collective_factory(rank, world) -> collective replaces the NCCL group
    (used to run the executor's host logic on CPU processes in tests)."""
    global _state
    if _state is not None:
        return _state
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if collective_factory is None:
        torch.cuda.set_device(local_rank)
    local = Device.cuda(local_rank)
    Device.setDefault(local)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s))
    devices = [local if r == rank else Device(None, f"rank{r}") for r in range(world)]
    if collective_factory is not None:
        _state = SpmdState(rank, world, local_rank, 0, collective_factory(rank, world), devices)
        return _state
    uid = bytearray(128)
    if rank == 0:
        buf = (C.c_char * 128)()
        call("j4c_comm_unique_id", C.cast(buf, C.c_void_p), 128)
        uid = bytearray(buf.raw)
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    raw = (C.c_char * 128).from_buffer_copy(obj[0])
    comm = C.c_void_p()
    call("j4c_comm_init_rank", C.cast(raw, C.c_void_p), 128, world, rank, local_rank,
         int(timeout_s * 1000) if timeout_s else COMM_TIMEOUT_MS, C.byref(comm))
    # The collective object is indexed by PmapContext.deviceIndex (= rank);
    # every index resolves to this process's own communicator.
    coll = NcclCollective([comm.value] * world)
    _state = SpmdState(rank, world, local_rank, comm.value, coll, devices)
    return _state


HEARTBEAT_S = float(os.environ.get("J4C_HEARTBEAT_S", "30"))


def heartbeat() -> None:
    """Host-side liveness check run before a pmap call enqueues any
    collective: every rank must reach it within HEARTBEAT_S.  A rank that has
    left (between steps) is reported here, on the host, before this rank
    launches a kernel that would wait for it on the GPU."""
    from .pmap import CollectiveError
    if _state is None or _state.world_size == 1 or not dist.is_initialized():
        return
    try:
        dist.monitored_barrier(timeout=datetime.timedelta(seconds=HEARTBEAT_S))
    except RuntimeError as e:
        raise CollectiveError(f"pmap: a peer rank did not reach the step within {HEARTBEAT_S} s: {e}") from e


# Collective signature check.  NCCL matches collectives by call order alone: a
# rank that all-reduces 100 floats while its peer all-reduces 200 hangs or
# reads past the smaller buffer.  The reference's SharedCollective.psum has
# the same hazard (api/SharedCollective.java:44-54: the sum loop runs over the
# caller's length and indexes every peer's deposit with it, so a shorter
# deposit throws on the longer caller while its peers wait at the barrier).
# Before a collective signature (kind, dtype, element counts) is used for the
# first time, every rank exchanges it over the host process group; ranks that
# disagree all raise CollectiveError naming each rank's signature, and no
# device work is enqueued.  A signature seen before is not exchanged again, so
# the steady state (and a step recorded as a CUDA graph) pays nothing.
CHECK_SIGNATURES = os.environ.get("J4C_CHECK_COLLECTIVES", "1") != "0"


def verify_collective(kind: str, dtype: str, counts: Tuple[int, ...]) -> None:
    """Raises CollectiveError on every rank when the ranks' collectives differ
    in kind, dtype or element counts (first use of each signature only)."""
    from .pmap import CollectiveError
    st = _state
    if st is None or st.world_size == 1 or not CHECK_SIGNATURES or not dist.is_initialized():
        return
    key = (kind, dtype, tuple(int(c) for c in counts))
    if key in st.verified:
        return
    sigs: list = [None] * st.world_size
    try:
        dist.all_gather_object(sigs, key)
    except RuntimeError as e:
        raise CollectiveError(f"{kind}: a peer rank did not reach the signature check: {e}") from e
    if any(s != key for s in sigs):
        desc = "; ".join(f"rank {r}: {s[0]} of {s[1]} {list(s[2])}" for r, s in enumerate(sigs))
        raise CollectiveError(f"{kind}: ranks issued different collectives ({desc})")
    st.verified.add(key)


def global_devices() -> List[Device]:
    if _state is None:
        raise RuntimeError("distributed.initialize() has not been called")
    return list(_state.devices)


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def shutdown() -> None:
    """Destroys the communicator and the process group."""
    global _state
    if _state is not None:
        from . import psum_sgd
        psum_sgd.close_all()  # peers' buffers unmapped while every rank is still here
        barrier()
        if _state.comm:
            call("j4c_comm_destroy", _state.comm)
        _state = None
    if dist.is_initialized():
        dist.destroy_process_group()
