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
from dataclasses import dataclass
from typing import List, Optional

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


_state: Optional[SpmdState] = None


def state() -> Optional[SpmdState]:
    return _state


def initialize(timeout_s: float = 120.0) -> SpmdState:
    """Joins the job described by RANK/WORLD_SIZE/LOCAL_RANK/MASTER_ADDR/MASTER_PORT."""
    global _state
    if _state is not None:
        return _state
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local_rank)
    local = Device.cuda(local_rank)
    Device.setDefault(local)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s))
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
    comms = [None] * world
    comms[0] = comm.value
    # The collective object is indexed by PmapContext.deviceIndex (= rank);
    # every index resolves to this process's own communicator.
    coll = NcclCollective([comm.value] * world)
    devices = [local if r == rank else Device(None, f"rank{r}") for r in range(world)]
    _state = SpmdState(rank, world, local_rank, comm.value, coll, devices)
    return _state


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
        call("j4c_comm_destroy", _state.comm)
        _state = None
    if dist.is_initialized():
        dist.destroy_process_group()
