"""The one-process-per-GPU pmap path (jax4j_b200.distributed + pmap.py) as
world_size-2 `gloo` process groups on CPU.

What runs here is the executor's host logic: each rank takes its shard
(global arrays or LocalShard), PmapContext is set, Lax.psum / Lax.allGather
dispatch to the rank's collective, the stacked output is an all-gather, and
failures surface within a deadline instead of hanging.  The collective is a
gloo stand-in defined in this file (CPU tensors, no kernels); the product's
collective is NCCL (j4c_psum), covered by the 2-GPU tests.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class GlooCollective:
    """psum / allGather of ConcreteNDArrays backed by CPU tensors, over gloo."""

    def __init__(self, rank, world):
        self.rank, self.world = rank, world

    def abort(self):
        pass

    def psum(self, index, x):
        from jax4j_b200 import ConcreteNDArray
        t = x.tensor().clone()
        dist.all_reduce(t)
        return ConcreteNDArray._wrap(t, x.shape(), x.dtype(), x.device())

    def allGather(self, index, x):
        from jax4j_b200 import ConcreteNDArray, Shape
        parts = [torch.empty_like(x.tensor()) for _ in range(self.world)]
        dist.all_gather(parts, x.tensor().contiguous())
        return ConcreteNDArray._wrap(torch.cat(parts), Shape((self.world,) + x.shape().dimensions()),
                                     x.dtype(), x.device())


def _cpu_array(values, shape):
    from jax4j_b200 import ConcreteNDArray, Device, DType, Shape
    t = torch.tensor(values, dtype=torch.float32).reshape(-1)
    return ConcreteNDArray._wrap(t, Shape(shape), DType.FLOAT32, Device.defaultDevice())


def _worker(rank, world, port, scenario, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), J4C_HEARTBEAT_S="4")
    try:
        from jax4j_b200 import JAX, Lax, LocalShard, distributed
        st = distributed.initialize(timeout_s=5.0, collective_factory=GlooCollective)
        devices = distributed.global_devices()
        assert len(devices) == world and devices[rank] is st.devices[rank]
        if scenario == "psum_global_input":
            # a [D, 3] global input: rank r runs shard r; psum adds the shards
            x = _cpu_array([1, 2, 3, 10, 20, 30], [2, 3])
            out = JAX.pmap(lambda s: Lax.psum(s), devices)(x)
            q.put((rank, "ok", out.tensor().tolist(), list(out.shape().dimensions())))
        elif scenario == "local_shard_allgather":
            local = _cpu_array([rank * 10.0 + i for i in range(4)], [4])
            out = JAX.pmap(lambda s: Lax.allGather(s, world), devices)(LocalShard(local, world))
            q.put((rank, "ok", out.tensor().tolist(), list(out.shape().dimensions())))
        elif scenario == "rank_fails_before_psum":
            x = _cpu_array([1, 2, 3, 4], [2, 2])

            def body(s):
                if rank == 1:
                    raise ValueError("shard 1 failed before psum")
                return Lax.psum(s)

            t0 = time.time()
            try:
                JAX.pmap(body, devices)(x)
                q.put((rank, "no error", None, time.time() - t0))
            except Exception as e:  # noqa: BLE001
                q.put((rank, type(e).__name__, str(e)[:200], time.time() - t0))
        elif scenario == "rank_leaves_between_steps":
            x = _cpu_array([1, 2, 3, 4], [2, 2])
            JAX.pmap(lambda s: Lax.psum(s), devices)(x)  # step 1: both ranks
            if rank == 1:
                q.put((rank, "left", None, None))
                q.close()
                q.join_thread()
                os._exit(0)  # leaves between steps, nothing in flight
            t0 = time.time()
            try:
                JAX.pmap(lambda s: Lax.psum(s), devices)(x)
                q.put((rank, "no error", None, time.time() - t0))
            except Exception as e:  # noqa: BLE001
                q.put((rank, type(e).__name__, str(e)[:200], time.time() - t0))
        elif scenario == "mismatched_psum":
            # rank r all-reduces 2 + r elements: every rank must get an error
            # naming both signatures, before any collective is enqueued
            from jax4j_b200 import ConcreteNDArray, Device, DType, Shape, distributed as dd
            n = 2 + rank
            local = _cpu_array([1.0] * n, [n])
            t0 = time.time()
            try:
                JAX.pmap(lambda s: Lax.psum(s), devices)(LocalShard(local, world))
                q.put((rank, "no error", None, time.time() - t0))
            except Exception as e:  # noqa: BLE001
                q.put((rank, type(e).__name__, str(e)[:300], time.time() - t0))
        elif scenario == "matched_psum_checked_once":
            from jax4j_b200 import distributed as dd
            calls = []
            real = dist.all_gather_object

            def counting(*a, **k):
                calls.append(1)
                return real(*a, **k)

            dist.all_gather_object = counting
            local = _cpu_array([float(rank)] * 3, [3])
            outs = [JAX.pmap(lambda s: Lax.psum(s), devices)(LocalShard(local, world)) for _ in range(3)]
            dist.all_gather_object = real
            sig = ("psum", "FLOAT32", (3,))
            q.put((rank, "ok", [o.tensor().tolist() for o in outs], (len(calls), sig in dd.state().verified)))
        elif scenario == "max_over_ranks":
            t = torch.tensor([float(rank + 1)], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            q.put((rank, "ok", float(t.item()), None))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "crash", repr(e), None))
    finally:
        try:
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(scenario, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + timeout
    while len(results) < world and time.time() < deadline:
        try:
            r = q.get(timeout=1)
            results[r[0]] = r[1:]
        except Exception:  # noqa: BLE001
            pass
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    return results


def test_spmd_psum_of_global_input():
    res = _run("psum_global_input")
    assert set(res) == {0, 1}
    for r in (0, 1):
        status, values, shape = res[r]
        assert status == "ok", values
        assert shape == [2, 3]
        # every rank sees the stacked [psum, psum] (PmapTest.java:68-76 pattern)
        assert values == [11, 22, 33, 11, 22, 33]


def test_spmd_local_shards_all_gather():
    res = _run("local_shard_allgather")
    for r in (0, 1):
        status, values, shape = res[r]
        assert status == "ok", values
        assert shape == [2, 2, 4]
        assert values == [0, 1, 2, 3, 10, 11, 12, 13] * 2


def test_spmd_failed_rank_surfaces_within_deadline():
    res = _run("rank_fails_before_psum")
    assert res[1][0] == "ValueError" and "shard 1 failed" in res[1][1]
    # the surviving rank does not hang in its psum: the collective's deadline ends it
    assert res[0][0] != "no error"
    assert res[0][2] < 30


def test_spmd_peer_that_left_is_detected_before_the_next_collective():
    res = _run("rank_leaves_between_steps")
    assert res[1][0] == "left"
    status, msg, elapsed = res[0]
    assert status == "CollectiveError", (status, msg)
    assert elapsed < 30


def test_spmd_mismatched_collective_sizes_raise_on_every_rank():
    res = _run("mismatched_psum")
    assert set(res) == {0, 1}
    for r in (0, 1):
        status, msg, elapsed = res[r]
        assert status == "CollectiveError", (r, status, msg)
        assert "different collectives" in msg and "[2]" in msg and "[3]" in msg, msg
        assert elapsed < 30


def test_spmd_collective_signature_is_exchanged_once():
    res = _run("matched_psum_checked_once")
    for r in (0, 1):
        status, values, (n_exchanges, recorded) = res[r]
        assert status == "ok", values
        assert values == [[1.0] * 6] * 3  # stacked [psum, psum] of ranks 0 and 1
        # the psum's signature once, the pmap output's all-gather once
        assert n_exchanges == 2 and recorded


def test_spmd_timing_is_max_over_ranks():
    res = _run("max_over_ranks")
    assert res[0][1] == 2.0 and res[1][1] == 2.0
