"""pmap across GPUs: in-process (one host thread per GPU, NCCL communicators
from ncclCommInitAll) and one process per GPU (torchrun, NCCL group with a
host heartbeat).  Skipped when fewer than two GPUs are visible."""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as orc
from tests.util import TOL_REDUCTION, assert_rel

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _ngpus():
    import torch
    return torch.cuda.device_count()


needs2 = pytest.mark.skipif("_ngpus() < 2", reason="needs two GPUs")


@needs2
def test_in_process_pmap_over_two_gpus():
    import jax4j_b200 as J
    devices = [J.Device.cuda(0), J.Device.cuda(1)]
    # PmapTest.java:68-76 / :92-100 / :118-138 with one shard per GPU
    x = J.ConcreteNDArray.of(np.float32([[10, 20], [10, 20]]))
    r = J.JAX.pmap(lambda s: J.Lax.psum(s), devices)(x)
    np.testing.assert_allclose(r.toFloatArray(), [20, 40, 20, 40], atol=1e-5)
    x = J.ConcreteNDArray.of(np.float32([[1, 2], [3, 4]]))
    r = J.JAX.pmap(lambda s: J.Lax.allGather(s, 2).sum(), devices)(x)
    np.testing.assert_allclose(r.toFloatArray(), [10, 10], atol=1e-5)
    two = J.ConcreteNDArray.scalar(2.0)
    fn = lambda v: J.JAX.pmap(lambda s: J.Lax.psum(s.mul(s).sum()).div(two), devices)(v).sum()
    np.testing.assert_allclose(J.JAX.grad(fn)(x).toFloatArray(), [2, 4, 6, 8], atol=1e-3)
    # the reduce-scatter ALL_GATHER VJP over NCCL (ncclReduceScatter)
    from jax4j_b200 import pmap as P
    c = J.ConcreteNDArray.of(np.float32([[1, 2], [3, 4]]))
    old = P.ALLGATHER_VJP
    try:
        J.Lax.setAllGatherVjp("reduce_scatter")
        fn = lambda v: J.JAX.pmap(lambda s: J.Lax.allGather(s, 2).mul(c).sum(), devices)(v).sum()
        np.testing.assert_allclose(J.JAX.grad(fn)(x).toFloatArray(), [2, 4, 6, 8], atol=1e-5)
    finally:
        P.ALLGATHER_VJP = old


def _torchrun(scenario, out, env_extra=None, timeout=240):
    env = dict(os.environ)
    env.update(env_extra or {})
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(29600 + (os.getpid() + 37 * len(scenario)) % 300),
           os.path.join(ROOT, "tests", "spmd_gpu_worker.py"), "--scenario", scenario, "--out", out]
    return subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout)


@needs2
def test_one_process_per_gpu_dp_step_matches_oracle(tmp_path):
    out = str(tmp_path / "dp.npz")
    r = _torchrun("dp_step", out)
    assert r.returncode == 0, r.stderr[-2000:]
    z = np.load(out)
    z1 = np.load(out + ".rank1.npz")
    ws, bs = [z["w1"], z["w2"]], [z["b1"], z["b2"]]
    per = [orc.mlp_loss_grad(ws, bs, z["x"], z["t"], act="tanh", threads=8),
           orc.mlp_loss_grad(ws, bs, z1["x"], z1["t"], act="tanh", threads=8)]
    np.testing.assert_allclose(z["losses"], [per[0][0], per[1][0]], rtol=TOL_REDUCTION)
    for i, k in enumerate(["w1", "w2"]):
        assert_rel(z["g_" + k], orc.psum([per[0][1][i], per[1][1][i]]), TOL_REDUCTION, k)
    for i, k in enumerate(["b1", "b2"]):
        assert_rel(z["g_" + k], orc.psum([per[0][2][i], per[1][2][i]]), TOL_REDUCTION, k)


@needs2
def test_one_process_per_gpu_grad_wrt_sharded_input(tmp_path):
    """JAX.grad of a pmap'd loss w.r.t. a LocalShard input: every rank gets
    the full [D, B, 64] cotangent, each slice equal to that shard's own gx."""
    out = str(tmp_path / "gx")
    r = _torchrun("grad_x", out)
    assert r.returncode == 0, r.stderr[-2000:]
    z = [np.load(out + f".rank{k}.npz") for k in range(2)]
    ws, bs = [z[0]["w1"], z[0]["w2"]], [z[0]["b1"], z[0]["b2"]]
    for k in range(2):
        for shard in range(2):
            ref = orc.mlp_loss_grad(ws, bs, z[shard]["x"], z[shard]["t"], act="tanh", want_gx=True,
                                    threads=4)[3]
            assert_rel(z[k]["gx"][shard], ref, TOL_REDUCTION, f"rank {k} shard {shard}")


@needs2
def test_rank_leaving_between_steps_is_reported_on_the_host(tmp_path):
    out = str(tmp_path / "leave.txt")
    r = _torchrun("leave", out, {"J4C_HEARTBEAT_S": "5", "NCCL_NVLS_ENABLE": "0"})
    assert os.path.exists(out), r.stderr[-2000:]
    assert open(out).read().startswith("CollectiveError")


@needs2
def test_psum_sgd_tree_fused_over_peer_memory_equals_psum_then_update(tmp_path):
    """Lax.psumSgdTree over two processes takes the fused path (the
    gradients summed out of the peer's memory, the update applied to each
    rank's slice, the slices gathered back) and, over three steps with three
    buckets (one cut at 16 leaves), gives the same bits as psumTree followed
    by the elementwise update: with two ranks the sum g0 + g1 is NCCL's too."""
    out = str(tmp_path / "psgd")
    r = _torchrun("psum_sgd", out, {"J4C_PSUM_SGD": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    z = [np.load(out + f".rank{k}.npz") for k in range(2)]
    for k in range(2):
        assert int(z[k]["status"]) == 0
        n = len([f for f in z[k].files if f.startswith("f")])
        assert n == 23
        for i in range(n):
            np.testing.assert_array_equal(z[k][f"f{i}"], z[k][f"r{i}"], err_msg=f"rank {k} leaf {i}")
            np.testing.assert_array_equal(z[k][f"f{i}"], z[0][f"f{i}"], err_msg=f"rank {k} leaf {i} vs rank 0")


@needs2
def test_psum_sgd_wait_runs_out_with_a_status(tmp_path):
    """Rank 0 runs the fused update while rank 1 stays on the host: rank 0's
    waits on flags that nothing sets run out after the 1 ms limit, and the
    kernels record status 0x7C05 and return (no fault, no hang)."""
    out = str(tmp_path / "ps_timeout.txt")
    r = _torchrun("psum_sgd_timeout", out, {"NCCL_NVLS_ENABLE": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert int(open(out).read()) == 0x7C05
