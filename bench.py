#!/usr/bin/env python
"""Headline benchmark: the pmap'd data-parallel grad step of jax4j.

Workload (one step per GPU): a 4-layer relu MLP 1024-4096-4096-4096-1000 with
Glorot-uniform weights (seed 3) and zero biases, softmax cross-entropy on a
batch of 8192 samples x ~ N(0,1) with one-hot labels uniform in [0, 1000)
(seeded SplitMix64 streams of the reference's Random), gradients over the
{w1,b1,...,w4,b4} pytree by JAX.valueAndGradTree inside JAX.pmap, psum
averaged over the D ranks (one NCCL all-reduce of all 41.9M gradients), then
an SGD update.  One process per GPU; weak scaling (8192 samples per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0).  `value` is device-timed throughput with the
inputs resident in HBM; `e2e` repeats the step through the same public API
with the step's inputs copied from pinned host memory and the loss read back
every step.  `--impl reference` times the reference's CPU algorithm (the C
restatement under oracle/, all host threads) on a bounded sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DIMS = [1024, 4096, 4096, 4096, 1000]
BATCH = 8192
LR = 0.01
SEED_W, SEED_X, SEED_Y = 3, 1, 2
METRIC = "pmap grad-step samples/s"
WORKLOAD = ("dp grad step: 4-layer relu MLP 1024-4096-4096-4096-1000, softmax cross-entropy, "
            "batch 8192 per GPU, psum-averaged grads over the param pytree + SGD")


def flops_per_sample() -> float:
    """Forward 2*sum(d_i*d_{i+1}), dW for every layer, dX for layers 2..4."""
    fwd = sum(2 * DIMS[i] * DIMS[i + 1] for i in range(len(DIMS) - 1))
    dx = sum(2 * DIMS[i] * DIMS[i + 1] for i in range(1, len(DIMS) - 1))
    return 2 * fwd + dx


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--batch", type=int, default=BATCH, help="samples per GPU (profiling runs only)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-graph", action="store_true", help="time the eager step only (no CUDA graph)")
    p.add_argument("--no-secondary", action="store_true",
                   help="skip the configuration 0-3 measurements that ride along in the headline line")
    p.add_argument("--workload", default="dp_step", choices=["dp_step", "gemm", "dot64", "sweep", "cfg0", "cfg2", "collectives", "psum_sgd",
                                                   "fft", "linalg"],
                   help="dp_step is the headline; gemm/sweep are single-kernel measurements "
                        "used for profiling")
    p.add_argument("--m", type=int, default=8192)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--trans", default="nn", choices=["nn", "tn", "nt", "tt"],
                   help="gemm workload: whether A and B are stored transposed")
    p.add_argument("--max-bytes", type=int, default=1 << 30, help="collectives: largest message per rank")
    p.add_argument("--rows", type=int, default=4096)
    p.add_argument("--cols", type=int, default=16384)
    return p.parse_args()


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None
        self.skip = 0

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        # wait for the first sample, then count only the samples taken from here on
        deadline = time.time() + 3.0
        while time.time() < deadline and self.proc.poll() is None:
            self.file.flush()
            with open(self.file.name) as f:
                n = sum(1 for l in f if l.strip())
            if n:
                self.skip = n
                break
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        with open(self.file.name) as f:
            rows = [l.strip().split(", ") for l in f if l.strip()][self.skip:]
        os.unlink(self.file.name)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                for name, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    import jax4j_b200 as J
    from jax4j_b200 import _lib, core, distributed

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        st = distributed.initialize(timeout_s=120.0)
        rank, devices = st.rank, distributed.global_devices()
    else:
        torch.cuda.set_device(0)
        rank, devices = 0, [J.Device.defaultDevice()]
    D = len(devices)
    dev = J.Device.defaultDevice()
    B = args.batch
    ordinal = dev.ordinal()

    # ---- parameters (replicated: every rank draws the same streams) ----
    keys = J.Random.split(J.PRNGKey.key(SEED_W), len(DIMS) - 1)
    params = {}
    for i in range(len(DIMS) - 1):
        params[f"w{i + 1}"] = J.Random.glorotUniform(keys[i], J.Shape(DIMS[i], DIMS[i + 1]), DIMS[i], DIMS[i + 1])
        params[f"b{i + 1}"] = J.ConcreteNDArray.full(J.Shape(DIMS[i + 1]), 0.0)

    # ---- this rank's rows of the global batch ----
    x_loc = J.Random.normal(J.PRNGKey.key(SEED_X), J.Shape(D * B, DIMS[0]), offset=rank * B * DIMS[0],
                            count=B * DIMS[0]).reshape(J.Shape(B, DIMS[0]))
    u = J.Random.uniform(J.PRNGKey.key(SEED_Y), J.Shape(D * B), offset=rank * B, count=B)
    labels = torch.clamp((u.tensor() * DIMS[-1]).to(torch.int64), max=DIMS[-1] - 1)
    t_t = torch.zeros(B * DIMS[-1], dtype=torch.float32, device=dev.torch_device())
    t_t.view(B, DIMS[-1]).scatter_(1, labels.view(B, 1), 1.0)
    t_loc = J.ConcreteNDArray._wrap(t_t, J.Shape(B, DIMS[-1]), J.DType.FLOAT32, dev)

    neg = J.ConcreteNDArray.scalar(-1.0)
    names = list(params)

    def loss(p, x, t):
        c = p.children
        a = x
        for i in range(1, len(DIMS) - 1):
            a = a.dot(c[f"w{i}"].value).add(c[f"b{i}"].value).relu()
        L = len(DIMS) - 1
        logits = a.dot(c[f"w{L}"].value).add(c[f"b{L}"].value)
        return J.Nn.softmax(logits).log().mul(t).sum(-1).mean().mul(neg)

    def step_fn(xs_arr, ts_arr, *ps):
        """One training step as a function of its buffers:
        (x, one-hot targets, *params) -> [per-shard losses, *updated params]."""
        p = dict(zip(names, ps))
        new = {}

        def body(xs, ts):
            value, grads = J.JAX.valueAndGradTree(lambda tr: loss(tr, xs, ts))(J.PyTree.dictOf(p))
            # psum-averaged gradient and SGD update, w - (psum(g) * (1/D)) * lr:
            # psumTree (NCCL, bucketed, overlapped) + one update kernel per
            # parameter, or with J4C_PSUM_SGD=1 the exchange fused with the
            # update over peer memory (j4c_psum_sgd)
            upd = J.Lax.psumSgdTree(J.PyTree.dictOf(p), grads, 1.0 / D, LR).children
            for k in names:
                new[k] = upd[k].value
            return value

        if world > 1:
            ins = (J.LocalShard(xs_arr, D), J.LocalShard(ts_arr, D))
        else:
            ins = (xs_arr.reshape(J.Shape(1, B, DIMS[0])), ts_arr.reshape(J.Shape(1, B, DIMS[-1])))
        losses = J.JAX.pmap(body, devices)(*ins)
        return [losses] + [new[k] for k in names]

    state = {"params": [params[k] for k in names]}

    def step():
        outs = step_fn(x_loc, t_loc, *state["params"])
        state["params"] = outs[1:]
        return outs[0]

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    sync_all()

    # ---- eager steps, timed (per-dot CUDA events for the roofline) ----
    launches0 = _lib.kernel_launches()
    core.DOT_TIMING = []
    sync_all()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    h0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # enqueue time per step (no sync inside)
    ev1.record()
    torch.cuda.synchronize()
    eager_ms_local = ev0.elapsed_time(ev1)
    eager_launches = _lib.kernel_launches() - launches0
    dots = core.DOT_TIMING
    core.DOT_TIMING = None
    eager_ms = max_over_ranks(eager_ms_local)
    dot_ms = sum(a.elapsed_time(b) for a, b, _, _ in dots)
    dot_flop = sum(f for _, _, f, _ in dots)
    dot_bytes_per_launch = sum(n for _, _, _, n in dots) / len(dots) if dots else None

    # ---- the same step recorded once as a CUDA graph and replayed ----
    graphs, graph_note, per_replay = [], None, None
    if not args.no_graph:
        try:
            from jax4j_b200.graphs import CapturedStep
            nparam = len(names)
            donate = {1 + j: 2 + j for j in range(nparam)}
            graphs.append(CapturedStep(step_fn, [x_loc, t_loc] + state["params"], donate, warmup=1))
            per_replay = graphs[0].kernels  # this library's kernels recorded by the capture
            state["params"] = graphs[0].inputs[2:]
        except Exception as e:  # noqa: BLE001 - reported in the line, eager numbers stand
            graph_note = f"capture failed: {type(e).__name__}: {str(e)[:200]}"
            graphs = []

    def replay():
        return graphs[0]()[0]

    timed_step = replay if graphs else step
    for _ in range(args.warmup):
        timed_step()
    sync_all()

    # ---- device-timed region (inputs resident in HBM) ----
    clocks = ClockSampler(ordinal)
    clocks.start()
    sync_all()
    ev0.record()
    for _ in range(args.steps):
        timed_step()
    ev1.record()
    torch.cuda.synchronize()
    ms_local = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    ms = max_over_ranks(ms_local)
    value = D * B * args.steps / (ms / 1e3)
    launches = per_replay * args.steps if graphs else eager_launches

    # ---- end to end: host inputs copied in, loss read back, every step ----
    e2e = None
    if not args.no_e2e:
        # Every step's x and one-hot targets are copied from pinned host
        # memory and every step's loss is read back to the host, as a
        # training loop does with a prefetching input pipeline: step i+1's
        # inputs go to the GPU on a copy stream (into the other of two
        # device slots) while step i computes, and step i's loss is read
        # once step i+1 has been launched.
        x_host = torch.empty(B * DIMS[0], dtype=torch.float32, pin_memory=True)
        t_host = torch.empty(B * DIMS[-1], dtype=torch.float32, pin_memory=True)
        x_host.copy_(x_loc.tensor().cpu())
        t_host.copy_(t_loc.tensor().cpu())
        h2d = (x_host.numel() + t_host.numel()) * 4
        slots = []
        for _ in range(2):
            xs = J.ConcreteNDArray._wrap(x_loc.tensor().clone(), J.Shape(B, DIMS[0]), J.DType.FLOAT32, dev)
            ts = J.ConcreteNDArray._wrap(t_loc.tensor().clone(), J.Shape(B, DIMS[-1]), J.DType.FLOAT32, dev)
            slots.append((xs, ts))
        slot_graphs = []
        if graphs:
            # one recorded step per input slot, both on the shared parameter buffers
            slot_graphs = [None, None]
            for k in range(2):
                slot_graphs[k] = CapturedStep(step_fn, [slots[k][0], slots[k][1]] + state["params"], donate,
                                              warmup=1)
        copy_stream = torch.cuda.Stream()
        compute = torch.cuda.current_stream()
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        loss_host = [torch.empty(D, dtype=torch.float32, pin_memory=True) for _ in range(2)]
        used = [False, False]

        def issue_copy(i):
            k = i % 2
            if used[k]:
                copy_stream.wait_event(free[k])
            xs, ts = slots[k]
            _lib.call("j4c_memcpy_h2d", xs.data_ptr(), x_host.data_ptr(), x_host.numel() * 4, copy_stream.cuda_stream)
            _lib.call("j4c_memcpy_h2d", ts.data_ptr(), t_host.data_ptr(), t_host.numel() * 4, copy_stream.cuda_stream)
            ready[k].record(copy_stream)

        def inputs_of(k):
            # fresh wrappers each step: the slot buffers are rewritten in place
            return [J.ConcreteNDArray._wrap(a.tensor(), a.shape(), a.dtype(), dev) for a in slots[k]]

        losses = []
        sync_all()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        issue_copy(0)
        for i in range(args.steps):
            k = i % 2
            compute.wait_event(ready[k])
            if slot_graphs:
                res = slot_graphs[k]()[0]
            else:
                res = step_fn(*inputs_of(k), *state["params"])
                state["params"] = res[1:]
                res = res[0]
            free[k].record(compute)
            used[k] = True
            if i + 1 < args.steps:
                issue_copy(i + 1)
            loss_host[k].copy_(res.tensor()[:D], non_blocking=True)
            done[k].record(compute)
            if i > 0:
                done[(i - 1) % 2].synchronize()
                losses.append(float(loss_host[(i - 1) % 2][0]))
        done[(args.steps - 1) % 2].synchronize()
        losses.append(float(loss_host[(args.steps - 1) % 2][0]))
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
        e2e = {"value": D * B * args.steps / (e2e_ms / 1e3), "unit": "samples/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4 * D,
               "ms_per_step": e2e_ms / args.steps, "loss": losses[-1],
               "pipeline": "inputs of step i+1 copied on a second stream during step i; "
                           "loss of step i read after step i+1 is launched"}
        for g in slot_graphs:
            g.release()

    replayed = bool(graphs)
    for g in graphs:
        g.release()  # before the process group goes away (a graph may hold NCCL work)
    graphs = []
    secondary = None
    if not args.no_secondary:
        # configurations 0-3, a few seconds each, on the same ranks (every rank
        # takes the same collective steps; rank 0 keeps the results)
        secondary = measure_secondary(args)
    if rank != 0:
        if world > 1:
            distributed.barrier()
            distributed.shutdown()
        return
    peaks = _measured_peaks()
    peak, peak_source = _tensor_peak(peaks, ms / 1e3)
    achieved = (dot_flop / (dot_ms / 1e3)) / 1e12 if dot_ms > 0 else None
    from jax4j_b200.core import split_kind
    f16 = split_kind() == 1
    # the three tensor-core products each FP32 product issues, against the dense rate of their kind
    mma_peak = (peak if f16 else peak / 2) if peak else None
    traffic = GEMM_DRAM_BYTES_PER_LAUNCH.get("fp16" if f16 else "tf32") if B == BATCH else None
    line = {
        "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": D, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded SplitMix64 streams (Random.normal/uniform), Glorot weights",
        "config": {"workload": WORKLOAD, "model": "mlp-1024-4096x3-1000-relu", "global_batch": D * B,
                   "per_gpu_batch": B, "parallelism": f"dp{D}",
                   "gradient_update": update_path(D),
                   "l2": "working set (167 MB params + >400 MB activations) exceeds the 126 MB L2"},
        "roofline": {"bound": "tensor",
                     "kernel": "dot (FP32 via 3xFP16 split, power-of-two scaled)" if f16
                               else "dot (FP32 via 3xTF32 split)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": (achieved / peak) if (achieved and peak) else None,
                     "peak_source": peak_source,
                     "dot_share_of_step": dot_ms / eager_ms_local if eager_ms_local else None,
                     "mma_issued": {"kind": "f16" if f16 else "tf32",
                                    "achieved": 3 * achieved if achieved else None, "peak": mma_peak,
                                    "frac": (3 * achieved / mma_peak) if (achieved and mma_peak) else None},
                     "algorithmic_bytes_per_launch": dot_bytes_per_launch,
                     "traffic": traffic,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum over the 11 GEMM "
                                       "launches of one step at batch 8192, averaged per launch "
                                       "(single-pass capture, cold L2)"},
        "gpu_launches": launches,
        "execution": ("CUDA graph replay of the recorded step (%d kernels per step)" % per_replay) if replayed
                     else "eager",
        "eager": {"ms_per_step": eager_ms / args.steps, "value": D * B * args.steps / (eager_ms / 1e3),
                  "gpu_launches": eager_launches},
        "host_enqueue_ms_per_step": host_ms,
        "clocks": clk,
        "timed_region_s": ms / 1e3,
        "flops_per_sample": flops_per_sample(),
    }
    if graph_note:
        line["graph_note"] = graph_note
    if e2e:
        line["e2e"] = e2e
    if D == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if secondary is not None:
        line["secondary"] = secondary
    print(json.dumps(line), flush=True)
    if world > 1:
        distributed.barrier()
        distributed.shutdown()


# DRAM bytes per GEMM launch of the batch-8192 step, from ncu captures of its
# 11 GEMM launches (dram__bytes_read.sum + dram__bytes_write.sum, averaged),
# per operand split kind: 3xFP16 with CTA-pair tiles (the default), 3xTF32
# with single-CTA tiles.
GEMM_DRAM_BYTES_PER_LAUNCH = {"tf32": 1.0663e9, "fp16": 4.747e8}


SUSTAINED_AFTER_S = 1.0  # timed regions at least this long are compared with the sustained peak


def _tensor_peak(peaks: dict, timed_s: float):
    """The bf16 denominator for a tensor-bound kernel, chosen by the length of
    the timed region: the burst figure (a short run, as the burst cuBLAS GEMM
    was timed) below SUSTAINED_AFTER_S, the sustained (seconds-long, power
    capped) figure above it."""
    burst, sustained = peaks.get("bf16_tflops"), peaks.get("bf16_tflops_sustained")
    src = peaks.get("source", "MEASURED_PEAKS.json")
    if sustained and timed_s >= SUSTAINED_AFTER_S:
        return sustained, (f"{src} bf16 sustained (timed region {timed_s:.2f} s >= {SUSTAINED_AFTER_S} s); "
                           "FP16 dense rate equal, TF32 half")
    return burst, (f"{src} bf16 burst (timed region {timed_s:.2f} s < {SUSTAINED_AFTER_S} s); "
                   "FP16 dense rate equal, TF32 half")


def _measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# the reference's CPU algorithm (oracle restatement), bounded samples
# ---------------------------------------------------------------------------
def _cpu_case(samples: int):
    import numpy as np
    from oracle import oracle as orc
    keys = orc.split(SEED_W, len(DIMS) - 1)
    ws = [orc.glorot_uniform(keys[i], (DIMS[i], DIMS[i + 1]), DIMS[i], DIMS[i + 1])
          for i in range(len(DIMS) - 1)]
    bs = [np.zeros(DIMS[i + 1], np.float32) for i in range(len(DIMS) - 1)]
    x = orc.normal(SEED_X, (samples * DIMS[0],)).reshape(samples, DIMS[0])
    lab = np.minimum((orc.uniform(SEED_Y, (samples,)) * DIMS[-1]).astype(np.int64), DIMS[-1] - 1)
    t = np.zeros((samples, DIMS[-1]), np.float32)
    t[np.arange(samples), lab] = 1
    return ws, bs, x, t


CPU_SLICE = 512        # samples of the batch the CPU arms time (CPU-N: all host threads)
CPU_SLICE_SERIAL = 32  # samples the reference's own threading (one-thread dot) is timed on


def _cpu_step(samples: int, threads: int) -> float:
    """Seconds of one grad step of the oracle's restatement of the
    reference's host path on `samples` samples of the batch."""
    from oracle import oracle as orc
    ws, bs, x, t = _cpu_case(samples)
    t0 = time.perf_counter()
    orc.mlp_loss_grad(ws, bs, x, t, act="relu", threads=threads)
    return time.perf_counter() - t0


def cpu_baseline() -> dict:
    """The oracle's restatement of the reference's host grad step on a fixed
    slice of the batch (CPU_SLICE samples) with its dot row-parallel over
    all host threads (the reference's CPU-N mode, BackendBenchmark.java:
    281-291, bit-identical to its serial loop), and beside it the
    reference's own threading -- the dot on one thread (ConcreteNDArray.java:
    452-459), elementwise work parallel -- on CPU_SLICE_SERIAL samples."""
    from oracle import oracle as orc
    threads = orc.nproc()
    dt = _cpu_step(CPU_SLICE, threads)
    dt1 = _cpu_step(CPU_SLICE_SERIAL, 1)
    return {"value": CPU_SLICE / dt, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{CPU_SLICE} samples of the batch, one grad step of the same model (sequential-k "
                      f"float dot, row-parallel over {threads} threads: the reference's CPU-N mode)",
            "reference_threading": {"value": CPU_SLICE_SERIAL / dt1, "unit": "samples/s", "cores": 1,
                                    "sample": f"{CPU_SLICE_SERIAL} samples, dot on one thread as the "
                                              "reference's ConcreteNDArray.dot runs it"}}


def run_reference(args):
    """The reference's CPU algorithm (the oracle's C restatement of its host
    path) with all host threads, each step one grad step on the fixed
    CPU_SLICE samples of the headline batch; rank 0 alone under torchrun."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as orc
    threads = orc.nproc()
    ws, bs, x, t = _cpu_case(CPU_SLICE)
    for _ in range(args.warmup):
        orc.mlp_loss_grad(ws, bs, x, t, act="relu", threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.mlp_loss_grad(ws, bs, x, t, act="relu", threads=threads)
    el = time.perf_counter() - t0
    value = CPU_SLICE * args.steps / el
    dt1 = _cpu_step(CPU_SLICE_SERIAL, 1)
    line = {"metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "model": "mlp-1024-4096x3-1000-relu",
                       "global_batch": BATCH * world, "parallelism": f"dp{world}",
                       "cpu_slice": f"{CPU_SLICE} samples of the batch per step"},
            "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                             "sample": f"{CPU_SLICE} samples per step (the reference's host algorithm, "
                                       f"C restatement, row-parallel dot over {threads} threads)",
                             "reference_threading": {"value": CPU_SLICE_SERIAL / dt1, "unit": "samples/s",
                                                     "cores": 1,
                                                     "sample": f"{CPU_SLICE_SERIAL} samples, dot on one "
                                                               "thread"}},
            "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_dot64(args):
    """One FLOAT64 dot C[M,N] = op(A)[M,K].op(B)[K,N] per step through j4c_dot
    (the DMMA kernel; J4C_DOT64=simt selects the CUDA-core kernel), A and B
    ~ U(-1, 1), inputs resident.  Reported against the B200's nominal dense
    FP64 rate (no measured FP64 peak exists on this pool)."""
    import torch
    import jax4j_b200 as J
    from jax4j_b200._lib import call
    torch.cuda.set_device(0)
    M, K, N = args.m, args.k, args.n
    ta, tb = args.trans[0] == "t", args.trans[1] == "t"
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.rand((K, M) if ta else (M, K), dtype=torch.float64, device="cuda", generator=g) * 2 - 1
    B = torch.rand((N, K) if tb else (K, N), dtype=torch.float64, device="cuda", generator=g) * 2 - 1
    out = torch.empty(M * N, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    fn = lambda: call("j4c_dot", 1, A.data_ptr(), B.data_ptr(), out.data_ptr(), M, K, N, int(ta), int(tb), stream)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ref = (A.t() if ta else A) @ (B.t() if tb else B)
    err = float((out.view(M, N) - ref).abs().max() / ref.abs().max())
    tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
    kernel = "simt" if os.environ.get("J4C_DOT64", "").startswith("s") else "dmma"
    print(json.dumps({"metric": "FLOAT64 dot TFLOP/s", "value": tf, "unit": "TFLOP/s", "ms_per_step": ms,
                      "kernel": kernel, "max_rel_diff_vs_torch": err, "dtype": "f64",
                      "config": {"workload": f"dot {M}x{K}x{N} op(A) op(B) = {args.trans}"},
                      "roofline": {"bound": "fp64", "achieved": tf, "peak": 40.0, "unit": "TFLOP/s",
                                   "frac": tf / 40.0, "peak_source": "nominal B200 dense FP64 (fallback)"}}),
          flush=True)


def run_gemm(args):
    """One FP32 dot C[M,N] = op(A)[M,K].op(B)[K,N] per step through j4c_dot_ws
    (both operand splits + the tcgen05 GEMM); the GEMM kernel alone is timed
    too, from cached splits."""
    import torch
    import jax4j_b200 as J
    from jax4j_b200 import core
    from jax4j_b200._lib import call, lib
    torch.cuda.set_device(0)
    M, K, N = args.m, args.k, args.n
    ta, tb = args.trans[0] == "t", args.trans[1] == "t"
    dev = J.Device.defaultDevice()
    A = J.Random.uniform(J.PRNGKey.key(2), J.Shape(*((K, M) if ta else (M, K))), -1.0, 1.0)
    B = J.Random.uniform(J.PRNGKey.key(3), J.Shape(*((N, K) if tb else (K, N))), -1.0, 1.0)
    ws_bytes = lib().j4c_dot_workspace_size(0, M, K, N)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty(M * N, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def full():
        call("j4c_dot_ws", 0, A.data_ptr(), B.data_ptr(), out.data_ptr(), M, K, N, int(ta), int(tb),
             ws.data_ptr(), ws_bytes, stream)

    def gemm_only():
        core._dot_raw(A, B, ta, tb, dev)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    ms = timed(full)
    gemm_ms = timed(gemm_only)
    flop = 2.0 * M * N * K
    from jax4j_b200.core import split_kind
    print(json.dumps({"metric": "dot TFLOP/s (FP32 accuracy, %s)" % ("3xFP16" if split_kind() == 1 else "3xTF32"),
                      "value": flop / (ms / 1e3) / 1e12,
                      "unit": "TFLOP/s", "ms_per_step": ms, "gemm_ms": gemm_ms,
                      "gemm_tflops": flop / (gemm_ms / 1e3) / 1e12,
                      "config": {"workload": f"dot {M}x{K}x{N} op(A){'T' if ta else ''} op(B){'T' if tb else ''}"},
                      "algorithmic_bytes": 4 * (M * K + K * N + M * N)}), flush=True)


SWEEP_ROWS, SWEEP_COLS = 4096, 16384


def _sweep_cpu(rows: int = 64) -> dict:
    """The oracle's restatement of the sweep (one thread) on `rows` rows."""
    from oracle import oracle as orc
    x = orc.normal(1, (rows * SWEEP_COLS,)).reshape(rows, SWEEP_COLS)
    y = orc.uniform(11, (rows * SWEEP_COLS,), -3.0, 3.0).reshape(rows, SWEEP_COLS)
    t0 = time.perf_counter()
    orc.sweep(x, y)
    dt = time.perf_counter() - t0
    n = rows * SWEEP_COLS
    return {"value": n / dt, "unit": "elements/s", "cores": 1, "kind": "port",
            "sample": f"{rows} rows x {SWEEP_COLS} of the sweep (where/tanh/sigmoid/clip + row sum + argmax), "
                      "one thread"}


def measure_sweep(args, quick: bool = False):
    """Config 1: z = where(x.gt(0), tanh(x)*sigmoid(y), relu(y).clip(-1,1)),
    z.sum(-1, keep) and z.argmax(-1) over this rank's [rows, cols] shard
    (x ~ N(0,1), y ~ U(-3,3)), one fused generated kernel via JAX.jit; no
    collective (each rank its own rows).  Returns rank 0's result."""
    import torch
    import jax4j_b200 as J
    from jax4j_b200 import grad as _g
    rank, world, _ = _spmd_setup()
    R, Cc = (SWEEP_ROWS, SWEEP_COLS) if quick else (args.rows, args.cols)
    x = J.Random.normal(J.PRNGKey.key(1), J.Shape(world * R, Cc), offset=rank * R * Cc,
                        count=R * Cc).reshape(J.Shape(R, Cc))
    y = J.Random.uniform(J.PRNGKey.key(11), J.Shape(world * R, Cc), -3.0, 3.0, offset=rank * R * Cc,
                         count=R * Cc).reshape(J.Shape(R, Cc))
    zero, lo, hi = (J.ConcreteNDArray.scalar(v) for v in (0.0, -1.0, 1.0))

    def sweep(xx, yy):
        z = J.Numpy.where(xx.gt(zero), xx.tanh().mul(yy.sigmoid()), yy.relu().clip(lo, hi))
        return z.sum(-1, True), z.argmax(-1)

    jitted = J.JAX.jit(sweep)
    steps = 10 if quick else args.steps

    def timed(fused: bool) -> float:
        _g.FUSION = fused
        try:
            return _timed(lambda: jitted(x, y), steps, max(3, args.warmup), world)
        finally:
            _g.FUSION = True

    ms_unfused = timed(False)
    ms = timed(True)
    # the fused launch replayed from a CUDA graph: device time without the
    # Python interpreter's per-call cost
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        jitted(x, y)
    ms_graph = _timed(graph.replay, 5 * steps, 3, world)
    del graph
    n = R * Cc
    min_bytes = 8 * n + 8 * R  # x, y read once; a sum and an argmax per row written
    if rank != 0:
        return None
    peaks = _measured_peaks()
    gbs = min_bytes / (ms_graph / 1e3) / 1e9
    out = {"metric": "config-1 sweep elements/s", "value": world * n / (ms_graph / 1e3), "unit": "elements/s",
           "n_gpus": world, "scaling": "weak", "ms_per_step": ms_graph, "ms_per_step_eager": ms,
           "ms_per_step_unfused": ms_unfused,
           "config": {"workload": f"where/tanh/sigmoid/clip + sum(-1) + argmax(-1), [{R},{Cc}] per GPU, "
                                  "fused (JAX.jit), CUDA graph replay"},
           "roofline": {"bound": "hbm", "kernel": "generated fused row kernel (fused.cu)", "achieved": gbs,
                        "peak": peaks.get("hbm_gbs"), "unit": "GB/s",
                        "frac": gbs / peaks["hbm_gbs"] if peaks.get("hbm_gbs") else None,
                        "traffic": None, "algorithmic_bytes_per_launch": min_bytes,
                        "peak_source": f"{peaks.get('source', 'MEASURED_PEAKS.json')} hbm_gbs (copy)"}}
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = _sweep_cpu()
    return out


def run_sweep(args):
    r = measure_sweep(args)
    if r is not None:
        print(json.dumps(r), flush=True)
    _finish(int(os.environ.get("WORLD_SIZE", "1")))


def run_fft(args):
    """Fft on the device: a 3-D complex transform of a 256^3 grid and a 1-D
    transform of 2^24 points, FLOAT32, resident real and imaginary arrays.
    Each input (128 MB) exceeds the 126 MB L2.  Roofline: HBM, with the
    minimum bytes of a transform = its inputs read once + outputs written
    once; the oracle (the reference's radix-2 transform) is timed on a 64^3
    grid beside it."""
    import numpy as np
    import torch
    import jax4j_b200 as J
    from oracle import oracle as orc
    torch.cuda.set_device(0)
    peaks = _measured_peaks()
    lines = []
    for shape, fn in (((256, 256, 256), J.Fft.fft3), ((1 << 24,), J.Fft.fft)):
        re = J.Random.normal(J.PRNGKey.key(21), J.Shape(shape))
        im = J.Random.normal(J.PRNGKey.key(22), J.Shape(shape))
        for _ in range(args.warmup):
            fn(re, im)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn(re, im)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        n = int(np.prod(shape))
        min_bytes = 16 * n  # re, im read + re, im written, 4 B each
        gbs = min_bytes / (ms / 1e3) / 1e9
        lines.append({"shape": list(shape), "ms": ms, "GBps_of_minimum_bytes": gbs,
                      "roofline_frac": gbs / peaks.get("hbm_gbs", 6650.0),
                      "gflops_5nlog2n": 5 * n * np.log2(n) / (ms / 1e3) / 1e9})
    # the reference's host algorithm (oracle restatement), one thread, on a 64^3 grid
    g = np.random.default_rng(0).standard_normal((2, 64, 64, 64)).astype(np.float32)
    t0 = time.perf_counter()
    orc.fft(g[0], g[1])
    cpu_s = time.perf_counter() - t0
    n_cpu = 64 ** 3
    print(json.dumps({"metric": "fft3 256^3 FP32 transforms/s", "value": 1e3 / lines[0]["ms"],
                      "unit": "transforms/s", "ms_per_step": lines[0]["ms"],
                      "config": {"workload": "Fft.fft3 on a 256^3 FP32 complex grid; Fft.fft of 2^24 points"},
                      "transforms": lines, "peak_hbm_GBps": peaks.get("hbm_gbs"),
                      "cpu_baseline": {"value": 1.0 / cpu_s, "unit": "transforms/s of a 64^3 grid",
                                       "cores": 1, "kind": "port",
                                       "sample": "the reference's radix-2 fft3 (oracle) on a 64^3 FP32 grid; "
                                                 f"{cpu_s * 1e3:.1f} ms, i.e. about "
                                                 f"{cpu_s * (256 ** 3 * 24) / (n_cpu * 18) * 1e3:.0f} ms "
                                                 "for 256^3 scaled by N log N"}}), flush=True)


B200_FP64_NOMINAL_TFLOPS = 40.0  # dense FP64 (tensor core) datasheet figure; no measured FP64 peak exists


def run_linalg(args):
    """Linalg on the device: Linalg.lu + LU.solve of an 8192 x 8192 FLOAT64
    system (a 512 MB matrix, above the 126 MB L2), then Linalg.cond, eig and
    svd at sizes the host algorithms take seconds on.  The factorisation is
    FP64 tensor-bound: 2/3 n^3 flops against the nominal FP64 peak.  e2e
    runs the same lu + solve from pinned host memory with the solution read
    back.  The oracle's restatement of the reference's unblocked elimination
    is timed beside it on n = 1024, one thread."""
    import numpy as np
    import torch
    import jax4j_b200 as J
    from oracle import oracle as orc
    torch.cuda.set_device(0)
    n = 8192
    rng = np.random.default_rng(5)
    a_host = torch.from_numpy(rng.standard_normal((n, n))).pin_memory()
    b_host = torch.from_numpy(rng.standard_normal(n)).pin_memory()
    A = J.ConcreteNDArray._wrap(a_host.view(-1).to("cuda"), J.Shape(n, n), J.DType.FLOAT64,
                                J.Device.defaultDevice())
    b = J.ConcreteNDArray._wrap(b_host.to("cuda"), J.Shape(n), J.DType.FLOAT64, J.Device.defaultDevice())

    def step():
        return J.Linalg.lu(A).solve(b)

    flops = 2.0 / 3.0 * n ** 3 + 2.0 * n * n
    ms = _timed(step, args.steps, args.warmup, 1)
    x = step().numpy()
    resid = float(np.abs(a_host.numpy() @ x - b_host.numpy()).max())

    dev = torch.device("cuda")
    x_host = torch.empty(n, dtype=torch.float64).pin_memory()

    def e2e_step():
        ad = a_host.view(-1).to(dev, non_blocking=True)
        bd = b_host.to(dev, non_blocking=True)
        Ad = J.ConcreteNDArray._wrap(ad, J.Shape(n, n), J.DType.FLOAT64, J.Device.defaultDevice())
        bb = J.ConcreteNDArray._wrap(bd, J.Shape(n), J.DType.FLOAT64, J.Device.defaultDevice())
        x_host.copy_(J.Linalg.lu(Ad).solve(bb).tensor(), non_blocking=True)

    e2e_ms = _timed(e2e_step, args.steps, args.warmup, 1)
    lu8 = J.Linalg.lu(A)
    cond_ms = _timed(lambda: J.Linalg.cond(lu8), 3, 1, 1)
    others = {"cond_hager_n8192_ms": cond_ms}
    m1 = J.ConcreteNDArray.of(rng.standard_normal((1024, 1024)), J.Shape(1024, 1024), J.DType.FLOAT64)
    others["eig_n1024_ms"] = _timed(lambda: J.Linalg.eig(m1), 2, 1, 1)
    m2 = J.ConcreteNDArray.of(rng.standard_normal((2048, 1024)), J.Shape(2048, 1024), J.DType.FLOAT64)
    others["svd_2048x1024_ms"] = _timed(lambda: J.Linalg.svd(m2), 2, 1, 1)

    nc = 1024
    ac = rng.standard_normal((nc, nc))
    t0 = time.perf_counter()
    st, lu_c, piv_c, _, _, _ = orc.lu_factor(ac)
    orc.lu_solve(lu_c, piv_c, rng.standard_normal(nc))
    cpu_s = time.perf_counter() - t0
    cpu_gflops = (2.0 / 3.0 * nc ** 3 + 2.0 * nc * nc) / cpu_s / 1e9
    achieved = flops / (ms / 1e3) / 1e12
    print(json.dumps({
        "metric": "lu + solve FP64 GFLOP/s (2/3 n^3 + 2 n^2)", "value": flops / (ms / 1e3) / 1e9, "unit": "GFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "f64", "data": "synthetic N(0,1) matrix and right-hand side",
        "config": {"workload": "Linalg.lu + LU.solve, n = 8192 FLOAT64 (512 MB matrix, above L2)"},
        "max_abs_residual": resid,
        "e2e": {"value": flops / (e2e_ms / 1e3) / 1e9, "unit": "GFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 8 * (n * n + n), "d2h_bytes_per_step": 8 * n},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": B200_FP64_NOMINAL_TFLOPS,
                     "unit": "TFLOP/s", "frac": achieved / B200_FP64_NOMINAL_TFLOPS,
                     "peak_source": "nominal B200 dense FP64 (no measured FP64 peak)", "traffic": None},
        "other_ops": others,
        "cpu_baseline": {"value": cpu_gflops, "unit": "GFLOP/s", "cores": 1, "kind": "port",
                         "sample": f"the reference's unblocked elimination + substitution (oracle) at n = {nc}: "
                                   f"{cpu_s * 1e3:.0f} ms"}}), flush=True)


# ---------------------------------------------------------------------------
# the other configurations: their own measurements (parity is in tests/)
# ---------------------------------------------------------------------------
def _spmd_setup():
    """(rank, world, devices) for this process: torchrun ranks or one GPU."""
    import torch
    import jax4j_b200 as J
    from jax4j_b200 import distributed
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        st = distributed.initialize(timeout_s=120.0)
        return st.rank, world, distributed.global_devices()
    torch.cuda.set_device(0)
    return 0, 1, [J.Device.defaultDevice()]


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed(fn, steps: int, warmup: int, world: int) -> float:
    """ms per call: device-timed on this rank's stream, max over ranks."""
    import torch
    from jax4j_b200 import distributed
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return _max_over_ranks(e0.elapsed_time(e1) / steps, world)


def _finish(world: int):
    from jax4j_b200 import distributed
    if world > 1:
        distributed.barrier()
        distributed.shutdown()


def measure_cfg0(args, quick: bool = False):
    """Config 0: 2-layer tanh MLP 784-512-10, x [2,256,784] ~ N(0,1) sharded
    over D = 2 pmap devices (two ranks, or two shards on one GPU).  (i) grad of
    pmap w.r.t. x; (ii) pmap of gradTree over {W1,b1,W2,b2} + psumTree.
    Each recorded as a CUDA graph and replayed; returns rank 0's result."""
    import torch
    import jax4j_b200 as J
    from jax4j_b200.graphs import CapturedStep
    rank, world, devices = _spmd_setup()
    if world == 1:
        devices = [J.Device.defaultDevice(), J.Device(None, "shard1")]
    elif world != 2:
        return {"note": "config 0 is defined on D = 2 pmap devices; it runs at 1 GPU (two shards) and 2 GPUs"} \
            if rank == 0 else None
    D = len(devices)
    B = 256
    keys = J.Random.split(J.PRNGKey.key(0), 3)
    params = {"w1": J.Random.glorotUniform(keys[0], J.Shape(784, 512), 784, 512),
              "b1": J.ConcreteNDArray.full(J.Shape(512), 0.0),
              "w2": J.Random.glorotUniform(keys[1], J.Shape(512, 10), 512, 10),
              "b2": J.ConcreteNDArray.full(J.Shape(10), 0.0)}
    x_all = J.Random.normal(J.PRNGKey.key(0), J.Shape(2, B, 784))
    lab = torch.clamp((J.Random.uniform(keys[2], J.Shape(2 * B)).tensor() * 10).to(torch.int64), max=9)
    t_t = torch.zeros(2 * B * 10, dtype=torch.float32, device="cuda")
    t_t.view(2 * B, 10).scatter_(1, lab.view(-1, 1), 1.0)
    t_all = J.ConcreteNDArray._wrap(t_t, J.Shape(2, B, 10), J.DType.FLOAT32, J.Device.defaultDevice())
    if world > 1:
        xa = J.ConcreteNDArray._wrap(x_all.tensor().view(2, -1)[rank].clone(), J.Shape(B, 784),
                                     J.DType.FLOAT32, J.Device.defaultDevice())
        ta = J.ConcreteNDArray._wrap(t_t.view(2, -1)[rank].clone(), J.Shape(B, 10), J.DType.FLOAT32,
                                     J.Device.defaultDevice())
    else:
        xa, ta = x_all, t_all
    neg = J.ConcreteNDArray.scalar(-1.0)

    def loss_fn(p, xs, ts):
        h = xs.dot(p["w1"]).add(p["b1"]).tanh()
        logits = h.dot(p["w2"]).add(p["b2"])
        return J.Nn.softmax(logits).log().mul(ts).sum(-1).mean().mul(neg)

    def wrap(a, b):
        return (J.LocalShard(a, D), J.LocalShard(b, D)) if world > 1 else (a, b)

    def fn_i(xx, tt):
        xi, ti = wrap(xx, tt)
        return [J.JAX.grad(lambda v: J.JAX.pmap(lambda xs, ts: loss_fn(params, xs, ts), devices)(v, ti).sum())(xi)]

    def fn_ii(xx, tt):
        xi, ti = wrap(xx, tt)
        outs = []

        def body(xs, ts):
            v, g = J.JAX.valueAndGradTree(
                lambda tr: loss_fn({k: tr.children[k].value for k in params}, xs, ts))(J.PyTree.dictOf(params))
            outs.extend(J.PyTrees.flatten(J.Lax.psumTree(g)))
            return v

        return [J.JAX.pmap(body, devices)(xi, ti)] + outs

    steps = 10 if quick else args.steps
    ms_i = _timed(lambda: fn_i(xa, ta), steps, max(3, args.warmup), world)
    ms_ii = _timed(lambda: fn_ii(xa, ta), steps, max(3, args.warmup), world)
    cs_i = CapturedStep(fn_i, [xa, ta])
    gms_i = _timed(cs_i, steps * 10, max(3, args.warmup), world)
    cs_i.release()
    cs_ii = CapturedStep(fn_ii, [xa, ta])
    gms_ii = _timed(cs_ii, steps * 10, max(3, args.warmup), world)
    cs_ii.release()
    if rank != 0:
        return None
    samples = 2 * B
    peaks = _measured_peaks()
    flop_ii = 1636352 * samples / (gms_ii / 1e3) / 1e12
    out = {"metric": "config-0 grad-step samples/s", "value": samples / (gms_ii / 1e3), "unit": "samples/s",
           "n_gpus": world,
           "config": {"workload": "2-layer tanh MLP 784-512-10, x [2,256,784], D=2 pmap devices; value = "
                                  "part (ii) gradTree + psumTree"},
           "grad_wrt_x": {"value": samples / (gms_i / 1e3), "ms_per_step": gms_i,
                          "eager_ms_per_step": ms_i, "flop_per_sample": 1626112},
           "grad_tree_psum": {"value": samples / (gms_ii / 1e3), "ms_per_step": gms_ii,
                              "eager_ms_per_step": ms_ii, "flop_per_sample": 1636352, "psum_floats": 407050},
           "execution": "CUDA graph replay of the recorded step (eager times beside)",
           "roofline": {"bound": "latency", "achieved": flop_ii, "peak": peaks.get("bf16_tflops"),
                        "unit": "TFLOP/s",
                        "frac": flop_ii / peaks["bf16_tflops"] if peaks.get("bf16_tflops") else None,
                        "note": "a 0.8 GFLOP step of 20-odd launches: bound by launch and kernel latency; "
                                "the tensor fraction is for information"}}
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = _cfg0_cpu(reps=2)
    return out


def run_cfg0(args):
    r = measure_cfg0(args)
    if r is not None:
        print(json.dumps(r), flush=True)
    _finish(int(os.environ.get("WORLD_SIZE", "1")))


def _cfg0_cpu(reps: int = 10) -> dict:
    import numpy as np
    from oracle import oracle as orc
    keys = orc.split(0, 3)
    ws = [orc.glorot_uniform(keys[0], (784, 512), 784, 512), orc.glorot_uniform(keys[1], (512, 10), 512, 10)]
    bs = [np.zeros(512, np.float32), np.zeros(10, np.float32)]
    x = orc.normal(0, (2 * 256 * 784,)).reshape(2, 256, 784)
    lab = np.minimum((orc.uniform(keys[2], (512,)) * 10).astype(np.int64), 9)
    t = np.zeros((512, 10), np.float32)
    t[np.arange(512), lab] = 1
    t = t.reshape(2, 256, 10)
    threads = orc.nproc()
    t0 = time.perf_counter()
    for _ in range(reps):
        for d in range(2):  # the two shards, as the reference's pmap runs them
            orc.mlp_loss_grad(ws, bs, x[d], t[d], act="tanh", threads=threads)
    dt = time.perf_counter() - t0
    return {"value": 512 * reps / dt, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{reps} full steps (both shards, grad over the params), row-parallel dot"}


def _cfg2_cpu(rows: int = 16) -> dict:
    """The oracle's sequential-k dot on `rows` rows of a shard's product,
    row-parallel over all host threads (the reference's CPU-N matmul)."""
    from oracle import oracle as orc
    K, N = 8192, 4096
    a = orc.uniform(2, (rows * K,), -1.0, 1.0).reshape(rows, K)
    b = orc.uniform(orc.split(2, 2)[1], (K * N,), -1.0, 1.0).reshape(K, N)
    threads = orc.nproc()
    t0 = time.perf_counter()
    orc.dot(a, b, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": 2.0 * rows * K * N / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} rows of a shard's [4096,8192].[8192,4096] product, row-parallel dot"}


def measure_cfg2(args, quick: bool = False):
    """Config 2: each shard computes A_i [4096,8192] . B [8192,4096]
    (A ~ U(-1,1) sharded on the leading axis, B replicated, seed 2) and the
    results are gathered with Lax.allGather.  Returns rank 0's result."""
    import jax4j_b200 as J
    from jax4j_b200 import core
    from jax4j_b200.core import split_kind
    rank, world, devices = _spmd_setup()
    D = len(devices)
    M, K, N = 4096, 8192, 4096
    A = J.Random.uniform(J.PRNGKey.key(2), J.Shape(D * M, K), -1.0, 1.0, offset=rank * M * K,
                         count=M * K).reshape(J.Shape(M, K))
    B = J.Random.uniform(J.Random.split(J.PRNGKey.key(2), 2)[1], J.Shape(K, N), -1.0, 1.0)
    a_in = J.LocalShard(A, D) if world > 1 else A.reshape(J.Shape(1, M, K))
    pm = J.JAX.pmap(lambda a: J.Lax.allGather(a.dot(B), D), devices)
    steps = 10 if quick else args.steps
    core.DOT_TIMING = []
    ms = _timed(lambda: pm(a_in), steps, max(3, args.warmup), world)
    dots = core.DOT_TIMING[-steps:]
    core.DOT_TIMING = None
    gemm_ms = sum(a.elapsed_time(b) for a, b, _, _ in dots) / max(1, len(dots))
    if rank != 0:
        return None
    flop = 2.0 * M * K * N
    peaks = _measured_peaks()
    f16 = split_kind() == 1
    peak, src = _tensor_peak(peaks, ms * steps / 1e3)
    ach = flop / (gemm_ms / 1e3) / 1e12
    mma_peak = peak if f16 else peak / 2
    out = {"metric": "config-2 pmap dot + allGather TFLOP/s", "unit": "TFLOP/s",
           "value": D * flop / (ms / 1e3) / 1e12, "ms_per_step": ms, "n_gpus": world, "scaling": "weak",
           "config": {"workload": "per shard [4096,8192].[8192,4096] FP32 (tensor-core split GEMM, "
                                  + ("3xFP16" if f16 else "3xTF32") + "), allGather of the [4096,4096] results"},
           "allgather_bytes_per_rank": 4 * M * N,
           "roofline": {"bound": "tensor", "kernel": "dot (gemm_3xtf32_kernel)", "achieved": ach, "peak": peak,
                        "unit": "TFLOP/s", "frac": ach / peak, "peak_source": src, "gemm_ms": gemm_ms,
                        "mma_issued": {"kind": "f16" if f16 else "tf32", "achieved": 3 * ach, "peak": mma_peak,
                                       "frac": 3 * ach / mma_peak}}}
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = _cfg2_cpu()
    return out


def run_cfg2(args):
    r = measure_cfg2(args)
    if r is not None:
        print(json.dumps(r), flush=True)
    _finish(int(os.environ.get("WORLD_SIZE", "1")))


PEER_COPY_GBS = 770.0  # measured NVLink peer copy per direction on this pool's B200s


def _collective_cpu(mb: int = 64, D: int = 8) -> dict:
    """The reference's in-process psum (SharedCollective.psum: each of the D
    shard threads sums all D slots in slot order) restated by the oracle,
    on D slots of `mb` MB."""
    import numpy as np
    from oracle import oracle as orc
    n = (mb << 20) // 4
    slots = [np.full(n, float(i + 1), np.float32) for i in range(D)]
    t0 = time.perf_counter()
    orc.psum(slots)
    dt = time.perf_counter() - t0
    return {"value": (n * 4) / dt * 2 * (D - 1) / D / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"psum over {D} slots of {mb} MB (one shard's thread), reported in the NCCL bus-bandwidth "
                      "convention"}


def measure_collectives(args, sizes=None):
    """Config 3: Lax.psum / Lax.allGather of float32 vectors ~ N(0,1) per
    rank.  Reports NCCL-convention bus GB/s for the raw device collective
    (back-to-back on the stream) and per call through JAX.pmap, plus grad
    through psum (its VJP is a psum) at 64 MB.  Returns rank 0's result."""
    import torch
    import jax4j_b200 as J
    from jax4j_b200 import _lib, distributed
    rank, world, devices = _spmd_setup()
    D = len(devices)
    if D == 1:
        if rank != 0:
            return None
        out = {"metric": "psum bus GB/s", "n_gpus": 1,
               "note": "a collective over one device moves no data; measured at N >= 2"}
        if not args.no_cpu_baseline:
            out["cpu_baseline"] = _collective_cpu()
        return out
    comm = distributed.state().comm
    stream = torch.cuda.current_stream().cuda_stream
    if sizes is None:
        sizes, size = [], 4096
        while size <= args.max_bytes:
            sizes.append(size)
            size *= 4
    rows = []
    for size in sizes:
        n = size // 4
        x = J.Random.normal(J.PRNGKey.key(4), J.Shape(n), offset=rank * n, count=n)
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        gat = torch.empty(n * D, dtype=torch.float32, device="cuda")
        iters = max(5, min(200, int(2e9 / max(size, 1) / 10)))
        ar_ms = _timed(lambda: _lib.call("j4c_psum", comm, 0, x.data_ptr(), out.data_ptr(), n, stream),
                       iters, 3, world)
        ag_ms = _timed(lambda: _lib.call("j4c_all_gather", comm, 0, x.data_ptr(), gat.data_ptr(), n, stream),
                       iters, 3, world)
        pm = J.JAX.pmap(lambda s: J.Lax.psum(s), devices)
        api_ms = _timed(lambda: pm(J.LocalShard(x, D)), max(3, iters // 10), 2, world)
        # the same all-reduce recorded as a CUDA graph of 10 calls: device
        # time without the host's per-call enqueue (as inside a recorded step)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            gs = torch.cuda.current_stream().cuda_stream
            for _ in range(10):
                _lib.call("j4c_psum", comm, 0, x.data_ptr(), out.data_ptr(), n, gs)
        graph_ms = _timed(g.replay, max(3, iters // 10), 2, world) / 10
        torch.cuda.synchronize()
        del g
        rows.append({"bytes": size, "allreduce_ms": ar_ms,
                     "allreduce_busbw_GBps": size / (ar_ms / 1e3) * 2 * (D - 1) / D / 1e9,
                     "allreduce_graph_ms": graph_ms,
                     "allreduce_graph_busbw_GBps": size / (graph_ms / 1e3) * 2 * (D - 1) / D / 1e9,
                     "allgather_ms": ag_ms,
                     "allgather_busbw_GBps": size * D / (ag_ms / 1e3) * (D - 1) / D / 1e9,
                     "pmap_psum_ms": api_ms})
        del x, out, gat
    n = (64 << 20) // 4
    x = J.Random.normal(J.PRNGKey.key(5), J.Shape(n), offset=rank * n, count=n)
    gpm = J.JAX.pmap(lambda s: J.JAX.grad(lambda v: J.Lax.psum(v.mul(v)).sum())(s), devices)
    grad_ms = _timed(lambda: gpm(J.LocalShard(x, D)), 5, 2, world)
    del x
    if rank != 0:
        return None
    at64 = next((r for r in rows if r["bytes"] == 64 << 20), rows[-1])
    return {"metric": "psum bus GB/s", "value": at64["allreduce_busbw_GBps"], "unit": "GB/s", "n_gpus": D,
            "config": {"workload": "Lax.psum / Lax.allGather, float32, per rank: "
                                   + ", ".join(f"{r['bytes'] >> 20} MB" if r["bytes"] >= 1 << 20
                                               else f"{r['bytes'] >> 10} KB" for r in rows)
                                   + "; value = all-reduce bus GB/s at %d MB" % (at64["bytes"] >> 20)},
            "sizes": rows, "grad_through_psum_64MB_ms": grad_ms,
            "roofline": {"bound": "nvlink", "achieved": at64["allreduce_busbw_GBps"], "peak": PEER_COPY_GBS,
                         "unit": "GB/s", "frac": at64["allreduce_busbw_GBps"] / PEER_COPY_GBS,
                         "peak_source": "measured NVLink peer copy per direction on this pool's B200s "
                                        "(NCCL bus-bandwidth convention: allreduce (S/t)*2(D-1)/D, "
                                        "allgather (D*S/t)*(D-1)/D)"}}


def measure_psum_sgd(args):
    """The headline's gradient exchange alone: Lax.psumSgdTree over the
    parameter tree of the 1024-4096x3-1000 MLP (167 MB of FLOAT32 per rank),
    fused over peer memory (j4c_psum_sgd) against psumTree (NCCL, per
    bucket) followed by one update kernel per parameter.  Each call is timed
    on the device, not overlapped with anything; bus GB/s in NCCL's
    all-reduce convention (2 (D - 1) / D x bytes / time).  Returns rank 0's
    result."""
    import numpy as np
    import torch
    import jax4j_b200 as J
    from jax4j_b200 import api as A, psum_sgd
    rank, world, devices = _spmd_setup()
    D = len(devices)
    if D == 1:
        return None if rank else {"metric": "psumSgdTree bus GB/s", "n_gpus": 1,
                                  "note": "the exchange moves no data on one device; measured at N >= 2"}
    shapes = []
    for i in range(1, len(DIMS)):
        shapes += [(DIMS[i - 1], DIMS[i]), (DIMS[i],)]
    r = np.random.default_rng(10 + rank)
    params = J.PyTree.list(*[J.PyTree.leaf(J.ConcreteNDArray.of(np.zeros(sh, np.float32))) for sh in shapes])
    grads = J.PyTree.list(*[J.PyTree.leaf(J.ConcreteNDArray.of(r.standard_normal(sh).astype(np.float32)))
                            for sh in shapes])
    nbytes = 4 * sum(int(np.prod(sh)) for sh in shapes)
    one = J.LocalShard(J.ConcreteNDArray.of(np.zeros(4, np.float32)), D)
    upd = A._sgd_update(1.0 / D, LR)

    def fused(dummy):
        J.Lax.psumSgdTree(params, grads, 1.0 / D, LR)
        return dummy

    def unfused(dummy):
        g = J.PyTrees.flatten(J.Lax.psumTree(grads))
        [upd(w, gg) for w, gg in zip(J.PyTrees.flatten(params), g)]
        return dummy

    pf, pu = J.JAX.pmap(fused, devices), J.JAX.pmap(unfused, devices)
    steps = max(5, args.steps)

    def graphed(fn):
        # device time of one call: recorded as a CUDA graph after eager
        # warm-up calls (peer buffers, communicators, kernels), then replayed
        for _ in range(2):
            fn(one)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn(one)
        ms = _timed(g.replay, steps, 3, world)
        torch.cuda.synchronize()
        del g
        return ms

    was = psum_sgd.ENABLED
    try:
        psum_sgd.ENABLED = True   # the fused exchange, whatever the default
        ms_f = graphed(pf)
        psum_sgd.ENABLED = False  # psumTree (NCCL) + update kernels
        ms_u = graphed(pu)
    finally:
        psum_sgd.ENABLED = was
    if rank != 0:
        return None
    bus = lambda ms: nbytes / (ms / 1e3) * 2 * (D - 1) / D / 1e9
    out = {"metric": "psumSgdTree bus GB/s", "value": bus(ms_f) if ms_f else None, "unit": "GB/s", "n_gpus": D,
           "config": {"workload": f"gradient all-reduce + SGD update of the headline's 8 parameters "
                                  f"({nbytes / 1e6:.0f} MB per rank), one call per step recorded as a CUDA "
                                  "graph, not overlapped with compute"},
           "fused_ms": ms_f, "nccl_then_update_ms": ms_u, "nccl_then_update_busbw_GBps": bus(ms_u),
           "roofline": {"bound": "nvlink", "achieved": bus(ms_f) if ms_f else None, "peak": PEER_COPY_GBS,
                        "unit": "GB/s", "frac": bus(ms_f) / PEER_COPY_GBS if ms_f else None,
                        "peak_source": "measured NVLink peer copy per direction on this pool's B200s"}}
    return out


def run_psum_sgd(args):
    r = measure_psum_sgd(args)
    if r is not None:
        print(json.dumps(r), flush=True)
    _finish(int(os.environ.get("WORLD_SIZE", "1")))


def run_collectives(args):
    r = measure_collectives(args)
    if r is not None:
        print(json.dumps(r), flush=True)
    _finish(int(os.environ.get("WORLD_SIZE", "1")))


def update_path(D: int) -> str:
    """Which path Lax.psumSgdTree takes for the headline's parameters."""
    from jax4j_b200 import psum_sgd
    if D == 1:
        return "one elementwise update kernel per parameter (no collective at N = 1)"
    if psum_sgd.ENABLED:
        return ("gradient all-reduce fused with the SGD update over peer memory (j4c_psum_sgd), "
                "bucketed and overlapped with the backward")
    return "NCCL all-reduce per bucket (psumTree), then one update kernel per parameter"


def measure_secondary(args) -> dict:
    """Configurations 0-3 beside the headline, a few seconds each: config 0
    samples/s, the config-1 fused sweep against HBM, the config-2 dot against
    the tensor peak, and at N >= 2 psum / allGather bus GB/s at 64 MB,
    256 MB and 1 GB.  Every rank runs them; rank 0 gets the results."""
    out = {}
    for name, fn in (("cfg0", lambda: measure_cfg0(args, quick=True)),
                     ("cfg1_sweep", lambda: measure_sweep(args, quick=True)),
                     ("cfg2", lambda: measure_cfg2(args, quick=True)),
                     ("cfg3_collectives", lambda: measure_collectives(args, sizes=[64 << 20, 256 << 20, 1 << 30]))):
        try:
            out[name] = fn()
        except Exception as e:  # noqa: BLE001 - one failed side measurement must not lose the headline
            out[name] = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
    return out


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "gemm":
        run_gemm(args)
    elif args.workload == "dot64":
        run_dot64(args)
    elif args.workload == "sweep":
        run_sweep(args)
    elif args.workload == "cfg0":
        run_cfg0(args)
    elif args.workload == "cfg2":
        run_cfg2(args)
    elif args.workload == "collectives":
        run_collectives(args)
    elif args.workload == "psum_sgd":
        run_psum_sgd(args)
    elif args.workload == "fft":
        run_fft(args)
    elif args.workload == "linalg":
        run_linalg(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
