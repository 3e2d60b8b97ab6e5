"""CUDA-graph capture of a whole step (forward, backward, collectives, update).

The reference runs every step through its interpreter (api/Grad.java:150-339)
and, on a device, one TornadoVM task per equation
(backend/TornadoJitCompiler.java:82-246).  Here one eager execution of a
step function is recorded as a CUDA graph -- every kernel, copy and NCCL
collective it launches on the current stream -- and later steps replay the
graph: one launch per step, no Python interpretation, no tracing.

    step = CapturedStep(fn, [params..., x, t], donate={1: 0, ...})
    loss = step()[0]            # runs the recorded step on the same buffers

`fn(*inputs)` must return a list of ConcreteNDArrays.  The inputs are the
graph's static buffers: refill them in place (`set_input`) between replays.
`donate={out_index: in_index}` copies output `out_index` into input
`in_index` at the end of every replay, which is how a training step carries
its updated parameters into the next replay.  Outputs are valid until the next
replay.  Requirements on `fn`: no host synchronisation and no host-dependent
control flow on device values (the graph replays the recorded launches).
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional, Sequence

import torch

from ._lib import call
from .core import ConcreteNDArray, stream_of


class CapturedStep:
    def __init__(self, fn: Callable[..., Sequence[ConcreteNDArray]], inputs: Sequence[ConcreteNDArray],
                 donate: Optional[Dict[int, int]] = None, warmup: int = 2):
        self.fn = fn
        self.inputs: List[ConcreteNDArray] = list(inputs)
        self.donate = dict(donate or {})
        dev = self.inputs[0].tensor().device
        for x in self.inputs:
            if x.tensor().device != dev:
                raise ValueError("CapturedStep: every input must live on the same GPU")
        for o, i in self.donate.items():
            if not (0 <= i < len(self.inputs)):
                raise ValueError(f"CapturedStep: donate target {i} is not an input")
        self._spmd = self._spmd_state()
        # Warm-up on a side stream: compiles generated kernels, configures
        # kernels, creates communicators and fills allocator caches, none of
        # which may happen during capture.  Warm-up results are discarded (the
        # inputs are not updated).
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        self._lines = {}  # input index -> static line-word buffer carried with a donated output's
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                warm = self._check(self.fn(*self._fresh_inputs()))
        # A donated output that carries its line maxima (an SGD-updated weight)
        # hands them to its input too: the recorded step's splits of that input
        # then take them instead of a max pass.  They start as the max pass of
        # the input's current contents.
        for o, i in self.donate.items():
            x = self.inputs[i]
            if getattr(warm[o], "_lines", None) is not None and x.shape().rank() == 2:
                rows, cols = x.shape().dimensions()
                buf = torch.empty(rows + cols + 1, dtype=torch.int32, device=dev)
                call("j4c_split_lines", x.data_ptr(), rows, cols, buf.data_ptr(), stream_of(dev.index))
                self._lines[i] = buf
        del warm
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        from ._lib import kernel_launches
        k0 = kernel_launches()
        with torch.cuda.graph(self.graph):
            outs = self._check(self.fn(*self._fresh_inputs()))
            s = torch.cuda.current_stream(dev).cuda_stream
            for o, i in self.donate.items():
                src, dst = outs[o], self.inputs[i]
                if src.tensor().numel() != dst.tensor().numel() or src.dtype() != dst.dtype():
                    raise ValueError(f"CapturedStep: output {o} does not match input {i}")
                call("j4c_memcpy_d2d", dst.data_ptr(), src.data_ptr(),
                     dst.tensor().numel() * dst.tensor().element_size(), s)
                if i in self._lines:
                    if getattr(src, "_lines", None) is None:
                        raise ValueError(f"CapturedStep: output {o} lost its line maxima during capture")
                    call("j4c_memcpy_d2d", self._lines[i].data_ptr(), src._lines.data_ptr(),
                         self._lines[i].numel() * 4, s)
        self.kernels = kernel_launches() - k0  # this library's kernels recorded in the graph
        self.outputs: List[ConcreteNDArray] = outs
        self.device = dev

    @staticmethod
    def _spmd_state():
        from . import distributed
        return distributed.state()

    @staticmethod
    def _check(outs) -> List[ConcreteNDArray]:
        outs = list(outs) if isinstance(outs, (list, tuple)) else [outs]
        for o in outs:
            if not isinstance(o, ConcreteNDArray):
                raise TypeError("CapturedStep: the step must return ConcreteNDArrays")
        return outs

    def _fresh_inputs(self) -> List[ConcreteNDArray]:
        # New wrappers around the static buffers: arrays are immutable and may
        # cache derived data (dot splits), while these buffers are refilled.
        out = [ConcreteNDArray._wrap(x.tensor(), x.shape(), x.dtype(), x.device()) for x in self.inputs]
        for i, buf in getattr(self, "_lines", {}).items():
            out[i]._lines = buf
        return out

    def set_input(self, index: int, src: ConcreteNDArray, stream: Optional[int] = None) -> None:
        """Copies `src` into static input `index` (device to device) on `stream`
        (default: the current stream), ordered before the next replay on it."""
        dst = self.inputs[index]
        if src.tensor().numel() != dst.tensor().numel() or src.dtype() != dst.dtype():
            raise ValueError(f"CapturedStep.set_input: {src.shape()} {src.dtype()} does not fit input {index}")
        if src.data_ptr() == dst.data_ptr():
            return
        s = stream if stream is not None else stream_of(self.device.index)
        call("j4c_memcpy_d2d", dst.data_ptr(), src.data_ptr(), dst.tensor().numel() * dst.tensor().element_size(), s)
        if index in self._lines:  # the new contents' line maxima
            rows, cols = dst.shape().dimensions()
            call("j4c_split_lines", dst.data_ptr(), rows, cols, self._lines[index].data_ptr(), s)

    def __call__(self) -> List[ConcreteNDArray]:
        """Replays the step on the current stream.  In one-process-per-GPU
        runs every rank first passes the host heartbeat, so a rank that has
        left is reported before this rank launches collectives that wait for it."""
        if self._spmd is not None and self._spmd.world_size > 1:
            from . import distributed
            distributed.heartbeat()
        self.graph.replay()
        return self.outputs

    def release(self) -> None:
        """Frees the graph (required before the process group is destroyed
        when the graph holds NCCL collectives)."""
        self.graph.reset()
        self.outputs = []
