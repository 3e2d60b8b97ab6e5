"""j4c_reduce_axis_noalloc: the per-axis reduction for callers that cannot
allocate device memory (a host runtime that gives all GPU memory to its own
arena, or code that must not block in cudaFree / a growing pool).

It is called here through the C ABI and compared with j4c_reduce_axis on the
same inputs, twice in a row, on shapes whose split axis makes it use its
static scratch array.  The file is named to be collected last so that a run
stopping at the first failure has already run every other test; it also
passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from tests.util import TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu

SUM_AXIS, MEAN_AXIS, FLOAT32, FLOAT64 = 11, 12, 0, 1


def _reduce(entry, prim, dtype, x, outer, axis, inner):
    import torch
    from jax4j_b200 import _lib
    out = torch.empty(outer * inner, dtype=x.dtype, device=x.device)
    rc = getattr(_lib.lib(), entry)(prim, dtype, x.data_ptr(), outer, axis, inner, out.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    return rc, out


def test_noalloc_matches_reduce_axis_on_consecutive_calls():
    import torch
    from jax4j_b200 import _lib
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(7)
    # (prim, dtype, outer, axis, inner): the first two split the axis across
    # CTAs and so go through the static scratch; the last is a row reduction.
    cases = [(SUM_AXIS, FLOAT32, 1, 2048, 1024),
             (MEAN_AXIS, FLOAT32, 1, 4096, 512),
             (SUM_AXIS, FLOAT64, 3, 1000, 40),
             (SUM_AXIS, FLOAT32, 333, 4096, 1)]
    for prim, dtype, outer, axis, inner in cases:
        tdt = torch.float32 if dtype == FLOAT32 else torch.float64
        for call in range(2):  # two calls in a row: the shared array's old contents must not matter
            x = torch.randn(outer * axis * inner, dtype=tdt, device="cuda", generator=g) * (call + 1)
            rc_ref, ref = _reduce("j4c_reduce_axis", prim, dtype, x, outer, axis, inner)
            rc_new, got = _reduce("j4c_reduce_axis_noalloc", prim, dtype, x, outer, axis, inner)
            assert rc_ref == 0, _lib.lib().j4c_last_error()
            assert rc_new == 0, _lib.lib().j4c_last_error()
            torch.cuda.synchronize()
            assert_rel(got.cpu().numpy(), ref.cpu().numpy(), TOL_REDUCTION,
                       f"noalloc vs reduce_axis {(prim, dtype, outer, axis, inner)} call {call}")


def test_noalloc_rejects_reductions_beyond_its_scratch():
    import torch
    from jax4j_b200 import _lib
    torch.cuda.set_device(0)
    # a [8192, 4096] column sum splits its axis across CTAs: its partial sums
    # (splits x 4096 floats) are more than the 256 KiB static array
    x = torch.zeros(8192 * 4096, dtype=torch.float32, device="cuda")
    rc, _ = _reduce("j4c_reduce_axis_noalloc", SUM_AXIS, FLOAT32, x, 1, 8192, 4096)
    assert rc == _lib.E_INVALID
    msg = _lib.lib().j4c_last_error().decode()
    assert "static maximum" in msg and "j4c_reduce_axis" in msg
    # the regular entry point still serves it
    rc, _ = _reduce("j4c_reduce_axis", SUM_AXIS, FLOAT32, x, 1, 8192, 4096)
    assert rc == 0
