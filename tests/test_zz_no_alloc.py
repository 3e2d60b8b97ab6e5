"""j4c_reduce_axis_noalloc: the per-axis reduction for callers that cannot
allocate device memory (a host runtime that gives all GPU memory to its own
arena, or code that must not block in cudaFree / a growing pool).

It is called here through the C ABI and compared with j4c_reduce_axis on the
same inputs, twice in a row, bit for bit (same kernels, same split of the
axis; only the partial-sum buffer differs), and with the CPU oracle's
sequential sum within the reduction tolerance.  The cases are chosen so that
their axis is split across CTAs -- the only plan that uses the static scratch
array -- and the test checks that from the same plan the library computes.
The file is named to be collected last so that a run stopping at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from tests.util import TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu

SUM_AXIS, MEAN_AXIS, FLOAT32, FLOAT64 = 11, 12, 0, 1
SCRATCH_BYTES = 256 * 1024  # J4C_REDUCE_NOALLOC_SCRATCH_BYTES in include/jax4j_cuda.h


def _col_splits(sms: int, esize: int, outer: int, axis: int, inner: int, aligned: bool = True) -> int:
    """How many chunks the library's column-reduction plan (col_plan in
    jax4j_b200/csrc/reduce.cu) cuts the axis into: > 1 means the partial sums
    go through scratch.  Restated here so the test can tell which branch a
    case takes."""
    vec = 4 if esize == 4 and inner % 4 == 0 and aligned else 1
    gx = -(-inner // (256 * vec))
    gy = min(outer, 65535)
    ctas, want = gx * gy, sms * 4
    splits = 1
    if ctas < want and axis >= 64:
        splits = min(-(-want // ctas), axis // 32, 64)
    chunk = -(-axis // splits)
    return -(-axis // chunk)


def _reduce(entry, prim, dtype, x, outer, axis, inner):
    import torch
    from jax4j_b200 import _lib
    out = torch.empty(outer * inner, dtype=x.dtype, device=x.device)
    rc = getattr(_lib.lib(), entry)(prim, dtype, x.data_ptr(), outer, axis, inner, out.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    return rc, out


def _host_reference(prim, dtype, x, outer, axis, inner):
    from oracle import oracle as orc
    a = x.cpu().numpy().reshape(outer, axis, inner)
    if dtype == FLOAT32:
        return orc.reduce_axis(prim, a, 1, False).reshape(-1)
    s = a.sum(axis=1, dtype=np.float64)  # the oracle restates FLOAT32 only
    return (s / axis if prim == MEAN_AXIS else s).reshape(-1)


def test_noalloc_matches_reduce_axis_on_consecutive_calls():
    import torch
    from jax4j_b200 import _lib
    torch.cuda.set_device(0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    g = torch.Generator(device="cuda").manual_seed(7)
    # (prim, dtype, outer, axis, inner): the first three split the axis
    # across CTAs and so go through the static scratch; the last is a row
    # reduction, which needs no scratch.
    cases = [(SUM_AXIS, FLOAT32, 1, 2048, 1024, True),
             (MEAN_AXIS, FLOAT32, 1, 4096, 512, True),
             (SUM_AXIS, FLOAT64, 3, 1000, 40, True),
             (SUM_AXIS, FLOAT32, 333, 4096, 1, False)]
    for prim, dtype, outer, axis, inner, uses_scratch in cases:
        esize = 4 if dtype == FLOAT32 else 8
        if uses_scratch:
            splits = _col_splits(sms, esize, outer, axis, inner)
            assert splits > 1, (outer, axis, inner, splits)
            assert splits * outer * inner * esize <= SCRATCH_BYTES, (outer, axis, inner, splits)
        tdt = torch.float32 if dtype == FLOAT32 else torch.float64
        for call in range(2):  # two calls in a row: the shared array's old contents must not matter
            x = torch.randn(outer * axis * inner, dtype=tdt, device="cuda", generator=g) * (call + 1)
            rc_ref, ref = _reduce("j4c_reduce_axis", prim, dtype, x, outer, axis, inner)
            rc_new, got = _reduce("j4c_reduce_axis_noalloc", prim, dtype, x, outer, axis, inner)
            assert rc_ref == 0, _lib.lib().j4c_last_error()
            assert rc_new == 0, _lib.lib().j4c_last_error()
            torch.cuda.synchronize()
            what = f"noalloc {(prim, dtype, outer, axis, inner)} call {call}"
            assert torch.equal(got, ref), f"{what}: differs from j4c_reduce_axis"
            assert_rel(got.cpu().numpy(), _host_reference(prim, dtype, x, outer, axis, inner),
                       TOL_REDUCTION, f"{what} vs the oracle")


def test_noalloc_rejects_reductions_beyond_its_scratch():
    import torch
    from jax4j_b200 import _lib
    torch.cuda.set_device(0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    # a [8192, 4096] column sum splits its axis across CTAs: its partial sums
    # (splits x 4096 floats) are more than the 256 KiB static array
    assert _col_splits(sms, 4, 1, 8192, 4096) * 4096 * 4 > SCRATCH_BYTES
    x = torch.zeros(8192 * 4096, dtype=torch.float32, device="cuda")
    rc, _ = _reduce("j4c_reduce_axis_noalloc", SUM_AXIS, FLOAT32, x, 1, 8192, 4096)
    assert rc == _lib.E_INVALID
    msg = _lib.lib().j4c_last_error().decode()
    assert "static maximum" in msg and "j4c_reduce_axis" in msg
    # the regular entry point still serves it
    rc, _ = _reduce("j4c_reduce_axis", SUM_AXIS, FLOAT32, x, 1, 8192, 4096)
    assert rc == 0
