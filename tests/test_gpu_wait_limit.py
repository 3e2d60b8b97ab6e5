"""The persistent GEMM's bounded waits, exercised without a fault: with the
wait limit set to 1 ns (j4c_set_wait_limit_ns) the first pipeline wait that
does not succeed at once gives up, so the kernel records status 0x7C05,
drains its own copies and tensor-core work (those waits keep their 2 s
limit), frees its tensor memory and returns.  The host reads the status
back, restores the limit, and the same context then computes a correct
product.  Nothing here traps, faults or hangs the GPU."""
import ctypes as C

import numpy as np
import pytest

from tests.util import TOL_REDUCTION, assert_rel

pytestmark = pytest.mark.gpu

STATUS_TIMEOUT = 0x7C05


def _status(L) -> int:
    code = C.c_int(0)
    assert L.j4c_device_status(C.byref(code)) == 0
    return code.value


def test_gemm_wait_limit_gives_up_with_a_status_and_the_context_stays_usable():
    import torch
    import jax4j_b200 as J
    from jax4j_b200 import _lib, core
    L = _lib.lib()
    torch.cuda.set_device(0)
    dev = J.Device.defaultDevice()
    r = np.random.default_rng(5)
    M, K, N = 2048, 2048, 1536
    A = r.uniform(-1, 1, (M, K)).astype(np.float32)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    a, b = J.ConcreteNDArray.of(A), J.ConcreteNDArray.of(B)
    core._dot_raw(a, b, False, False, dev)  # splits made, module loaded
    torch.cuda.synchronize()
    assert _status(L) == 0
    prev = C.c_uint64(0)
    assert L.j4c_set_wait_limit_ns(1, C.byref(prev)) == 0
    try:
        assert prev.value == 2_000_000_000
        core._dot_raw(a, b, False, False, dev)  # gives up: C is unspecified
        torch.cuda.synchronize()  # returns: the kernel ended on its own
        assert _status(L) == STATUS_TIMEOUT
    finally:
        assert L.j4c_set_wait_limit_ns(prev.value, None) == 0
    assert L.j4c_set_wait_limit_ns(0, None) == _lib.E_INVALID  # a limit must be positive
    got = core._dot_raw(a, b, False, False, dev).numpy()
    torch.cuda.synchronize()
    assert _status(L) == 0
    ref = (A.astype(np.float64) @ B.astype(np.float64)).astype(np.float32)
    assert_rel(got, ref, TOL_REDUCTION, "product after the timed-out launch")
