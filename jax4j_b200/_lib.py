"""ctypes binding of libjax4j_cuda.so (the C ABI declared in include/jax4j_cuda.h).

The product path has no fallback: if the library or a CUDA device is missing,
`lib()` raises instead of computing anything on the host.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch  # noqa: F401  (loads the CUDA runtime and NCCL before our library)

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libjax4j_cuda.so")

# status codes (include/jax4j_cuda.h)
OK, E_INVALID, E_UNSUPPORTED, E_CUDA, E_OOM, E_NCCL, E_TIMEOUT, E_DEVICE = range(8)
STATUS_NAMES = {0: "OK", 1: "INVALID", 2: "UNSUPPORTED", 3: "CUDA", 4: "OOM", 5: "NCCL",
                6: "TIMEOUT", 7: "DEVICE"}


class J4CError(RuntimeError):
    """A libjax4j_cuda call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{STATUS_NAMES.get(code, code)}] {message}")
        self.code = code


class J4CTimeout(J4CError):
    pass


_lib = None
_lock = threading.Lock()

P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int
PI64 = C.POINTER(C.c_int64)

# name -> argtypes; every function returns int unless listed in _RESTYPES.
SIGNATURES = {
    "j4c_abi_version": [],
    "j4c_kernel_launches": [C.POINTER(C.c_uint64)],
    "j4c_last_error": [],
    "j4c_device_count": [C.POINTER(C.c_int)],
    "j4c_set_device": [I32],
    "j4c_get_device": [C.POINTER(C.c_int)],
    "j4c_enable_peer_access": [I32, I32],
    "j4c_stream_synchronize": [P],
    "j4c_stream_create": [C.POINTER(P)],
    "j4c_stream_destroy": [P],
    "j4c_device_status": [C.POINTER(C.c_int)],
    "j4c_malloc": [C.c_size_t, C.POINTER(P), P],
    "j4c_free": [P, P],
    "j4c_memcpy_h2d": [P, P, C.c_size_t, P],
    "j4c_memcpy_d2h": [P, P, C.c_size_t, P],
    "j4c_memcpy_d2d": [P, P, C.c_size_t, P],
    "j4c_fill": [I32, P, I64, C.c_double, P],
    "j4c_binary": [I32, I32, P, PI64, I32, P, PI64, I32, P, P],
    "j4c_compare": [I32, I32, P, PI64, I32, P, PI64, I32, P, P],
    "j4c_unary": [I32, I32, P, I64, P, P],
    "j4c_cast": [I32, I32, P, I64, P, P],
    "j4c_reduce_all": [I32, I32, P, I64, P, P],
    "j4c_reduce_axis": [I32, I32, P, I64, I64, I64, P, P],
    "j4c_reduce_axis_noalloc": [I32, I32, P, I64, I64, I64, P, P],
    "j4c_argreduce": [I32, I32, P, I64, I64, I64, P, P],
    "j4c_broadcast_like": [I32, P, PI64, I32, P, PI64, I32, P],
    "j4c_relu_grad": [I32, P, P, I64, P, P],
    "j4c_maxmin_grad": [I32, I32, P, PI64, I32, P, PI64, I32, P, PI64, I32, P, P, P],
    "j4c_transpose": [I32, P, I64, I64, P, P],
    "j4c_gather_rows": [I32, P, I64, I64, I32, P, I64, P, P],
    "j4c_scatter_add_rows": [I32, P, I64, I64, I32, P, I64, P, P],
    "j4c_dot": [I32, P, P, P, I64, I64, I64, I32, I32, P],
    "j4c_dot_ws": [I32, P, P, P, I64, I64, I64, I32, I32, P, C.c_size_t, P],
    "j4c_dot_workspace_size": [I32, I64, I64, I64],
    "j4c_split_pitch": [I64],
    "j4c_dot_split_kind": [],
    "j4c_split_f32": [P, I64, I64, P, P, P],
    "j4c_split_f32_transposed": [P, I64, I64, P, P, P],
    "j4c_dot_split": [P, P, P, P, P, I64, I64, I64, I32, I32, P],
    "j4c_dot_split_ep": [P, P, P, P, P, I64, I64, I64, I32, I32, P, P, P, P],
    "j4c_split_f32_both": [P, I64, I64, P, P, P, P, P],
    "j4c_split_f32_ex": [P, I64, I64, P, P, P, P, P, P, P, P],
    "j4c_split_f32_cols": [P, I64, I64, P, P, P],
    "j4c_split_lines": [P, I64, I64, P, P],
    "j4c_split_floats": [I64, I64],
    "j4c_set_wait_limit_ns": [C.c_uint64, C.POINTER(C.c_uint64)],
    "j4c_dot_split_ep_max": [P, P, P, P, P, I64, I64, I64, I32, I32, P, P, P, P, P],
    "j4c_dot_split_ep_bits": [P, P, P, P, P, I64, I64, I64, I32, I32, P, P, P, P, P, P, P],
    "j4c_fft": [I32, I32, PI64, P, P, P, P, I32, P],
    "j4c_rfft": [I32, I32, PI64, P, P, P, P],
    "j4c_irfft": [I32, I32, PI64, P, P, P, P],
    "j4c_dct1": [I32, I64, P, P, P],
    "j4c_lu_factor": [I32, I64, P, P, P, P, P, P],
    "j4c_lu_solve": [I64, I64, P, P, I32, I32, P, P, P],
    "j4c_lu_rcond": [I64, P, P, C.c_double, P, P],
    "j4c_eig": [I32, I64, P, P, P, P],
    "j4c_svd": [I32, I64, I64, P, P, P, P, P],
    "j4c_dot_split_batched": [P, P, P, P, P, I64, I64, I64, I64, I32, I32, I32, I32, P],
    "j4c_fused_compile": [P, C.POINTER(P)],
    "j4c_fused_source": [P, I32, P, C.c_size_t, C.POINTER(C.c_size_t)],
    "j4c_fused_launch": [P, I64, I64, C.POINTER(P), C.POINTER(P), C.POINTER(P), P],
    "j4c_random_permutation": [C.c_uint64, I64, P, P],
    "j4c_random_uniform": [C.c_uint64, I64, I64, C.c_float, C.c_float, P, P],
    "j4c_random_normal": [C.c_uint64, I64, I64, P, P],
    "j4c_comm_unique_id": [P, C.c_size_t],
    "j4c_comm_init_rank": [P, C.c_size_t, I32, I32, I32, I64, C.POINTER(P)],
    "j4c_comm_init_all": [C.POINTER(C.c_int), I32, I64, C.POINTER(P)],
    "j4c_comm_rank": [P, C.POINTER(C.c_int), C.POINTER(C.c_int)],
    "j4c_comm_destroy": [P],
    "j4c_comm_abort": [P],
    "j4c_psum": [P, I32, P, P, I64, P],
    "j4c_all_gather": [P, I32, P, P, I64, P],
    "j4c_reduce_scatter": [P, I32, P, P, I64, P],
    "j4c_comm_wait": [P, P],
    "j4c_psum_slots": [I32, C.POINTER(P), I32, P, I64, P],
    "j4c_sgd_update_lines": [P, P, I64, I64, C.c_float, C.c_float, P, P, P],
    "j4c_peer_alloc": [C.c_size_t, C.POINTER(P), P, C.c_size_t],
    "j4c_peer_open": [P, C.c_size_t, C.POINTER(P)],
    "j4c_peer_close": [P],
    "j4c_peer_free": [P],
    "j4c_psum_sgd_flag_bytes": [],
    "j4c_psum_sgd": [C.POINTER(P), C.POINTER(P), C.POINTER(P), I32, I32, I64, I32, C.POINTER(I64), C.POINTER(P),
                     C.c_float, C.c_float, P, P, P],
}
_RESTYPES = {"j4c_last_error": C.c_char_p, "j4c_dot_workspace_size": C.c_size_t,
             "j4c_split_pitch": C.c_int64, "j4c_split_floats": C.c_int64,
             "j4c_psum_sgd_flag_bytes": C.c_size_t}


def lib() -> C.CDLL:
    """Loads the library once; raises if it is missing."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python -m jax4j_b200.build` "
                        "(jax4j_b200 has no host fallback)")
                L = C.CDLL(LIB_PATH)
                for name, args in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = _RESTYPES.get(name, C.c_int)
                _lib = L
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != OK:
        msg = lib().j4c_last_error().decode(errors="replace")
        cls = J4CTimeout if rc == E_TIMEOUT else J4CError
        raise cls(rc, f"{what}: {msg}" if what else msg)


def dims(shape) -> C.Array:
    n = len(shape)
    arr = (C.c_int64 * max(n, 1))(*shape)
    return arr


def kernel_launches() -> int:
    v = C.c_uint64(0)
    check(lib().j4c_kernel_launches(C.byref(v)), "j4c_kernel_launches")
    return int(v.value)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
