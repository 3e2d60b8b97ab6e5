"""The C-ABI library without a GPU: it loads, exports every entry point the
header declares, agrees with the reference's enum ordinals, and rejects bad
arguments with a status code and a message (checks that run before any CUDA
call)."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "jax4j_cuda.h")


def _declared():
    return set(re.findall(r"J4C_API[^;]*?\b(j4c_\w+)\(", open(HEADER).read()))


def _defines():
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (J4C_\w+) (\d+)", open(HEADER).read())}


def test_library_exports_every_declared_symbol():
    from jax4j_b200 import _lib
    L = _lib.lib()
    out = subprocess.check_output(["nm", "-D", "--defined-only", _lib.LIB_PATH]).decode()
    exported = {l.split()[-1] for l in out.splitlines() if " T j4c_" in l}
    declared = _declared()
    assert declared, "no declarations parsed"
    assert declared == exported, (declared - exported, exported - declared)
    # the Python binding declares a signature for every entry point
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)
    assert L.j4c_abi_version() == _defines()["J4C_ABI_VERSION"]


def test_ordinals_match_reference_enums():
    from jax4j_b200 import DType, Primitive
    d = _defines()
    for p in Primitive:
        key = "J4C_" + p.name
        if key in d:
            assert d[key] == int(p), p
    for t in DType:
        assert d["J4C_" + t.name] == t.ordinal


def _err(L):
    return L.j4c_last_error().decode()


def test_invalid_arguments_report_status_and_message():
    from jax4j_b200 import _lib
    L = _lib.lib()
    one = (C.c_int64 * 1)(3)
    fake = C.c_void_p(0x1000)
    # DOT is not an elementwise binary primitive
    rc = L.j4c_binary(4, 0, fake, one, 1, fake, one, 1, fake, None)
    assert rc == _lib.E_INVALID and "not a binary op" in _err(L)
    # integer arithmetic is rejected like the reference (DTypeTest.java:138-143)
    rc = L.j4c_binary(0, 2, fake, one, 1, fake, one, 1, fake, None)
    assert rc == _lib.E_INVALID and "requires FLOAT32 or FLOAT64" in _err(L)
    # shapes that do not broadcast (BroadcastTest.java:35-40)
    two = (C.c_int64 * 1)(2)
    rc = L.j4c_binary(0, 0, fake, one, 1, fake, two, 1, fake, None)
    assert rc == _lib.E_INVALID and "broadcast" in _err(L)
    # BOOL comparisons are rejected (ConcreteNDArray.java:393-394)
    rc = L.j4c_compare(19, 4, fake, one, 1, fake, one, 1, fake, None)
    assert rc == _lib.E_INVALID
    rc = L.j4c_reduce_axis(9, 0, fake, 1, 1, 1, fake, None)
    assert rc == _lib.E_INVALID
    rc = L.j4c_argreduce(27, 0, fake, 1, 0, 1, fake, None)
    assert rc == _lib.E_INVALID and "axis_len" in _err(L)
    rc = L.j4c_cast(9, 0, fake, 4, fake, None)
    assert rc == _lib.E_INVALID
    rc = L.j4c_psum_slots(0, None, 0, fake, 4, None)
    assert rc == _lib.E_INVALID
    buf = (C.c_char * 8)()
    rc = L.j4c_comm_unique_id(C.cast(buf, C.c_void_p), 8)
    assert rc == _lib.E_INVALID and "bytes" in _err(L)
    rc = L.j4c_dot(2, fake, fake, fake, 4, 4, 4, 0, 0, None)
    assert rc == _lib.E_INVALID and "FLOAT32 or FLOAT64" in _err(L)


def test_product_fails_loudly_without_library(tmp_path, monkeypatch):
    from jax4j_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(ImportError, match="no host fallback"):
        _lib.lib()
