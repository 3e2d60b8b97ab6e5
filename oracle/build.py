"""Build recipe for the CPU oracle (test infrastructure, not product code).

Compiles oracle/ref_cpu.c into oracle/_build/libj4c_oracle.so.  The flags keep
Java's float semantics: no fused multiply-add (-ffp-contract=off), no
value-changing optimisations (-fno-fast-math), SSE arithmetic on x86-64.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libj4c_oracle.so")
SRC = os.path.join(HERE, "ref_cpu.c")


def build(force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if (not force and os.path.exists(LIB)
            and os.path.getmtime(LIB) >= max(os.path.getmtime(SRC),
                                             os.path.getmtime(os.path.join(HERE, "ref_cpu.h")))):
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-D_GNU_SOURCE", "-ffp-contract=off", "-fno-fast-math",
           "-fPIC", "-shared", "-pthread", "-Wall", "-Wextra", "-Wno-unused-parameter",
           "-o", LIB, SRC, "-lm"]
    subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
