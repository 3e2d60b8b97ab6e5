"""The 3xTF32 split kind (J4C_GEMM_SPLIT=tf32), which the library fixes per
process: the dot, split-format and MLP-gradient parity tests run again in a
child process with it selected, so both kinds stay covered."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_tf32_split_kind_parity():
    env = dict(os.environ, J4C_GEMM_SPLIT="tf32")
    probe = subprocess.run([sys.executable, "-c", "from jax4j_b200.core import split_kind; print(split_kind())"],
                           cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert probe.returncode == 0 and probe.stdout.strip() == "0", probe.stdout + probe.stderr
    run = subprocess.run([sys.executable, "-m", "pytest", "tests/test_gpu_ops.py", "tests/test_gpu_models.py",
                          "tests/test_gpu_vmap.py", "-q", "-x", "-p", "no:cacheprovider"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert run.returncode == 0, run.stdout[-4000:] + run.stderr[-2000:]
