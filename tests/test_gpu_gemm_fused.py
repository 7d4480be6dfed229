"""The fused single-kernel GEMM (dequant warps feeding the tensor cores), which
VOXQ_GEMM_TWO_PHASE=-1 selects in place of the default two-phase path.  The
switch is read once per process, so the GEMM parity tests and the epilogue
tests run again in a child process with it set."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_fused_gemm_parity_in_child_process():
    env = dict(os.environ, VOXQ_GEMM_TWO_PHASE="-1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        os.path.join(HERE, "test_gpu_matmul.py"), "-k", "gemm or epilogues"],
                       env=env, cwd=os.path.dirname(HERE), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
