"""GEMM launch-plan switches, each read once per process, so the GEMM parity
tests run again in a child process with the switch set:

- VOXQ_GEMM_TWO_PHASE=-1 selects the fused single-kernel GEMM (dequant warps
  feeding the tensor cores) in place of the default two-phase path;
- VOXQ_GEMM_SPLIT forces the split-K factor: 1 (no split) and the largest the
  K range allows, on the whole config-3 sweep.  Every case must meet the same
  tolerance against the CPU checker whatever the split;
- VOXQ_GEMM_CLUSTER=0 sums the K-split partials of batches of up to 256 rows
  through global memory and a reduction kernel instead of inside a cluster."""
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


@pytest.mark.parametrize("split", ["1", "16"])
def test_c3_sweep_with_forced_split_in_child_process(split):
    env = dict(os.environ, VOXQ_GEMM_SPLIT=split)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        os.path.join(HERE, "test_gpu_matmul.py"), "-k", "c3_sweep"],
                       env=env, cwd=os.path.dirname(HERE), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert "16 passed" in r.stdout


def test_gemm_without_cluster_split_in_child_process():
    env = dict(os.environ, VOXQ_GEMM_CLUSTER="0")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        os.path.join(HERE, "test_gpu_matmul.py"), "-k", "gemm or epilogues"],
                       env=env, cwd=os.path.dirname(HERE), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
