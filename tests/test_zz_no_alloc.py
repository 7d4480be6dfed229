"""voxq_matmul_nt_q_noalloc: the quantized GEMV for callers that cannot let a
library allocate device memory (engines holding a fixed device-memory budget,
or hosts that forbid allocation after set-up because cudaMalloc/cudaFree can
synchronise the device mid-stream).  Its scratch is a fixed array inside the
library's device image, so it must give the same results as the allocating
entry point, voxq_matmul_nt_q, call after call.

Named to be collected last: a failure here leaves every other test already run.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import voxq  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 1e-3  # the GEMV tolerance of the other matmul tests


def _scale(a, qw):
    """sum_k |a w| / sqrt(K), the per-element tolerance scale, in fp64."""
    wd = voxq.dequantize(qw.to_blocks(), qw.N * qw.K, qw.qtype).view(qw.N, qw.K).double()
    return (a.double().abs() @ wd.abs().T) / np.sqrt(qw.K)


def _noalloc(a, qw, out, epi=None, stream=None):
    d = qw.desc()
    return voxq.lib().voxq_matmul_nt_q_noalloc(a.data_ptr(), a.shape[0], a.stride(0), C.byref(d), out.data_ptr(),
                                               out.stride(0), C.byref(epi) if epi is not None else None,
                                               int(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("qt", [voxq.Q4, voxq.Q8], ids=["q4", "q8"])
@pytest.mark.parametrize("M,N,K", [(1, 4096, 1024), (3, 1000, 4096), (8, 257, 512)])
def test_noalloc_matches_allocating_entry_point(qt, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 100 + K)
    qw = voxq.QWeight.from_float(torch.randn(N, K, device="cuda", generator=g) * 0.02, qt)
    a = torch.randn(M, K, device="cuda", generator=g)
    ref = voxq.matmul_nt_q(a, qw)
    bound = TOL * torch.maximum(ref.double().abs(), _scale(a, qw))
    for call in range(2):  # two calls in a row share (and reuse) the fixed scratch
        out = torch.full((M, N), float("nan"), device="cuda")
        assert _noalloc(a, qw, out) == 0
        torch.cuda.synchronize()
        assert bool(((out.double() - ref.double()).abs() <= bound).all()), f"call {call}"
    assert voxq.lib().voxq_device_error(0) == 0


def test_noalloc_epilogue_and_limits():
    g = torch.Generator(device="cuda").manual_seed(7)
    N, K = 384, 1024
    qw = voxq.QWeight.from_float(torch.randn(N, K, device="cuda", generator=g) * 0.02, voxq.Q8)
    a = torch.randn(2, K, device="cuda", generator=g)
    bias = torch.randn(N, device="cuda", generator=g)
    ref = voxq.matmul_nt_q(a, qw, bias=bias)
    for _ in range(2):
        out = torch.empty(2, N, device="cuda")
        epi = voxq.Epilogue(bias.data_ptr(), 0, 0, None)
        assert _noalloc(a, qw, out, epi) == 0
        torch.cuda.synchronize()
        bound = TOL * torch.maximum(ref.double().abs(), _scale(a, qw))
        assert bool(((out.double() - ref.double()).abs() <= bound).all())
    # more than 8 activation rows is the GEMM path, which this entry point does not take
    a9 = torch.randn(9, K, device="cuda", generator=g)
    assert _noalloc(a9, qw, torch.empty(9, N, device="cuda")) == voxq.UNSUPPORTED
