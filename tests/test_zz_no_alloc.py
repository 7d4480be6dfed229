"""voxq_matmul_nt_q_noalloc: the quantized GEMV for callers that cannot let a
library allocate device memory (engines holding a fixed device-memory budget,
or hosts that forbid allocation after set-up because cudaMalloc/cudaFree can
synchronise the device mid-stream).  Its scratch is a fixed array inside the
library's device image, so it must give the reference's results (the CPU
checker's tensor_matmul_nt on the dequantized weight, src/tensor.c:617-678)
and the allocating entry point's results, call after call, up to the largest
shapes the GEMV accepts.

Named to be collected last: a failure here leaves every other test already run.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import assert_matmul_close
from oracle import oracle as O

torch = pytest.importorskip("torch")
import voxq  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 1e-3  # the GEMV tolerance of the other matmul tests


def _weight(N, K, qt, seed):
    w = O.rand_normal(seed, N * K, 0.02).reshape(N, K)
    blocks = O.quantize(w, qt)
    wdeq = O.dequantize(blocks, N * K, qt).reshape(N, K)
    return voxq.QWeight.from_blocks(torch.from_numpy(blocks).cuda(), N, K, qt), wdeq


def _noalloc(a, qw, out, epi=None):
    d = qw.desc()
    return voxq.lib().voxq_matmul_nt_q_noalloc(a.data_ptr(), a.shape[0], a.stride(0), C.byref(d), out.data_ptr(),
                                               out.stride(0), C.byref(epi) if epi is not None else None,
                                               int(torch.cuda.current_stream().cuda_stream))


def _two_calls(a, qw, ref, sc, epi=None, tol=TOL):
    """Two calls in a row share (and reuse) the fixed scratch: both must match."""
    alloc = None
    for call in range(2):
        out = torch.full((a.shape[0], qw.N), float("nan"), device="cuda")
        assert _noalloc(a, qw, out, epi) == 0
        torch.cuda.synchronize()
        y = out.cpu().numpy()
        assert_matmul_close(y, ref, sc, tol, f"call {call}")
        if alloc is None:
            alloc = y
        else:
            assert np.array_equal(y, alloc), "second call differs from the first"
    assert voxq.lib().voxq_noalloc_device_error(0) == 0
    return alloc


@pytest.mark.parametrize("qt", [voxq.Q4, voxq.Q8], ids=["q4", "q8"])
@pytest.mark.parametrize("M,N,K", [(1, 4096, 1024), (3, 1000, 4096), (8, 257, 512), (2, 64, 8192)])
def test_noalloc_matches_reference_and_allocating_entry_point(qt, M, N, K):
    qw, wdeq = _weight(N, K, qt, seed=M * 100 + K)
    a_np = O.rand_normal(M * 100 + K + 1, M * K).reshape(M, K)
    a = torch.from_numpy(a_np).cuda()
    ref = O.matmul_nt(a_np, wdeq)
    _, sc = O.matmul_nt_f64(a_np, wdeq)
    y = _two_calls(a, qw, ref, sc)
    # the allocating entry point computes the same thing
    assert_matmul_close(y, voxq.matmul_nt_q(a, qw).cpu().numpy(), sc, 2 * TOL, "vs voxq_matmul_nt_q")


@pytest.mark.parametrize("qt,K", [(voxq.Q4, 32768), (voxq.Q8, 16384)], ids=["q4", "q8"])
def test_noalloc_largest_k_fits_the_array(qt, K):
    """M = 8 at the GEMV's largest K: the limb scratch (M * 3.5 * K bytes for
    Q4, M * 4 * K for Q8) is at its largest and must fit the fixed array."""
    M, N = 8, 48
    qw, wdeq = _weight(N, K, qt, seed=K + qt)
    a_np = O.rand_normal(K + 7, M * K).reshape(M, K)
    ref = O.matmul_nt(a_np, wdeq)
    _, sc = O.matmul_nt_f64(a_np, wdeq)
    _two_calls(torch.from_numpy(a_np).cuda(), qw, ref, sc)


def test_noalloc_epilogues():
    """bias + residual, then SwiGLU (silu(a W^T) * (a Up^T), src/nn.c:148-169)."""
    N, K, M = 384, 1024, 2
    qw, wdeq = _weight(N, K, voxq.Q8, seed=71)
    up, updeq = _weight(N, K, voxq.Q8, seed=72)
    a_np = O.rand_normal(73, M * K).reshape(M, K)
    bias = O.rand_normal(74, N)
    res = O.rand_normal(75, M * N).reshape(M, N)
    a = torch.from_numpy(a_np).cuda()
    g = O.matmul_nt(a_np, wdeq)
    _, gsc = O.matmul_nt_f64(a_np, wdeq)
    u = O.matmul_nt(a_np, updeq)
    _, usc = O.matmul_nt_f64(a_np, updeq)
    bias_d, res_d = torch.from_numpy(bias).cuda(), torch.from_numpy(res).cuda()
    epi = voxq.Epilogue(bias_d.data_ptr(), res_d.data_ptr(), res_d.stride(0), None)
    _two_calls(a, qw, g + bias[None, :] + res, gsc, epi)

    ud = up.desc()
    epi = voxq.Epilogue(0, 0, 0, C.pointer(ud))
    g64 = g.astype(np.float64)
    sg = 1 / (1 + np.exp(-g64))
    want = g64 * sg * u
    # error of silu(g) * u from errors in g and u, each within TOL of its scale
    scale = np.abs(sg * (1 + g64 * (1 - sg))) * gsc * np.abs(u) + np.abs(g64 * sg) * usc
    for _ in range(2):
        out = torch.full((M, N), float("nan"), device="cuda")
        assert _noalloc(a, qw, out, epi) == 0
        torch.cuda.synchronize()
        err = np.abs(out.cpu().numpy() - want)
        assert np.all(err <= TOL * np.maximum(np.abs(want), scale) + 1e-30), "swiglu"
    assert voxq.lib().voxq_noalloc_device_error(0) == 0


def test_noalloc_rejects_what_it_cannot_run():
    qw, _ = _weight(64, 1024, voxq.Q8, seed=81)
    # more than 8 activation rows is the GEMM path, which this entry point does not take
    a9 = torch.zeros(9, 1024, device="cuda")
    assert _noalloc(a9, qw, torch.empty(9, 64, device="cuda")) == voxq.UNSUPPORTED
    # a code row longer than the GEMV accepts (Q8, K > 16384)
    big, _ = _weight(16, 16416, voxq.Q8, seed=82)
    a = torch.zeros(8, 16416, device="cuda")
    assert _noalloc(a, big, torch.empty(8, 16, device="cuda")) == voxq.UNSUPPORTED
    # the error word reads (and clears) without a launch; voxq_device_error reports it too
    assert voxq.lib().voxq_noalloc_device_error(1) == 0
    assert voxq.lib().voxq_device_error(0) == 0
