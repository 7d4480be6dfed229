"""The reference's tensor.h CUDA block, driven exactly as the reference engine
drives it: tensor_cuda_init -> tensor_to_cuda(weights) -> tensor_matmul_nt_cuda
with host activations and host outputs -> tensor_to_cpu / tensor_free.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import assert_matmul_close
from oracle import oracle as O

torch = pytest.importorskip("torch")
import voxq  # noqa: E402

pytestmark = pytest.mark.gpu
L = None


@pytest.fixture()
def abi(request):
    """Initialises the library in the quant mode given by the test's param."""
    global L
    L = voxq.lib()
    mode = getattr(request, "param", "f32")
    L.tensor_cuda_shutdown()
    old = os.environ.get("VOXCPM_QUANT")
    os.environ["VOXCPM_QUANT"] = mode
    assert L.tensor_cuda_init() == 0
    yield mode
    L.tensor_cuda_shutdown()
    if old is None:
        os.environ.pop("VOXCPM_QUANT", None)
    else:
        os.environ["VOXCPM_QUANT"] = old


def run_matmul(a_np, w_t, M, N):
    a = voxq.host_tensor(a_np)
    out = voxq.host_tensor(np.zeros((M, N), np.float32))
    try:
        rc = L.tensor_matmul_nt_cuda(a, w_t, out)
        assert rc == 0, rc
        return voxq.host_tensor_view(out)
    finally:
        voxq.free_tensor(a)
        voxq.free_tensor(out)


@pytest.mark.parametrize("M", [1, 3, 20])
def test_f32_weights_host_io(abi, M):
    N, K = 257, 96
    w = O.rand_normal(1, N * K, 0.02).reshape(N, K)
    a = O.rand_normal(2, M * K).reshape(M, K)
    wt = voxq.host_tensor(w)
    assert L.tensor_to_cuda(wt) == 0 and wt.contents.is_cuda
    y = run_matmul(a, wt, M, N)
    y_ref, sc = O.matmul_nt(a, w), O.matmul_nt_f64(a, w)[1]
    assert_matmul_close(y, y_ref, sc, 1e-5, "f32 weights")
    # a host weight is uploaded for the call only
    wh = voxq.host_tensor(w)
    y2 = run_matmul(a, wh, M, N)
    np.testing.assert_array_equal(y, y2)
    voxq.free_tensor(wt)
    voxq.free_tensor(wh)


def test_fp16_weights(abi):
    M, N, K = 2, 64, 128
    w = O.rand_normal(3, N * K, 0.02).reshape(N, K).astype(np.float16)
    a = O.rand_normal(4, M * K).reshape(M, K)
    wt = voxq.host_tensor(w, fp16=True)
    assert L.tensor_to_cuda(wt) == 0
    y = run_matmul(a, wt, M, N)
    wf = w.astype(np.float32)
    assert_matmul_close(y, O.matmul_nt(a, wf), O.matmul_nt_f64(a, wf)[1], 1e-5, "fp16 weights")
    # round trip back to the host keeps the fp16 payload
    assert L.tensor_to_cpu(wt) == 0 and not wt.contents.is_cuda and wt.contents.is_fp16
    voxq.free_tensor(wt)


@pytest.mark.parametrize("abi", ["q8", "q4"], indirect=True)
@pytest.mark.parametrize("M", [1, 2, 8, 24])
def test_quantized_upload_and_matmul(abi, M):
    qt = voxq.Q8 if abi == "q8" else voxq.Q4
    N, K = 1024, 1024
    w = O.rand_normal(5, N * K, 0.02).reshape(N, K)
    a = O.rand_normal(6, M * K).reshape(M, K)
    wt = voxq.host_tensor(w)
    assert L.tensor_to_cuda(wt) == 0 and wt.contents.is_cuda
    y = run_matmul(a, wt, M, N)
    wdeq = O.dequantize(O.quantize(w, qt), N * K, qt, q8_signed=False).reshape(N, K)
    tol = 1e-3 if M <= 8 else 5e-3
    assert_matmul_close(y, O.matmul_nt(a, wdeq), O.matmul_nt_f64(a, wdeq)[1], tol, f"{abi} M{M}")
    # tensor_to_cpu returns the dequantized weight, bit-exact with the checker
    assert L.tensor_to_cpu(wt) == 0
    back = voxq.host_tensor_view(wt)
    np.testing.assert_array_equal(back.view(np.uint32), wdeq.view(np.uint32))
    voxq.free_tensor(wt)


@pytest.mark.parametrize("abi", ["q8"], indirect=True)
def test_quantize_skips_non_block_shapes(abi):
    """K % 32 != 0 weights stay fp32 (the packed layout needs row-contained blocks)."""
    M, N, K = 2, 10, 40
    w = O.rand_normal(7, N * K, 0.02).reshape(N, K)
    a = O.rand_normal(8, M * K).reshape(M, K)
    wt = voxq.host_tensor(w)
    assert L.tensor_to_cuda(wt) == 0
    y = run_matmul(a, wt, M, N)
    assert_matmul_close(y, O.matmul_nt(a, w), O.matmul_nt_f64(a, w)[1], 1e-5, "fp32 fallback shape")
    assert L.tensor_to_cpu(wt) == 0
    np.testing.assert_array_equal(voxq.host_tensor_view(wt), w)
    voxq.free_tensor(wt)


def test_device_activation_and_output(abi):
    M, N, K = 4, 96, 64
    w = O.rand_normal(9, N * K, 0.02).reshape(N, K)
    a = O.rand_normal(10, M * K).reshape(M, K)
    wt, at = voxq.host_tensor(w), voxq.host_tensor(a)
    ot = voxq.host_tensor(np.zeros((M, N), np.float32))
    for t in (wt, at, ot):
        assert L.tensor_to_cuda(t) == 0
    assert L.tensor_matmul_nt_cuda(at, wt, ot) == 0
    assert L.tensor_to_cpu(ot) == 0
    y = voxq.host_tensor_view(ot)
    assert_matmul_close(y, O.matmul_nt(a, w), O.matmul_nt_f64(a, w)[1], 1e-5, "device io")
    for t in (wt, at, ot):
        voxq.free_tensor(t)


def test_error_codes(abi):
    a = voxq.host_tensor(np.ones((2, 64), np.float32))
    w = voxq.host_tensor(np.ones((3, 64), np.float32))
    bad_out = voxq.host_tensor(np.zeros((2, 4), np.float32))
    bad_w = voxq.host_tensor(np.ones((3, 32), np.float32))
    out = voxq.host_tensor(np.zeros((2, 3), np.float32))
    try:
        assert L.tensor_matmul_nt_cuda(a, w, bad_out) == voxq.SHAPE_MISMATCH
        assert L.tensor_matmul_nt_cuda(a, bad_w, out) == voxq.SHAPE_MISMATCH
        assert L.tensor_matmul_nt_cuda(None, w, out) == voxq.INTERNAL
        L.tensor_cuda_shutdown()
        assert L.tensor_matmul_nt_cuda(a, w, out) == voxq.CUDA_NOT_FOUND
        assert L.tensor_cuda_init() == 0
        assert L.tensor_matmul_nt_cuda(a, w, out) == 0
        np.testing.assert_allclose(voxq.host_tensor_view(out), np.full((2, 3), 64.0))
    finally:
        for t in (a, w, bad_out, bad_w, out):
            voxq.free_tensor(t)


def test_upload_weight_helper(abi):
    w = voxq.host_tensor(np.ones((4, 32), np.float32))
    import ctypes as C
    p = C.pointer(w)
    assert L.tensor_cuda_upload_weight(p) == 0 and w.contents.is_cuda
    assert L.tensor_cuda_upload_weight(None) == 0
    voxq.free_tensor(w)


@pytest.mark.parametrize("abi", ["q8"], indirect=True)
def test_fp16_uploads_land_before_quantization(abi):
    """Many fp16 host weights of the engine's shapes, uploaded back to back by
    tensor_to_cuda (VOXCPM_QUANT=q8): each must come back from tensor_to_cpu as
    exactly its Q8 dequantization -- every row, the last ones included (the
    quantizer must not read the upload before its copy has landed)."""
    rs = np.random.RandomState(11)
    shapes = [(2048, 2048), (256, 2048), (256, 2048), (6144, 2048), (2048, 6144), (1024, 64), (64, 1024)] * 3
    for i, (N, K) in enumerate(shapes):
        w = (rs.standard_normal((N, K)) * 0.02).astype(np.float16)
        wt = voxq.host_tensor(w, fp16=True)
        assert L.tensor_to_cuda(wt) == 0 and wt.contents.is_cuda
        want = O.dequantize(O.quantize(w.astype(np.float32), voxq.Q8), N * K, voxq.Q8).reshape(N, K)
        assert L.tensor_to_cpu(wt) == 0
        back = voxq.host_tensor_view(wt)
        bad = np.where((back.view(np.uint32) != want.view(np.uint32)).any(1))[0]
        assert bad.size == 0, f"upload {i} ({N}x{K}): rows {bad[:8].tolist()} differ"
        voxq.free_tensor(wt)
