"""voxq_conv1d_forward / voxq_conv1d_transpose_forward against the CPU
checker's restatement of the reference's conv1d_forward and
conv1d_transpose_forward (src/nn.c:765-931), on the shapes of the AudioVAE
decoder (src/audio_vae.c:579-690) and odd ones, with host and device tensors.
fp32 on both sides; rule: |y - y_ref| <= 1e-4 * sum |w x| (+ |b|) per element."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
import voxq  # noqa: E402

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def lib():
    L = voxq.lib()
    L.tensor_cuda_shutdown()
    assert L.tensor_cuda_init() == 0
    yield L
    L.tensor_cuda_shutdown()


def device_tensor(t):
    """A Tensor borrowing a CUDA torch tensor (is_cuda, not owned)."""
    T = voxq.Tensor()
    shp = (C.c_int * t.dim())(*t.shape)
    T.data = C.cast(C.c_void_p(t.data_ptr()), C.POINTER(C.c_float))
    T.shape = C.cast(shp, C.POINTER(C.c_int))
    T.ndim = t.dim()
    T.size = t.numel()
    T.is_cuda = True
    return T, shp


def check(y, ref, sc, what):
    err = np.abs(y.astype(np.float64) - ref)
    assert np.all(err <= TOL * np.maximum(sc, 1e-30)), f"{what}: max scaled err {float((err / sc).max()):.3e}"


# (Cin, Cout, K, stride, pad, groups, T): conv_in, proj_up, residual depthwise / pointwise at
# the decoder's channel widths and lengths, conv_out, and odd shapes
CONV = [(64, 64, 7, 1, 3, 64, 4), (64, 2048, 1, 1, 0, 1, 4), (1024, 1024, 7, 1, 3, 1024, 32),
        (1024, 1024, 1, 1, 0, 1, 32), (256, 256, 1, 1, 0, 1, 960), (32, 1, 7, 1, 3, 1, 7680),
        (12, 18, 3, 2, 1, 3, 101), (5, 7, 4, 3, 0, 1, 10)]
# (Cin, Cout, K, stride, pad, T): the six upsampling blocks (kernel 2 x stride) and odd ones
CONVT = [(2048, 1024, 16, 8, 4, 4), (1024, 512, 12, 6, 3, 32), (512, 256, 10, 5, 2, 192),
         (256, 128, 4, 2, 1, 960), (64, 32, 4, 2, 1, 3840), (7, 5, 5, 3, 0, 9), (3, 4, 3, 1, 1, 6)]


@pytest.mark.parametrize("Cin,Cout,K,stride,pad,groups,T", CONV)
def test_conv1d(lib, Cin, Cout, K, stride, pad, groups, T):
    rs = np.random.RandomState(Cin + Cout + T)
    x = rs.standard_normal((1, Cin, T)).astype(np.float32)
    w = (rs.standard_normal((Cout, Cin // groups, K)) * 0.05).astype(np.float32)
    b = rs.standard_normal(Cout).astype(np.float32)
    ref, sc = O.conv1d(x, w, b, stride, pad, groups)
    wt, bt = voxq.host_tensor(w), voxq.host_tensor(b)
    desc = voxq.Conv1dDesc(C.cast(wt, C.c_void_p), C.cast(bt, C.c_void_p), Cin, Cout, K, stride, pad, groups)
    try:
        for call in range(2):  # the second call uses the cached device weight
            xt, ot = voxq.host_tensor(x), voxq.host_tensor(np.zeros(ref.shape, np.float32))
            assert lib.voxq_conv1d_forward(C.byref(desc), xt, ot) == 0
            check(voxq.host_tensor_view(ot), ref, sc, f"conv1d host call {call}")
            voxq.free_tensor(xt)
            voxq.free_tensor(ot)
        xd, od = torch.from_numpy(x).cuda(), torch.zeros(ref.shape, device="cuda")
        (tx, s1), (to, s2) = device_tensor(xd), device_tensor(od)
        assert lib.voxq_conv1d_forward(C.byref(desc), C.byref(tx), C.byref(to)) == 0
        torch.cuda.synchronize()
        check(od.cpu().numpy(), ref, sc, "conv1d device")
    finally:
        voxq.free_tensor(wt)
        voxq.free_tensor(bt)


@pytest.mark.parametrize("Cin,Cout,K,stride,pad,T", CONVT)
def test_conv1d_transpose(lib, Cin, Cout, K, stride, pad, T):
    rs = np.random.RandomState(Cin * 3 + T)
    x = rs.standard_normal((1, Cin, T)).astype(np.float32)
    w = (rs.standard_normal((Cin, Cout, K)) * 0.05).astype(np.float32)
    b = rs.standard_normal(Cout).astype(np.float32)
    ref, sc = O.conv1d_transpose(x, w, b, stride, pad)
    wt, bt = voxq.host_tensor(w), voxq.host_tensor(b)
    desc = voxq.Conv1dTransposeDesc(C.cast(wt, C.c_void_p), C.cast(bt, C.c_void_p), Cin, Cout, K, stride, pad)
    xt, ot = voxq.host_tensor(x), voxq.host_tensor(np.zeros(ref.shape, np.float32))
    try:
        assert lib.voxq_conv1d_transpose_forward(C.byref(desc), xt, ot) == 0
        check(voxq.host_tensor_view(ot), ref, sc, "conv1d_transpose")
    finally:
        for t in (wt, bt, xt, ot):
            voxq.free_tensor(t)


def test_conv_shape_errors_and_no_bias(lib):
    x = np.ones((1, 4, 8), np.float32)
    w = np.ones((6, 4, 3), np.float32)
    wt, xt = voxq.host_tensor(w), voxq.host_tensor(x)
    ot = voxq.host_tensor(np.zeros((1, 6, 8), np.float32))
    desc = voxq.Conv1dDesc(C.cast(wt, C.c_void_p), None, 4, 6, 3, 1, 1, 1)
    assert lib.voxq_conv1d_forward(C.byref(desc), xt, ot) == 0
    ref, _ = O.conv1d(x, w, None, 1, 1, 1)
    np.testing.assert_allclose(voxq.host_tensor_view(ot), ref, rtol=1e-6)
    bad = voxq.Conv1dDesc(C.cast(wt, C.c_void_p), None, 5, 6, 3, 1, 1, 1)  # in_channels disagree with x
    assert lib.voxq_conv1d_forward(C.byref(bad), xt, ot) == voxq.SHAPE_MISMATCH
    for t in (wt, xt, ot):
        voxq.free_tensor(t)


def test_vae_decode_steps(lib):
    """voxq_vae_decode: the decoder's step list (conv_in, proj_up, snake, a transposed upsampling
    conv, a residual sub-block with its saved input, the final snake, conv_out, tanh) on a resident
    activation, against the checker's convolutions and a float64 snake / tanh
    (src/audio_vae.c:310-351, 354-421, 941-1116), fp32 between steps.  Rule: the tanh-bounded
    output within 2e-4 absolute."""
    rs = np.random.RandomState(7)
    B, T, D, C1, C2 = 1, 4, 16, 32, 8
    keep = []

    def host(a):
        t = voxq.host_tensor(a.astype(np.float32))
        keep.append(t)
        return t

    def conv_desc(w, b, cin, cout, k, stride, pad, groups):
        d = voxq.Conv1dDesc(C.cast(host(w), C.c_void_p), C.cast(host(b), C.c_void_p) if b is not None else None,
                            cin, cout, k, stride, pad, groups)
        keep.append(d)
        return d

    def convt_desc(w, b, cin, cout, k, stride, pad):
        d = voxq.Conv1dTransposeDesc(C.cast(host(w), C.c_void_p),
                                     C.cast(host(b), C.c_void_p) if b is not None else None, cin, cout, k, stride, pad)
        keep.append(d)
        return d

    z = rs.standard_normal((B, T, D)).astype(np.float32)
    w_in = (rs.standard_normal((D, 1, 7)) * 0.3).astype(np.float32)
    w_up = (rs.standard_normal((C1, D, 1)) * 0.3).astype(np.float32)
    b_up = (rs.standard_normal(C1) * 0.1).astype(np.float32)
    a0 = (0.5 + rs.random_sample(C1)).astype(np.float32)
    w_t = (rs.standard_normal((C1, C2, 4)) * 0.2).astype(np.float32)
    b_t = (rs.standard_normal(C2) * 0.1).astype(np.float32)
    a1 = (0.5 + rs.random_sample(C2)).astype(np.float32)
    w_dw = (rs.standard_normal((C2, 1, 7)) * 0.3).astype(np.float32)
    a2 = (0.5 + rs.random_sample(C2)).astype(np.float32)
    w_pw = (rs.standard_normal((C2, C2, 1)) * 0.3).astype(np.float32)
    af = (0.5 + rs.random_sample(C2)).astype(np.float32)
    w_out = (rs.standard_normal((1, C2, 7)) * 0.3).astype(np.float32)
    b_out = np.array([0.05], np.float32)

    ops_spec = [("conv", conv_desc(w_in, None, D, D, 7, 1, 3, D)),
                ("conv", conv_desc(w_up, b_up, D, C1, 1, 1, 0, 1)),
                ("snake", host(a0)),
                ("convt", convt_desc(w_t, b_t, C1, C2, 4, 2, 1)),
                ("save", None), ("snake", host(a1)), ("conv", conv_desc(w_dw, None, C2, C2, 7, 1, 3, C2)),
                ("snake", host(a2)), ("conv", conv_desc(w_pw, None, C2, C2, 1, 1, 0, 1)), ("add", None),
                ("snake", host(af)), ("conv", conv_desc(w_out, b_out, C2, 1, 7, 1, 3, 1)), ("tanh", None)]
    kinds = {"conv": 1, "convt": 2, "snake": 3, "save": 4, "add": 5, "tanh": 6}
    ops = (voxq.VaeOp * len(ops_spec))()
    for i, (k, v) in enumerate(ops_spec):
        ops[i].kind = kinds[k]
        if k == "conv":
            ops[i].conv = C.pointer(v)
        elif k == "convt":
            ops[i].convt = C.pointer(v)
        elif k == "snake":
            ops[i].alpha = v

    # reference chain: the checker's convolutions, float64 elementwise steps, float32 between steps
    def snake(h, a):
        return (h + np.sin(a[None, :, None].astype(np.float64) * h) ** 2 / 1.0).astype(np.float32)

    h = np.ascontiguousarray(z.transpose(0, 2, 1))
    h, _ = O.conv1d(h, w_in, None, 1, 3, D)
    h, _ = O.conv1d(h, w_up, b_up, 1, 0, 1)
    h = snake(h, a0)
    h, _ = O.conv1d_transpose(h, w_t, b_t, 2, 1)
    skip = h.copy()
    h = snake(h, a1)
    h, _ = O.conv1d(h, w_dw, None, 1, 3, C2)
    h = snake(h, a2)
    h, _ = O.conv1d(h, w_pw, None, 1, 0, 1)
    h = h + skip
    h = snake(h, af)
    h, _ = O.conv1d(h, w_out, b_out, 1, 3, 1)
    ref = np.tanh(h.astype(np.float64))
    wave = voxq.host_tensor(np.zeros((B, ref.shape[2]), np.float32))
    keep.append(wave)
    try:
        assert lib.voxq_vae_decode(ops, len(ops_spec), C.c_float(1.0), host(z), wave) == 0
        got = voxq.host_tensor_view(wave)
        err = np.abs(got.astype(np.float64) - ref[:, 0, :])
        # the chain amplifies the per-step 1e-4 bound; its output is tanh-bounded
        assert float(err.max()) <= 2e-4, f"max err {float(err.max()):.3e}"
        # a wrong waveform shape is the reference's shape error
        bad = voxq.host_tensor(np.zeros((B, ref.shape[2] + 1), np.float32))
        keep.append(bad)
        assert lib.voxq_vae_decode(ops, len(ops_spec), C.c_float(1.0), host(z), bad) == voxq.SHAPE_MISMATCH
    finally:
        for t in keep:
            if isinstance(t, C.POINTER(voxq.Tensor)):
                voxq.free_tensor(t)
