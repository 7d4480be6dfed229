"""Quantized matmul (GEMV M <= 8, GEMM M > 8) vs the reference's CPU path.

Reference value: tensor_matmul_nt (src/tensor.c:617-678, restated in
oracle/voxq_oracle.c) on the dequantized weight.  Tolerance rule from the
north star, per element: |y - y_ref| <= tol * max(|y_ref|, sum_k |w x| / sqrt(K)),
tol = 1e-3 for the fp32 GEMV, 5e-3 for the fp16-operand tensor-core GEMM.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_matmul_close
from oracle import oracle as O

torch = pytest.importorskip("torch")
import voxq  # noqa: E402

pytestmark = pytest.mark.gpu

TOL_GEMV = 1e-3
TOL_GEMM = 5e-3


def tol_for(M):
    return TOL_GEMV if M <= 8 else TOL_GEMM


def make_weight(N, K, qt, seed, signed=False, mult=0.02):
    w = O.rand_normal(seed, N * K, mult).reshape(N, K)
    blocks = O.quantize(w, qt)
    wdeq = O.dequantize(blocks, N * K, qt, q8_signed=signed).reshape(N, K)
    qw = voxq.QWeight.from_blocks(torch.from_numpy(blocks).cuda(), N, K, qt, q8_signed=signed)
    return qw, wdeq


def ref(a, wdeq):
    y = O.matmul_nt(a, wdeq)
    _, sc = O.matmul_nt_f64(a, wdeq)
    return y, sc


SHAPES = [
    # (M, N, K): C1 shape, decode shapes of C2, ragged N, small and large K, M up to 8
    (1, 4096, 1024), (1, 1024, 1024), (1, 128, 1024), (1, 1024, 4096),
    (2, 1000, 1024), (3, 33, 96), (5, 7, 32), (8, 257, 512), (4, 64, 64), (1, 1, 4096), (6, 300, 2048),
]


@pytest.mark.parametrize("qt", [voxq.Q8, voxq.Q4], ids=["q8", "q4"])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemv_matches_tensor_c(qt, M, N, K):
    qw, wdeq = make_weight(N, K, qt, seed=N * 31 + K)
    a = O.rand_normal(M + 2 * K + 1, M * K).reshape(M, K)
    y = voxq.matmul_nt_q(torch.from_numpy(a).cuda(), qw).cpu().numpy()
    y_ref, sc = ref(a, wdeq)
    assert_matmul_close(y, y_ref, sc, TOL_GEMV, f"M{M} N{N} K{K} q{qt}")


@pytest.mark.parametrize("qt", [voxq.Q8, voxq.Q4], ids=["q8", "q4"])
@pytest.mark.parametrize("M", [1, 2, 5])
def test_gemv_outlier_activations(qt, M):
    """Activations with rare huge entries (heavy tails, one dominant channel):
    the case where the activation limbs need their third int8 term."""
    N, K = 256, 1024
    qw, wdeq = make_weight(N, K, qt, seed=31)
    rs = np.random.RandomState(32)
    a = rs.randn(M, K).astype(np.float32)
    a[rs.rand(M, K) < 0.01] *= 300.0          # sparse outliers
    a[:, 17] = 5e4                              # one channel dominating every row
    a[:, 500:532] *= 1e-6                       # a near-silent block
    y = voxq.matmul_nt_q(torch.from_numpy(a).cuda(), qw).cpu().numpy()
    y_ref, sc = ref(a, wdeq)
    assert_matmul_close(y, y_ref, sc, TOL_GEMV, f"outliers M{M} q{qt}")


@pytest.mark.parametrize("M", [1, 3, 8])
def test_gemv_q8_signed_mode(M):
    N, K = 200, 1024
    qw, wdeq = make_weight(N, K, voxq.Q8, seed=77, signed=True)
    a = O.rand_normal(78, M * K).reshape(M, K)
    y = voxq.matmul_nt_q(torch.from_numpy(a).cuda(), qw).cpu().numpy()
    y_ref, sc = ref(a, wdeq)
    assert_matmul_close(y, y_ref, sc, TOL_GEMV, "signed q8")


@pytest.mark.parametrize("qt", [voxq.Q8, voxq.Q4], ids=["q8", "q4"])
@pytest.mark.parametrize("M", [1, 4, 16, 64])
def test_epilogues(qt, M):
    N, K = 384, 1024
    qw, wdeq = make_weight(N, K, qt, seed=5)
    up, updeq = make_weight(N, K, qt, seed=6)
    a = O.rand_normal(7, M * K).reshape(M, K)
    bias = O.rand_normal(8, N)
    res = O.rand_normal(9, M * N).reshape(M, N)
    ad = torch.from_numpy(a).cuda()
    g, gsc = ref(a, wdeq)
    u, usc = ref(a, updeq)
    tol = tol_for(M)
    # bias + residual, residual aliasing the output (in-place residual add)
    out = torch.from_numpy(res.copy()).cuda()
    voxq.matmul_nt_q(ad, qw, out=out, bias=torch.from_numpy(bias).cuda(), residual=out)
    want = g + bias[None, :] + res
    assert_matmul_close(out.cpu().numpy(), want, gsc, tol, "bias+residual")
    # SwiGLU: silu(a W^T) * (a Up^T)   (src/nn.c:148-169)
    y = voxq.matmul_nt_q(ad, qw, up=up).cpu().numpy()
    g64 = g.astype(np.float64)
    sil = g64 / (1 + np.exp(-g64))
    want = sil * u
    # error of silu(g)*u from errors in g and u, each within tol of its scale
    dsil = np.abs(1 / (1 + np.exp(-g64)) * (1 + g64 * (1 - 1 / (1 + np.exp(-g64)))))
    scale = dsil * gsc * np.abs(u) + np.abs(sil) * usc
    err = np.abs(y - want)
    assert np.all(err <= tol * np.maximum(np.abs(want), scale) + 1e-30), "swiglu"


def test_batch_equals_single_calls():
    """voxq_gemv_batch runs each item exactly as a single call would (bitwise)."""
    rng_seed = 100
    specs, singles = [], []
    shapes = [(1, 1024, 1024, voxq.Q4), (1, 128, 1024, voxq.Q4), (3, 4096, 1024, voxq.Q4),
              (1, 1024, 4096, voxq.Q4), (2, 96, 64, voxq.Q4)]
    for i, (M, N, K, qt) in enumerate(shapes):
        qw, _ = make_weight(N, K, qt, seed=rng_seed + i)
        a = torch.from_numpy(O.rand_normal(rng_seed + 50 + i, M * K).reshape(M, K)).cuda()
        out = torch.full((M, N), float("nan"), device="cuda")
        specs.append(dict(w=qw, a=a, out=out))
        singles.append(voxq.matmul_nt_q(a, qw))
    items = voxq.make_gemv_items(specs)
    voxq.gemv_batch(items)
    torch.cuda.synchronize()
    for s, ref_out in zip(specs, singles):
        assert torch.equal(s["out"], ref_out)


@pytest.mark.parametrize("qt", [voxq.Q4, voxq.Q8])
def test_gemv_result_independent_of_launch_size(qt):
    """A single-row GEMV gives the same bits alone (small launch: short tiles)
    and inside a large batch (full-height tiles), and matches the oracle."""
    N, K, n = 4096, 1024, 48
    qw, wdeq = make_weight(N, K, qt, seed=900)
    a = O.rand_normal(901, K).reshape(1, K)
    at = torch.from_numpy(a).cuda()
    alone = voxq.matmul_nt_q(at, qw)
    outs = [torch.full((1, N), float("nan"), device="cuda") for _ in range(n)]
    voxq.gemv_batch(voxq.make_gemv_items([dict(w=qw, a=at, out=o) for o in outs]))
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, alone)
    y, sc = ref(a, wdeq)
    assert_matmul_close(alone.cpu().numpy(), y, sc, TOL_GEMV)


@pytest.mark.parametrize("qt,K", [(voxq.Q4, 160), (voxq.Q4, 96), (voxq.Q8, 96), (voxq.Q4, 4160)])
def test_gemv_single_row_unaligned_trailer_rows(qt, K):
    """Single-row GEMVs whose trailer rows are not 16-byte multiples (K % 128 != 0
    for Q4, K % 64 != 0 for Q8): odd trailer windows, partial 4-chunk groups."""
    N = 300
    qw, wdeq = make_weight(N, K, qt, seed=950 + K)
    a = O.rand_normal(951 + K, K).reshape(1, K)
    bias = O.rand_normal(952 + K, N)
    y = voxq.matmul_nt_q(torch.from_numpy(a).cuda(), qw, bias=torch.from_numpy(bias).cuda()).cpu().numpy()
    want, sc = ref(a, wdeq)
    assert_matmul_close(y, want + bias[None, :], sc, TOL_GEMV)


def test_batch_mixed_formats_and_epilogues():
    specs, wants = [], []
    for i, (qt, M, swi) in enumerate([(voxq.Q8, 1, False), (voxq.Q4, 2, True), (voxq.Q8, 5, True),
                                      (voxq.Q4, 1, False)]):
        N, K = 160 + 32 * i, 512
        qw, wdeq = make_weight(N, K, qt, seed=200 + i)
        a = O.rand_normal(300 + i, M * K).reshape(M, K)
        spec = dict(w=qw, a=torch.from_numpy(a).cuda(), out=torch.empty(M, N, device="cuda"))
        g, gsc = ref(a, wdeq)
        if swi:
            up, updeq = make_weight(N, K, qt, seed=400 + i)
            spec["up"] = up
            u, _ = ref(a, updeq)
            want = (g / (1 + np.exp(-g.astype(np.float64)))) * u
            sc = None
        else:
            bias = O.rand_normal(500 + i, N)
            spec["bias"] = torch.from_numpy(bias).cuda()
            want, sc = g + bias[None, :], gsc
        specs.append(spec)
        wants.append((want, sc))
    voxq.gemv_batch(voxq.make_gemv_items(specs))
    torch.cuda.synchronize()
    for s, (want, sc) in zip(specs, wants):
        y = s["out"].cpu().numpy()
        if sc is not None:
            assert_matmul_close(y, want, sc, TOL_GEMV, "batch bias item")
        else:
            assert np.allclose(y, want, rtol=5e-3, atol=1e-4)


def test_c2_decode_step_full_size():
    """Config 2 at full size: 24 layers x (Q, K, V, O, gate, up, down), Q4, one
    grouped launch; checked against an fp64 product of the device-dequantized
    weights (whose dequantizer is bit-exact with the CPU checker)."""
    H, F, KV, L = 1024, 4096, 128, 24
    shapes = [(H, H), (KV, H), (KV, H), (H, H), (F, H), (F, H), (H, F)]
    g = torch.Generator(device="cuda").manual_seed(1)
    specs = []
    for layer in range(L):
        for (N, K) in shapes:
            w = torch.randn(N, K, device="cuda", generator=g) * 0.02
            qw = voxq.QWeight.from_float(w, voxq.Q4)
            a = torch.randn(1, K, device="cuda", generator=g)
            specs.append(dict(w=qw, a=a, out=torch.empty(1, N, device="cuda")))
    voxq.gemv_batch(voxq.make_gemv_items(specs))
    torch.cuda.synchronize()
    worst = 0.0
    for s in specs:
        qw = s["w"]
        wdeq = voxq.dequantize(qw.to_blocks(), qw.N * qw.K, qw.qtype).view(qw.N, qw.K).double()
        a = s["a"].double()
        y_ref = a @ wdeq.T
        sc = (a.abs() @ wdeq.abs().T) / np.sqrt(qw.K)
        bound = TOL_GEMV * torch.maximum(y_ref.abs(), sc)
        err = (s["out"].double() - y_ref).abs()
        assert bool((err <= bound).all()), f"N{qw.N} K{qw.K}"
        worst = max(worst, float((err / bound).max()) * TOL_GEMV)
    assert worst < TOL_GEMV


@pytest.mark.parametrize("qt", [voxq.Q8, voxq.Q4], ids=["q8", "q4"])
@pytest.mark.parametrize("M,N", [(16, 1024), (64, 1024), (256, 4096), (100, 200), (9, 64)])
def test_gemm_matches_tensor_c(qt, M, N):
    K = 1024
    qw, wdeq = make_weight(N, K, qt, seed=M * 7 + N)
    a = O.rand_normal(M + 5, M * K).reshape(M, K)
    y = voxq.matmul_nt_q(torch.from_numpy(a).cuda(), qw).cpu().numpy()
    y_ref, sc = ref(a, wdeq)
    assert_matmul_close(y, y_ref, sc, TOL_GEMM, f"gemm M{M} N{N}")


# Rows of the M = 2048 outputs checked against the CPU checker: eight rows in
# each 256-row activation tile (its first and last rows, both sides of the
# 64- and 128-row boundaries), 64 in all.
C3_ROWS_2048 = np.array([t * 256 + r for t in range(8) for r in (0, 1, 63, 64, 127, 128, 200, 255)])


@pytest.mark.parametrize("qt", [voxq.Q8, voxq.Q4], ids=["q8", "q4"])
@pytest.mark.parametrize("M", [16, 64, 256, 2048])
@pytest.mark.parametrize("N", [1024, 4096])
def test_gemm_c3_sweep_vs_tensor_c(qt, M, N):
    """Every config-3 case (K = 1024), each of which takes its own launch plan
    (tile width, split-K factor, one or two weight sub-tiles per tile), against
    tensor_matmul_nt (src/tensor.c:617-678) on the dequantized weight."""
    K = 1024
    qw, wdeq = make_weight(N, K, qt, seed=3000 + 7 * M + N)
    a = O.rand_normal(4000 + M + N, M * K).reshape(M, K)
    y = voxq.matmul_nt_q(torch.from_numpy(a).cuda(), qw).cpu().numpy()
    rows = np.arange(M) if M <= 256 else C3_ROWS_2048
    y_ref, sc = ref(a[rows], wdeq)
    assert_matmul_close(y[rows], y_ref, sc, TOL_GEMM, f"c3 M{M} N{N} q{qt}")
    if M == 2048:
        # all rows against an fp64 product of the same operands
        yd = torch.from_numpy(y).double()
        wd = torch.from_numpy(wdeq).double()
        ad = torch.from_numpy(a).double()
        y64 = ad @ wd.T
        sc64 = (ad.abs() @ wd.abs().T) / np.sqrt(K)
        assert bool(((yd - y64).abs() <= TOL_GEMM * torch.maximum(y64.abs(), sc64)).all())


def test_gemm_c3_largest_against_fp64():
    """C3's largest shape (M=2048, N=4096, K=1024) on device data, fp64 torch check."""
    M, N, K = 2048, 4096, 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    for qt in (voxq.Q8, voxq.Q4):
        w = torch.randn(N, K, device="cuda", generator=g) * 0.02
        qw = voxq.QWeight.from_float(w, qt)
        a = torch.randn(M, K, device="cuda", generator=g)
        y = voxq.matmul_nt_q(a, qw)
        wdeq = voxq.dequantize(qw.to_blocks(), N * K, qt).view(N, K).double()
        y_ref = a.double() @ wdeq.T
        sc = (a.double().abs() @ wdeq.abs().T) / np.sqrt(K)
        err = (y.double() - y_ref).abs()
        assert bool((err <= TOL_GEMM * torch.maximum(y_ref.abs(), sc)).all())


def test_dense_fp32_and_fp16_weights():
    for M in (1, 5, 40):
        N, K = 300, 200
        a = O.rand_normal(11, M * K).reshape(M, K)
        w = O.rand_normal(12, N * K, 0.02).reshape(N, K)
        y = voxq.matmul_nt_dense(torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()).cpu().numpy()
        y_ref, sc = ref(a, w)
        assert_matmul_close(y, y_ref, sc, 1e-5, "dense fp32")
        wh = w.astype(np.float16)
        y = voxq.matmul_nt_dense(torch.from_numpy(a).cuda(), torch.from_numpy(wh).cuda()).cpu().numpy()
        y_ref, sc = ref(a, wh.astype(np.float32))
        assert_matmul_close(y, y_ref, sc, 1e-5, "dense fp16")


def test_matmul_rejects_bad_shapes():
    qw, _ = make_weight(64, 64, voxq.Q8, seed=1)
    a = torch.zeros(2, 64, device="cuda")
    out = torch.zeros(2, 64, device="cuda")
    L = voxq.lib()
    d = qw.desc()
    import ctypes as C
    # lda shorter than K
    assert L.voxq_matmul_nt_q(a.data_ptr(), 2, 32, C.byref(d), out.data_ptr(), 64, None, None) == voxq.SHAPE_MISMATCH
    # up-projection with another N
    up, _ = make_weight(32, 64, voxq.Q8, seed=2)
    ud = up.desc()
    epi = voxq.Epilogue(0, 0, 0, C.pointer(ud))
    assert L.voxq_matmul_nt_q(a.data_ptr(), 2, 64, C.byref(d), out.data_ptr(), 64, C.byref(epi),
                              None) == voxq.SHAPE_MISMATCH
    # M = 0 / N = 0 are no-ops
    assert L.voxq_matmul_nt_q(a.data_ptr(), 0, 64, C.byref(d), out.data_ptr(), 64, None, None) == 0
