"""Pre-quantized weights in the engine's VXCP container, on the device.

voxq_vxcp_quantize rewrites a VXCP model file with its 2-D weights as Q4_1 /
Q8 blocks (include/voxq.h), quantized on the GPU: the blocks must be the
oracle's restatement of scripts/quantize.py's quantizer (:42-75) on the same
values byte for byte, every other tensor copied unchanged, both CRC32C
checksums valid.  voxq_tensor_attach_blocks hands such blocks to
tensor_to_cuda: the device weight must then hold exactly those blocks
(tensor_to_cpu returns the oracle's dequantization bit for bit) and multiply
like any uploaded weight (oracle matmul, the library's 1e-3 / 5e-3 rule).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

from conftest import assert_matmul_close
from oracle import oracle as O

torch = pytest.importorskip("torch")
import voxq  # noqa: E402
from voxq import vxcp  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture()
def lib_f32():
    L = voxq.lib()
    L.tensor_cuda_shutdown()
    old = os.environ.pop("VOXCPM_QUANT", None)
    assert L.tensor_cuda_init() == 0
    yield L
    L.tensor_cuda_shutdown()
    if old is not None:
        os.environ["VOXCPM_QUANT"] = old


def _model(rng):
    """A small VXCP model: (name, dtype, shape, raw, fp32 values or None)."""
    out = []
    w = (rng.standard_normal((64, 128)) * 0.02).astype(np.float32)
    out.append(("base_lm.layers.0.self_attn.q_proj.weight", vxcp.FP32, w.shape, w.tobytes(), w))
    h = (rng.standard_normal((32, 64)) * 0.02).astype(np.float16)
    out.append(("base_lm.layers.0.mlp.up_proj.weight", vxcp.FP16, h.shape, h.tobytes(), h.astype(np.float32)))
    b = (rng.standard_normal((16, 32)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    out.append(("feat_decoder.proj.weight", vxcp.BF16, b.shape, b.tobytes(),
                (b.astype(np.uint32) << 16).view(np.float32)))
    e = (rng.standard_normal((50, 64)) * 0.02).astype(np.float16)
    out.append(("base_lm.embed_tokens.weight", vxcp.FP16, e.shape, e.tobytes(), None))  # kept by name
    n = np.ones(64, np.float32)
    out.append(("base_lm.norm.weight", vxcp.FP32, n.shape, n.tobytes(), None))         # 1-D
    o = rng.standard_normal((7, 40)).astype(np.float32)
    out.append(("stop_head.weight", vxcp.FP32, o.shape, o.tobytes(), None))            # rows of 40
    s = O.quantize(rng.standard_normal(64).astype(np.float32), voxq.Q8)
    out.append(("already.q8", vxcp.Q8_BLOCKS, (2, 32), vxcp.stream_to_blocks(s, voxq.Q8).tobytes(), None))
    return out


@pytest.mark.parametrize("qtype", [voxq.Q8, voxq.Q4])
def test_vxcp_quantize_file(tmp_path, qtype):
    torch.cuda.init()
    rng = np.random.default_rng(5)
    ts = _model(rng)
    src, dst = str(tmp_path / "m.vxcpm"), str(tmp_path / "mq.vxcpm")
    vxcp.write(src, [(n, d, s, r) for n, d, s, r, _ in ts])
    st = vxcp.quantize_file(src, dst, qtype, keep=("embed_tokens",))
    assert st == {"tensors": len(ts), "quantized": 3, "bytes_in": os.path.getsize(src),
                  "bytes_out": os.path.getsize(dst)}
    hdr, entries = vxcp.read_index(dst)
    assert hdr["data_end"] == os.path.getsize(dst)
    data = open(dst, "rb").read()
    head = bytearray(data[:64])
    head[56:64] = bytes(8)
    assert vxcp.crc32c(bytes(head)) == hdr["header_crc32c"]
    assert vxcp.crc32c(data[64:]) == hdr["data_crc32c"]
    qdt = vxcp.Q4_1 if qtype == voxq.Q4 else vxcp.Q8_BLOCKS
    for (name, dt, shape, raw, vals), e in zip(ts, entries):
        assert e.name == name and e.shape == shape
        got = vxcp.read_raw(dst, e)
        if vals is None:
            assert e.dtype == dt and got == raw, f"{name} changed"
        else:
            assert e.dtype == qdt, name
            want = np.asarray(O.quantize(vals.reshape(-1), qtype), np.uint8)
            np.testing.assert_array_equal(vxcp.blocks_to_stream(got, qdt), want, err_msg=name)


def test_vxcp_quantize_errors(tmp_path):
    torch.cuda.init()
    L = voxq.lib()
    bad = str(tmp_path / "bad.vxcpm")
    open(bad, "wb").write(b"NOTVXCP" + bytes(100))
    rc = L.voxq_vxcp_quantize(bad.encode(), str(tmp_path / "o").encode(), voxq.Q8, None, 0, None)
    assert rc == -2 and not os.path.exists(tmp_path / "o")
    assert L.voxq_vxcp_quantize(str(tmp_path / "none").encode(), bad.encode(), voxq.Q8, None, 0, None) == -1
    ok = str(tmp_path / "ok.vxcpm")
    vxcp.write(ok, [("w", vxcp.FP32, (4, 32), np.ones((4, 32), np.float32).tobytes())])
    assert L.voxq_vxcp_quantize(ok.encode(), bad.encode(), voxq.F16, None, 0, None) == voxq.UNSUPPORTED
    q40 = str(tmp_path / "q40.vxcpm")
    vxcp.write(q40, [("w", vxcp.Q4_0, (1, 32), bytes(18))])
    assert L.voxq_vxcp_quantize(q40.encode(), str(tmp_path / "o2").encode(), voxq.Q8, None, 0, None) == \
        voxq.UNSUPPORTED


def _attach(L, t, stream, qtype):
    """Attaches a malloc'd copy of `stream`; frees it again if refused."""
    buf = voxq._libc.malloc(len(stream))
    C.memmove(buf, bytes(stream), len(stream))
    rc = L.voxq_tensor_attach_blocks(t, qtype, buf, len(stream))
    if rc != 0:
        voxq._libc.free(buf)
    return rc


@pytest.mark.parametrize("qtype", [voxq.Q8, voxq.Q4])
@pytest.mark.parametrize("M", [1, 24])
def test_attached_blocks_upload(lib_f32, qtype, M):
    L = lib_f32
    N, K = 512, 256
    w = O.rand_normal(21, N * K, 0.02).reshape(N, K)
    stream = np.asarray(O.quantize(w, qtype), np.uint8)
    wdeq = O.dequantize(stream, N * K, qtype).reshape(N, K).astype(np.float32)
    # the loader's tensor: the dequantized values on the host, the blocks attached
    wt = voxq.host_tensor(wdeq)
    assert _attach(L, wt, stream, qtype) == 0
    assert L.tensor_to_cuda(wt) == 0 and wt.contents.is_cuda
    a = O.rand_normal(22, M * K).reshape(M, K)
    at = voxq.host_tensor(a)
    ot = voxq.host_tensor(np.zeros((M, N), np.float32))
    assert L.tensor_matmul_nt_cuda(at, wt, ot) == 0
    tol = 1e-3 if M <= 8 else 5e-3
    assert_matmul_close(voxq.host_tensor_view(ot), O.matmul_nt(a, wdeq), O.matmul_nt_f64(a, wdeq)[1], tol,
                        f"attached q{qtype} M{M}")
    # the device weight is exactly the attached blocks
    assert L.tensor_to_cpu(wt) == 0
    np.testing.assert_array_equal(voxq.host_tensor_view(wt).view(np.uint32), wdeq.view(np.uint32))
    for t in (wt, at, ot):
        voxq.free_tensor(t)


def test_attach_rules(lib_f32):
    L = lib_f32
    w = np.ones((8, 64), np.float32)
    stream = np.asarray(O.quantize(w, voxq.Q8), np.uint8)
    t = voxq.host_tensor(w)
    # wrong byte count / non-block rows / 1-D are refused, ownership stays with the caller
    buf = voxq._libc.malloc(10)
    assert L.voxq_tensor_attach_blocks(t, voxq.Q8, buf, 10) == voxq.SHAPE_MISMATCH
    voxq._libc.free(buf)
    odd = voxq.host_tensor(np.ones((4, 40), np.float32))
    assert _attach(L, odd, stream, voxq.Q8) == voxq.SHAPE_MISMATCH
    one_d = voxq.host_tensor(np.ones(512, np.float32))
    assert _attach(L, one_d, stream, voxq.Q8) == voxq.SHAPE_MISMATCH
    # detach frees them; a later upload quantizes nothing (VOXCPM_QUANT unset: fp32)
    assert _attach(L, t, stream, voxq.Q8) == 0
    assert L.voxq_tensor_detach_blocks(t) == 1 and L.voxq_tensor_detach_blocks(t) == 0
    assert L.tensor_to_cuda(t) == 0 and L.tensor_to_cpu(t) == 0
    np.testing.assert_array_equal(voxq.host_tensor_view(t), w)
    # blocks attached to a tensor whose host buffer has since changed (another
    # tensor at the same address) are dropped, not uploaded
    t2 = voxq.host_tensor(np.full((8, 64), 2.0, np.float32))
    assert _attach(L, t2, stream, voxq.Q8) == 0
    new = voxq.host_tensor(np.full((8, 64), 3.0, np.float32))
    fp = C.POINTER(C.c_float)
    a_old = C.cast(t2.contents.data, C.c_void_p).value
    a_new = C.cast(new.contents.data, C.c_void_p).value
    t2.contents.data = C.cast(a_new, fp)
    new.contents.data = C.cast(a_old, fp)
    assert L.tensor_to_cuda(t2) == 0 and L.tensor_to_cpu(t2) == 0
    np.testing.assert_array_equal(voxq.host_tensor_view(t2), np.full((8, 64), 3.0, np.float32))
    for x in (t, odd, one_d, t2, new):
        voxq.free_tensor(x)
