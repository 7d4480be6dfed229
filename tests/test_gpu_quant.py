"""Device quantizer / dequantizer / layout packing vs the reference bytes.

Bit-exact bar: the device quantize.py restatement must reproduce the SHA-256
of quantize.py's own output (tests/golden/quant_cases.json) on every case.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest

import cases
from oracle import oracle as O

torch = pytest.importorskip("torch")
import voxq  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


@pytest.fixture(scope="module")
def qcases():
    with open(os.path.join(GOLD, "quant_cases.json")) as f:
        return {c["name"]: c for c in json.load(f)["cases"]}


@pytest.mark.parametrize("name", cases.CASES)
def test_device_quantizer_matches_quantize_py(qcases, name):
    x = cases.make_case(name)
    xd = torch.from_numpy(x).cuda()
    rec = qcases[name]
    for qt, tag in ((voxq.Q4, "q4"), (voxq.Q8, "q8")):
        packed = voxq.quantize(xd, qt)
        torch.cuda.synchronize()
        got = packed.cpu().numpy()
        assert sha(got) == rec[f"{tag}_sha256"], f"{name}/{tag}: device bytes differ from quantize.py"
        deq_s = voxq.dequantize(packed, x.size, qt, q8_signed=True).cpu().numpy()
        assert sha(deq_s.tobytes()) == rec[f"{tag}_dequant_sha256"], f"{name}/{tag}: dequant differs"
        deq_u = voxq.dequantize(packed, x.size, qt, q8_signed=False).cpu().numpy()
        want_u = O.dequantize(got, x.size, qt, q8_signed=False)
        np.testing.assert_array_equal(deq_u.view(np.uint32), want_u.view(np.uint32))


def test_ref_gen_test_data_packs_on_device():
    for name, qt in [("q4_uniform", voxq.Q4), ("q4_extreme", voxq.Q4), ("q4_zero", voxq.Q4),
                     ("q8_uniform", voxq.Q8), ("q8_spread", voxq.Q8)]:
        tag = "q4" if qt == voxq.Q4 else "q8"
        x = np.load(os.path.join(GOLD, "ref_quant", f"{tag}_input_{name}.npy"))
        want = open(os.path.join(GOLD, "ref_quant", f"{tag}_packed_{name}.bin"), "rb").read()
        got = voxq.quantize(torch.from_numpy(x).cuda(), qt).cpu().numpy().tobytes()
        assert got == want, name


@pytest.mark.parametrize("qt", [voxq.Q4, voxq.Q8])
@pytest.mark.parametrize("N,K", [(1, 32), (7, 96), (64, 1024), (130, 4096)])
def test_packed_layout_roundtrip(qt, N, K):
    w = torch.from_numpy(O.rand_normal(N * 7 + K, N * K, 0.02).reshape(N, K)).cuda()
    blocks = torch.zeros(voxq.quant_bytes(N * K, qt), dtype=torch.uint8, device="cuda")
    qw = voxq.QWeight.from_float(w, qt, blocks_out=blocks)
    # the packed layout is the block stream split into codes and trailers
    np.testing.assert_array_equal(blocks.cpu().numpy(), O.quantize(w.cpu().numpy(), qt))
    qw2 = voxq.QWeight.from_blocks(blocks, N, K, qt)
    assert torch.equal(qw.codes, qw2.codes) and torch.equal(qw.scales, qw2.scales)
    assert torch.equal(qw.to_blocks(), blocks)
    # row multipliers: powers of two putting each row's largest |w| in [2^13, 2^14)
    nb = K // 32
    tb = N * nb * (4 if qt == voxq.Q4 else 8)
    off = (tb + 15) // 16 * 16
    rowmul = qw.scales[off:off + 4 * N].view(torch.float32).cpu().numpy()
    wd = O.dequantize(blocks.cpu().numpy(), N * K, qt).reshape(N, K)
    wmax = np.abs(wd).max(axis=1) * rowmul
    mant, _ = np.frexp(rowmul)
    assert np.all(mant == 0.5)
    assert np.all((wmax < 2.0 ** 14) & ((wmax >= 2.0 ** 12) | (wmax == 0)))


def test_quantize_rejects_bad_arguments():
    L = voxq.lib()
    x = torch.zeros(64, device="cuda")
    out = torch.zeros(80, dtype=torch.uint8, device="cuda")
    assert L.voxq_quantize(x.data_ptr(), 64, voxq.F32, out.data_ptr(), None) == voxq.UNSUPPORTED
    assert L.voxq_quantize(x.data_ptr(), 0, voxq.Q8, out.data_ptr(), None) == 0
    codes = torch.zeros(64, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(64, dtype=torch.uint8, device="cuda")
    assert L.voxq_quantize_weight(x.data_ptr(), 2, 31, voxq.Q8, codes.data_ptr(), sc.data_ptr(), None,
                                  None) == voxq.SHAPE_MISMATCH
