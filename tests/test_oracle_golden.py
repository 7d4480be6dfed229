"""The CPU checker (oracle/) pinned against the reference's own outputs.

Golden data (tests/golden, made by gen_golden.py from the reference):
  * ref_quant/: the reference gen_test_data.py's Q4/Q8 packs (gen_test_data.py:216-278)
  * quant_cases.json / quant_small.npz: scripts/quantize.py:42-82 over seeded cases
  * ref_matmul.npz: the reference tensor.c (tensor_matmul_nt, tensor_rand_normal)
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest

import cases
from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


@pytest.fixture(scope="module")
def qcases():
    with open(os.path.join(GOLD, "quant_cases.json")) as f:
        return {c["name"]: c for c in json.load(f)["cases"]}


@pytest.mark.parametrize("name", ["q4_uniform", "q4_spread", "q4_extreme", "q4_zero"])
def test_ref_gen_test_data_q4(name):
    x = np.load(os.path.join(GOLD, "ref_quant", f"q4_input_{name}.npy"))
    want = open(os.path.join(GOLD, "ref_quant", f"q4_packed_{name}.bin"), "rb").read()
    assert O.quantize(x, O.QTYPE_Q4).tobytes() == want


@pytest.mark.parametrize("name", ["q8_uniform", "q8_spread"])
def test_ref_gen_test_data_q8(name):
    x = np.load(os.path.join(GOLD, "ref_quant", f"q8_input_{name}.npy"))
    want = open(os.path.join(GOLD, "ref_quant", f"q8_packed_{name}.bin"), "rb").read()
    assert O.quantize(x, O.QTYPE_Q8).tobytes() == want


@pytest.mark.parametrize("name", cases.CASES)
def test_quantize_py_cases(qcases, name):
    """Bit-exact with quantize.py's bytes over every seeded case (~10^6 blocks)."""
    x = cases.make_case(name)
    rec = qcases[name]
    assert rec["n"] == x.size
    for qt, tag in ((O.QTYPE_Q4, "q4"), (O.QTYPE_Q8, "q8")):
        packed = O.quantize(x, qt)
        assert sha(packed) == rec[f"{tag}_sha256"], f"{name} {tag} bytes differ from quantize.py"
        # quantize.py's dequantizer reads Q8 codes as int8 (scripts/quantize.py:79)
        deq = O.dequantize(packed, x.size, qt, q8_signed=True)
        assert sha(deq.tobytes()) == rec[f"{tag}_dequant_sha256"], f"{name} {tag} dequant differs"


def test_small_cases_verbatim():
    z = np.load(os.path.join(GOLD, "quant_small.npz"))
    seen = 0
    for name in cases.SMALL_CASES:
        x = cases.make_case(name)
        for qt, tag in ((O.QTYPE_Q4, "q4"), (O.QTYPE_Q8, "q8")):
            key = f"{name}.{tag}"
            if key not in z:
                continue
            seen += 1
            got = O.quantize(x, qt)
            np.testing.assert_array_equal(got, z[key], err_msg=key)
            deq = O.dequantize(got, x.size, qt, q8_signed=True)
            np.testing.assert_array_equal(deq.view(np.uint32), z[key + ".dequant"].view(np.uint32), err_msg=key)
    assert seen >= 8


def test_q8_unsigned_reading_is_the_quantizer_intent():
    """Unsigned Q8 reading reconstructs within half a step; quantize.py's signed read does not."""
    x = cases.make_case("normal1")[: 32 * 4096]
    p = O.quantize(x, O.QTYPE_Q8)
    blocks = p.reshape(-1, 40)
    step = blocks[:, 32:36].copy().view(np.float32).ravel()
    u = O.dequantize(p, x.size, O.QTYPE_Q8, q8_signed=False).reshape(-1, 32)
    s = O.dequantize(p, x.size, O.QTYPE_Q8, q8_signed=True).reshape(-1, 32)
    xr = x.reshape(-1, 32)
    # half a quantization step, plus the two fp32 roundings of q*scale+min
    slack = 4 * np.spacing(np.abs(xr).astype(np.float32)) + 4 * np.spacing(np.float32(1e-30))
    assert np.all(np.abs(u - xr) <= 0.5 * step[:, None] * (1 + 1e-5) + slack)
    assert np.abs(s - xr).max() > 10 * np.abs(u - xr).max()


def test_double_to_half_matches_numpy():
    r = np.random.RandomState(5)
    vals = np.concatenate([
        r.randn(20000) * 10.0 ** r.uniform(-10, 6, 20000),
        [0.0, -0.0, 65504.0, 65519.99, 65520.0, 65536.0, 1e300, -1e300, 2.0 ** -24, 2.0 ** -25,
         2.0 ** -25 * 1.0000001, 3 * 2.0 ** -26, 6.1e-5, 5.96e-8, np.inf, -np.inf, np.nan],
    ])
    got = np.array([O.double_to_half(v) for v in vals], dtype=np.uint16)
    want = np.array([np.float16(v).view(np.uint16) for v in vals], dtype=np.uint16)
    np.testing.assert_array_equal(got, want)


def test_ref_matmul_kat():
    """tests/test_tensor.c:130-161 known answer, NT layout."""
    z = np.load(os.path.join(GOLD, "ref_matmul.npz"))
    np.testing.assert_array_equal(z["kat.out"], np.array([[58, 64], [139, 154]], dtype=np.float32))
    a = np.array([[1, 2, 3], [4, 5, 6]], dtype=np.float32)
    bt = np.array([[7, 9, 11], [8, 10, 12]], dtype=np.float32)
    np.testing.assert_array_equal(O.matmul_nt(a, bt), z["kat.out"])


@pytest.mark.parametrize("shape", cases.MATMUL_CASES, ids=lambda s: f"{s[0]}x{s[1]}x{s[2]}")
def test_oracle_matmul_vs_reference_tensor_c(shape):
    M, N, K, _, _ = shape
    z = np.load(os.path.join(GOLD, "ref_matmul.npz"))
    a, w, ref = z[f"{M}x{N}x{K}.a"], z[f"{M}x{N}x{K}.w"], z[f"{M}x{N}x{K}.out"]
    got = O.matmul_nt(a, w)
    # same single fp32 accumulator order; the compiled reference may fuse the
    # multiply-add (x86-64-v3 has FMA), so allow a few ulps of the running sum
    _, absscale = O.matmul_nt_f64(a, w)
    assert np.all(np.abs(got - ref) <= 1e-5 * np.maximum(np.abs(ref), absscale))


def test_rng_matches_reference():
    z = np.load(os.path.join(GOLD, "ref_matmul.npz"))
    np.testing.assert_array_equal(O.rand_normal(1, 1001), z["rng.seed1"])
    np.testing.assert_array_equal(O.rand_normal(2, 64), z["rng.seed2"])


@pytest.mark.skipif(not O.ref_available(), reason="reference tensor.c not built here")
def test_oracle_vs_live_reference():
    for (M, N, K) in [(1, 17, 64), (4, 96, 320), (7, 5, 1024)]:
        a = O.rand_normal(3, M * K).reshape(M, K)
        w = O.rand_normal(4, N * K, 0.02).reshape(N, K)
        ref = O.ref_matmul_nt(a, w)
        got = O.matmul_nt(a, w)
        _, absscale = O.matmul_nt_f64(a, w)
        assert np.all(np.abs(got - ref) <= 1e-5 * np.maximum(np.abs(ref), absscale))


def test_tail_padding_and_sizes():
    for n in (1, 7, 31, 32, 33, 481):
        x = cases.make_case("tail481")[:n]
        p4 = O.quantize(x, O.QTYPE_Q4)
        p8 = O.quantize(x, O.QTYPE_Q8)
        nb = (n + 31) // 32
        assert p4.size == nb * 20 and p8.size == nb * 40
        # the padded tail equals quantizing the explicitly zero-padded block
        xp = np.zeros(nb * 32, dtype=np.float32)
        xp[:n] = x
        np.testing.assert_array_equal(p4, O.quantize(xp, O.QTYPE_Q4))
        np.testing.assert_array_equal(p8, O.quantize(xp, O.QTYPE_Q8))
