"""quantize.py containers (VXCPM2) read by the library, no GPU needed.

Fixtures: tests/golden/vxcpm2_{f32,q4,q8,f16}.bin, made by
tests/golden/make_vxcpm2.py -- the f32 file from seeded tensors, the others by
the reference's own convert_quant (scripts/quantize.py:110-312).  The stored
Q4/Q8 blocks are checked against the oracle's quantizer, which is pinned to
quantize.py's block functions (scripts/quantize.py:42-82) elsewhere.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import struct
import sys

import numpy as np
import pytest

import voxq
from voxq.container import VXCPM2
from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
sys.path.insert(0, GOLD)
import make_vxcpm2 as MK  # noqa: E402

KINDS = {"f32": 0, "f16": 1, "q4": 2, "q8": 3}


def path(kind):
    return os.path.join(GOLD, f"vxcpm2_{kind}.bin")


@pytest.mark.parametrize("kind", list(KINDS))
def test_header_and_tensor_table(kind):
    with VXCPM2(path(kind)) as f:
        h = f.header
        assert h["quant"] == KINDS[kind]
        assert h["n_groups"] == MK.N_GROUPS
        for name in MK.HEADER_ORDER:
            if name != "quant":
                assert h[name] == MK.HEADER[name], name
        assert h["rope_theta"] == pytest.approx(MK.HEADER["rope_theta"])
        assert len(f.tensors) == len(MK.TENSORS)  # group 1 is empty and skipped
        for t, (g, name, shape, _) in zip(f.tensors, MK.TENSORS):
            assert t.shape == shape and t.group == g and t.name_hash == MK.name_hash(name)
            n = int(np.prod(shape))
            nb = (n + 31) // 32
            assert t.nbytes == {0: 4 * n, 1: 2 * n, 2: 20 * nb, 3: 40 * nb}[t.dtype]


@pytest.mark.parametrize("kind", ["q4", "q8"])
def test_blocks_are_the_reference_quantizer_output(kind):
    qt = KINDS[kind]
    with VXCPM2(path(kind)) as f:
        for t in f.tensors:
            v = MK.tensor_values(t.index).reshape(-1)
            assert np.array_equal(f.raw(t.index), O.quantize(v, qt)), t


@pytest.mark.parametrize("kind", list(KINDS))
def test_dequantize_matches_oracle(kind):
    with VXCPM2(path(kind)) as f:
        for t in f.tensors:
            v = MK.tensor_values(t.index).reshape(-1)
            got = f.dequantize(t.index).reshape(-1)
            if kind == "f32":
                want = v
            elif kind == "f16":
                want = v.astype(np.float16).astype(np.float32)
            else:
                want = O.dequantize(O.quantize(v, KINDS[kind]), v.size, KINDS[kind]).astype(np.float32)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), t
        if kind == "q8":  # the reference's signed reading (scripts/quantize.py:77-82)
            v = MK.tensor_values(0).reshape(-1)
            want = O.dequantize(O.quantize(v, 3), v.size, 3, q8_signed=True).astype(np.float32)
            assert np.array_equal(f.dequantize(0, q8_signed=True).reshape(-1), want)


def with_checksum(src, dst):
    data = bytearray(open(src, "rb").read())
    digest = hashlib.sha256(bytes(data[:72]) + b"\0" * 8 + bytes(data[80:])).digest()
    data[72:80] = digest[:8]
    open(dst, "wb").write(bytes(data))


def test_checksum(tmp_path):
    with VXCPM2(path("f32")) as f:
        assert f.verify() is True
    # the reference quantizer leaves the field 0 (it raises before writing it)
    for kind in ("q4", "q8", "f16"):
        with VXCPM2(path(kind)) as f:
            assert f.header["checksum"] == 0 and f.verify() is None
    good = tmp_path / "good.bin"
    with_checksum(path("q4"), good)
    with VXCPM2(good) as f:
        assert f.verify() is True
    bad = bytearray(open(good, "rb").read())
    bad[-5] ^= 0x40
    (tmp_path / "bad.bin").write_bytes(bytes(bad))
    with VXCPM2(tmp_path / "bad.bin") as f:
        assert f.verify() is False


def open_code(p):
    with pytest.raises(voxq.VoxqError) as e:
        VXCPM2(p)
    return e.value.code


def test_malformed_files(tmp_path):
    assert open_code(tmp_path / "missing.bin") == -1                 # VOXCPM_ERR_FILE_NOT_FOUND
    data = open(path("q4"), "rb").read()
    (tmp_path / "magic.bin").write_bytes(b"VXCP" + data[4:5] + b"1" + data[6:])  # "VXCPM1"
    assert open_code(tmp_path / "magic.bin") == -2                   # VOXCPM_ERR_INVALID_MODEL
    (tmp_path / "trunc.bin").write_bytes(data[:-7])                  # last tensor cut short
    assert open_code(tmp_path / "trunc.bin") == -2
    (tmp_path / "short.bin").write_bytes(data[:100])                 # no full header
    assert open_code(tmp_path / "short.bin") == -2
    q = bytearray(data)
    struct.pack_into("<I", q, 56, 7)                                  # unknown quant type
    (tmp_path / "quant.bin").write_bytes(bytes(q))
    assert open_code(tmp_path / "quant.bin") == -9                   # VOXCPM_ERR_UNSUPPORTED
    g = bytearray(data)
    struct.pack_into("<I", g, 80, 1 << 20)                            # offset table past the end
    (tmp_path / "groups.bin").write_bytes(bytes(g))
    assert open_code(tmp_path / "groups.bin") == -2
    # an empty file and a directory
    (tmp_path / "empty.bin").write_bytes(b"")
    assert open_code(tmp_path / "empty.bin") == -2
