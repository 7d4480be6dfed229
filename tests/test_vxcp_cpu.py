"""The VXCP loader with voxq's quantized dtypes, on the host.

`vxcp_load_check` runs voxq_vxcp_load.c -- the weight_index_build /
weight_load_tensor that the qfile engine build links in place of the engine's
own (src/model.c:1628-1877) -- on a small file written here, and prints what
it loaded.  Expected values come from the oracle: Q4 / Q8 blocks from its
restatement of quantize.py's quantizer (scripts/quantize.py:42-75), the
loaded floats from its dequantizer (scripts/quantize.py:56-82, unsigned Q8
codes), the other dtypes as src/model.c:1811-1858 converts them.  Checked:
data offsets of every dtype (the engine's loader sizes Q4_0 / Q4_1 as 0
bytes), the fp32 / fp16 payload bit for bit, NaN -> 0, which tensors get
their blocks attached for tensor_to_cuda (2-D, rows a multiple of 32) and
that those blocks are the quantize.py stream byte for byte.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "voxcpm2-c_b200"))
sys.path.insert(0, REPO)

from oracle import oracle  # noqa: E402
from voxq import Q4, Q8  # noqa: E402
from voxq import vxcp  # noqa: E402

CHECK = os.path.join(REPO, "voxcpm2-c_b200", "engine", "_build", "vxcp_load_check")


def fnv(b: bytes) -> str:
    h = 1469598103934665603
    for x in b:
        h = ((h ^ x) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return f"{h:016x}"


def _tensors(rng):
    """(name, dtype, shape, raw, expected host data bytes, kept fp16, attached qtype, stream)."""
    out = []

    def q(name, shape, qtype, scale=0.05):
        x = (rng.standard_normal(int(np.prod(shape))) * scale).astype(np.float32)
        stream = oracle.quantize(x, qtype)
        raw = vxcp.stream_to_blocks(stream, qtype).tobytes()
        dt = vxcp.Q4_1 if qtype == Q4 else vxcp.Q8_BLOCKS
        deq = oracle.dequantize(stream, x.size, qtype).astype(np.float32)
        att = (2 if qtype == Q4 else 3) if len(shape) == 2 and shape[1] % 32 == 0 else 0
        out.append((name, dt, shape, raw, deq.tobytes(), 0, att, bytes(stream) if att else None))

    q("layers.1.attn.wq.weight", (6, 64), Q8)
    q("layers.0.ffn.w1.weight", (5, 96), Q4)
    q("special.q8_1d", (70,), Q8)          # 1-D: dequantized only; last block padded
    q("zz.q4_rows20", (3, 20), Q4)          # rows not a multiple of 32: dequantized only
    h = (rng.standard_normal((3, 40)) * 0.1).astype(np.float16)
    out.append(("proj.fp16", vxcp.FP16, (3, 40), h.tobytes(), h.tobytes(), 1, 0, None))
    h1 = (rng.standard_normal(17)).astype(np.float16)
    out.append(("norm.fp16_1d", vxcp.FP16, (17,), h1.tobytes(), h1.astype(np.float32).tobytes(), 0, 0, None))
    b = (rng.standard_normal((4, 8)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    out.append(("emb.bf16", vxcp.BF16, (4, 8), b.tobytes(),
                (b.astype(np.uint32) << 16).view(np.float32).tobytes(), 0, 0, None))
    f = rng.standard_normal(9).astype(np.float32)
    f[3] = np.nan
    g = f.copy()
    g[3] = 0.0
    out.append(("bias.f32", vxcp.FP32, (9,), f.tobytes(), g.tobytes(), 0, 0, None))
    return out


@pytest.mark.skipif(not os.path.exists(CHECK), reason="engine harness not built (needs the reference checkout)")
def test_loader_reads_quantized_dtypes(tmp_path):
    rng = np.random.default_rng(7)
    ts = _tensors(rng)
    path = str(tmp_path / "m.vxcpm")
    vxcp.write(path, [(n, d, s, r) for n, d, s, r, *_ in ts])
    hdr, entries = vxcp.read_index(path)
    assert hdr["data_end"] == os.path.getsize(path)
    r = subprocess.run([CHECK, path], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    lines = [json.loads(x) for x in r.stdout.strip().splitlines()]
    assert lines[-1] == {"tensors": len(ts), "status": 0}, r.stdout
    got = {x["name"]: x for x in lines[:-1]}
    assert list(got) == sorted(got), "index not sorted by name"
    by_name = {e.name: e for e in entries}
    for name, dt, shape, raw, want, f16, att, stream in ts:
        g, e = got[name], by_name[name]
        assert (g["dtype"], tuple(g["shape"]), g["offset"], g["bytes"]) == (dt, shape, e.offset, len(raw)), name
        assert g["load"] == 0 and g["fp16"] == f16, (name, g)
        assert g["fnv"] == fnv(want), f"{name}: loaded data differs"
        assert g["attached"] == att, (name, g)
        if att:
            assert g["blocks_fnv"] == fnv(stream), f"{name}: attached blocks are not the quantize.py stream"


@pytest.mark.skipif(not os.path.exists(CHECK), reason="engine harness not built (needs the reference checkout)")
def test_loader_sizes_and_rejects_q4_0(tmp_path):
    """Q4_0 has no producer and no dequantization: the index sizes it (18-byte
    blocks, docs/WEIGHT_FORMAT.md §5) so later tensors stay in place; loading it fails."""
    a = np.arange(8, dtype=np.float32)
    path = str(tmp_path / "q40.vxcpm")
    vxcp.write(path, [("a.q40", vxcp.Q4_0, (2, 32), bytes(36)), ("b.f32", vxcp.FP32, (8,), a.tobytes())])
    r = subprocess.run([CHECK, path], capture_output=True, text=True, timeout=60)
    lines = [json.loads(x) for x in r.stdout.strip().splitlines()]
    got = {x["name"]: x for x in lines[:-1]}
    assert got["a.q40"]["bytes"] == 36 and got["a.q40"]["load"] == -9
    assert got["b.f32"]["load"] == 0 and got["b.f32"]["fnv"] == fnv(a.tobytes())
    assert got["b.f32"]["offset"] == got["a.q40"]["offset"] + 36


@pytest.mark.skipif(not os.path.exists(CHECK), reason="engine harness not built (needs the reference checkout)")
def test_loader_rejects_corrupt_shapes(tmp_path):
    """Malformed index entries end in VOXCPM_ERR_INVALID_MODEL (-2), never in a read outside
    the file or the entry: a shape whose value count would wrap 64 bits (the index is refused),
    and an ndim of 0 (sized by the index as one value, src/model.c:1715-1719) whose shape[0]
    names 1000 values (the load of that tensor is refused; the engine's loader would read them)."""
    import struct
    a = np.arange(1000, dtype=np.float32)
    base = str(tmp_path / "ok.vxcpm")
    vxcp.write(base, [("a.f32", vxcp.FP32, (1000,), a.tobytes()), ("b.f32", vxcp.FP32, (8,), a[:8].tobytes())])
    raw = bytearray(open(base, "rb").read())
    wrap = bytearray(raw)
    struct.pack_into("<5I", wrap, 64 + 12, 4, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF)
    p = tmp_path / "wrap.vxcpm"
    p.write_bytes(bytes(wrap))
    r = subprocess.run([CHECK, str(p)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and json.loads(r.stdout.strip().splitlines()[-1]) == {"tensors": 0, "status": -2}
    assert "impossible shape" in r.stderr
    flat = bytearray(raw)
    struct.pack_into("<I", flat, 64 + 12, 0)  # a.f32: ndim 0, shape[0] still 1000
    p = tmp_path / "ndim0.vxcpm"
    p.write_bytes(bytes(flat))
    r = subprocess.run([CHECK, str(p)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    got = {x["name"]: x for x in map(json.loads, r.stdout.strip().splitlines()[:-1])}
    assert got["a.f32"]["bytes"] == 4 and got["a.f32"]["load"] == -2


def test_writer_checksums_and_block_order(tmp_path):
    """The writer's header / data CRC32C and the VXCP <-> quantize.py block order round trip."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal(96).astype(np.float32)
    for qtype, dt in ((Q4, vxcp.Q4_1), (Q8, vxcp.Q8_BLOCKS)):
        s = oracle.quantize(x, qtype)
        b = vxcp.stream_to_blocks(s, qtype)
        assert np.array_equal(vxcp.blocks_to_stream(b.tobytes(), dt), np.asarray(s, np.uint8))
        if qtype == Q4:  # header first: fp16 scale, fp16 min at the block start
            assert bytes(b[:4]) == bytes(np.asarray(s, np.uint8)[16:20])
    path = str(tmp_path / "c.vxcpm")
    vxcp.write(path, [("t", vxcp.FP32, (96,), x.tobytes())])
    data = open(path, "rb").read()
    head = bytearray(data[:64])
    head[56:64] = bytes(8)
    assert vxcp.crc32c(bytes(head)) == int.from_bytes(data[56:60], "little")
    assert vxcp.crc32c(data[64:]) == int.from_bytes(data[60:64], "little")
