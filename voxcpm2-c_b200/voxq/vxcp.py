"""The engine's VXCP weight container with voxq's quantized dtypes.

VXCP is the format the reference engine loads (docs/WEIGHT_FORMAT.md, read by
src/model.c:1628-1877): a 64-byte header ("VXCP", version 1, tensor count,
CRC32C of the header at 56 and of metadata + names + data at 60), one 32-byte
entry per tensor (name offset, name length, dtype, ndim, shape[4]), the string
table, then the tensors' data back to back in entry order from the byte after
the last name's NUL.  The format names Q4_0 / Q4_1 but the engine's loader
cannot read them; include/voxq.h defines the quantized dtypes voxq writes:

    4  Q4_1  20-byte blocks: fp16 d, fp16 m, 16 code bytes (quantize.py nibbles)
    5  Q8    40-byte blocks: fp32 d, fp32 m, 32 code bytes (unsigned)

with d, m and the codes of scripts/quantize.py's blocks, header fields first.

`quantize_file` runs the library's device converter (voxq_vxcp_quantize);
`read_index` / `read_raw` / `write` are host code for inspecting and writing
such files (no device needed).
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass
from typing import Iterable, Sequence

import numpy as np

from . import Q4, Q8, check, lib

FP32, BF16, FP16, Q4_0, Q4_1, Q8_BLOCKS = 0, 1, 2, 3, 4, 5
MAGIC = 0x56435850
HEADER, META = 64, 32
_BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q8_BLOCKS: 40}


class VoxqStats(C.Structure):
    """voxq_vxcp_stats (include/voxq.h)."""
    _fields_ = [("tensors", C.c_uint32), ("quantized", C.c_uint32), ("bytes_in", C.c_uint64),
                ("bytes_out", C.c_uint64)]


@dataclass(frozen=True)
class Entry:
    name: str
    dtype: int
    shape: tuple
    offset: int
    nbytes: int

    @property
    def elements(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64))


def dtype_bytes(dtype: int, n: int) -> int:
    """Bytes of n values stored as `dtype`."""
    if dtype == FP32:
        return 4 * n
    if dtype in (BF16, FP16):
        return 2 * n
    if dtype in _BLOCK_BYTES:
        return _BLOCK_BYTES[dtype] * ((n + 31) // 32)
    raise ValueError(f"unknown VXCP dtype {dtype}")


def crc32c(data, crc: int = 0) -> int:
    """CRC32C (Castagnoli) of bytes-like `data`, continuing from `crc`."""
    table = _crc_table()
    c = crc ^ 0xFFFFFFFF
    for b in memoryview(data).cast("B"):
        c = table[(c ^ b) & 0xFF] ^ (c >> 8)
    return c ^ 0xFFFFFFFF


_TABLE = None


def _crc_table():
    global _TABLE
    if _TABLE is None:
        t = []
        for i in range(256):
            c = i
            for _ in range(8):
                c = (c >> 1) ^ 0x82F63B78 if c & 1 else c >> 1
            t.append(c)
        _TABLE = t
    return _TABLE


def read_index(path: str) -> tuple[dict, list[Entry]]:
    """(header fields, entries in file order) of a VXCP file."""
    with open(path, "rb") as f:
        head = f.read(HEADER)
        magic, version, n = struct.unpack_from("<III", head)
        if magic != MAGIC or version != 1:
            raise ValueError(f"{path}: not a VXCP version-1 file")
        meta = f.read(META * n)
        metas = [struct.unpack_from("<8I", meta, META * i) for i in range(n)]
        name_end = max(m[0] + m[1] for m in metas)
        names = f.read(name_end + 1)
    pos = HEADER + META * n + name_end + 1
    entries = []
    for no, nl, dt, nd, *shape in metas:
        shp = tuple(shape[:nd])
        nb = dtype_bytes(dt, int(np.prod(shp, dtype=np.int64)))
        entries.append(Entry(names[no:no + nl].decode(), dt, shp, pos, nb))
        pos += nb
    hdr = {"tensors": n, "header_crc32c": struct.unpack_from("<I", head, 56)[0],
           "data_crc32c": struct.unpack_from("<I", head, 60)[0], "data_end": pos}
    return hdr, entries


def read_raw(path: str, e: Entry) -> bytes:
    with open(path, "rb") as f:
        f.seek(e.offset)
        return f.read(e.nbytes)


def blocks_to_stream(raw: bytes, dtype: int) -> np.ndarray:
    """VXCP Q4_1 / Q8 blocks -> the quantize.py block stream (codes first)."""
    bb = _BLOCK_BYTES[dtype]
    hb = 4 if dtype == Q4_1 else 8
    b = np.frombuffer(raw, np.uint8).reshape(-1, bb)
    return np.concatenate([b[:, hb:], b[:, :hb]], axis=1).reshape(-1)


def stream_to_blocks(stream, qtype: int) -> np.ndarray:
    """The quantize.py block stream (Q4 or Q8) -> VXCP Q4_1 / Q8 blocks."""
    bb, hb = (20, 4) if qtype == Q4 else (40, 8)
    b = np.asarray(stream, np.uint8).reshape(-1, bb)
    return np.concatenate([b[:, bb - hb:], b[:, :bb - hb]], axis=1).reshape(-1)


def write(path: str, tensors: Sequence[tuple[str, int, tuple, bytes]]) -> None:
    """Writes (name, dtype, shape, raw data) tensors as a VXCP file with both checksums."""
    names = b""
    meta = b""
    for name, dt, shape, raw in tensors:
        if len(raw) != dtype_bytes(dt, int(np.prod(shape, dtype=np.int64))):
            raise ValueError(f"{name}: {len(raw)} bytes for dtype {dt} shape {shape}")
        nb = name.encode()
        shp = list(shape) + [1] * (4 - len(shape))
        meta += struct.pack("<8I", len(names), len(nb), dt, len(shape), *shp)
        names += nb + b"\0"
    data_crc = crc32c(meta + names)
    for _, _, _, raw in tensors:
        data_crc = crc32c(raw, data_crc)
    head = bytearray(HEADER)
    struct.pack_into("<III", head, 0, MAGIC, 1, len(tensors))
    struct.pack_into("<I", head, 56, crc32c(bytes(head)))
    struct.pack_into("<I", head, 60, data_crc)
    with open(path, "wb") as f:
        f.write(bytes(head))
        f.write(meta)
        f.write(names)
        for _, _, _, raw in tensors:
            f.write(raw)


def quantize_file(src: str, dst: str, qtype: int, keep: Iterable[str] = ("embed_tokens",)) -> dict:
    """voxq_vxcp_quantize: src's 2-D fp32/fp16/bf16 tensors (rows a multiple of
    32, names without any `keep` substring) quantized on the current device
    into dst as Q4_1 (qtype Q4) or Q8 (qtype Q8) blocks."""
    keep = [k.encode() for k in keep]
    arr = (C.c_char_p * max(1, len(keep)))(*keep)
    st = VoxqStats()
    check(lib().voxq_vxcp_quantize(str(src).encode(), str(dst).encode(), qtype, arr, len(keep), C.byref(st)),
          f"voxq_vxcp_quantize({src})")
    return {"tensors": st.tensors, "quantized": st.quantized, "bytes_in": st.bytes_in, "bytes_out": st.bytes_out}


__all__ = ["Entry", "read_index", "read_raw", "write", "quantize_file", "blocks_to_stream", "stream_to_blocks",
           "dtype_bytes", "crc32c", "FP32", "BF16", "FP16", "Q4_0", "Q4_1", "Q8_BLOCKS"]
