#!/usr/bin/env python3
"""Regenerates the VXCPM2 container fixtures in this folder.

    python tests/golden/make_vxcpm2.py [--ref <reference checkout>]

vxcpm2_f32.bin is written here from seeded tensors in the container layout
that the reference's quantizer reads (scripts/quantize.py:119-162: 256-byte
header, layer-group offset table, tensors as name_hash, ndim, dims[3] + data,
checksum of :309-315).  vxcpm2_q4.bin, vxcpm2_q8.bin and vxcpm2_f16.bin are
the reference's own ``convert_quant`` (scripts/quantize.py:110-312) run on it,
imported from the reference checkout -- the bytes the tests compare against
(with its magic constant given the 8 bytes it writes, and its checksum field
left at the 0 that the reference leaves there; see main()).
The tensor list (TENSORS) is imported by the tests to rebuild the inputs.
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import importlib.util
import io
import json
import os
import struct
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (group, name, shape, scale); group 1 is left empty on purpose
TENSORS = [
    (0, "layers.0.attn.q_proj.weight", (48, 64), 0.02),
    (0, "layers.0.attn_norm.weight", (64,), 1.0),
    (2, "layers.1.mlp.down_proj.weight", (32, 96), 0.02),
    (2, "layers.1.mlp.down_proj.bias", (32,), 0.1),
    (2, "feat_encoder.conv.weight", (8, 4, 3), 0.5),
    (3, "lm_head.weight", (40, 128), 0.02),
]
N_GROUPS = 4
HEADER = dict(version=2, n_layers=2, n_layers_enc=1, n_ralm_layers=1, n_dit_layers=1, d_model=64, d_ff=96,
              n_heads=4, n_kv_heads=2, head_dim=16, max_seq_len=512, vocab_size=40, quant=0, sample_rate=16000,
              audio_vae_dim=64, rope_theta=10000.0)
HEADER_ORDER = ["version", "n_layers", "n_layers_enc", "n_ralm_layers", "n_dit_layers", "d_model", "d_ff", "n_heads",
                "n_kv_heads", "head_dim", "max_seq_len", "vocab_size", "quant", "sample_rate", "audio_vae_dim"]


def default_ref():
    """The reference checkout: $VOXCPM_REF, else BASELINE.json's reference_path."""
    if os.environ.get("VOXCPM_REF"):
        return os.environ["VOXCPM_REF"]
    try:
        with open(os.path.join(os.path.dirname(os.path.dirname(HERE)), "BASELINE.json")) as f:
            return json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None


def tensor_values(i: int) -> np.ndarray:
    _, _, shape, scale = TENSORS[i]
    rs = np.random.RandomState(7000 + i)
    v = (rs.standard_normal(int(np.prod(shape))) * scale).astype(np.float32)
    if i == 1:
        v += 1.0  # a norm weight around 1
    return v.reshape(shape)


def name_hash(name: str) -> int:
    return zlib.crc32(name.encode()) & 0xFFFFFFFF


def write_f32(path: str) -> None:
    groups = [bytearray() for _ in range(N_GROUPS)]
    for i, (g, name, shape, _) in enumerate(TENSORS):
        dims = list(shape) + [0] * (3 - len(shape))
        groups[g] += struct.pack("<5I", name_hash(name), len(shape), *dims) + tensor_values(i).tobytes()
    header = bytearray(256)
    struct.pack_into("8s", header, 0, b"VXCPM2\0")
    for k, name in enumerate(HEADER_ORDER):
        struct.pack_into("<I", header, 8 + 4 * k, HEADER[name])
    struct.pack_into("<f", header, 68, HEADER["rope_theta"])
    struct.pack_into("<I", header, 80, N_GROUPS)
    offsets, pos = [], 256 + (N_GROUPS + 1) * 8
    for g in groups:
        offsets.append(pos)
        pos += len(g)
    offsets.append(pos)
    data = bytes(header) + struct.pack(f"<{N_GROUPS + 1}Q", *offsets) + b"".join(bytes(g) for g in groups)
    digest = hashlib.sha256(data[:72] + b"\0" * 8 + data[80:]).digest()
    data = data[:72] + digest[:8] + data[80:]
    with open(path, "wb") as f:
        f.write(data)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=default_ref(), required=default_ref() is None,
                    help="reference checkout (default: $VOXCPM_REF or BASELINE.json reference_path)")
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location("ref_quantize", os.path.join(args.ref, "scripts", "quantize.py"))
    q = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(q)
    # The reference compares header[:8] with the 7-byte VOXCPM_MAGIC
    # (scripts/quantize.py:25, 122-126), so convert_quant rejects every input.
    # The 8-byte form is what it writes (struct '8s' pads with \0,
    # scripts/quantize.py:285), so the output bytes are unchanged.
    q.VOXCPM_MAGIC = b"VXCPM2\0\0"
    src = os.path.join(HERE, "vxcpm2_f32.bin")
    write_f32(src)
    for kind in ("q4", "q8", "f16"):
        # convert_quant then reads back its write-only output to checksum it
        # (scripts/quantize.py:308-310) and raises; header, index and tensors are
        # written by then and the checksum field keeps its placeholder 0 -- the
        # file the reference produces, kept as it is.
        try:
            with contextlib.redirect_stdout(io.StringIO()):
                q.convert_quant(src, os.path.join(HERE, f"vxcpm2_{kind}.bin"), kind)
        except io.UnsupportedOperation:
            pass
    for kind in ("f32", "q4", "q8", "f16"):
        p = os.path.join(HERE, f"vxcpm2_{kind}.bin")
        print(p, os.path.getsize(p))


if __name__ == "__main__":
    main()
