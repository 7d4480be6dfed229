#!/usr/bin/env python3
"""Regenerates the golden fixtures in this folder from the reference itself.

Run where the reference checkout is available (its path from --ref, else the
VOXCPM_REF environment variable, else BASELINE.json's "reference_path"):

    python tests/golden/gen_golden.py [--ref <reference checkout>]

It writes:
  ref_quant/            output of the reference's ``scripts/gen_test_data.py
                        --only quant`` (8-block Q4/Q8 packs, RandomState(42))
  quant_cases.json      for each seeded case: SHA-256 of the bytes that the
                        reference's ``quantize_q4_block`` / ``quantize_q8_block``
                        (scripts/quantize.py:42-75) produce over the flattened,
                        zero-padded tensor (scripts/quantize.py:239-260), and of
                        ``dequantize_*_block``'s output (scripts/quantize.py:56-82)
  quant_small.npz       raw bytes and dequant values of a few small cases
  ref_matmul.npz        the reference ``tensor_matmul_nt`` (src/tensor.c:617-678,
                        compiled unchanged by oracle/Makefile) on small seeded
                        shapes, and ``tensor_rand_normal`` (src/tensor.c:361-371)

Inputs of every case come from ``cases.make_case`` (numpy RandomState), so a
test can rebuild them anywhere without the reference.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import subprocess
import sys
import tempfile
import warnings

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, REPO)

import cases  # noqa: E402


def default_ref():
    """The reference checkout: $VOXCPM_REF, else BASELINE.json's reference_path."""
    if os.environ.get("VOXCPM_REF"):
        return os.environ["VOXCPM_REF"]
    try:
        with open(os.path.join(os.path.dirname(os.path.dirname(HERE)), "BASELINE.json")) as f:
            return json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None


def load_quantize(ref: str):
    spec = importlib.util.spec_from_file_location("ref_quantize", os.path.join(ref, "scripts", "quantize.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def ref_pack(Q, x: np.ndarray, qtype: int) -> bytes:
    """scripts/quantize.py:239-260: blocks over the flattened tensor, last block zero-padded."""
    fn = Q.quantize_q4_block if qtype == 2 else Q.quantize_q8_block
    n = x.size
    out = bytearray()
    nb = (n + 31) // 32
    for b in range(nb):
        blk = x[b * 32:min(b * 32 + 32, n)]
        if blk.size < 32:
            blk = np.pad(blk, (0, 32 - blk.size), "constant")
        out.extend(fn(blk))
    return bytes(out)


def ref_unpack(Q, packed: bytes, n: int, qtype: int) -> np.ndarray:
    """scripts/quantize.py:225-231 style: dequantize every block, keep n values."""
    bb = 20 if qtype == 2 else 40
    fn = Q.dequantize_q4_block if qtype == 2 else Q.dequantize_q8_block
    blocks = [fn(packed[i:i + bb]) for i in range(0, len(packed), bb)]
    return np.concatenate(blocks).astype(np.float32)[:n]


def run_ref_gen_quant(path: str, outdir: str) -> None:
    """Runs ``gen_quant_tests`` of the reference's gen_test_data.py unchanged.

    Under Python 3.12 that file as a whole fails to compile (its ``main`` reads
    OUTPUT_DIR before declaring it ``global``, gen_test_data.py:535-542), so
    only the module-level constants and the helper / generator functions it
    needs are compiled from the parsed source and executed.
    """
    import ast
    import contextlib
    import io

    tree = ast.parse(open(path, encoding="utf-8").read(), filename=path)
    keep = []
    for node in tree.body:
        if isinstance(node, (ast.Import, ast.ImportFrom)):
            keep.append(node)
        elif isinstance(node, ast.Assign) and all(isinstance(t, ast.Name) for t in node.targets):
            keep.append(node)
        elif isinstance(node, ast.FunctionDef) and node.name in ("save_npy", "save_bin", "gen_quant_tests"):
            keep.append(node)
    mod = ast.Module(body=keep, type_ignores=[])
    ns: dict = {"__name__": "ref_gen_test_data"}
    exec(compile(mod, path, "exec"), ns)
    ns["OUTPUT_DIR"] = outdir
    with contextlib.redirect_stdout(io.StringIO()):
        ns["gen_quant_tests"]()


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=default_ref(), required=default_ref() is None,
                    help="reference checkout (default: $VOXCPM_REF or BASELINE.json reference_path)")
    args = ap.parse_args()
    warnings.simplefilter("ignore")
    Q = load_quantize(args.ref)

    # 1. The reference's own quant fixture generator.
    outdir = os.path.join(HERE, "ref_quant")
    os.makedirs(outdir, exist_ok=True)
    run_ref_gen_quant(os.path.join(args.ref, "scripts", "gen_test_data.py"), outdir)

    # 2. Seeded cases through quantize.py, hashed.
    records = []
    small = {}
    for name in cases.CASES:
        x = cases.make_case(name)
        rec = {"name": name, "n": int(x.size)}
        for qtype, tag in ((2, "q4"), (3, "q8")):
            packed = ref_pack(Q, x, qtype)
            rec[f"{tag}_sha256"] = sha(packed)
            deq = ref_unpack(Q, packed, x.size, qtype)
            rec[f"{tag}_dequant_sha256"] = sha(deq.tobytes())
            if x.size <= 4096:
                small[f"{name}.{tag}"] = np.frombuffer(packed, dtype=np.uint8)
                small[f"{name}.{tag}.dequant"] = deq
        records.append(rec)
        print(f"  {name}: n={x.size}", flush=True)
    with open(os.path.join(HERE, "quant_cases.json"), "w") as f:
        json.dump({"generator": "reference scripts/quantize.py, numpy " + np.__version__,
                   "cases": records}, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "quant_small.npz"), **small)

    # 3. The reference tensor.c (compiled unchanged) for matmul_nt and the RNG.
    subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), f"REF={args.ref}"], check=True)
    from oracle import oracle as O

    mm = {}
    for (M, N, K, sa, sw) in cases.MATMUL_CASES:
        a = O.ref_rand_normal(sa, M * K).reshape(M, K)
        w = (O.ref_rand_normal(sw, N * K) * np.float32(0.02)).reshape(N, K)
        mm[f"{M}x{N}x{K}.a"] = a
        mm[f"{M}x{N}x{K}.w"] = w
        mm[f"{M}x{N}x{K}.out"] = O.ref_matmul_nt(a, w)
    # tests/test_tensor.c:130-161 known answer, restated in the NT layout
    a = np.array([[1, 2, 3], [4, 5, 6]], dtype=np.float32)
    bt = np.array([[7, 9, 11], [8, 10, 12]], dtype=np.float32)
    mm["kat.out"] = O.ref_matmul_nt(a, bt)
    mm["rng.seed1"] = O.ref_rand_normal(1, 1001)
    mm["rng.seed2"] = O.ref_rand_normal(2, 64)
    np.savez_compressed(os.path.join(HERE, "ref_matmul.npz"), **mm)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
