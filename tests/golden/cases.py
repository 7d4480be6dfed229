"""Seeded quantizer / matmul input cases shared by the golden generator and the tests.

Every case is rebuilt from numpy's legacy ``RandomState`` (stable across
platforms and numpy versions), so the fixtures only store hashes and a few
small byte dumps.  The adversarial cases cover what the reference quantizer
(scripts/quantize.py:42-75) has to get right bit for bit: round-half-even
ties, blocks whose min/max is a signed zero, constant blocks, f32 subnormals,
f32 overflow in ``x - min``, infinities, NaN, a zero-padded tail block, scales
that underflow / overflow binary16, and scales whose double -> half rounding
differs from double -> float -> half.
"""
from __future__ import annotations

import numpy as np

BLK = 32


def _rs(seed: int) -> np.random.RandomState:
    return np.random.RandomState(seed)


def _ties(seed: int, nblk: int, levels: int) -> np.ndarray:
    """Blocks with min 0, max levels*s and interior values (m + 1/2) * s (exact ties)."""
    r = _rs(seed)
    out = np.empty((nblk, BLK), dtype=np.float32)
    for b in range(nblk):
        s = np.float32(2.0 ** r.randint(-20, 10))
        m = r.randint(0, levels, size=BLK).astype(np.float64) + 0.5
        row = (m * float(s)).astype(np.float32)
        row[r.randint(BLK)] = 0.0
        row[r.randint(BLK)] = np.float32(levels * float(s))
        out[b] = row
    return out.ravel()


def _signed_zero(seed: int, nblk: int) -> np.ndarray:
    """Blocks whose min (or max) is zero, holding both +0 and -0."""
    r = _rs(seed)
    out = np.empty((nblk, BLK), dtype=np.float32)
    for b in range(nblk):
        row = (r.rand(BLK).astype(np.float32) + np.float32(0.25))
        if b % 2:
            row = -row
        nz = r.randint(1, 8)
        for i in r.choice(BLK, nz, replace=False):
            row[i] = np.float32(-0.0) if r.rand() < 0.5 else np.float32(0.0)
        out[b] = row
    return out.ravel()


def _const(seed: int) -> np.ndarray:
    vals = [0.0, -0.0, 1.0, -3.5, 1e-30, -1e-42, 65504.0, 1e20, 3.0e38]
    r = _rs(seed)
    rows = [np.full(BLK, v, dtype=np.float32) for v in vals]
    rows += [np.full(BLK, np.float32(r.randn()), dtype=np.float32) for _ in range(23)]
    return np.concatenate(rows)


def _special(seed: int) -> np.ndarray:
    """Subnormals, f32 overflow of x - min, +-inf and NaN (one feature per block)."""
    r = _rs(seed)
    rows = []
    for _ in range(8):
        rows.append((r.randn(BLK) * 1e-40).astype(np.float32))  # f32 subnormals
        rows.append((r.rand(BLK) * 4e38 - 1e38).astype(np.float32) * np.float32(1.0))
        rows[-1][r.randint(BLK)] = np.float32(-3.0e38)
        rows[-1][r.randint(BLK)] = np.float32(3.3e38)
        x = r.randn(BLK).astype(np.float32)
        x[r.randint(BLK)] = np.inf
        rows.append(x)
        x = r.randn(BLK).astype(np.float32)
        x[r.randint(BLK)] = -np.inf
        rows.append(x)
        x = r.randn(BLK).astype(np.float32)
        x[r.randint(BLK)] = np.nan
        rows.append(x)
    rows.append(np.full(BLK, np.inf, dtype=np.float32))
    rows.append(np.full(BLK, -np.inf, dtype=np.float32))
    return np.concatenate(rows)


def _mixed_scale(seed: int, nblk: int) -> np.ndarray:
    """Per-block magnitude log-uniform over 1e-12 .. 1e12 (binary16 under/overflow)."""
    r = _rs(seed)
    mag = 10.0 ** r.uniform(-12, 12, size=(nblk, 1))
    return (r.randn(nblk, BLK) * mag).astype(np.float32).ravel()


def _half_double_rounding(seed: int, nblk: int) -> np.ndarray:
    """Blocks [mn, mx, ...] whose Q4 scale (double(mx) - double(mn)) / 15 rounds
    differently to binary16 when it goes through float first (seeded search).

    With mn = 0 this cannot happen (mx / 15 never lands within half a float ulp
    of a binary16 midpoint); a tiny negative mn makes mx - mn carry more than
    24 significant bits in double, which is where the two roundings part."""
    r = _rs(seed)
    found = []
    for _ in range(400):
        if len(found) >= nblk:
            break
        mx = (10.0 ** r.uniform(-4, 4.5, size=200000)).astype(np.float32)
        mn = (-mx.astype(np.float64) * 10.0 ** r.uniform(-12, -4, size=200000)).astype(np.float32)
        d = (mx.astype(np.float64) - mn.astype(np.float64)) / 15.0
        direct = d.astype(np.float16)
        via = d.astype(np.float32).astype(np.float16)
        hit = np.nonzero(direct.view(np.uint16) != via.view(np.uint16))[0]
        found.extend(zip(mn[hit].tolist(), mx[hit].tolist()))
    if len(found) < nblk:
        raise RuntimeError(f"only {len(found)} double-rounding blocks found")
    out = np.empty((nblk, BLK), dtype=np.float32)
    for b in range(nblk):
        mn, mx = found[b]
        row = (np.float32(mn) + r.rand(BLK) * (mx - mn)).astype(np.float32)
        row = np.clip(row, np.float32(mn), np.float32(mx))
        row[0] = np.float32(mn)
        row[1 + r.randint(BLK - 1)] = np.float32(mx)
        out[b] = row
    return out.ravel()


def make_case(name: str) -> np.ndarray:
    if name == "w002":
        return (_rs(11).randn(524288 * BLK) * 0.02).astype(np.float32)
    if name == "normal1":
        return _rs(12).randn(131072 * BLK).astype(np.float32)
    if name == "normal100":
        return (_rs(13).randn(65536 * BLK) * 100.0).astype(np.float32)
    if name == "mixed_scale":
        return _mixed_scale(14, 131072)
    if name == "ties_q4":
        return _ties(15, 2048, 15)
    if name == "ties_q8":
        return _ties(16, 2048, 255)
    if name == "signed_zero":
        return _signed_zero(17, 4096)
    if name == "const":
        return _const(18)
    if name == "special":
        return _special(19)
    if name == "half_double_rounding":
        return _half_double_rounding(20, 64)
    if name == "tail481":
        return _rs(21).randn(481).astype(np.float32)
    if name == "tail7":
        return (_rs(22).randn(7) * 5).astype(np.float32)
    raise KeyError(name)


CASES = ["w002", "normal1", "normal100", "mixed_scale", "ties_q4", "ties_q8", "signed_zero",
         "const", "special", "half_double_rounding", "tail481", "tail7"]

# Small cases where the golden bytes are stored verbatim (quant_small.npz).
SMALL_CASES = [c for c in CASES if c in ("ties_q4", "const", "special", "half_double_rounding",
                                         "tail481", "tail7")]

# (M, N, K, seed_a, seed_w) for the reference tensor_matmul_nt fixtures
MATMUL_CASES = [(1, 64, 96, 2, 1), (3, 40, 64, 4, 3), (5, 33, 128, 6, 5), (2, 130, 1024, 8, 7)]
