"""The roofline arithmetic of bench.py, on the host: the algorithmic bytes and
flops its lines divide by must be the workload's own figures.

Config 2: 24 layers of Q/K/V/O/gate/up/down at hidden 1024, kv 128, FFN 4096,
Q4 (0.625 B per weight): 224,133,120 weight bytes per step, plus each GEMV's
fp32 activation read and output write.  Config 3 at K = 1024: quantized weight
+ fp32 A + fp32 out per call (Q8, N = 4096: 5.57 / 6.55 / 10.49 / 47.2 MB for
M = 16 / 64 / 256 / 2048), 2 M N K flops, and only M = 2048 above the ridge of
the bf16 tensor peak over the HBM copy bandwidth.
"""
from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402

Q4, Q8 = 2, 3


def test_c2_step_bytes():
    algo, weights = bench.c2_bytes_per_step(Q4)
    assert weights == 224_133_120
    per_layer_io = sum(4 * K + 4 * N for (_, N, K, _) in bench.C2_LAYER)
    # activation reads: six GEMVs over hidden 1024, down over FFN 4096; outputs: q, o, down at 1024,
    # k, v at 128, gate, up at 4096
    assert per_layer_io == 4 * (1024 * 6 + 4096) + 4 * (1024 * 3 + 128 * 2 + 4096 * 2) == 87_040
    assert algo == weights + 24 * per_layer_io == 226_222_080
    assert bench.c2_bytes_per_step(Q8)[1] == 2 * weights


@pytest.mark.parametrize("M,mb", [(16, 5_570_560), (64, 6_553_600), (256, 10_485_760), (2048, 47_185_920)])
def test_c3_bytes_and_bound(M, mb):
    ms = 0.01
    r = bench.c3_roof(M, 4096, 1024, True, ms)
    assert r["algorithmic_bytes"] == mb
    assert r["GBps"] == pytest.approx(mb / (ms * 1e-3) / 1e9, rel=1e-3)
    assert r["TFLOPs"] == pytest.approx(2 * M * 4096 * 1024 / (ms * 1e-3) / 1e12, rel=1e-2)
    assert r["bound"] == ("tensor" if M == 2048 else "hbm")
    hbm, bf16, _, _ = bench.peaks()
    want = r["TFLOPs"] / bf16 if M == 2048 else r["GBps"] / hbm
    assert r["frac"] == pytest.approx(want, rel=1e-2)
    # Q4 halves the weight bytes only
    assert bench.c3_roof(M, 4096, 1024, False, ms)["algorithmic_bytes"] == mb - 4096 * 1024 * 5 // 8
