"""The CPU checker's restatement of the AudioVAE convolutions (src/nn.c:765-931)
against an independent numpy formulation of the same definitions."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O


def np_conv1d(x, w, b, stride, pad, groups):
    B, Cin, T = x.shape
    Cout, ipg, K = w.shape
    Tout = (T + 2 * pad - K) // stride + 1
    xp = np.pad(x.astype(np.float64), ((0, 0), (0, 0), (pad, pad)))
    out = np.zeros((B, Cout, Tout))
    opg = Cout // groups
    for o in range(Cout):
        c0 = (o // opg) * ipg
        for k in range(K):
            sl = xp[:, c0:c0 + ipg, k:k + stride * (Tout - 1) + 1:stride]  # [B, ipg, Tout]
            out[:, o, :] += np.einsum("c,bct->bt", w[o, :, k].astype(np.float64), sl)
    return out + (b[None, :, None] if b is not None else 0)


def np_conv1d_transpose(x, w, b, stride, pad):
    B, Cin, T = x.shape
    _, Cout, K = w.shape
    full = (T - 1) * stride + K
    out = np.zeros((B, Cout, full))
    for k in range(K):
        contrib = np.einsum("bct,co->bot", x.astype(np.float64), w[:, :, k].astype(np.float64))
        out[:, :, k:k + stride * (T - 1) + 1:stride] += contrib
    out = out[:, :, pad:full - pad]
    return out + (b[None, :, None] if b is not None else 0)


@pytest.mark.parametrize("Cin,Cout,K,stride,pad,groups,T", [
    (8, 8, 7, 1, 3, 8, 20), (6, 10, 1, 1, 0, 1, 9), (4, 6, 3, 2, 1, 2, 11), (5, 3, 4, 4, 2, 1, 16)])
def test_conv1d_matches_definition(Cin, Cout, K, stride, pad, groups, T):
    rs = np.random.RandomState(Cin * 7 + K)
    x = rs.standard_normal((2, Cin, T)).astype(np.float32)
    w = rs.standard_normal((Cout, Cin // groups, K)).astype(np.float32)
    b = rs.standard_normal(Cout).astype(np.float32)
    y, sc = O.conv1d(x, w, b, stride, pad, groups)
    want = np_conv1d(x, w, b, stride, pad, groups)
    assert y.shape == want.shape
    assert np.all(np.abs(y - want) <= 1e-5 * np.maximum(sc, 1.0))


@pytest.mark.parametrize("Cin,Cout,K,stride,pad,T", [(8, 4, 16, 8, 4, 4), (6, 3, 12, 6, 3, 5), (4, 2, 4, 2, 1, 7)])
def test_conv1d_transpose_matches_definition(Cin, Cout, K, stride, pad, T):
    rs = np.random.RandomState(Cin * 11 + K)
    x = rs.standard_normal((1, Cin, T)).astype(np.float32)
    w = rs.standard_normal((Cin, Cout, K)).astype(np.float32)
    b = rs.standard_normal(Cout).astype(np.float32)
    y, sc = O.conv1d_transpose(x, w, b, stride, pad)
    want = np_conv1d_transpose(x, w, b, stride, pad)
    assert y.shape == want.shape
    assert np.all(np.abs(y - want) <= 1e-5 * np.maximum(sc, 1.0))
