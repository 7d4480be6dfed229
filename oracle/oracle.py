"""ctypes loader for the CPU checker libraries.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the product library or its timed paths.

- ``liboracle.so``: the C restatement in ``voxq_oracle.c`` of the reference's
  ``scripts/quantize.py:42-104`` block math and ``src/tensor.c:339-371,617-678``.
- ``_ref/libref_tensor.so``: the reference's own ``src/tensor.c`` compiled
  unchanged (see ``Makefile``); ``tensor_matmul_nt`` is called through the
  reference's ``Tensor`` struct (``include/tensor.h:45-56``).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libref_tensor.so")

QTYPE_Q4 = 2  # scripts/quantize.py:28 QUANT_TYPES
QTYPE_Q8 = 3
BLOCK = 32
BLOCK_BYTES = {QTYPE_Q4: 20, QTYPE_Q8: 40}

_lib = None
_ref = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        fp, u8p, dp = C.POINTER(C.c_float), C.POINTER(C.c_uint8), C.POINTER(C.c_double)
        L.oracle_quantize.argtypes = [fp, C.c_size_t, C.c_int, u8p]
        L.oracle_quantize.restype = C.c_size_t
        L.oracle_dequantize.argtypes = [u8p, C.c_size_t, C.c_int, C.c_int, fp]
        L.oracle_matmul_nt.argtypes = [fp, fp, fp, C.c_int, C.c_int, C.c_int]
        L.oracle_matmul_nt_f64.argtypes = [fp, fp, dp, dp, C.c_int, C.c_int, C.c_int]
        L.oracle_rand_normal.argtypes = [C.POINTER(C.c_uint64), fp, C.c_size_t, C.c_float]
        ip = C.c_int
        L.oracle_conv1d.argtypes = [fp, fp, fp, fp, fp, ip, ip, ip, ip, ip, ip, ip, ip]
        L.oracle_conv1d_transpose.argtypes = [fp, fp, fp, fp, fp, ip, ip, ip, ip, ip, ip, ip]
        L.oracle_double_to_half.argtypes = [C.c_double]
        L.oracle_double_to_half.restype = C.c_uint16
        _lib = L
    return _lib


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(C.POINTER(C.c_float))


def quant_nbytes(n: int, qtype: int) -> int:
    return (n + BLOCK - 1) // BLOCK * BLOCK_BYTES[qtype]


def quantize(x, qtype: int) -> np.ndarray:
    """Flattened-tensor quantization (scripts/quantize.py:239-260)."""
    x, xp = _f32(np.ravel(x))
    out = np.zeros(quant_nbytes(x.size, qtype), dtype=np.uint8)
    lib().oracle_quantize(xp, x.size, qtype, out.ctypes.data_as(C.POINTER(C.c_uint8)))
    return out


def dequantize(blocks, n: int, qtype: int, q8_signed: bool = False) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.zeros(n, dtype=np.float32)
    lib().oracle_dequantize(b.ctypes.data_as(C.POINTER(C.c_uint8)), n, qtype, int(q8_signed),
                            out.ctypes.data_as(C.POINTER(C.c_float)))
    return out


def matmul_nt(a, w) -> np.ndarray:
    """out = a @ w.T with one sequential fp32 accumulator (src/tensor.c:666-675)."""
    a, ap = _f32(a)
    w, wp = _f32(w)
    M, K = a.shape
    N = w.shape[0]
    out = np.zeros((M, N), dtype=np.float32)
    lib().oracle_matmul_nt(ap, wp, out.ctypes.data_as(C.POINTER(C.c_float)), M, N, K)
    return out


def matmul_nt_f64(a, w):
    """fp64 product and the tolerance scale sum_k |a w| / sqrt(K)."""
    a, ap = _f32(a)
    w, wp = _f32(w)
    M, K = a.shape
    N = w.shape[0]
    out = np.zeros((M, N), dtype=np.float64)
    sc = np.zeros((M, N), dtype=np.float64)
    dp = C.POINTER(C.c_double)
    lib().oracle_matmul_nt_f64(ap, wp, out.ctypes.data_as(dp), sc.ctypes.data_as(dp), M, N, K)
    return out, sc


def conv1d(x, w, b, stride: int, pad: int, groups: int):
    """conv1d_forward (src/nn.c:765-834): x [B, Cin, T], w [Cout, Cin/groups, k].
    Returns (out, sum of |w x| + |b|) -- the error scale of the parity tests."""
    x, xp = _f32(x)
    w, wp = _f32(w)
    B, Cin, Tin = x.shape
    Cout, _, Kw = w.shape
    Tout = (Tin + 2 * pad - Kw) // stride + 1
    out = np.zeros((B, Cout, Tout), np.float32)
    sc = np.zeros_like(out)
    bp = _f32(b)[1] if b is not None else None
    lib().oracle_conv1d(xp, wp, bp, out.ctypes.data_as(C.POINTER(C.c_float)), sc.ctypes.data_as(C.POINTER(C.c_float)),
                        B, Cin, Tin, Cout, Kw, stride, pad, groups)
    return out, sc


def conv1d_transpose(x, w, b, stride: int, pad: int):
    """conv1d_transpose_forward (src/nn.c:864-931): x [B, Cin, T], w [Cin, Cout, k]."""
    x, xp = _f32(x)
    w, wp = _f32(w)
    B, Cin, Tin = x.shape
    _, Cout, Kw = w.shape
    Tout = (Tin - 1) * stride - 2 * pad + Kw
    out = np.zeros((B, Cout, Tout), np.float32)
    sc = np.zeros_like(out)
    bp = _f32(b)[1] if b is not None else None
    lib().oracle_conv1d_transpose(xp, wp, bp, out.ctypes.data_as(C.POINTER(C.c_float)),
                                  sc.ctypes.data_as(C.POINTER(C.c_float)), B, Cin, Tin, Cout, Kw, stride, pad)
    return out, sc


def rand_normal(seed: int, n: int, mult: float = 1.0) -> np.ndarray:
    """xorshift64 + Box-Muller stream of the reference (src/tensor.c:339-371)."""
    s = C.c_uint64(seed)
    out = np.zeros(n, dtype=np.float32)
    lib().oracle_rand_normal(C.byref(s), out.ctypes.data_as(C.POINTER(C.c_float)), n, mult)
    return out


def double_to_half(d: float) -> int:
    return int(lib().oracle_double_to_half(float(d)))


# ---------------------------------------------------------------------------
# The reference's own tensor.c (compiled unchanged into _ref/libref_tensor.so)
# ---------------------------------------------------------------------------

class RefTensor(C.Structure):
    """Layout of ``Tensor`` in the reference's include/tensor.h:45-56."""

    _fields_ = [
        ("data", C.POINTER(C.c_float)),
        ("shape", C.POINTER(C.c_int)),
        ("ndim", C.c_int),
        ("strides", C.c_int64 * 5),
        ("size", C.c_size_t),
        ("is_cuda", C.c_bool),
        ("is_owned", C.c_bool),
        ("data_fp16", C.POINTER(C.c_uint16)),
        ("is_fp16", C.c_bool),
        ("name", C.c_char * 64),
    ]


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(REF_PATH + " (build with `make -C oracle` where the reference is present)")
        L = C.CDLL(REF_PATH)
        TP = C.POINTER(RefTensor)
        L.tensor_create_from_buffer.argtypes = [C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_float)]
        L.tensor_create_from_buffer.restype = TP
        L.tensor_free.argtypes = [TP]
        L.tensor_matmul_nt.argtypes = [TP, TP, TP]
        L.tensor_matmul_nt.restype = C.c_int
        L.tensor_rand_normal.argtypes = [TP, C.POINTER(C.c_uint64)]
        _ref = L
    return _ref


class _Wrapped:
    """A reference Tensor that borrows a numpy buffer (no ownership)."""

    def __init__(self, arr: np.ndarray):
        self.arr = arr
        shape = (C.c_int * arr.ndim)(*arr.shape)
        self.t = ref().tensor_create_from_buffer(arr.ndim, shape, arr.ctypes.data_as(C.POINTER(C.c_float)))
        if not self.t:
            raise MemoryError("tensor_create_from_buffer failed")

    def close(self):
        if self.t:
            ref().tensor_free(self.t)  # is_owned=false: frees only the struct and shape
            self.t = None


def ref_matmul_nt(a, w, out=None) -> np.ndarray:
    """The reference's tensor_matmul_nt (src/tensor.c:617-678), single-threaded."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    if out is None:
        out = np.zeros((a.shape[0], w.shape[0]), dtype=np.float32)
    ta, tw, to = _Wrapped(a), _Wrapped(w), _Wrapped(out)
    try:
        rc = ref().tensor_matmul_nt(ta.t, tw.t, to.t)
    finally:
        ta.close(); tw.close(); to.close()
    if rc != 0:
        raise RuntimeError(f"tensor_matmul_nt returned {rc}")
    return out


def ref_rand_normal(seed: int, n: int) -> np.ndarray:
    """The reference's tensor_rand_normal (src/tensor.c:361-371)."""
    out = np.zeros(n, dtype=np.float32)
    t = _Wrapped(out)
    s = C.c_uint64(seed)
    try:
        ref().tensor_rand_normal(t.t, C.byref(s))
    finally:
        t.close()
    return out
