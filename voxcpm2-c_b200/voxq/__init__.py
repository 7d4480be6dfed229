"""Python binding of libvoxq (the C ABI in include/voxq.h), via ctypes.

The reference ships a ctypes binding of its engine (python/voxcpm2.py); this
module is the matching host-side view of the quantized-matmul path.  It keeps
the reference's names and error convention: every call returns a VoxCPMError
code (include/voxcpm.h:45-58) and a non-zero code raises ``VoxqError``.

PyTorch is used only to own device memory and streams; the library itself
takes raw pointers.  There is no CPU fallback: importing this module on a
machine without the built library raises, and GPU calls without a device fail.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Optional, Sequence

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "libvoxq.so")

F32, F16, Q4, Q8 = 0, 1, 2, 3  # scripts/quantize.py:28 QUANT_TYPES
BLOCK = 32
MAX_BATCH = 192

ERRORS = {
    0: "VOXCPM_SUCCESS", -1: "VOXCPM_ERR_FILE_NOT_FOUND", -2: "VOXCPM_ERR_INVALID_MODEL",
    -3: "VOXCPM_ERR_INVALID_TEXT", -4: "VOXCPM_ERR_INVALID_AUDIO", -5: "VOXCPM_ERR_SHAPE_MISMATCH",
    -6: "VOXCPM_ERR_OOM", -7: "VOXCPM_ERR_GPU", -8: "VOXCPM_ERR_INTERNAL", -9: "VOXCPM_ERR_UNSUPPORTED",
    -10: "VOXCPM_ERR_TIMEOUT", -11: "VOXCPM_ERR_CUDA_NOT_FOUND",
}
SHAPE_MISMATCH, OOM, INTERNAL, UNSUPPORTED, CUDA_NOT_FOUND = -5, -6, -8, -9, -11


class VoxqError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        super().__init__(f"{what}: {ERRORS.get(code, code)} ({code})")


class Tensor(C.Structure):
    """The reference's ``Tensor`` (include/tensor.h:45-56)."""

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


class QWeightDesc(C.Structure):
    """``voxq_qweight``: the packed device layout of one quantized weight."""

    _fields_ = [("codes", C.c_void_p), ("scales", C.c_void_p), ("N", C.c_int32), ("K", C.c_int32),
                ("qtype", C.c_int32), ("q8_signed", C.c_int32)]


class Conv1dDesc(C.Structure):
    """voxq_conv1d_desc: the layout of the engine's Conv1D (include/nn.h:198-207)."""

    _fields_ = [("weight", C.c_void_p), ("bias", C.c_void_p), ("in_channels", C.c_int), ("out_channels", C.c_int),
                ("kernel_size", C.c_int), ("stride", C.c_int), ("padding", C.c_int), ("groups", C.c_int)]


class Conv1dTransposeDesc(C.Structure):
    """voxq_conv1d_transpose_desc: the layout of the engine's Conv1DTranspose (include/nn.h:221-229)."""

    _fields_ = [("weight", C.c_void_p), ("bias", C.c_void_p), ("in_channels", C.c_int), ("out_channels", C.c_int),
                ("kernel_size", C.c_int), ("stride", C.c_int), ("padding", C.c_int)]


class Epilogue(C.Structure):
    _fields_ = [("bias", C.c_void_p), ("residual", C.c_void_p), ("ldr", C.c_int64),
                ("up", C.POINTER(QWeightDesc))]


class GemvItem(C.Structure):
    _fields_ = [("w", QWeightDesc), ("a", C.c_void_p), ("out", C.c_void_p), ("bias", C.c_void_p),
                ("residual", C.c_void_p), ("up_codes", C.c_void_p), ("up_scales", C.c_void_p),
                ("M", C.c_int32), ("lda", C.c_int32), ("ldo", C.c_int32), ("ldr", C.c_int32)]


# Every symbol include/voxq.h declares, with its ctypes signature.
class Vxcpm2Header(C.Structure):
    """voxq_vxcpm2_header (include/voxq.h)."""
    _fields_ = [(n, C.c_uint32) for n in ("version", "n_layers", "n_layers_enc", "n_ralm_layers", "n_dit_layers",
                                           "d_model", "d_ff", "n_heads", "n_kv_heads", "head_dim", "max_seq_len",
                                           "vocab_size", "quant", "sample_rate", "audio_vae_dim")] + \
               [("rope_theta", C.c_float), ("checksum", C.c_uint64), ("n_groups", C.c_uint32)]


class Vxcpm2Tensor(C.Structure):
    """voxq_vxcpm2_tensor (include/voxq.h)."""
    _fields_ = [("name_hash", C.c_uint32), ("ndim", C.c_uint32), ("dims", C.c_uint32 * 3), ("dtype", C.c_int32),
                ("group", C.c_int32), ("elements", C.c_uint64), ("offset", C.c_uint64), ("bytes", C.c_uint64)]


class VaeOp(C.Structure):
    """voxq_vae_op (include/voxq.h)."""
    _fields_ = [("kind", C.c_int), ("conv", C.POINTER(Conv1dDesc)), ("convt", C.POINTER(Conv1dTransposeDesc)),
                ("alpha", C.POINTER(Tensor))]


class RmsNormDesc(C.Structure):
    """voxq_rmsnorm_desc (include/voxq.h; the engine's RmsNorm)."""
    _fields_ = [("weight", C.POINTER(Tensor)), ("eps", C.c_float)]


class AttentionDesc(C.Structure):
    """voxq_attention_desc (the engine's Attention)."""
    _fields_ = [("wq", C.POINTER(Tensor)), ("wk", C.POINTER(Tensor)), ("wv", C.POINTER(Tensor)),
                ("wo", C.POINTER(Tensor)), ("d_model", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int)]


class SwigluDesc(C.Structure):
    """voxq_swiglu_desc (the engine's SwiGLU)."""
    _fields_ = [("w1", C.POINTER(Tensor)), ("w2", C.POINTER(Tensor)), ("w3", C.POINTER(Tensor)),
                ("d_model", C.c_int), ("d_ff", C.c_int)]


class BlockDesc(C.Structure):
    """voxq_block_desc (the engine's TransformerBlock)."""
    _fields_ = [("rms_attn", C.POINTER(RmsNormDesc)), ("attn", C.POINTER(AttentionDesc)),
                ("rms_ffn", C.POINTER(RmsNormDesc)), ("ffn", C.POINTER(SwigluDesc))]


class LocEncDesc(C.Structure):
    """voxq_locenc_desc (the engine's LocEnc)."""
    _fields_ = [("in_proj_weight", C.POINTER(Tensor)), ("in_proj_bias", C.POINTER(Tensor)),
                ("special_token", C.POINTER(Tensor)), ("layers", C.POINTER(BlockDesc)), ("n_layers", C.c_int),
                ("output_norm", C.POINTER(RmsNormDesc)), ("d_model", C.c_int), ("patch_size", C.c_int)]


_vp, _sz, _i, _i64 = C.c_void_p, C.c_size_t, C.c_int, C.c_int64
_TP = C.POINTER(Tensor)
SIGNATURES = {
    "tensor_cuda_init": ([], _i),
    "tensor_cuda_shutdown": ([], None),
    "tensor_to_cuda": ([_TP], _i),
    "tensor_to_cpu": ([_TP], _i),
    "tensor_cuda_free": ([_TP], _i),
    "tensor_matmul_nt_cuda": ([_TP, _TP, _TP], _i),
    "tensor_cuda_upload_weight": ([C.POINTER(_TP)], _i),
    "voxq_version": ([], C.c_char_p),
    "voxq_set_device": ([_i], _i),
    "voxq_device_error": ([_i], _i),
    "voxq_matmul_traffic": ([C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), _i], None),
    "voxq_selftest_wait_timeout": ([_i], _i),
    "voxq_quant_bytes": ([_sz, _i], _sz),
    "voxq_quantize": ([_vp, _sz, _i, _vp, _vp], _i),
    "voxq_dequantize": ([_vp, _sz, _i, _i, _vp, _vp], _i),
    "voxq_codes_bytes": ([_i, _i, _i], _sz),
    "voxq_scales_bytes": ([_i, _i, _i], _sz),
    "voxq_quantize_weight": ([_vp, _i, _i, _i, _vp, _vp, _vp, _vp], _i),
    "voxq_pack_blocks": ([_vp, _i, _i, _i, _vp, _vp, _vp], _i),
    "voxq_unpack_blocks": ([_vp, _vp, _i, _i, _i, _vp, _vp], _i),
    "voxq_matmul_nt_q": ([_vp, _i, _i64, C.POINTER(QWeightDesc), _vp, _i64, C.POINTER(Epilogue), _vp], _i),
    "voxq_matmul_nt_q_noalloc": ([_vp, _i, _i64, C.POINTER(QWeightDesc), _vp, _i64, C.POINTER(Epilogue), _vp], _i),
    "voxq_noalloc_device_error": ([_i], _i),
    "voxq_matmul_nt_dense": ([_vp, _i, _i64, _vp, _i, _i, _i, _vp, _i64, _vp], _i),
    "voxq_gemv_batch": ([C.POINTER(GemvItem), _i, _vp], _i),
    "voxq_conv1d_forward": ([C.POINTER(Conv1dDesc), _TP, _TP], _i),
    "voxq_conv1d_transpose_forward": ([C.POINTER(Conv1dTransposeDesc), _TP, _TP], _i),
    "voxq_conv_cache_clear": ([], None),
    "voxq_vae_decode": ([C.POINTER(VaeOp), _i, C.c_float, _TP, _TP], _i),
    "voxq_transformer_block_forward": ([C.POINTER(BlockDesc), _TP, _TP, _TP, _TP, _TP, _i, _TP], _i),
    "voxq_block_cache_clear": ([], None),
    "voxq_locdit_sample": ([_vp, _TP, _TP, _i, C.c_float, _TP, _TP], _i),
    "voxq_locenc_forward": ([_vp, _TP, _TP], _i),
    "voxq_vxcpm2_open": ([C.c_char_p, C.POINTER(_vp)], _i),
    "voxq_vxcpm2_close": ([_vp], None),
    "voxq_vxcpm2_info": ([_vp, C.POINTER(Vxcpm2Header), C.POINTER(_i)], _i),
    "voxq_vxcpm2_tensor_info": ([_vp, _i, C.POINTER(Vxcpm2Tensor)], _i),
    "voxq_vxcpm2_data": ([_vp, _i], _vp),
    "voxq_vxcpm2_verify": ([_vp], _i),
    "voxq_vxcpm2_dequantize": ([_vp, _i, _i, _vp], _i),
    "voxq_vxcpm2_upload_qweight": ([_vp, _i, _vp, _vp, _vp], _i),
    "voxq_vxcp_quantize": ([C.c_char_p, C.c_char_p, _i, C.POINTER(C.c_char_p), _i, _vp], _i),
    "voxq_tensor_attach_blocks": ([_TP, _i, _vp, _sz], _i),
    "voxq_tensor_detach_blocks": ([_TP], _i),
}

_lib = None


def lib():
    """Loads libvoxq.so; raises if it has not been built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python voxcpm2-c_b200/build.py` "
                              "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(code: int, what: str) -> None:
    if code != 0:
        raise VoxqError(code, what)


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        import torch
        return int(torch.cuda.current_stream().cuda_stream)
    return int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream)


# ---------------------------------------------------------------------------
# Quantizer (device)
# ---------------------------------------------------------------------------

def quant_bytes(n: int, qtype: int) -> int:
    return int(lib().voxq_quant_bytes(n, qtype))


def quantize(x, qtype: int, stream=None):
    """Device quantize.py block stream of a float32 CUDA tensor (flattened)."""
    import torch
    x = x.contiguous().view(-1)
    out = torch.zeros(quant_bytes(x.numel(), qtype), dtype=torch.uint8, device=x.device)
    check(lib().voxq_quantize(_ptr(x), x.numel(), qtype, _ptr(out), _stream(stream)), "voxq_quantize")
    return out


def dequantize(blocks, n: int, qtype: int, q8_signed: bool = False, stream=None):
    import torch
    out = torch.empty(n, dtype=torch.float32, device=blocks.device)
    check(lib().voxq_dequantize(_ptr(blocks), n, qtype, int(q8_signed), _ptr(out), _stream(stream)),
          "voxq_dequantize")
    return out


@dataclass
class QWeight:
    """A packed device weight W[N, K] (codes + per-block scale/min)."""

    codes: "object"
    scales: "object"
    N: int
    K: int
    qtype: int
    q8_signed: bool = False

    def desc(self) -> QWeightDesc:
        return QWeightDesc(_ptr(self.codes), _ptr(self.scales), self.N, self.K, self.qtype, int(self.q8_signed))

    @property
    def nbytes(self) -> int:
        return self.codes.numel() + self.scales.numel()

    @staticmethod
    def alloc(N: int, K: int, qtype: int, device="cuda", q8_signed: bool = False) -> "QWeight":
        import torch
        cb = int(lib().voxq_codes_bytes(N, K, qtype))
        sb = int(lib().voxq_scales_bytes(N, K, qtype))
        return QWeight(torch.empty(cb, dtype=torch.uint8, device=device),
                       torch.empty(sb, dtype=torch.uint8, device=device), N, K, qtype, q8_signed)

    @staticmethod
    def from_float(w, qtype: int, blocks_out=None, stream=None, q8_signed: bool = False) -> "QWeight":
        """Quantizes a float32 CUDA tensor [N, K] (K % 32 == 0) on the device."""
        w = w.contiguous()
        N, K = w.shape
        q = QWeight.alloc(N, K, qtype, w.device, q8_signed)
        check(lib().voxq_quantize_weight(_ptr(w), N, K, qtype, _ptr(q.codes), _ptr(q.scales), _ptr(blocks_out),
                                         _stream(stream)), "voxq_quantize_weight")
        return q

    @staticmethod
    def from_blocks(blocks, N: int, K: int, qtype: int, stream=None, q8_signed: bool = False) -> "QWeight":
        """Packs a quantize.py block stream (uint8 CUDA tensor) into the device layout."""
        q = QWeight.alloc(N, K, qtype, blocks.device, q8_signed)
        check(lib().voxq_pack_blocks(_ptr(blocks), N, K, qtype, _ptr(q.codes), _ptr(q.scales), _stream(stream)),
              "voxq_pack_blocks")
        return q

    def to_blocks(self, stream=None):
        import torch
        out = torch.empty(quant_bytes(self.N * self.K, self.qtype), dtype=torch.uint8, device=self.codes.device)
        check(lib().voxq_unpack_blocks(_ptr(self.codes), _ptr(self.scales), self.N, self.K, self.qtype, _ptr(out),
                                       _stream(stream)), "voxq_unpack_blocks")
        return out


# ---------------------------------------------------------------------------
# Matmul
# ---------------------------------------------------------------------------

def matmul_nt_q(a, w: QWeight, out=None, bias=None, residual=None, up: Optional[QWeight] = None, stream=None):
    """out[M, N] = epilogue(a[M, K] @ W^T) on the device (voxq_matmul_nt_q)."""
    import torch
    M, K = a.shape
    if out is None:
        out = torch.empty(M, w.N, dtype=torch.float32, device=a.device)
    d = w.desc()
    epi = None
    keep = []
    if bias is not None or residual is not None or up is not None:
        ud = up.desc() if up is not None else None
        keep.append(ud)
        epi = Epilogue(_ptr(bias), _ptr(residual), residual.stride(0) if residual is not None else 0,
                       C.pointer(ud) if ud is not None else None)
    check(lib().voxq_matmul_nt_q(_ptr(a), M, a.stride(0), C.byref(d), _ptr(out), out.stride(0),
                                 C.byref(epi) if epi is not None else None, _stream(stream)), "voxq_matmul_nt_q")
    return out


def matmul_nt_dense(a, w, out=None, stream=None):
    import torch
    M, K = a.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=a.device)
    check(lib().voxq_matmul_nt_dense(_ptr(a), M, a.stride(0), _ptr(w), int(w.dtype == torch.float16), N, K,
                                     _ptr(out), out.stride(0), _stream(stream)), "voxq_matmul_nt_dense")
    return out


def make_gemv_items(specs: Sequence[dict]):
    """specs: dicts with keys w (QWeight), a, out, and optional bias, residual, up."""
    arr = (GemvItem * len(specs))()
    for i, s in enumerate(specs):
        w: QWeight = s["w"]
        a, out = s["a"], s["out"]
        it = arr[i]
        it.w = w.desc()
        it.a, it.out = _ptr(a), _ptr(out)
        it.bias = _ptr(s.get("bias"))
        r = s.get("residual")
        it.residual = _ptr(r)
        it.ldr = r.stride(0) if r is not None else 0
        up = s.get("up")
        if up is not None:
            it.up_codes, it.up_scales = _ptr(up.codes), _ptr(up.scales)
        it.M = a.shape[0]
        it.lda = a.stride(0)
        it.ldo = out.stride(0)
    return arr


def gemv_batch(items, stream=None) -> None:
    """One launch for many independent GEMVs (voxq_gemv_batch)."""
    check(lib().voxq_gemv_batch(items, len(items), _stream(stream)), "voxq_gemv_batch")


def set_device(d: int) -> None:
    check(lib().voxq_set_device(d), "voxq_set_device")


def version() -> str:
    return lib().voxq_version().decode()


# ---------------------------------------------------------------------------
# Reference Tensor ABI helpers (host side of tensor.h's CUDA block)
# ---------------------------------------------------------------------------

_libc = C.CDLL(None)
_libc.malloc.restype = C.c_void_p
_libc.malloc.argtypes = [C.c_size_t]
_libc.calloc.restype = C.c_void_p
_libc.calloc.argtypes = [C.c_size_t, C.c_size_t]
_libc.free.argtypes = [C.c_void_p]


def host_tensor(arr, fp16: bool = False) -> "C.POINTER(Tensor)":
    """A reference Tensor owning malloc'd copies of arr (as tensor_create would)."""
    import numpy as np
    arr = np.ascontiguousarray(arr, dtype=np.float16 if fp16 else np.float32)
    t = C.cast(_libc.calloc(1, C.sizeof(Tensor)), C.POINTER(Tensor))
    shp = C.cast(_libc.calloc(arr.ndim, C.sizeof(C.c_int)), C.POINTER(C.c_int))
    st = 1
    for i in range(arr.ndim - 1, -1, -1):
        shp[i] = arr.shape[i]
        t.contents.strides[i] = st
        st *= arr.shape[i]
    t.contents.shape = shp
    t.contents.ndim = arr.ndim
    t.contents.size = arr.size
    t.contents.is_owned = True
    buf = _libc.malloc(max(arr.nbytes, 1))
    C.memmove(buf, arr.ctypes.data, arr.nbytes)
    if fp16:
        t.contents.data_fp16 = C.cast(buf, C.POINTER(C.c_uint16))
        t.contents.is_fp16 = True
    else:
        t.contents.data = C.cast(buf, C.POINTER(C.c_float))
    return t


def host_tensor_view(t) -> "object":
    """numpy copy of a host fp32 Tensor's data."""
    import numpy as np
    c = t.contents
    shape = tuple(c.shape[i] for i in range(c.ndim))
    n = int(c.size)
    buf = (C.c_float * n).from_address(C.cast(c.data, C.c_void_p).value)
    return np.frombuffer(buf, dtype=np.float32, count=n).reshape(shape).copy()


def free_tensor(t) -> None:
    """The reference tensor_free (src/tensor.c:131-150) for tensors made here."""
    c = t.contents
    if c.is_cuda:
        lib().tensor_cuda_free(t)
    else:
        if c.data:
            _libc.free(C.cast(c.data, C.c_void_p))
        if c.data_fp16:
            _libc.free(C.cast(c.data_fp16, C.c_void_p))
    _libc.free(C.cast(c.shape, C.c_void_p))
    _libc.free(C.cast(t, C.c_void_p))
