"""quantize.py weight containers (VXCPM2) -> packed device weights.

Thin wrapper over the library's voxq_vxcpm2_* entry points (include/voxq.h),
which read the container written by the reference's quantizer
(scripts/quantize.py:110-312): 256-byte header, layer-group offset table,
tensors as (name_hash, ndim, dims[3]) + f32 / f16 / Q4 / Q8 data.  2-D Q4/Q8
tensors become QWeight objects without requantization (the block bytes are
packed as they are); other tensors are returned as float32 arrays.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import QWeight, Vxcpm2Header, Vxcpm2Tensor, check, lib, _stream

QUANT_NAMES = {0: "f32", 1: "f16", 2: "q4", 3: "q8"}


@dataclass(frozen=True)
class TensorInfo:
    index: int
    name_hash: int
    shape: tuple
    dtype: int        # the file's quant type (0 f32, 1 f16, 2 q4, 3 q8)
    group: int        # layer group
    offset: int       # data offset in the file
    nbytes: int


class VXCPM2:
    """An open container: `header` (dict), `tensors` (list of TensorInfo)."""

    def __init__(self, path: str):
        self._h = C.c_void_p()
        check(lib().voxq_vxcpm2_open(str(path).encode(), C.byref(self._h)), f"voxq_vxcpm2_open({path})")
        hdr, n = Vxcpm2Header(), C.c_int()
        check(lib().voxq_vxcpm2_info(self._h, C.byref(hdr), C.byref(n)), "voxq_vxcpm2_info")
        self.header = {name: getattr(hdr, name) for name, _ in Vxcpm2Header._fields_}
        self.tensors = []
        for i in range(n.value):
            t = Vxcpm2Tensor()
            check(lib().voxq_vxcpm2_tensor_info(self._h, i, C.byref(t)), "voxq_vxcpm2_tensor_info")
            self.tensors.append(TensorInfo(i, t.name_hash, tuple(t.dims[: t.ndim]), t.dtype, t.group, t.offset,
                                           t.bytes))

    def close(self) -> None:
        if self._h:
            lib().voxq_vxcpm2_close(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def verify(self):
        """True / False: the stored SHA-256 checksum matches / does not match;
        None: no checksum stored (0, as the reference quantizer leaves it)."""
        r = lib().voxq_vxcpm2_verify(self._h)
        return None if r == -9 else r == 0

    def raw(self, i: int) -> np.ndarray:
        """Tensor i's stored bytes (a copy)."""
        t = self.tensors[i]
        p = lib().voxq_vxcpm2_data(self._h, i)
        return np.frombuffer((C.c_uint8 * t.nbytes).from_address(p), dtype=np.uint8).copy()

    def dequantize(self, i: int, q8_signed: bool = False) -> np.ndarray:
        """Tensor i as float32, in its stored shape."""
        t = self.tensors[i]
        n = int(np.prod(t.shape)) if t.shape else 1
        out = np.empty(n, dtype=np.float32)
        check(lib().voxq_vxcpm2_dequantize(self._h, i, int(q8_signed), out.ctypes.data), "voxq_vxcpm2_dequantize")
        return out.reshape(t.shape)

    def qweight(self, i: int, device="cuda", q8_signed: bool = False, stream=None) -> QWeight:
        """2-D Q4/Q8 tensor i ([N, K], K % 32 == 0) as a packed device weight."""
        t = self.tensors[i]
        if len(t.shape) != 2:
            raise ValueError(f"tensor {i} has shape {t.shape}; a 2-D [N, K] weight is needed")
        q = QWeight.alloc(t.shape[0], t.shape[1], t.dtype, device, q8_signed)
        check(lib().voxq_vxcpm2_upload_qweight(self._h, i, q.codes.data_ptr(), q.scales.data_ptr(), _stream(stream)),
              "voxq_vxcpm2_upload_qweight")
        return q
