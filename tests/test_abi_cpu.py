"""The C-ABI library on a machine without a GPU: it loads, exports every
symbol include/voxq.h declares, and reports VOXCPM_ERR_CUDA_NOT_FOUND so the
reference's tensor_matmul_nt falls back to its CPU loop (src/tensor.c:629-640)."""
from __future__ import annotations

import os
import re

import pytest

import voxq

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(REPO, "include", "voxq.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.findall(r"^VOXQ_API\s+(?:VoxCPMError|void|size_t|int|const char\s*\*|const uint8_t\s*\*)\s*(\w+)\s*\(",
                      src, flags=re.M)


def test_header_declares_reference_block():
    fns = set(header_functions())
    for f in ("tensor_cuda_init", "tensor_cuda_shutdown", "tensor_to_cuda", "tensor_to_cpu",
              "tensor_cuda_free", "tensor_matmul_nt_cuda", "tensor_cuda_upload_weight"):
        assert f in fns


def test_library_exports_every_declared_symbol():
    lib = voxq.lib()
    fns = header_functions()
    assert len(fns) >= 20
    for f in fns:
        assert hasattr(lib, f), f"libvoxq.so does not export {f}"
    assert set(fns) == set(voxq.SIGNATURES), "Python binding and header disagree"


def test_no_internal_symbols_leak():
    out = os.popen(f"nm -D --defined-only {voxq.LIB_PATH}").read()
    names = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert set(header_functions()) <= names
    assert not any(n.startswith("_ZN4voxq") for n in names)


def test_sizes_and_layout_math():
    assert voxq.quant_bytes(0, voxq.Q4) == 0
    assert voxq.quant_bytes(1, voxq.Q4) == 20
    assert voxq.quant_bytes(33, voxq.Q8) == 80
    assert voxq.lib().voxq_quant_bytes(64, voxq.F32) == 0
    L = voxq.lib()
    assert L.voxq_codes_bytes(4096, 1024, voxq.Q8) == 4096 * 1024
    assert L.voxq_codes_bytes(4096, 1024, voxq.Q4) == 4096 * 512
    # trailers, a float row multiplier per row at a 16-byte boundary, 16 bytes of padding
    assert L.voxq_scales_bytes(4096, 1024, voxq.Q8) == 4096 * 32 * 8 + 4 * 4096 + 16
    assert L.voxq_scales_bytes(4096, 1024, voxq.Q4) == 4096 * 32 * 4 + 4 * 4096 + 16
    assert L.voxq_scales_bytes(3, 32, voxq.Q4) == 16 + 12 + 16
    # same block bytes per weight as the block stream (1.25 / 0.625)
    for qt in (voxq.Q4, voxq.Q8):
        assert (L.voxq_codes_bytes(64, 1024, qt) + L.voxq_scales_bytes(64, 1024, qt) - 4 * 64 - 16
                == L.voxq_quant_bytes(64 * 1024, qt))


def test_tensor_struct_layout_matches_reference():
    import ctypes as C
    from oracle import oracle as O
    assert C.sizeof(voxq.Tensor) == C.sizeof(O.RefTensor)
    for (a, _), (b, _) in zip(voxq.Tensor._fields_, O.RefTensor._fields_):
        assert getattr(voxq.Tensor, a).offset == getattr(O.RefTensor, b).offset


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU contract")
def test_no_gpu_reports_cuda_not_found():
    import numpy as np
    L = voxq.lib()
    assert L.tensor_cuda_init() == voxq.CUDA_NOT_FOUND
    a = voxq.host_tensor(np.ones((2, 64), np.float32))
    w = voxq.host_tensor(np.ones((3, 64), np.float32))
    o = voxq.host_tensor(np.zeros((2, 3), np.float32))
    try:
        assert L.tensor_matmul_nt_cuda(a, w, o) == voxq.CUDA_NOT_FOUND
        bad = voxq.host_tensor(np.zeros((2, 4), np.float32))
        assert L.tensor_matmul_nt_cuda(a, w, bad) == voxq.SHAPE_MISMATCH
        voxq.free_tensor(bad)
    finally:
        for t in (a, w, o):
            voxq.free_tensor(t)
