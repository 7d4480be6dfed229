"""quantize.py containers on the device: the 2-D Q4/Q8 tensors of the
reference quantizer's output (tests/golden/vxcpm2_q4.bin, vxcpm2_q8.bin, see
tests/golden/make_vxcpm2.py) become packed weights with their bytes unchanged,
and multiply like the reference's tensor_matmul_nt (src/tensor.c:617-678) on
the dequantized weight."""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import assert_matmul_close
from oracle import oracle as O

torch = pytest.importorskip("torch")
import voxq  # noqa: E402
from voxq.container import VXCPM2  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("kind,qt", [("q4", voxq.Q4), ("q8", voxq.Q8)])
@pytest.mark.parametrize("M", [1, 3, 64])
def test_container_weights_on_device(kind, qt, M):
    with VXCPM2(os.path.join(GOLD, f"vxcpm2_{kind}.bin")) as f:
        mats = [t for t in f.tensors if len(t.shape) == 2]
        assert len(mats) == 3
        for t in mats:
            N, K = t.shape
            w = f.qweight(t.index)
            torch.cuda.synchronize()
            assert np.array_equal(w.to_blocks().cpu().numpy(), f.raw(t.index))  # bytes unchanged
            wdeq = f.dequantize(t.index)
            a = O.rand_normal(500 + t.index + M, M * K).reshape(M, K)
            y = voxq.matmul_nt_q(torch.from_numpy(a).cuda(), w).cpu().numpy()
            want = O.matmul_nt(a, wdeq)
            _, sc = O.matmul_nt_f64(a, wdeq)
            assert_matmul_close(y, want, sc, 1e-3 if M <= 8 else 5e-3, f"{kind} {t.shape} M={M}")
        with pytest.raises(ValueError):
            f.qweight(1)  # a 1-D norm weight is not a matmul weight
