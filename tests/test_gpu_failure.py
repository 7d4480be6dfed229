"""Failure detection on the GPU without a fault: a bounded wait that can never complete gives
up, records its site in the device error word and returns; the context stays usable."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    import torch
    import voxq
    L = voxq.lib()
    assert L.voxq_device_error(1) >= 0          # start clean
    code = L.voxq_selftest_wait_timeout(3)      # ~3 ms: nothing ever arrives on the barrier
    assert code == 1                            # VOXQ_DEVERR_WAIT_FULL, recorded and cleared
    assert L.voxq_device_error(0) == 0
    # a normal call afterwards runs and is correct
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((256, 128)) * 0.02).astype(np.float32)
    x = rng.standard_normal((1, 128)).astype(np.float32)
    qw = voxq.QWeight.from_float(torch.from_numpy(w).cuda(), voxq.Q8)
    y = voxq.matmul_nt_q(torch.from_numpy(x).cuda(), qw).cpu().numpy()
    wd = O.dequantize(O.quantize(w.reshape(-1), 3), w.size, 3).reshape(w.shape)
    ref, scale = O.matmul_nt_f64(x, wd)
    assert np.all(np.abs(y - ref) <= 1e-3 * np.maximum(np.abs(ref), scale))
    assert L.voxq_device_error(1) == 0


def test_selftest_repeats():
    import voxq
    L = voxq.lib()
    for polls in (1, 2):
        assert L.voxq_selftest_wait_timeout(polls) == 1
    assert L.voxq_device_error(0) == 0
