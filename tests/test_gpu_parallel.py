"""Column-sharded matmul (config-3 multi-GPU partitioning) on one GPU: the ranks of a world are
emulated one after another; each quantizes only its weight rows and writes its output columns
of the shared [M, N] output (row stride N).  The assembled output is checked against the CPU
oracle on the full quantized weight (blocks are row-contained, so the shards quantize to the
same bytes)."""
import numpy as np
import pytest

from conftest import assert_matmul_close
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M", [1, 8, 64, 300])
@pytest.mark.parametrize("world", [2, 4])
def test_column_sharded_matmul_matches_full(M, world):
    import torch
    import voxq
    from voxq import parallel
    rng = np.random.default_rng(M * 10 + world)
    N, K = 1024, 512
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    a = rng.standard_normal((M, K)).astype(np.float32)
    wt = torch.from_numpy(w).cuda()
    at = torch.from_numpy(a).cuda()
    out = torch.full((M, N), float("nan"), device="cuda")
    for r in range(world):
        rows, n0, n1 = parallel.shard_weight_rows(wt, world, r, align=128)
        qw = voxq.QWeight.from_float(rows.contiguous(), voxq.Q8)
        parallel.matmul_column_shard(at, qw, out, n0)
    torch.cuda.synchronize()
    assert voxq.lib().voxq_device_error(1) == 0
    y = out.cpu().numpy()
    wd = O.dequantize(O.quantize(w.reshape(-1), 3), w.size, 3).reshape(N, K)
    ref, scale = O.matmul_nt_f64(a, wd)
    assert_matmul_close(y, ref, scale, 1e-3 if M <= 8 else 5e-3, f"M={M} world={world}")
