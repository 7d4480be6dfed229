"""Host-side multi-GPU logic (voxq.parallel): shards, LPT assignment, heartbeat deadlines.

The multi-process cases run as gloo ranks on the CPU (world size 2, rendezvous on 127.0.0.1);
the failure cases make a rank exit or raise on the host, never a GPU fault."""
import ast
import itertools
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from voxq import parallel

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("n,world,align", [(4096, 2, 128), (4096, 8, 128), (1024, 3, 1), (300, 4, 32), (5, 8, 1), (0, 2, 1)])
def test_column_shard_partitions(n, world, align):
    ranges = [parallel.column_shard(n, world, r, align) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a0 <= a1
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= align
    assert all(a % align == 0 for a, _ in ranges)


def test_column_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        parallel.column_shard(10, 2, 2)


def _opt_makespan(costs, workers):
    best = float("inf")
    for assign in itertools.product(range(workers), repeat=len(costs)):
        load = [0.0] * workers
        for c, w in zip(costs, assign):
            load[w] += c
        best = min(best, max(load))
    return best


@pytest.mark.parametrize("seed", range(6))
def test_lpt_partition_bound_and_determinism(seed):
    rng = np.random.default_rng(seed)
    costs = list(rng.integers(32, 129, size=7))  # config-5 token lengths
    for workers in (1, 2, 3):
        plan = parallel.lpt_partition(costs, workers)
        assert sorted(i for u in plan for i in u) == list(range(len(costs)))
        assert plan == parallel.lpt_partition(costs, workers)
        mk = max(parallel.loads(plan, costs))
        assert mk <= (4 / 3 - 1 / (3 * workers)) * _opt_makespan(costs, workers) + 1e-9


def test_lpt_partition_config5_balance():
    rng = np.random.default_rng(5)
    costs = list(rng.integers(32, 129, size=256))
    for g in (1, 2, 4, 8):
        ld = parallel.loads(parallel.lpt_partition(costs, g), costs)
        assert max(ld) - min(ld) <= max(costs)


def test_reassign_moves_only_unfinished_units_of_dead_workers():
    costs = [9, 8, 7, 6, 5, 4, 3, 2]
    plan = parallel.lpt_partition(costs, 3)
    done = [plan[1][0]]
    new = parallel.reassign(plan, done, [1], costs)
    assert new[1] == []
    remaining = sorted(i for u in new for i in u)
    assert remaining == sorted(set(range(8)) - set(done))
    for w in (0, 2):  # live workers keep their own units first, in order
        assert new[w][:len(plan[w])] == plan[w]
    with pytest.raises(RuntimeError):
        parallel.reassign(plan, [], [0, 1, 2], costs)


def test_gloo_column_shards_reassemble_the_full_product(tmp_path):
    from oracle import oracle
    port = _free_port()
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "mp_parallel_worker.py"), "shard", str(r), "2",
                               str(port), str(tmp_path)]) for r in range(2)]
    assert [p.wait(timeout=120) for p in procs] == [0, 0]
    sharded = np.load(tmp_path / "sharded.npy")
    M, N, K = 5, 300, 64
    w = oracle.rand_normal(7, N * K, 0.02).reshape(N, K)
    a = oracle.rand_normal(8, M * K).reshape(M, K)
    wd = oracle.dequantize(oracle.quantize(w.reshape(-1), 2), N * K, 2).reshape(N, K)
    full = oracle.matmul_nt(a, wd)
    # blocks never straddle rows (K % 32 == 0), so the sharded result is bit-identical
    assert np.array_equal(sharded.view(np.uint32), np.asarray(full, dtype=np.float32).view(np.uint32))


@pytest.mark.parametrize("fail", ["exit", "raise"])
def test_watchdog_detects_a_dead_worker_and_reassigns(tmp_path, fail):
    port = _free_port()
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "mp_parallel_worker.py"), "watchdog", str(r), "2",
                               str(port), str(tmp_path), fail], stderr=subprocess.DEVNULL) for r in range(2)]
    rc0 = procs[0].wait(timeout=120)
    procs[1].wait(timeout=120)
    assert rc0 == 0
    rec = ast.literal_eval((tmp_path / "watchdog.txt").read_text())
    assert rec["dead"] == [1]
    assert rec["done"] == rec["plan"][1][:1]
    assert rec["new"][1] == []
    assert sorted(i for u in rec["new"] for i in u) == sorted(set(range(8)) - set(rec["done"]))
