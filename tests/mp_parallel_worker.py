"""Worker process for the multi-process (gloo, CPU) tests of voxq.parallel.

Usage: python mp_parallel_worker.py <mode> <rank> <world> <port> <outdir>
  shard     each rank computes its output-column shard of A W^T with the CPU oracle on its own
            quantized weight rows; rank 0 gathers the shards (test-only gather) and saves them.
  watchdog  rank 1 publishes one heartbeat then stops (or raises); rank 0 detects it dead after
            the deadline and re-assigns its unfinished utterances.
"""
import os
import sys
import time

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "voxcpm2-c_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch.distributed as dist  # noqa: E402

from voxq import parallel  # noqa: E402


def shard(rank, world, port, outdir):
    from oracle import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    M, N, K, qt = 5, 300, 64, 2  # Q4
    w = oracle.rand_normal(7, N * K, 0.02).reshape(N, K)
    a = oracle.rand_normal(8, M * K).reshape(M, K)
    n0, n1 = parallel.column_shard(N, world, rank, align=32)
    blocks = oracle.quantize(w[n0:n1].reshape(-1), qt)          # this rank's rows only
    wd = oracle.dequantize(blocks, (n1 - n0) * K, qt).reshape(n1 - n0, K)
    y = oracle.matmul_nt(a, wd)
    got = [None] * world
    dist.all_gather_object(got, (n0, n1, y.tolist()))           # test-only gather of the results
    if rank == 0:
        out = np.zeros((M, N), dtype=np.float32)
        for (s0, s1, ys) in got:
            out[:, s0:s1] = np.asarray(ys, dtype=np.float32)
        np.save(os.path.join(outdir, "sharded.npy"), out)
    dist.barrier()
    dist.destroy_process_group()


def watchdog(rank, world, port, outdir, fail):
    from torch.distributed import TCPStore
    store = TCPStore("127.0.0.1", port, world, rank == 0, timeout=__import__("datetime").timedelta(seconds=30))
    costs = [100, 80, 75, 60, 40, 35, 20, 10]
    plan = parallel.lpt_partition(costs, world)
    hb = parallel.Heartbeat(store, rank)
    if rank == 1:
        mine = plan[1]
        hb.beat(mine[:1])          # finished its first utterance
        if fail == "raise":
            raise RuntimeError("worker 1 failed")
        os._exit(3)                # dies silently, no further heartbeat
    wd = parallel.Watchdog(store, world, deadline_s=1.0)
    done = []
    t_end = time.time() + 20
    dead = []
    while time.time() < t_end:
        hb.beat(done)
        dead, done_all = wd.poll()
        if dead:
            break
        time.sleep(0.1)
    new = parallel.reassign(plan, done_all, dead, costs)
    with open(os.path.join(outdir, "watchdog.txt"), "w") as f:
        f.write(repr({"dead": dead, "done": done_all, "plan": plan, "new": new}))


if __name__ == "__main__":
    mode, rank, world, port, outdir = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]), sys.argv[5]
    if mode == "shard":
        shard(rank, world, port, outdir)
    else:
        watchdog(rank, world, port, outdir, sys.argv[6] if len(sys.argv) > 6 else "exit")
