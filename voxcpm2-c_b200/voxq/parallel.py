"""Multi-GPU partitioning for the quantized matmul path: shards and work lists, no collectives.

One process per GPU (launched by torchrun); nothing here moves tensors between GPUs.

- Batched GEMM (config 3): GPU g owns the weight rows, i.e. the output columns,
  ``[g*N/G, (g+1)*N/G)``.  Quantized blocks never straddle rows when K % 32 == 0, so each
  rank quantizes (or loads) only its rows and writes its column slice of ``out`` in place.
- Serving (config 5): independent utterances are assigned to GPUs by longest-processing-time
  first on their cost (token count), one model replica per GPU.
- Fault handling: workers publish heartbeats in a ``torch.distributed`` key-value store; a
  coordinator declares workers whose heartbeat is older than a deadline dead and re-assigns
  their unfinished utterances to live workers (LPT again).  Detection is on the host, between
  steps; no GPU wait depends on another rank.
"""
from __future__ import annotations

import heapq
import time
from typing import Dict, Iterable, List, Optional, Sequence, Tuple


def column_shard(n: int, world: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """Half-open output-column range of ``rank`` when ``n`` columns are split over ``world`` ranks.

    Ranges are contiguous, disjoint, cover [0, n) and differ in size by at most ``align``
    (boundaries are multiples of ``align``, e.g. 128 to keep whole GEMM tiles on one rank)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if align <= 0:
        raise ValueError("align must be positive")
    units = (n + align - 1) // align
    lo = units * rank // world
    hi = units * (rank + 1) // world
    return min(n, lo * align), min(n, hi * align)


def lpt_partition(costs: Sequence[float], workers: int) -> List[List[int]]:
    """Longest-processing-time-first assignment of units to ``workers``.

    Units are taken in decreasing cost (ties by index) and each goes to the currently least
    loaded worker (ties by worker index), so the result is deterministic.  The makespan is at
    most (4/3 - 1/(3 workers)) of the optimum.  Returns, per worker, the unit indices in the
    order they were assigned."""
    if workers <= 0:
        raise ValueError("workers must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, w) for w in range(workers)]
    out: List[List[int]] = [[] for _ in range(workers)]
    for i in order:
        load, w = heapq.heappop(heap)
        out[w].append(i)
        heapq.heappush(heap, (load + float(costs[i]), w))
    return out


def loads(assignment: Sequence[Sequence[int]], costs: Sequence[float]) -> List[float]:
    return [float(sum(costs[i] for i in units)) for units in assignment]


def reassign(assignment: Sequence[Sequence[int]], done: Iterable[int], dead: Iterable[int],
             costs: Sequence[float]) -> List[List[int]]:
    """Moves the unfinished units of ``dead`` workers onto the live ones (LPT on top of the live
    workers' remaining load).  Finished units are dropped from every list."""
    done_set, dead_set = set(done), set(dead)
    live = [w for w in range(len(assignment)) if w not in dead_set]
    if not live:
        raise RuntimeError("no live worker left")
    out: List[List[int]] = [[] if w in dead_set else [i for i in units if i not in done_set]
                            for w, units in enumerate(assignment)]
    orphans = [i for w in sorted(dead_set) if w < len(assignment) for i in assignment[w] if i not in done_set]
    heap = [(sum(costs[i] for i in out[w]), w) for w in live]
    heapq.heapify(heap)
    for i in sorted(orphans, key=lambda i: (-costs[i], i)):
        load, w = heapq.heappop(heap)
        out[w].append(i)
        heapq.heappush(heap, (load + float(costs[i]), w))
    return out


class Heartbeat:
    """Worker side: publishes ``(time, units done)`` under ``hb/<rank>`` in a store."""

    def __init__(self, store, rank: int, prefix: str = "hb"):
        self.store, self.rank, self.prefix = store, rank, prefix

    def beat(self, units_done: Sequence[int] = ()) -> None:
        done = ",".join(str(i) for i in units_done)
        self.store.set(f"{self.prefix}/{self.rank}", f"{time.time():.6f};{done}")


class Watchdog:
    """Coordinator side: reads every worker's heartbeat and reports the ones that are late.

    A worker that never published counts from the watchdog's creation; one whose last beat is
    older than ``deadline_s`` is dead.  ``poll`` never blocks on a missing key."""

    def __init__(self, store, world: int, deadline_s: float, prefix: str = "hb"):
        self.store, self.world, self.deadline, self.prefix = store, world, deadline_s, prefix
        self.t0 = time.time()

    def _read(self, rank: int) -> Optional[Tuple[float, List[int]]]:
        key = f"{self.prefix}/{rank}"
        if self.store.check([key]):
            t, _, done = self.store.get(key).decode().partition(";")
            return float(t), [int(x) for x in done.split(",") if x]
        return None

    def poll(self) -> Tuple[List[int], List[int]]:
        """Returns (dead ranks, units reported done by any rank)."""
        now = time.time()
        dead: List[int] = []
        done: List[int] = []
        for r in range(self.world):
            rec = self._read(r)
            last = rec[0] if rec else self.t0
            if rec:
                done.extend(rec[1])
            if now - last > self.deadline:
                dead.append(r)
        return dead, sorted(set(done))


def shard_weight_rows(w_fp32, world: int, rank: int, align: int = 128):
    """Rows of an fp32 weight [N, K] (torch) owned by ``rank``: (view, n0, n1)."""
    n0, n1 = column_shard(int(w_fp32.shape[0]), world, rank, align)
    return w_fp32[n0:n1], n0, n1


def matmul_column_shard(a, w_shard, out, n0: int, stream=None, **epi):
    """out[:, n0:n0+Ns] = epilogue(a @ w_shard^T) for this rank's rows (a QWeight of Ns rows);
    ``out`` is the full [M, N] output (row stride N), written only in this rank's columns."""
    from . import matmul_nt_q
    ns = w_shard.N
    return matmul_nt_q(a, w_shard, out=out[:, n0:n0 + ns], stream=stream, **epi)


__all__ = ["column_shard", "lpt_partition", "loads", "reassign", "Heartbeat", "Watchdog",
           "shard_weight_rows", "matmul_column_shard"]
