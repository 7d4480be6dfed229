"""Config-5 serving: many independent utterances over G GPUs, W engine workers per GPU.

Each worker is one process of the engine harness in serving mode
(``voxq_engine_run_gpu --serve``: the unchanged voxcpm2-c engine, src/model.c
voxcpm_create -> voxcpm_to_cuda -> voxcpm_generate per utterance, linked
against libvoxq).  It loads its own model replica on the GPU named by
``CUDA_VISIBLE_DEVICES``, prints ``{"ready": ...}``, then synthesises one
utterance per request line ``"INDEX TOKENS TOKEN_SEED PATCHES"`` and answers
with one JSON line.  The reference engine is single-utterance (``B = 1``,
src/model.c:653), so concurrency comes from workers, never from batching
inside one.

Scheduling (host side, no inter-GPU traffic):
- utterances are assigned to workers longest-processing-time first on their
  cost (``parallel.lpt_partition``), all requests written up front;
- a worker's answers are its heartbeats: one that stays silent for
  ``deadline_s`` while it owes answers, or whose process ends, is declared
  dead, its process group (started here) is killed, and its unanswered
  utterances move to the live workers (``parallel.reassign``);
- an utterance answered twice (a late answer from a worker declared dead) is
  kept once.
"""
from __future__ import annotations

import json
import os
import queue
import signal
import subprocess
import threading
import time
from typing import Dict, List, Optional, Sequence

from .parallel import lpt_partition, reassign

VOCAB = 73448


def workload(n: int, patches: int, seed: int = 5, lo: int = 32, hi: int = 128) -> List[dict]:
    """``n`` utterances: token counts uniform in [lo, hi], token-id seeds distinct and non-zero
    (the harness draws ids uniformly from the 73448-entry vocabulary with xorshift64)."""
    import numpy as np
    rs = np.random.RandomState(seed)
    lens = rs.randint(lo, hi + 1, size=n)
    return [{"index": i, "tokens": int(lens[i]), "token_seed": int(seed) * 1000003 + i + 1, "patches": int(patches)}
            for i in range(n)]


def cost(u: dict) -> float:
    """Scheduling cost of an utterance: its patches dominate (each runs the DiT sampler, the
    AudioVAE decode and a RALM step); the prefill grows with the token count."""
    return float(u["patches"]) + u["tokens"] / 32.0


class _Worker:
    def __init__(self, wid: int, gpu: int, cmd: Sequence[str], env: dict, events: "queue.Queue"):
        self.wid, self.gpu = wid, gpu
        self.proc = subprocess.Popen(list(cmd), stdin=subprocess.PIPE, stdout=subprocess.PIPE,
                                     stderr=subprocess.PIPE, env=env, text=True, bufsize=1,
                                     start_new_session=True)
        self.ready = None
        self.owed: List[int] = []  # requests written and not answered, in order
        self.last = time.time()
        self.dead = False
        self.stderr_tail: List[str] = []
        threading.Thread(target=self._read_out, args=(events,), daemon=True).start()
        threading.Thread(target=self._read_err, daemon=True).start()

    def _read_out(self, events):
        for line in self.proc.stdout:
            events.put((self.wid, line))
        events.put((self.wid, None))  # end of output: the process is gone

    def _read_err(self):
        for line in self.proc.stderr:
            self.stderr_tail = (self.stderr_tail + [line.rstrip()])[-20:]

    def send(self, u: dict) -> bool:
        try:
            self.proc.stdin.write(f"{u['index']} {u['tokens']} {u['token_seed']} {u['patches']}\n")
            self.proc.stdin.flush()
        except (BrokenPipeError, OSError, ValueError):
            return False
        self.owed.append(u["index"])
        return True

    def stop(self, timeout: float = 30.0):
        try:
            self.proc.stdin.write("quit\n")
            self.proc.stdin.close()
        except (BrokenPipeError, OSError, ValueError):
            pass
        try:
            self.proc.wait(timeout=timeout)
        except subprocess.TimeoutExpired:
            self.kill()

    def kill(self):
        """Ends the process group this worker was started in (and nothing else)."""
        if self.proc.poll() is None:
            try:
                os.killpg(self.proc.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
        try:
            self.proc.wait(timeout=30)
        except subprocess.TimeoutExpired:
            pass


def visible_device(g: int, env: dict) -> str:
    """The ``CUDA_VISIBLE_DEVICES`` value that pins a worker to GPU ``g`` as the calling process
    numbers its GPUs: the g-th entry of the caller's own ``CUDA_VISIBLE_DEVICES`` when that is set
    (an index or a UUID), else ``g`` itself (also for an index past the caller's list)."""
    ids = [x.strip() for x in env.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip()]
    return ids[g] if 0 <= g < len(ids) else str(g)


def serve(cmd: Sequence[str], utterances: Sequence[dict], gpus: Sequence[int], workers_per_gpu: int = 1,
          env: Optional[dict] = None, deadline_s: float = 120.0, ready_timeout_s: float = 900.0) -> dict:
    """Runs ``utterances`` (dicts from ``workload``) on ``len(gpus) * workers_per_gpu`` workers of
    ``cmd`` and returns the per-utterance answers and the throughput.  Throughput is measured from
    the moment the requests are written (every worker loaded) to the last answer.  ``gpus`` are
    indices as this process sees its GPUs (``visible_device``)."""
    if not gpus or workers_per_gpu < 1:
        raise ValueError("need at least one GPU and one worker per GPU")
    by_index = {u["index"]: u for u in utterances}
    costs = {u["index"]: cost(u) for u in utterances}
    events: "queue.Queue" = queue.Queue()
    base_env = dict(os.environ if env is None else env)
    workers: List[_Worker] = []
    for g in gpus:
        for _ in range(workers_per_gpu):
            e = dict(base_env, CUDA_VISIBLE_DEVICES=visible_device(g, base_env))
            workers.append(_Worker(len(workers), g, cmd, e, events))
    results: Dict[int, dict] = {}
    errors: List[dict] = []
    dead: List[int] = []
    reassigned: List[int] = []
    t_load = time.time()
    try:
        # ---- every worker loads its replica; one that fails to is dead from the start
        pending_ready = {w.wid for w in workers}
        while pending_ready:
            left = ready_timeout_s - (time.time() - t_load)
            if left <= 0:
                break
            try:
                wid, line = events.get(timeout=min(left, 1.0))
            except queue.Empty:
                continue
            w = workers[wid]
            if line is None:
                w.dead = True
                pending_ready.discard(wid)
                continue
            try:
                msg = json.loads(line)
            except json.JSONDecodeError:
                continue
            if msg.get("ready"):
                w.ready = msg
                pending_ready.discard(wid)
        for wid in pending_ready:
            workers[wid].dead = True
        for w in workers:
            if w.dead:
                dead.append(w.wid)
                w.kill()
        live = [w for w in workers if not w.dead]
        if not live:
            raise RuntimeError("no serving worker came up: " +
                               " | ".join(" ".join(w.stderr_tail[-3:]) for w in workers))
        load_s = time.time() - t_load

        # ---- LPT assignment over the live workers, all requests written up front
        order = [u["index"] for u in utterances]
        plan = lpt_partition([costs[i] for i in order], len(live))
        t0 = time.time()
        for w, units in zip(live, plan):
            w.last = t0
            for k in units:
                if not w.send(by_index[order[k]]):
                    break
        t_last = t0

        def declare_dead(w: _Worker):
            w.dead = True
            dead.append(w.wid)
            w.kill()
            owed = [i for i in w.owed if i not in results]
            w.owed = []
            alive = [x for x in workers if not x.dead]
            if not owed:
                return
            if not alive:
                raise RuntimeError(f"every serving worker died; {len(owed)} utterances unanswered")
            cur = [[i for i in x.owed if i not in results] for x in alive] + [owed]
            moved = reassign(cur, results.keys(), [len(alive)], costs)
            for x, mine in zip(alive, moved):
                new = [i for i in mine if i not in x.owed]
                if new and not x.owed:
                    x.last = time.time()  # an idle worker's silence so far is not late
                for i in new:
                    reassigned.append(i)
                    x.send(by_index[i])

        # ---- answers (heartbeats) until every utterance is answered
        while len(results) < len(utterances):
            try:
                wid, line = events.get(timeout=0.5)
            except queue.Empty:
                wid, line = None, ""
            if wid is not None:
                w = workers[wid]
                if line is None:
                    if not w.dead and [i for i in w.owed if i not in results]:
                        declare_dead(w)
                    continue
                try:
                    msg = json.loads(line)
                except json.JSONDecodeError:
                    continue
                if "utt" in msg:
                    i = int(msg["utt"])
                    w.last = time.time()
                    if i in w.owed:
                        w.owed.remove(i)
                    if "error" in msg:
                        errors.append(dict(msg, worker=w.wid))
                        results.setdefault(i, dict(msg, worker=w.wid, gpu=w.gpu))
                    elif i not in results or "error" in results[i]:
                        results[i] = dict(msg, worker=w.wid, gpu=w.gpu, t_done=w.last - t0)
                    t_last = max(t_last, w.last)
            now = time.time()
            for w in workers:
                if not w.dead and w.owed and now - w.last > deadline_s:
                    declare_dead(w)
        wall = t_last - t0
    finally:
        for w in workers:
            if not w.dead:
                w.stop()
            else:
                w.kill()

    ok = [r for r in results.values() if "error" not in r]
    per_gpu = {}
    for g in sorted(set(gpus)):
        rs = [r for r in ok if r["gpu"] == g]
        wb = sum(int(r.get("weight_bytes", 0)) for r in rs)
        per_gpu[str(g)] = {"utterances": len(rs), "patches": sum(int(r["patches"]) for r in rs),
                           "weight_bytes": wb, "GBps": round(wb / wall / 1e9, 2) if wall > 0 else None}
    audio = sum(float(r.get("audio_s", 0.0)) for r in ok)
    return {
        "utterances": len(utterances), "answered": len(ok), "errors": errors,
        "workers": len(workers), "workers_per_gpu": workers_per_gpu, "gpus": list(gpus),
        "load_s": round(load_s, 3), "wall_s": round(wall, 4),
        "utt_per_s": round(len(ok) / wall, 4) if wall > 0 else None,
        "audio_s": round(audio, 3), "rtf_aggregate": round(wall / audio, 4) if audio > 0 else None,
        "per_gpu": per_gpu, "dead_workers": dead, "reassigned": sorted(set(reassigned)),
        "results": [results[i] for i in sorted(results)],
    }


__all__ = ["workload", "cost", "serve", "visible_device", "VOCAB"]
