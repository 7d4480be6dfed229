"""Config 5 scheduling on the host: the serving orchestrator (voxq.serve) driving
stand-in workers that speak the engine worker's protocol (tests/fake_serve_worker.py).

Checks LPT placement, that every utterance is answered exactly once, and the
failure path of SURVEY 8(e): a worker that stops answering (hangs) or exits is
declared dead after the deadline, its process group is killed, and its
unanswered utterances move to the live workers.  No GPU is used.
"""
from __future__ import annotations

import os
import sys
import time

import pytest

from voxq import serve as S
from voxq.parallel import lpt_partition

HERE = os.path.dirname(os.path.abspath(__file__))
FAKE = [sys.executable, os.path.join(HERE, "fake_serve_worker.py")]


def test_workload_is_seeded_and_in_range():
    a = S.workload(64, patches=100, seed=5)
    b = S.workload(64, patches=100, seed=5)
    assert a == b
    assert all(32 <= u["tokens"] <= 128 and u["patches"] == 100 and u["token_seed"] != 0 for u in a)
    assert len({u["token_seed"] for u in a}) == 64
    assert S.workload(64, patches=100, seed=6) != a


def test_all_answered_once_with_lpt_balance():
    utts = S.workload(24, patches=3, seed=1)
    r = S.serve(FAKE, utts, gpus=[0, 1], workers_per_gpu=2, env=dict(os.environ, FAKE_SLEEP="0.005"),
                deadline_s=20)
    assert r["answered"] == 24 and not r["errors"] and not r["dead_workers"]
    assert [x["utt"] for x in r["results"]] == list(range(24))
    # placement follows lpt_partition over the 4 workers
    plan = lpt_partition([S.cost(u) for u in utts], 4)
    for w, units in enumerate(plan):
        assert sorted(x["utt"] for x in r["results"] if x["worker"] == w) == sorted(units)
    assert set(r["per_gpu"]) == {"0", "1"}
    assert sum(g["utterances"] for g in r["per_gpu"].values()) == 24
    assert r["utt_per_s"] > 0 and r["wall_s"] > 0


@pytest.mark.parametrize("mode", ["hang", "exit"])
def test_dead_worker_is_replaced(tmp_path, mode):
    # worker on "GPU" 1 fails after one answer; the others take over its utterances
    wrapper = tmp_path / "w.py"
    knob = "FAKE_HANG_AFTER" if mode == "hang" else "FAKE_EXIT_AFTER"
    wrapper.write_text(
        "import os, runpy, sys\n"
        f"if os.environ.get('CUDA_VISIBLE_DEVICES') == '1': os.environ['{knob}'] = '1'\n"
        f"sys.argv = [{FAKE[1]!r}]\n"
        f"runpy.run_path({FAKE[1]!r}, run_name='__main__')\n")
    utts = S.workload(12, patches=2, seed=3)
    t0 = time.time()
    r = S.serve([sys.executable, str(wrapper)], utts, gpus=[0, 1, 2], workers_per_gpu=1,
                env=dict(os.environ, FAKE_SLEEP="0.01"), deadline_s=1.5)
    assert time.time() - t0 < 60
    assert r["answered"] == 12 and [x["utt"] for x in r["results"]] == list(range(12))
    assert r["dead_workers"] == [1]
    assert r["reassigned"], "the dead worker's utterances were not moved"
    assert all(x["gpu"] != 1 for x in r["results"] if x["utt"] in r["reassigned"])
    assert r["per_gpu"]["1"]["utterances"] == 1


def test_worker_that_never_loads_is_skipped(tmp_path):
    wrapper = tmp_path / "w.py"
    wrapper.write_text(
        "import os, runpy, sys\n"
        "if os.environ.get('CUDA_VISIBLE_DEVICES') == '0': os.environ['FAKE_NO_READY'] = '1'\n"
        f"sys.argv = [{FAKE[1]!r}]\n"
        f"runpy.run_path({FAKE[1]!r}, run_name='__main__')\n")
    utts = S.workload(6, patches=1, seed=2)
    r = S.serve([sys.executable, str(wrapper)], utts, gpus=[0, 1], workers_per_gpu=1,
                env=dict(os.environ), deadline_s=5, ready_timeout_s=30)
    assert r["dead_workers"] == [0]
    assert r["answered"] == 6 and all(x["gpu"] == 1 for x in r["results"])


def test_no_worker_up_raises(tmp_path):
    with pytest.raises(RuntimeError, match="no serving worker"):
        S.serve(FAKE, S.workload(2, patches=1), gpus=[0], workers_per_gpu=1,
                env=dict(os.environ, FAKE_NO_READY="1"), deadline_s=2, ready_timeout_s=10)


def test_workers_follow_the_callers_visible_devices(tmp_path):
    """A caller that itself sees only some GPUs (CUDA_VISIBLE_DEVICES=6,3) numbers them 0 and 1;
    its worker for GPU 1 must be pinned to physical GPU 3, not 1: here the worker on "3" never
    loads, so worker 1 is the dead one and GPU 0 ("6") answers everything."""
    assert S.visible_device(1, {"CUDA_VISIBLE_DEVICES": "6,3"}) == "3"
    assert S.visible_device(0, {"CUDA_VISIBLE_DEVICES": "GPU-aa, GPU-bb"}) == "GPU-aa"
    assert S.visible_device(2, {"CUDA_VISIBLE_DEVICES": "6,3"}) == "2"
    assert S.visible_device(1, {}) == "1"
    wrapper = tmp_path / "w.py"
    wrapper.write_text(
        "import os, runpy, sys\n"
        "if os.environ.get('CUDA_VISIBLE_DEVICES') == '3': os.environ['FAKE_NO_READY'] = '1'\n"
        f"sys.argv = [{FAKE[1]!r}]\n"
        f"runpy.run_path({FAKE[1]!r}, run_name='__main__')\n")
    utts = S.workload(4, patches=1, seed=4)
    r = S.serve([sys.executable, str(wrapper)], utts, gpus=[0, 1], workers_per_gpu=1,
                env=dict(os.environ, CUDA_VISIBLE_DEVICES="6,3"), deadline_s=5, ready_timeout_s=30)
    assert r["dead_workers"] == [1]
    assert r["answered"] == 4 and all(x["gpu"] == 0 for x in r["results"])
