"""Config 5: many utterances served by several engine workers sharing one GPU.

Each worker is the unchanged reference engine on libvoxq in serving mode
(voxq_engine_run_gpu --serve); voxq.serve assigns utterances by LPT and
collects the answers.  Checks on the seeded random-init model (Q8, whose
projection weights are exactly representable, so the CPU engine's golden
latents apply):
- the golden utterance (64 tokens, token seed 1, 4 patches) served next to
  other utterances on a shared GPU gives latents within 1e-2 max-abs of the
  CPU engine's (tests/golden/engine_c4_q8.npz) -- the north-star rule;
- every utterance's latents are bit-identical whether it is served by two
  concurrent workers or by one worker in another order: nothing leaks between
  utterances or between workers of one GPU.
"""
from __future__ import annotations

import json
import os
import shutil
import tempfile

import numpy as np
import pytest

from voxq import serve as S

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(REPO, "voxcpm2-c_b200", "engine", "_build")
GOLDEN = os.path.join(REPO, "tests", "golden")


def _workdir():
    for base in (os.environ.get("VOXQ_MODEL_DIR"), tempfile.gettempdir(), REPO):
        if base and os.path.isdir(base) and shutil.disk_usage(base).free > 12e9:
            return tempfile.mkdtemp(prefix="voxq_serve_", dir=base)
    pytest.skip("no folder with 12 GB free for the 5 GB random-init model")


def test_served_utterances_match_cpu_engine_and_each_other():
    import subprocess
    meta = json.load(open(os.path.join(GOLDEN, "engine_c4_q8.json")))
    want = np.load(os.path.join(GOLDEN, "engine_c4_q8.npz"))["latents"]
    for exe in ("make_model", "voxq_engine_run_gpu"):
        assert os.path.exists(os.path.join(BUILD, exe)), f"{exe} missing: make -C voxcpm2-c_b200/engine"
    work = _workdir()
    try:
        prefix = os.path.join(work, "rand")
        gen = json.loads(subprocess.run([os.path.join(BUILD, "make_model"), prefix, "--seed",
                                         str(meta["model"]["seed"])], check=True, capture_output=True,
                                        text=True).stdout.strip().splitlines()[-1])
        assert gen["model_data_crc32c"] == meta["model"]["model_data_crc32c"]
        utts = [{"index": 0, "tokens": meta["tokens"], "token_seed": meta["token_seed"], "patches": meta["patches"]},
                {"index": 1, "tokens": 40, "token_seed": 77, "patches": 2},
                {"index": 2, "tokens": 128, "token_seed": 78, "patches": 2},
                {"index": 3, "tokens": 97, "token_seed": 79, "patches": 3}]
        runs = {}
        for name, wpg, order in (("two_workers", 2, utts), ("one_worker", 1, utts[::-1])):
            lat = os.path.join(work, name)
            os.makedirs(lat)
            cmd = [os.path.join(BUILD, "voxq_engine_run_gpu"), "--model", prefix + ".vxcpm", "--gpu", "--serve",
                   "--latents-dir", lat]
            r = S.serve(cmd, order, gpus=[0], workers_per_gpu=wpg, env=dict(os.environ, VOXCPM_QUANT="q8"),
                        deadline_s=600)
            assert r["answered"] == 4 and not r["errors"] and not r["dead_workers"], r
            runs[name] = (r, {u["index"]: np.fromfile(os.path.join(lat, f"utt{u['index']}.f32"), dtype=np.float32)
                              for u in utts})
    finally:
        shutil.rmtree(work, ignore_errors=True)
    r2, lat2 = runs["two_workers"]
    r1, lat1 = runs["one_worker"]
    assert len({x["worker"] for x in r2["results"]}) == 2, "both workers should have served"
    for u in utts:
        assert lat2[u["index"]].size == 256 * u["patches"]
        assert np.array_equal(lat2[u["index"]], lat1[u["index"]]), f"utterance {u['index']} differs between runs"
    got = lat2[0].reshape(want.shape)
    err = float(np.abs(got.astype(np.float64) - want).max())
    assert err <= 1e-2, f"golden utterance latents max-abs error {err:.3e}"
    assert all(x["weight_bytes"] > 0 and x["matmul_calls"] > 0 for x in r2["results"])
    print(f"served: {r2['utt_per_s']} utt/s with 2 workers, {r1['utt_per_s']} with 1; golden err {err:.2e}")
