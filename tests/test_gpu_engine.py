"""Config 4: the unchanged reference engine on libvoxq.

The reference's src/*.c, compiled as they are with VOXCPM_CUDA (so
tensor_matmul_nt calls tensor_matmul_nt_cuda, src/tensor.c:629-640) and
linked against libvoxq.so, loads the seeded random-init model, uploads it with
voxcpm_to_cuda (src/model.c:498-560) under VOXCPM_QUANT=q8 -- every projection
weight quantized on the device, bit-exactly as scripts/quantize.py would --
and runs voxcpm_generate (src/model.c:630-1048): TSLM and RALM prefill over 64
token ids, then per patch the LocDiT sampler (10 Euler steps, CFG 2.0), the
AudioVAE decode and the LocEnc -> fusion -> RALM update.

Oracle: the same engine built without VOXCPM_CUDA (the reference CPU path, one
scalar loop per output, src/tensor.c:617-678) on the same model, whose latents
are committed in tests/golden/engine_c4_q8.npz (tests/golden/make_engine_golden.py).
The model's projection weights are exactly representable in Q8, so both runs
multiply by identical weights.  Rule (north star): latents within 1e-2 max-abs.
"""
from __future__ import annotations

import json
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(REPO, "voxcpm2-c_b200", "engine", "_build")
GOLDEN = os.path.join(REPO, "tests", "golden")
TOL = 1e-2


def _workdir():
    """A scratch folder with room for the ~5 GB model."""
    for base in (os.environ.get("VOXQ_MODEL_DIR"), tempfile.gettempdir(), REPO):
        if base and os.path.isdir(base) and shutil.disk_usage(base).free > 12e9:
            return tempfile.mkdtemp(prefix="voxq_engine_", dir=base)
    pytest.skip("no folder with 12 GB free for the 5 GB random-init model")


def test_unchanged_engine_on_libvoxq_matches_cpu_engine():
    meta = json.load(open(os.path.join(GOLDEN, "engine_c4_q8.json")))
    want = np.load(os.path.join(GOLDEN, "engine_c4_q8.npz"))["latents"]
    for exe in ("make_model", "voxq_engine_run_gpu"):
        assert os.path.exists(os.path.join(BUILD, exe)), \
            f"{exe} missing: build it with `make -C voxcpm2-c_b200/engine REF=<reference checkout>`"
    work = _workdir()
    try:
        prefix = os.path.join(work, "rand")
        gen = json.loads(subprocess.run([os.path.join(BUILD, "make_model"), prefix, "--seed",
                                         str(meta["model"]["seed"])], check=True, capture_output=True,
                                        text=True).stdout.strip().splitlines()[-1])
        for k in ("model_data_crc32c", "audiovae_data_crc32c", "model_bytes", "audiovae_bytes"):
            assert gen[k] == meta["model"][k], f"regenerated model differs from the golden run's ({k})"
        lat = os.path.join(work, "gpu_latents.f32")
        env = dict(os.environ, VOXCPM_QUANT="q8")
        r = subprocess.run([os.path.join(BUILD, "voxq_engine_run_gpu"), "--model", prefix + ".vxcpm", "--gpu",
                            "--patches", str(meta["patches"]), "--tokens", str(meta["tokens"]),
                            "--token-seed", str(meta["token_seed"]), "--latents", lat],
                           env=env, capture_output=True, text=True, timeout=1200)
        assert r.returncode == 0, r.stderr[-3000:]
        assert "GPU upload complete" in r.stderr
        run = json.loads(r.stdout.strip().splitlines()[-1])
        got = np.fromfile(lat, dtype=np.float32).reshape(want.shape)
    finally:
        shutil.rmtree(work, ignore_errors=True)
    assert run["build"] == "gpu"
    mm = run["stages"]["tensor_matmul_nt"]
    assert mm["calls"] == meta["cpu_run"]["stages"]["tensor_matmul_nt"]["calls"]
    # the projections ran on the device: the CPU loop takes ~80 ms per call here
    assert mm["s"] / mm["calls"] < 2e-3, f"{mm['s'] / mm['calls'] * 1e3:.2f} ms per tensor_matmul_nt"
    err = np.abs(got.astype(np.float64) - want)
    assert np.isfinite(got).all()
    assert float(err.max()) <= TOL, f"latents max-abs error {float(err.max()):.3e} per patch " \
                                    f"{[float(e) for e in err.reshape(len(err), -1).max(1)]}"
