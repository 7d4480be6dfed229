"""Config 4: the unchanged reference engine on libvoxq.

The reference's src/*.c, compiled as they are with VOXCPM_CUDA (so
tensor_matmul_nt calls tensor_matmul_nt_cuda, src/tensor.c:629-640) and
linked against libvoxq.so, loads the seeded random-init model, uploads it with
voxcpm_to_cuda (src/model.c:498-560) under VOXCPM_QUANT=q8 -- every projection
weight quantized on the device, bit-exactly as scripts/quantize.py would --
and runs voxcpm_generate (src/model.c:630-1048): TSLM and RALM prefill over 64
token ids, then per patch the LocDiT sampler (10 Euler steps, CFG 2.0), the
AudioVAE decode and the LocEnc -> fusion -> RALM update.

The libvoxq build also sends every transformer block
(transformer_block_forward, src/nn.c:579-700: norms, attention with its KV
cache, SwiGLU, residuals) to libvoxq's device block, and the AudioVAE
decoder's convolutions (conv1d_forward / conv1d_transpose_forward,
src/nn.c:765-931), which the reference runs on the host even in its GPU
build, to libvoxq's device convolutions.

Oracle: the same engine built without VOXCPM_CUDA (the reference CPU path, one
scalar loop per output, src/tensor.c:617-678, and the host convolutions) on the
same model, whose latents and audio are committed in
tests/golden/engine_c4_q8.npz (tests/golden/make_engine_golden.py).  The
model's projection weights are exactly representable in Q8, so both runs
multiply by identical weights.  Rule (north star): latents within 1e-2
max-abs.

The device convolutions are checked on the engine's own data by a second run
of the libvoxq build with VOXQ_ENGINE_VAE=cpu (the reference's host
convolutions): both runs have bit-identical latents, so their audio differs
only by the convolution path (fp32 on both sides, different summation order).
The random-init AudioVAE saturates: its peak-normalised output sits at +-1
except for isolated transition samples between the two, which move with the
last bits of their inputs (one sample seen at -0.30 vs -0.35).  Rules on the
audio: mean |difference| <= 5e-4 and 99th percentile <= 5e-3.  (It is not
compared with the CPU engine's audio, whose slightly different latents move
the transitions.)
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
AUDIO_MEAN_TOL, AUDIO_P99_TOL = 5e-4, 5e-3


def _workdir():
    """A scratch folder with room for the ~5 GB model."""
    for base in (os.environ.get("VOXQ_MODEL_DIR"), tempfile.gettempdir(), REPO):
        if base and os.path.isdir(base) and shutil.disk_usage(base).free > 12e9:
            return tempfile.mkdtemp(prefix="voxq_engine_", dir=base)
    pytest.skip("no folder with 12 GB free for the 5 GB random-init model")


@pytest.fixture(scope="module")
def model():
    """The golden run's seeded random-init model, written once for this module:
    (folder, model path prefix, golden metadata)."""
    meta = json.load(open(os.path.join(GOLDEN, "engine_c4_q8.json")))
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
        yield work, prefix, meta
    finally:
        shutil.rmtree(work, ignore_errors=True)


def _run(exe, model_path, meta, work, tag, **env):
    """One engine run; returns (its JSON line, latents, audio)."""
    lat = os.path.join(work, f"lat_{tag}.f32")
    aud = os.path.join(work, f"audio_{tag}.f32")
    r = subprocess.run([os.path.join(BUILD, exe), "--model", model_path, "--gpu",
                        "--patches", str(meta["patches"]), "--tokens", str(meta["tokens"]),
                        "--token-seed", str(meta["token_seed"]), "--latents", lat, "--audio", aud],
                       env=dict(os.environ, **env), capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "GPU upload complete" in r.stderr
    out = (json.loads(r.stdout.strip().splitlines()[-1]), np.fromfile(lat, dtype=np.float32),
           np.fromfile(aud, dtype=np.float32))
    os.remove(lat)
    os.remove(aud)
    return out


def test_unchanged_engine_on_libvoxq_matches_cpu_engine(model):
    work, prefix, meta = model
    gold = np.load(os.path.join(GOLDEN, "engine_c4_q8.npz"))
    want, want_audio = gold["latents"], gold["audio"]
    runs = {}
    for vae in ("gpu", "cpu"):
        run_, lat, aud = _run("voxq_engine_run_gpu", prefix + ".vxcpm", meta, work, vae, VOXCPM_QUANT="q8",
                              VOXQ_ENGINE_VAE=vae)
        runs[vae] = (run_, lat.reshape(want.shape), aud)
    run, got, got_audio = runs["gpu"]
    _, got_cpu_vae, host_audio = runs["cpu"]
    assert run["build"] == "gpu" and run["vae"] == "device"
    # every transformer block (TSLM, RALM, LocDiT, LocEnc) ran on the device
    assert run["blocks"]["device"] > 0 and run["blocks"]["host"] == 0, run["blocks"]
    mm = run["stages"]["tensor_matmul_nt"]
    # the projections outside the blocks ran on the device: the CPU loop takes ~80 ms per call here
    assert 0 < mm["calls"] < meta["cpu_run"]["stages"]["tensor_matmul_nt"]["calls"]
    assert mm["s"] / mm["calls"] < 2e-3, f"{mm['s'] / mm['calls'] * 1e3:.2f} ms per tensor_matmul_nt"
    err = np.abs(got.astype(np.float64) - want)
    assert np.isfinite(got).all()
    assert float(err.max()) <= TOL, f"latents max-abs error {float(err.max()):.3e} per patch " \
                                    f"{[float(e) for e in err.reshape(len(err), -1).max(1)]}"
    print(f"latents max-abs error per patch: {[float(e) for e in err.reshape(len(err), -1).max(1)]}")
    # the convolution path: same latents, device vs host convolutions
    assert np.array_equal(got, got_cpu_vae)
    assert got_audio.shape == want_audio.shape == host_audio.shape and np.isfinite(got_audio).all()
    d = np.abs(got_audio.astype(np.float64) - host_audio)
    mean, p99 = float(d.mean()), float(np.quantile(d, 0.99))
    print(f"audio, device vs host convolutions on the same latents: mean |d| {mean:.2e}, p99 {p99:.2e}, "
          f"max {float(d.max()):.2e}")
    assert mean <= AUDIO_MEAN_TOL and p99 <= AUDIO_P99_TOL, f"audio mean |d| {mean:.2e}, p99 {p99:.2e}"


@pytest.mark.parametrize("quant", ["q8", "q4"])
def test_prequantized_vxcp_file(model, quant):
    """The engine starting from a pre-quantized VXCP file (voxq_vxcp_quantize:
    every 2-D projection weight stored as Q8 / Q4_1 blocks, the host-read token
    embedding kept as it is) through the qfile build, whose loader reads those
    dtypes and hands the blocks to tensor_to_cuda, with VOXCPM_QUANT unset,
    must produce the same latents bit for bit as the fp32/fp16 file quantized
    on upload (VOXCPM_QUANT=q8 / q4): the device weights are the same
    quantize.py blocks either way.  For Q8 that also ties it to the CPU
    engine's golden latents (the model's weights are exact in Q8)."""
    import sys
    sys.path.insert(0, os.path.join(REPO, "voxcpm2-c_b200"))
    import voxq
    from voxq import vxcp
    work, prefix, meta = model
    exe = "voxq_engine_run_gpu_qfile"
    assert os.path.exists(os.path.join(BUILD, exe)), f"{exe} missing: build the engine harness"
    qdir = os.path.join(work, quant)
    os.makedirs(qdir, exist_ok=True)
    qpath = os.path.join(qdir, "rand.vxcpm")
    st = vxcp.quantize_file(prefix + ".vxcpm", qpath, voxq.Q8 if quant == "q8" else voxq.Q4,
                            keep=("embed_tokens",))
    os.symlink(prefix + "_audiovae.vxcpm", os.path.join(qdir, "rand_audiovae.vxcpm"))
    try:
        assert st["quantized"] > 0 and st["bytes_out"] < st["bytes_in"], st
        ref_run, ref_lat, _ = _run("voxq_engine_run_gpu", prefix + ".vxcpm", meta, work, "up_" + quant,
                                   VOXCPM_QUANT=quant)
        env = {k: v for k, v in os.environ.items() if k != "VOXCPM_QUANT"}
        lat = os.path.join(work, f"lat_file_{quant}.f32")
        r = subprocess.run([os.path.join(BUILD, exe), "--model", qpath, "--gpu", "--patches", str(meta["patches"]),
                            "--tokens", str(meta["tokens"]), "--token-seed", str(meta["token_seed"]),
                            "--latents", lat], env=env, capture_output=True, text=True, timeout=1200)
        assert r.returncode == 0, r.stderr[-3000:]
        run = json.loads(r.stdout.strip().splitlines()[-1])
        got = np.fromfile(lat, dtype=np.float32)
    finally:
        shutil.rmtree(qdir, ignore_errors=True)
    assert run["blocks"]["device"] > 0 and run["blocks"]["host"] == 0, run["blocks"]
    print(f"{quant}: file {st['bytes_in'] / 1e9:.2f} GB -> {st['bytes_out'] / 1e9:.2f} GB, "
          f"{st['quantized']} of {st['tensors']} tensors quantized; upload {run['upload_s']:.2f} s "
          f"vs {ref_run['upload_s']:.2f} s quantizing on upload")
    assert got.shape == ref_lat.shape and np.isfinite(got).all()
    assert np.array_equal(got, ref_lat), f"max |d| {float(np.abs(got - ref_lat).max()):.3e}"
