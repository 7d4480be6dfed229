#!/usr/bin/env python3
"""Golden latents of the unchanged reference engine on its CPU path.

    python tests/golden/make_engine_golden.py [--workdir DIR] [--patches 4]

Needs the engine binaries of voxcpm2-c_b200/engine (``make -C
voxcpm2-c_b200/engine REF=<reference checkout>``).  It writes the seeded
random-init model (make_model, seed 1) into DIR (a temporary folder by
default; about 5 GB), runs ``voxq_engine_run_cpu`` -- the reference's
src/*.c built without VOXCPM_CUDA, so every projection runs through
tensor_matmul_nt's scalar loop (src/tensor.c:617-678) -- for a 64-token
input (token seed 1) and writes into this folder:

  engine_c4_q8.npz    latents [patches, 64, 4] of loc_dit_sample, and the
                      peak-normalised audio voxcpm_generate returns
  engine_c4_q8.json   the model files' CRC32C (to pin that a GPU host
                      regenerates the same bytes), the run's settings and
                      its per-stage CPU times (one host thread)

The model's projection weights are exactly representable in Q8 (see
make_model.c), so a GPU run that quantizes them on upload (VOXCPM_QUANT=q8)
multiplies by the same weights as this CPU run.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
BUILD = os.path.join(REPO, "voxcpm2-c_b200", "engine", "_build")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workdir", default=None)
    ap.add_argument("--patches", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--token-seed", type=int, default=1)
    ap.add_argument("--model-seed", type=int, default=1)
    args = ap.parse_args()
    work = args.workdir or tempfile.mkdtemp(prefix="voxq_engine_")
    os.makedirs(work, exist_ok=True)
    prefix = os.path.join(work, f"rand_s{args.model_seed}")
    gen = json.loads(subprocess.run([os.path.join(BUILD, "make_model"), prefix, "--seed", str(args.model_seed)],
                                    check=True, capture_output=True, text=True).stdout.strip().splitlines()[-1])
    lat = os.path.join(work, "cpu_latents.f32")
    aud = os.path.join(work, "cpu_audio.f32")
    r = subprocess.run([os.path.join(BUILD, "voxq_engine_run_cpu"), "--model", prefix + ".vxcpm", "--patches",
                        str(args.patches), "--tokens", str(args.tokens), "--token-seed", str(args.token_seed),
                        "--latents", lat, "--audio", aud], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stderr[-4000:])
        raise SystemExit(f"CPU engine failed ({r.returncode})")
    run = json.loads(r.stdout.strip().splitlines()[-1])
    latents = np.fromfile(lat, dtype=np.float32).reshape(args.patches, 64, 4)
    audio = np.fromfile(aud, dtype=np.float32)
    np.savez_compressed(os.path.join(HERE, "engine_c4_q8.npz"), latents=latents, audio=audio)
    meta = {"model": {k: gen[k] for k in ("model_bytes", "model_tensors", "model_data_crc32c", "audiovae_bytes",
                                          "audiovae_tensors", "audiovae_data_crc32c", "seed")},
            "patches": args.patches, "tokens": args.tokens, "token_seed": args.token_seed,
            "cfg_value": 2.0, "inference_timesteps": 10,
            "cpu_run": run, "cpu": open("/proc/cpuinfo").read().split("model name")[1].split("\n")[0].strip(" :\t")}
    with open(os.path.join(HERE, "engine_c4_q8.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print(json.dumps({"latents": list(latents.shape), "generate_s": run["generate_s"], "workdir": work}))


if __name__ == "__main__":
    main()
