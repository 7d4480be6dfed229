#!/usr/bin/env python3
"""Benchmark of the quantized-matmul hot path on B200 (one JSON line on rank 0).

Default workload = BASELINE config 2: one batch-1 decode step of a 24-layer
decoder (hidden 1024, 16/2 heads x 64, SwiGLU 4096): the Q, K, V, O, gate, up
and down GEMVs of every layer (168 GEMVs, Q4 weights, 224 MB), executed as one
grouped voxq launch.  Metric: algorithmic HBM bytes per second (quantized
weight bytes + fp32 activation and output bytes).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c1|c3]

Multi-GPU: the batch-1 path does not shard (replicas only); under torchrun
each rank runs its own replica and `value` sums the ranks' bytes over the
slowest rank's device time.  `--impl reference` times the reference's own CPU
implementation (tensor_matmul_nt from src/tensor.c, built unchanged into
oracle/_ref) on a bounded sample of the same workload, on all host threads.
"""
from __future__ import annotations

import argparse
import csv
import ctypes as C
import io
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "voxcpm2-c_b200"))

H, F, KV, LAYERS = 1024, 4096, 128, 24
# (name, N, K, input index) per layer; Q/K/V share the attention input, gate/up the FFN input
C2_LAYER = [("q", H, H, 0), ("k", KV, H, 0), ("v", KV, H, 0), ("o", H, H, 1),
            ("gate", F, H, 2), ("up", F, H, 2), ("down", H, F, 3)]
C2_INPUT_K = [H, H, H, F]


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def c2_bytes_per_step(qtype: int) -> tuple[int, int]:
    """(algorithmic bytes, weight bytes) of one C2 step."""
    per_w = 0.625 if qtype == 2 else 1.25
    wbytes = abyte = 0
    for (_, N, K, _) in C2_LAYER:
        wbytes += int(N * K * per_w)
        abyte += 4 * K + 4 * N
    return LAYERS * (wbytes + abyte), LAYERS * wbytes


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = [r for r in csv.reader(io.StringIO(self.out or "")) if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def build_c2(torch, voxq, dev, qtype, copies, seed):
    """`copies` independent weight sets (alternated so no step reuses L2)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    sets = []
    for c in range(copies):
        specs = []
        for layer in range(LAYERS):
            xs = [torch.randn(1, k, device=dev, generator=g) for k in C2_INPUT_K]
            for (name, N, K, xi) in C2_LAYER:
                w = torch.randn(N, K, device=dev, generator=g) * 0.02
                qw = voxq.QWeight.from_float(w, qtype)
                del w
                specs.append(dict(w=qw, a=xs[xi], out=torch.empty(1, N, device=dev)))
        sets.append(specs)
    torch.cuda.synchronize(dev)
    return sets


def run_ours(args, torch, dist, rank, world, local_rank):
    import voxq
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    voxq.set_device(local_rank)
    qtype = voxq.Q4
    stream = torch.cuda.Stream(dev)
    hbm, bf16, bf16s, peak_kind = peaks()
    algo_bytes, wbytes = c2_bytes_per_step(qtype)

    sets = build_c2(torch, voxq, dev, qtype, copies=2, seed=1234 + rank)
    item_arrays = [voxq.make_gemv_items(s) for s in sets]
    n_items = len(sets[0])

    def step(i):
        voxq.gemv_batch(item_arrays[i & 1], stream=stream)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize(dev)

    # soak so the clock sampler sees the device under this load, then time K steps
    def barrier():
        if dist is not None:
            dist.barrier()
    sampler = ClockSampler(local_rank)
    with sampler:
        t_end = time.time() + args.soak
        i = 0
        while time.time() < t_end:
            for _ in range(200):
                step(i)
                i += 1
            torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
    ms = e0.elapsed_time(e1)
    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = world * algo_bytes / (ms_per_step * 1e-3) / 1e9
    achieved = algo_bytes / (ms / args.steps * 1e-3) / 1e9  # this rank's kernel, one launch per step

    # ---- end to end through the public C ABI with host buffers ----
    e2e = run_e2e(torch, voxq, dev, stream, sets[0], args, algo_bytes)
    e2e_abi = run_e2e_tensor_abi(torch, voxq, dev, args, algo_bytes, rank) if args.tensor_abi else None

    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        cpu = cpu_baseline(args.cpu_seconds, threads=1)

    # the single-row launch runs the tensor-path GEMV unless VOXQ_GEMV_MMA=0
    mma = os.environ.get("VOXQ_GEMV_MMA", "1")[:1] != "0"
    kernel = "voxq::gemv_mma_kernel<Q4,false,192>" if mma else "voxq::gemv_kernel<Q4,1,4,false,false,192>"
    traffic = None
    tp = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tp):
        t = json.load(open(tp)).get("gemv_mma_c2_q4" if mma else "gemv_c2_q4")
        if t:  # dram__bytes_read.sum + dram__bytes_write.sum of one launch (ncu)
            traffic = t["dram_read_bytes"] + t["dram_write_bytes"]

    if rank == 0:
        line = {
            "metric": "c2_q4_decode_gemv_hbm_GBps",
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q4 weights, fp32 activations/accumulate",
            "data": "synthetic: weights 0.02*N(0,1) quantized on device to Q4, activations N(0,1)",
            "config": {
                "workload": "BASELINE config 2: 24-layer batch-1 decode step, Q/K/V/O/gate/up/down GEMVs, Q4, one grouped launch",
                "gemvs_per_step": n_items, "hidden": H, "ffn": F, "kv_dim": KV, "layers": LAYERS,
                "weight_bytes_per_step": wbytes, "algorithmic_bytes_per_step": algo_bytes,
                "l2": "inputs larger than L2: two 224 MB weight sets alternated between steps",
                "parallelism": f"replicas x{world} (batch-1 GEMV does not shard)",
            },
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                         "traffic": traffic, "kernel": kernel},
            "e2e": e2e,
            # per step: the tensor-path GEMV splits its activations itself (one launch);
            # the dp4a kernel needs the limb prepass before it (two)
            "gpu_launches": (1 if mma else 2) * args.steps,
            "clocks": sampler.summary(),
        }
        if e2e_abi is not None:
            line["e2e_tensor_abi"] = e2e_abi
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


def run_e2e(torch, voxq, dev, stream, specs, args, algo_bytes):
    """Same step through voxq_gemv_batch with host buffers: H2D of every
    input vector from pinned memory, the launch, D2H of every output."""
    in_sizes = []
    seen = {}
    for s in specs:
        if id(s["a"]) not in seen:
            seen[id(s["a"])] = s["a"]
            in_sizes.append(s["a"].numel())
    n_in = sum(in_sizes)
    n_out = sum(s["out"].numel() for s in specs)
    h_in = torch.randn(n_in).pin_memory()
    h_out = torch.empty(n_out).pin_memory()
    d_in = torch.empty(n_in, device=dev)
    d_out = torch.empty(n_out, device=dev)
    # re-point the items at the packed device staging buffers
    off = 0
    views = {}
    for k, t in seen.items():
        views[k] = d_in[off:off + t.numel()].view_as(t)
        off += t.numel()
    off = 0
    e_specs = []
    for s in specs:
        o = d_out[off:off + s["out"].numel()].view_as(s["out"])
        off += s["out"].numel()
        e_specs.append(dict(w=s["w"], a=views[id(s["a"])], out=o))
    items = voxq.make_gemv_items(e_specs)

    def step():
        d_in.copy_(h_in, non_blocking=True)
        voxq.gemv_batch(items, stream=stream)
        h_out.copy_(d_out, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        k = max(args.steps, 1)
        e0.record(stream)
        for _ in range(k):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / k
    return {"value": round(algo_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 5),
            "h2d_bytes_per_step": 4 * n_in, "d2h_bytes_per_step": 4 * n_out,
            "path": "voxq_gemv_batch, pinned host inputs/outputs, copies inside the timed region"}


def run_e2e_tensor_abi(torch, voxq, dev, args, algo_bytes, rank):
    """The unchanged-engine path: 168 tensor_matmul_nt_cuda calls per step with
    host activations and host outputs (weights uploaded by tensor_to_cuda in
    VOXCPM_QUANT=q4 mode), wall-clock per step (each call is synchronous)."""
    L = voxq.lib()
    os.environ["VOXCPM_QUANT"] = "q4"
    L.tensor_cuda_shutdown()
    if L.tensor_cuda_init() != 0:
        return {"unavailable": "tensor_cuda_init failed"}
    g = torch.Generator().manual_seed(99 + rank)
    ws, ins, outs = [], [], []
    try:
        for layer in range(LAYERS):
            for (_, N, K, _) in C2_LAYER:
                w = voxq.host_tensor((torch.randn(N, K, generator=g) * 0.02).numpy())
                voxq.check(L.tensor_to_cuda(w), "tensor_to_cuda")
                ws.append(w)
                ins.append(voxq.host_tensor(torch.randn(1, K, generator=g).numpy()))
                outs.append(voxq.host_tensor(np.zeros((1, N), np.float32)))

        def step():
            for w, a, o in zip(ws, ins, outs):
                rc = L.tensor_matmul_nt_cuda(a, w, o)
                if rc:
                    raise RuntimeError(rc)
        for _ in range(args.warmup):
            step()
        k = max(3, min(args.steps, 50))
        t0 = time.perf_counter()
        for _ in range(k):
            step()
        ms = (time.perf_counter() - t0) * 1e3 / k
    finally:
        for t in ws + ins + outs:
            voxq.free_tensor(t)
        L.tensor_cuda_shutdown()
    h2d = sum(4 * C2_LAYER[i % 7][2] for i in range(len(ws)))
    d2h = sum(4 * C2_LAYER[i % 7][1] for i in range(len(ws)))
    return {"value": round(algo_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "168 x tensor_matmul_nt_cuda (reference ABI), host a/out, synchronous per call (wall clock)"}


# ---------------------------------------------------------------------------
# CPU: the reference's tensor_matmul_nt (src/tensor.c:617-678), unchanged
# ---------------------------------------------------------------------------

def _cpu_sample(n_layers: int, seed: int):
    sys.path.insert(0, REPO)
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    jobs = []
    for layer in range(n_layers):
        xs = [rng.standard_normal((1, k), dtype=np.float32) for k in C2_INPUT_K]
        for (_, N, K, xi) in C2_LAYER:
            w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
            wd = O.dequantize(O.quantize(w, 2), N * K, 2).reshape(N, K)  # Q4 weight, dequantized to fp32
            jobs.append((xs[xi], wd, np.zeros((1, N), np.float32)))
    return O, jobs


def _ref_kind():
    sys.path.insert(0, REPO)
    from oracle import oracle as O
    return ("reference", O.ref_matmul_nt) if O.ref_available() else ("port", O.matmul_nt)


def cpu_baseline(seconds: float, threads: int = 1):
    """Reference tensor_matmul_nt over one layer's 7 GEMVs, repeated ~`seconds`."""
    O, jobs = _cpu_sample(1, 7)
    kind, fn = _ref_kind()
    algo_layer = c2_bytes_per_step(2)[0] // LAYERS
    n = 0
    t0 = time.perf_counter()
    while True:
        for (a, w, o) in jobs:
            fn(a, w, o)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(n * algo_layer / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{n} x one C2 layer (7 GEMVs, Q4 weights dequantized to fp32), {dt:.1f} s, single thread"}


def run_reference(args, rank, world):
    """Reference arm: the reference's CPU tensor_matmul_nt on every host thread."""
    if rank != 0:
        return
    kind, fn = _ref_kind()
    nthreads = os.cpu_count() or 1
    O, jobs = _cpu_sample(1, 11)
    algo_layer = c2_bytes_per_step(2)[0] // LAYERS
    # one step = each thread runs one full layer (7 GEMVs) on its own buffers
    per_thread = [[(a, w, np.zeros_like(o)) for (a, w, o) in jobs] for _ in range(nthreads)]

    def one_step():
        ths = [threading.Thread(target=lambda js=js: [fn(a, w, o) for (a, w, o) in js]) for js in per_thread]
        for t in ths:
            t.start()
        for t in ths:
            t.join()

    for _ in range(args.warmup):
        one_step()
    k = args.steps
    t0 = time.perf_counter()
    for _ in range(k):
        one_step()
    dt = (time.perf_counter() - t0) / k
    value = nthreads * algo_layer / dt / 1e9
    line = {
        "impl": "reference", "metric": "c2_q4_decode_gemv_hbm_GBps", "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": k, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 (Q4 weights dequantized to fp32)", "data": "synthetic",
        "config": {"workload": "BASELINE config 2 sample: one decoder layer's 7 GEMVs per host thread per step",
                   "parallelism": f"{nthreads} host threads"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": nthreads, "kind": kind,
                         "sample": f"{nthreads} threads x one C2 layer (7 GEMVs) per step"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_c1(args, torch):
    """one Q8 GEMV, W [4096, 1024] = 0.02 N(0,1) quantized on device, x [1, 1024]
    N(0,1), y [1, 4096].  The weight fits in L2, so 64 weight copies (> 335 MB) are rotated and the
    calls are replayed from a CUDA graph (device time per call; host launch cost excluded)."""
    import voxq
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm, bf16, bf16s, peak_kind = peaks()
    st = torch.cuda.Stream(dev)
    N, K, copies = 4096, 1024, 64
    g = torch.Generator(device=dev).manual_seed(1)
    ws = [voxq.QWeight.from_float(torch.randn(N, K, device=dev, generator=g) * 0.02, voxq.Q8) for _ in range(copies)]
    x = torch.randn(1, K, device=dev, generator=g)
    y = torch.empty(1, N, device=dev)
    with torch.cuda.stream(st):
        for i in range(max(args.warmup, 3)):
            voxq.matmul_nt_q(x, ws[i % copies], out=y, stream=st)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for i in range(copies):
            voxq.matmul_nt_q(x, ws[i], out=y, stream=st)
    loops = max(1, args.steps // copies)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        graph.replay()
        e0.record(st)
        for _ in range(loops):
            graph.replay()
        e1.record(st)
    torch.cuda.synchronize(dev)
    calls = loops * copies
    ms = e0.elapsed_time(e1) / calls
    byts = N * K * 5 // 4 + 4 * K + 4 * N  # 5,263,360 B
    gbs = byts / (ms * 1e-3) / 1e9
    print(json.dumps({"metric": "c1_q8_gemv_hbm_GBps", "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1,
                      "steps": calls, "warmup": max(args.warmup, 3), "us_per_call": round(ms * 1e3, 3),
                      "higher_is_better": True, "dtype": "q8 weights, fp32 activations/accumulate",
                      "data": "synthetic: 0.02*N(0,1) weights quantized on device to Q8, N(0,1) activation",
                      "config": {"workload": "BASELINE config 1: Q8 GEMV N=4096 K=1024",
                                 "algorithmic_bytes_per_call": byts, "weight_copies": copies,
                                 "l2": "64 rotated weight copies (335 MB > L2)"},
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                   "frac": round(gbs / hbm, 4), "peak_kind": peak_kind},
                      "gpu_launches": (1 if os.environ.get("VOXQ_GEMV_MMA", "1")[:1] != "0" else 2) * calls,
                      "device_error": voxq.lib().voxq_device_error(1)}), flush=True)


def run_c3(args, torch):
    """BASELINE config 3 sweep (one JSON line per shape): K = 1024, N in {1024, 4096},
    M in {16, 64, 256, 2048}, Q8 and Q4, one voxq_matmul_nt_q call per step.

    `us` is device time per call: the calls (prepass, GEMM and any split-K reduction
    kernel each) are captured in a CUDA graph and replayed, so host launch cost is
    excluded; `us_eager` is the same loop launched from Python call by call.  Weight
    copies are rotated so the weights of consecutive calls never share L2 (> 126 MB
    in total)."""
    import voxq
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm, bf16, bf16s, peak_kind = peaks()
    st = torch.cuda.Stream(dev)
    K = 1024
    g = torch.Generator(device=dev).manual_seed(3)
    only = None
    if args.shape:  # "M,N,q8|q4": one shape (profiling)
        m_, n_, q_ = args.shape.split(",")
        only = (int(m_), int(n_), voxq.Q8 if q_.lower() == "q8" else voxq.Q4)
    for qt in (voxq.Q8, voxq.Q4):
        for N in (1024, 4096):
            if only and (qt != only[2] or N != only[1]):
                continue
            wbytes = int(N * K * (1.25 if qt == voxq.Q8 else 0.625))
            # rotate > 300 MB of weights (no L2 reuse); a single profiled shape uses 4 copies
            copies = 4 if only else max(2, int(300e6 // wbytes) + 1)
            ws = [voxq.QWeight.from_float(torch.randn(N, K, device=dev, generator=g) * 0.02, qt)
                  for _ in range(copies)]
            for M in (16, 64, 256, 2048):
                if only and M != only[0]:
                    continue
                a = torch.randn(M, K, device=dev, generator=g)
                out = torch.empty(M, N, device=dev)
                reps = max(copies, 64)
                with torch.cuda.stream(st):
                    for i in range(max(args.warmup, 3)):
                        voxq.matmul_nt_q(a, ws[i % copies], out=out, stream=st)
                torch.cuda.synchronize(dev)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=st):
                    for i in range(reps):
                        voxq.matmul_nt_q(a, ws[i % copies], out=out, stream=st)
                with torch.cuda.stream(st):
                    graph.replay()
                torch.cuda.synchronize(dev)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                loops = max(1, args.steps // reps)
                with torch.cuda.stream(st):  # replay() launches on the current stream
                    e0.record(st)
                    for _ in range(loops):
                        graph.replay()
                    e1.record(st)
                torch.cuda.synchronize(dev)
                ms = e0.elapsed_time(e1) / (loops * reps)
                del graph
                with torch.cuda.stream(st):
                    e0.record(st)
                    for i in range(reps):
                        voxq.matmul_nt_q(a, ws[i % copies], out=out, stream=st)
                    e1.record(st)
                torch.cuda.synchronize(dev)
                ms_eager = e0.elapsed_time(e1) / reps
                err = voxq.lib().voxq_device_error(1)
                flops = 2.0 * M * N * K
                byts = wbytes + 4 * M * K + 4 * M * N
                tf = flops / (ms * 1e-3) / 1e12
                gbs = byts / (ms * 1e-3) / 1e9
                ai = flops / byts
                bound = "tensor" if ai > bf16 * 1e12 / (hbm * 1e9) else "hbm"
                frac = tf / bf16 if bound == "tensor" else gbs / hbm
                print(json.dumps({"config": "c3", "qtype": "q8" if qt == voxq.Q8 else "q4", "M": M, "N": N, "K": K,
                                  "us": round(ms * 1e3, 2), "us_eager": round(ms_eager * 1e3, 2),
                                  "TFLOPs": round(tf, 1), "GBps": round(gbs, 1), "bound": bound,
                                  "frac": round(frac, 4), "peak_kind": peak_kind,
                                  "path": "gemv" if M <= 8 else "tcgen05 gemm", "weight_copies": copies,
                                  "device_error": err}), flush=True)
            del ws


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--soak", type=float, default=1.0, help="seconds of untimed load before timing (clock sampling)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-tensor-abi", dest="tensor_abi", action="store_false")
    ap.add_argument("--shape", default="", help="c3 only: one shape 'M,N,q8|q4'")
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3"],
                    help="c2: the headline decode step (default); c1: one Q8 GEMV; c3: GEMM sweep, one line per shape")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.config in ("c1", "c3"):
        import torch
        (run_c1 if args.config == "c1" else run_c3)(args, torch)
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist_mod
        torch.cuda.set_device(local_rank)
        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local_rank))
        dist = dist_mod
    try:
        run_ours(args, torch, dist, rank, world, local_rank)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
