#!/usr/bin/env python3
"""Benchmark of the quantized-matmul hot path on B200 (one JSON line on rank 0).

Default workload = BASELINE config 2: one batch-1 decode step of a 24-layer
decoder (hidden 1024, 16/2 heads x 64, SwiGLU 4096): the Q, K, V, O, gate, up
and down GEMVs of every layer (168 GEMVs, Q4 weights, 224 MB), executed as one
grouped voxq launch.  Metric: algorithmic HBM bytes per second (quantized
weight bytes + fp32 activation and output bytes).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c1|c3]

The default line also carries, under "configs", the other BASELINE configs
measured in the same run on GPU 0: config 1 (one Q8 GEMV), the config-3 GEMM
sweep (16 shapes), the config-2 step as a dependent chain (each layer's
inputs are the previous outputs: QKV -> O -> gate/up -> down, 120 launches
replayed from a CUDA graph), per-call costs through the reference ABI
(tensor_matmul_nt_cuda with host buffers), and the reference's own GPU path
(src/tensor_cuda.cu + src/tensor.c built unchanged for sm_100: cuBLAS FP32
SGEMM on dequantized weights) on the same workloads.

Multi-GPU: the batch-1 path does not shard (replicas only); under torchrun
each rank runs its own replica and `value` sums the ranks' bytes over the
slowest rank's device time.  Each rank also runs its column shard of a
config-3 GEMM (weight rows split across ranks, no collective on the data
path) and the line reports per-rank device times.  `--impl reference` times
the reference's own CPU implementation (tensor_matmul_nt from src/tensor.c,
built unchanged into oracle/_ref) on a bounded sample of the same workload,
on all host threads.
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
    per_rank_ms = [ms]
    if dist is not None:
        t = torch.zeros(world, device=dev)
        t[rank] = ms
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        per_rank_ms = [float(v) for v in t.tolist()]
    ms_max = max(per_rank_ms)
    ms_per_step = ms_max / args.steps
    value = world * algo_bytes / (ms_per_step * 1e-3) / 1e9
    achieved = algo_bytes / (ms / args.steps * 1e-3) / 1e9  # this rank's kernel, one launch per step

    # ---- end to end through the public C ABI with host buffers (every rank; summed) ----
    e2e = run_e2e(torch, voxq, dev, stream, sets[0], args, algo_bytes)
    if dist is not None:
        t = torch.zeros(world, device=dev)
        t[rank] = e2e["ms_per_step"]
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        e2e_ms = [float(v) for v in t.tolist()]
        e2e["per_rank_ms_per_step"] = [round(v, 5) for v in e2e_ms]
        e2e["ms_per_step"] = round(max(e2e_ms), 5)
        e2e["value"] = round(world * algo_bytes / (max(e2e_ms) * 1e-3) / 1e9, 1)
        e2e["aggregate"] = "all ranks' bytes over the slowest rank's time"
    e2e_abi = run_e2e_tensor_abi(torch, voxq, dev, args, algo_bytes, rank) if (args.tensor_abi and rank == 0) else None

    configs = {}
    if world > 1:
        configs["c3_sharded"] = measure_sharded_c3(torch, voxq, dist, dev, stream, rank, world, args.steps,
                                                    args.warmup)
    cpu = None
    if rank == 0 and world == 1:
        if args.configs:
            configs["c1"] = measure_c1(torch, voxq, dev, stream, args.steps, args.warmup)
            configs["c2_chain"] = measure_c2_chain(torch, voxq, dev, stream, qtype, max(20, args.steps // 20),
                                                   args.warmup)
            configs["c3"] = measure_c3(torch, voxq, dev, stream, args.steps, args.warmup, eager=False)
            if args.tensor_abi:
                shapes = [(M, N, 1024) for N in C3_N for M in C3_M]
                configs["tensor_abi_per_call"] = {
                    "what": "wall-clock us per tensor_matmul_nt_cuda call, host a/out, quantized device weights",
                    "q4_c2_shapes": measure_abi_calls(torch, voxq, "q4", [(1, N, K) for (_, N, K, _) in C2_LAYER[:5]]
                                                      + [(1, H, F)], 200, breakdown=True),
                    "q8_c3": measure_abi_calls(torch, voxq, "q8", shapes, 40),
                }
            configs["reference_gpu"] = measure_ref_gpu(args)
        if args.cpu_seconds > 0:
            cpu = cpu_baseline(args.cpu_seconds, threads=1)
    if args.configs:
        configs.update(engine_configs(args, dist, rank, world, local_rank))

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
                "workload": "BASELINE config 2: 24-layer batch-1 decode step, Q/K/V/O/gate/up/down GEMVs, Q4, "
                            "independent inputs, one grouped launch (the dependent chain is configs.c2_chain)",
                "gemvs_per_step": n_items, "hidden": H, "ffn": F, "kv_dim": KV, "layers": LAYERS,
                "weight_bytes_per_step": wbytes, "algorithmic_bytes_per_step": algo_bytes,
                "l2": "inputs larger than L2: two 224 MB weight sets alternated between steps",
                "parallelism": f"replicas x{world} (batch-1 GEMV does not shard)",
            },
            "per_rank_ms": [round(v, 4) for v in per_rank_ms],
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                         "traffic": traffic,
                         "traffic_source": "profiles/traffic.json: dram__bytes_read.sum + dram__bytes_write.sum "
                                           "of one launch of this kernel on this workload from an ncu capture "
                                           "(copied, not measured in this run)" if traffic else None,
                         "kernel": kernel},
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
        if configs:
            line["configs"] = configs
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


def measure_c1(torch, voxq, dev, st, steps, warmup):
    """one Q8 GEMV, W [4096, 1024] = 0.02 N(0,1) quantized on device, x [1, 1024]
    N(0,1), y [1, 4096].  The weight fits in L2, so 64 weight copies (> 335 MB) are rotated and the
    calls are replayed from a CUDA graph (device time per call; host launch cost excluded)."""
    hbm, bf16, bf16s, peak_kind = peaks()
    N, K, copies = 4096, 1024, 64
    g = torch.Generator(device=dev).manual_seed(1)
    ws = [voxq.QWeight.from_float(torch.randn(N, K, device=dev, generator=g) * 0.02, voxq.Q8) for _ in range(copies)]
    x = torch.randn(1, K, device=dev, generator=g)
    y = torch.empty(1, N, device=dev)
    with torch.cuda.stream(st):
        for i in range(max(warmup, 3)):
            voxq.matmul_nt_q(x, ws[i % copies], out=y, stream=st)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for i in range(copies):
            voxq.matmul_nt_q(x, ws[i], out=y, stream=st)
    loops = max(2, steps // copies)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        graph.replay()
        e0.record(st)
        for _ in range(loops):
            graph.replay()
        e1.record(st)
    torch.cuda.synchronize(dev)
    del graph
    calls = loops * copies
    ms = e0.elapsed_time(e1) / calls
    byts = N * K * 5 // 4 + 4 * K + 4 * N  # 5,263,360 B
    gbs = byts / (ms * 1e-3) / 1e9
    mma = os.environ.get("VOXQ_GEMV_MMA", "1")[:1] != "0"
    return {"metric": "c1_q8_gemv_hbm_GBps", "value": round(gbs, 1), "unit": "GB/s", "us_per_call": round(ms * 1e3, 3),
            "calls": calls, "workload": "BASELINE config 1: Q8 GEMV N=4096 K=1024, CUDA-graph replay",
            "algorithmic_bytes_per_call": byts, "l2": "64 rotated weight copies (335 MB > L2)",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4), "peak_kind": peak_kind},
            "gpu_launches": (1 if mma else 2) * calls, "device_error": voxq.lib().voxq_device_error(1)}


def run_c1(args, torch):
    import voxq
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    print(json.dumps(measure_c1(torch, voxq, dev, torch.cuda.Stream(dev), args.steps, args.warmup)), flush=True)


def run_chain(args, torch):
    """The dependent C2 decode step alone (configs.c2_chain of the default line)."""
    import voxq
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    r = measure_c2_chain(torch, voxq, dev, torch.cuda.Stream(dev), voxq.Q4, max(20, args.steps // 20),
                         args.warmup)
    print(json.dumps(r), flush=True)


C3_M = (16, 64, 256, 2048)
C3_N = (1024, 4096)


def c3_roof(M, N, K, qt_q8, ms):
    hbm, bf16, bf16s, peak_kind = peaks()
    wbytes = int(N * K * (1.25 if qt_q8 else 0.625))
    flops = 2.0 * M * N * K
    byts = wbytes + 4 * M * K + 4 * M * N
    tf = flops / (ms * 1e-3) / 1e12
    gbs = byts / (ms * 1e-3) / 1e9
    bound = "tensor" if flops / byts > bf16 * 1e12 / (hbm * 1e9) else "hbm"
    frac = tf / bf16 if bound == "tensor" else gbs / hbm
    return {"TFLOPs": round(tf, 1), "GBps": round(gbs, 1), "bound": bound, "frac": round(frac, 4),
            "peak_kind": peak_kind, "algorithmic_bytes": byts}


def measure_c3(torch, voxq, dev, st, steps, warmup, only=None, eager=True):
    """BASELINE config 3 sweep: K = 1024, N in {1024, 4096}, M in {16, 64, 256, 2048}, Q8 and Q4,
    one voxq_matmul_nt_q call per step.

    `us` is device time per call: the calls (prepass, GEMM and any split-K reduction
    kernel each) are captured in a CUDA graph and replayed, so host launch cost is
    excluded; `us_eager` is the same loop launched from Python call by call.  Weight
    copies are rotated so the weights of consecutive calls never share L2 (> 300 MB
    in total).  Returns one dict per shape."""
    K = 1024
    g = torch.Generator(device=dev).manual_seed(3)
    rows = []
    for qt in (voxq.Q8, voxq.Q4):
        for N in C3_N:
            if only and (qt != only[2] or N != only[1]):
                continue
            wbytes = int(N * K * (1.25 if qt == voxq.Q8 else 0.625))
            # rotate > 300 MB of weights (no L2 reuse); a single profiled shape uses 4 copies
            copies = 4 if only else max(2, int(300e6 // wbytes) + 1)
            ws = [voxq.QWeight.from_float(torch.randn(N, K, device=dev, generator=g) * 0.02, qt)
                  for _ in range(copies)]
            for M in C3_M:
                if only and M != only[0]:
                    continue
                a = torch.randn(M, K, device=dev, generator=g)
                out = torch.empty(M, N, device=dev)
                reps = max(copies, 64)
                with torch.cuda.stream(st):
                    for i in range(max(warmup, 3)):
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
                loops = max(2, steps // reps)
                with torch.cuda.stream(st):  # replay() launches on the current stream
                    e0.record(st)
                    for _ in range(loops):
                        graph.replay()
                    e1.record(st)
                torch.cuda.synchronize(dev)
                ms = e0.elapsed_time(e1) / (loops * reps)
                del graph
                row = {"qtype": "q8" if qt == voxq.Q8 else "q4", "M": M, "N": N, "K": K, "us": round(ms * 1e3, 2)}
                if eager:
                    with torch.cuda.stream(st):
                        e0.record(st)
                        for i in range(reps):
                            voxq.matmul_nt_q(a, ws[i % copies], out=out, stream=st)
                        e1.record(st)
                    torch.cuda.synchronize(dev)
                    row["us_eager"] = round(e0.elapsed_time(e1) / reps * 1e3, 2)
                row.update(c3_roof(M, N, K, qt == voxq.Q8, ms))
                row.update({"path": "gemv" if M <= 8 else "tcgen05 gemm", "weight_copies": copies,
                            "device_error": voxq.lib().voxq_device_error(1)})
                rows.append(row)
            del ws
    return rows


def run_c3(args, torch):
    import voxq
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    only = None
    if args.shape:  # "M,N,q8|q4": one shape (profiling)
        m_, n_, q_ = args.shape.split(",")
        only = (int(m_), int(n_), voxq.Q8 if q_.lower() == "q8" else voxq.Q4)
    for row in measure_c3(torch, voxq, dev, torch.cuda.Stream(dev), args.steps, args.warmup, only):
        row["config"] = "c3"
        print(json.dumps(row), flush=True)


def measure_c2_chain(torch, voxq, dev, st, qtype, steps, warmup, seed=77):
    """Config 2 as a dependent decode step: per layer, Q/K/V from the layer input
    (one grouped launch), O from Q (+ the layer input as residual), gate/up from
    O with the fused SwiGLU epilogue, down from that (+ O as residual); the down
    output is the next layer's input.  Attention and the norms are not on the
    matmul path and are left out, so O reads Q directly.  Each step is captured
    once in a CUDA graph (one per weight set; two sets alternate so every step
    streams its 224 MB of weights from HBM) and replayed."""
    g = torch.Generator(device=dev).manual_seed(seed)
    graphs, launches = [], 0
    keep = []
    mma = os.environ.get("VOXQ_GEMV_MMA", "1")[:1] != "0"
    for copy in range(2):
        W = []
        for layer in range(LAYERS):
            W.append({name: voxq.QWeight.from_float(torch.randn(N, K, device=dev, generator=g) * 0.02, qtype)
                      for (name, N, K, _) in C2_LAYER})
        xs = [torch.randn(1, H, device=dev, generator=g)] + [torch.empty(1, H, device=dev) for _ in range(LAYERS)]
        qs = [torch.empty(1, H, device=dev) for _ in range(LAYERS)]
        kvs = [torch.empty(1, KV, device=dev) for _ in range(2 * LAYERS)]
        os_ = [torch.empty(1, H, device=dev) for _ in range(LAYERS)]
        hs = [torch.empty(1, F, device=dev) for _ in range(LAYERS)]
        qkv = [voxq.make_gemv_items([dict(w=W[l]["q"], a=xs[l], out=qs[l]), dict(w=W[l]["k"], a=xs[l], out=kvs[2 * l]),
                                     dict(w=W[l]["v"], a=xs[l], out=kvs[2 * l + 1])]) for l in range(LAYERS)]

        def step(W=W, xs=xs, qs=qs, os_=os_, hs=hs, qkv=qkv):
            for l in range(LAYERS):
                voxq.gemv_batch(qkv[l], stream=st)
                voxq.matmul_nt_q(qs[l], W[l]["o"], out=os_[l], residual=xs[l], stream=st)
                voxq.matmul_nt_q(os_[l], W[l]["gate"], out=hs[l], up=W[l]["up"], stream=st)
                voxq.matmul_nt_q(hs[l], W[l]["down"], out=xs[l + 1], residual=os_[l], stream=st)
        with torch.cuda.stream(st):
            for _ in range(max(warmup, 3)):
                step()
        torch.cuda.synchronize(dev)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            step()
        graphs.append(gr)
        keep.append((W, xs, qs, kvs, os_, hs, qkv, step))
    # QKV, O, down: one launch each on the tensor-path GEMV; gate/up with SwiGLU: limb prepass + GEMV
    launches = LAYERS * ((3 if mma else 6) + 2)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        for i in range(4):
            graphs[i & 1].replay()
        torch.cuda.synchronize(dev)
        e0.record(st)
        for i in range(steps):
            graphs[i & 1].replay()
        e1.record(st)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    # the same chain launched call by call from Python (host launch cost included)
    k_eager = max(3, min(steps, 50))
    with torch.cuda.stream(st):
        e0.record(st)
        for i in range(k_eager):
            keep[i & 1][-1]()
        e1.record(st)
    torch.cuda.synchronize(dev)
    ms_eager = e0.elapsed_time(e1) / k_eager
    del graphs
    hbm, _, _, peak_kind = peaks()
    algo_bytes, _ = c2_bytes_per_step(qtype)
    gbs = algo_bytes / (ms * 1e-3) / 1e9
    return {"metric": "c2_q4_decode_chain_hbm_GBps", "value": round(gbs, 1), "unit": "GB/s",
            "ms_per_step": round(ms, 5), "ms_per_step_eager": round(ms_eager, 4),
            "value_eager": round(algo_bytes / (ms_eager * 1e-3) / 1e9, 1),
            "workload": "BASELINE config 2, dependent: 24 layers x (QKV grouped -> O(+res) -> gate/up SwiGLU -> "
                        "down(+res)), each input the previous output; CUDA-graph replay (value) and Python "
                        "launches (value_eager)",
            "launches_per_step": launches, "algorithmic_bytes_per_step": algo_bytes,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4), "peak_kind": peak_kind},
            "device_error": voxq.lib().voxq_device_error(1)}


def _device_tensor(voxq, t):
    """A reference Tensor that borrows a CUDA torch tensor (is_cuda, not owned)."""
    T = voxq.Tensor()
    shp = (C.c_int * t.dim())(*t.shape)
    T.data = C.cast(C.c_void_p(t.data_ptr()), C.POINTER(C.c_float))
    T.shape = C.cast(shp, C.POINTER(C.c_int))
    T.ndim = t.dim()
    T.size = t.numel()
    T.is_cuda = True
    return T, shp


def measure_abi_calls(torch, voxq, qname, shapes, reps, breakdown=False):
    """Per-call cost of tensor_matmul_nt_cuda (the reference ABI the unchanged
    engine calls) with host activations and outputs, weights uploaded and
    quantized by tensor_to_cuda under VOXCPM_QUANT=qname.  Wall clock per call.
    With `breakdown`, the same call also with a device activation (no staging
    or host->device copy), with a device output (no output path or wait), and
    with both on the device (launch only; one device synchronisation per loop)."""
    L = voxq.lib()
    os.environ["VOXCPM_QUANT"] = qname
    L.tensor_cuda_shutdown()
    if L.tensor_cuda_init() != 0:
        return [{"unavailable": "tensor_cuda_init failed"}]
    g = torch.Generator().manual_seed(5)
    rows = []

    def timed(a, w, o, k, sync=False):
        for _ in range(3):
            voxq.check(L.tensor_matmul_nt_cuda(a, w, o), "tensor_matmul_nt_cuda")
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(k):
            L.tensor_matmul_nt_cuda(a, w, o)
        if sync:
            torch.cuda.synchronize()
        return round((time.perf_counter() - t0) * 1e6 / k, 2)
    try:
        for (M, N, K) in shapes:
            w = voxq.host_tensor((torch.randn(N, K, generator=g) * 0.02).numpy())
            a_np = torch.randn(M, K, generator=g).numpy()
            a = voxq.host_tensor(a_np)
            o = voxq.host_tensor(np.zeros((M, N), np.float32))
            try:
                voxq.check(L.tensor_to_cuda(w), "tensor_to_cuda")
                k = max(3, reps if M <= 256 else reps // 4)
                row = {"M": M, "N": N, "K": K, "us": timed(a, w, o, k)}
                if breakdown:
                    ad = torch.from_numpy(a_np).cuda()
                    od = torch.empty(M, N, device="cuda")
                    (ta, s1), (to, s2) = _device_tensor(voxq, ad), _device_tensor(voxq, od)
                    row["us_device_a"] = timed(C.byref(ta), w, o, k)
                    row["us_device_out"] = timed(a, w, C.byref(to), k, sync=True)
                    row["us_device_both"] = timed(C.byref(ta), w, C.byref(to), k, sync=True)
                rows.append(row)
            finally:
                for t in (w, a, o):
                    voxq.free_tensor(t)
    finally:
        L.tensor_cuda_shutdown()
        os.environ.pop("VOXCPM_QUANT", None)
    return rows


REF_GPU_LIB = os.path.join(REPO, "oracle", "_ref", "libref_tensor_cuda.so")


def ref_gpu_worker(args):
    """Runs in its own process (the reference library exports the same tensor_*
    symbols as libvoxq): the reference's GPU path, src/tensor_cuda.cu + src/tensor.c
    built unchanged for sm_100.  tensor_matmul_nt -> tensor_matmul_nt_cuda ->
    cuBLAS FP32 SGEMM on device fp32 weights (the reference has no quantized GPU
    path; Q4/Q8 files are dequantized to fp32 at load), per-call cudaMalloc,
    copies and cudaDeviceSynchronize.  Prints one JSON object."""
    sys.path.insert(0, REPO)
    from oracle import oracle as O
    L = C.CDLL(REF_GPU_LIB)
    TP = C.POINTER(O.RefTensor)
    L.tensor_create.argtypes = [C.c_int, C.POINTER(C.c_int)]
    L.tensor_create.restype = TP
    L.tensor_free.argtypes = [TP]
    for f in ("tensor_to_cuda", "tensor_matmul_nt"):
        getattr(L, f).restype = C.c_int
    L.tensor_to_cuda.argtypes = [TP]
    L.tensor_matmul_nt.argtypes = [TP, TP, TP]
    L.tensor_cuda_init.restype = C.c_int
    if L.tensor_cuda_init() != 0:
        print(json.dumps({"unavailable": "reference tensor_cuda_init failed"}))
        return
    rng = np.random.default_rng(17)

    def make(shape, scale=1.0):
        t = L.tensor_create(len(shape), (C.c_int * len(shape))(*shape))
        n = int(np.prod(shape))
        buf = (C.c_float * n).from_address(C.cast(t.contents.data, C.c_void_p).value)
        np.frombuffer(buf, dtype=np.float32)[:] = rng.standard_normal(n, dtype=np.float32) * np.float32(scale)
        return t

    out = {}
    # config 2: 168 synchronous calls per step, host activations and outputs
    ws, ins, outs = [], [], []
    for layer in range(LAYERS):
        for (_, N, K, _) in C2_LAYER:
            w = make((N, K), 0.02)
            if L.tensor_to_cuda(w) != 0:
                print(json.dumps({"unavailable": "reference tensor_to_cuda failed"}))
                return
            ws.append(w)
            ins.append(make((1, K)))
            outs.append(make((1, N)))

    def c2_step():
        for w, a, o in zip(ws, ins, outs):
            if L.tensor_matmul_nt(a, w, o) != 0:
                raise RuntimeError("reference tensor_matmul_nt failed")
    for _ in range(3):
        c2_step()
    k = max(3, min(args.steps, 20))
    t0 = time.perf_counter()
    for _ in range(k):
        c2_step()
    ms = (time.perf_counter() - t0) * 1e3 / k
    algo_bytes, _ = c2_bytes_per_step(2)
    out["c2"] = {"ms_per_step": round(ms, 3), "value": round(algo_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                 "us_per_call": round(ms * 1e3 / len(ws), 2),
                 "path": "168 x tensor_matmul_nt (reference, VOXCPM_CUDA): host a/out, fp32 device weights, cuBLAS"}
    for t in ws + ins + outs:
        L.tensor_free(t)
    # config 3: per shape, host a/out (engine path) and device a/out (kernel + the call's sync)
    rows = []
    K = 1024
    for N in C3_N:
        w = make((N, K), 0.02)
        L.tensor_to_cuda(w)
        for M in C3_M:
            a, o = make((M, K)), make((M, N))
            for _ in range(2):
                L.tensor_matmul_nt(a, w, o)
            reps = 20 if M < 2048 else 6
            t0 = time.perf_counter()
            for _ in range(reps):
                L.tensor_matmul_nt(a, w, o)
            us_host = (time.perf_counter() - t0) * 1e6 / reps
            L.tensor_to_cuda(a)
            L.tensor_to_cuda(o)
            for _ in range(2):
                L.tensor_matmul_nt(a, w, o)
            t0 = time.perf_counter()
            for _ in range(reps):
                L.tensor_matmul_nt(a, w, o)
            us_dev = (time.perf_counter() - t0) * 1e6 / reps
            rows.append({"M": M, "N": N, "K": K, "us_host_io": round(us_host, 1), "us_device_io": round(us_dev, 1),
                         "TFLOPs_device_io": round(2.0 * M * N * K / (us_dev * 1e-6) / 1e12, 2)})
            L.tensor_free(a)
            L.tensor_free(o)
        L.tensor_free(w)
    out["c3"] = rows
    print(json.dumps(out), flush=True)


def measure_ref_gpu(args):
    """The reference's GPU bar, timed in a child process (see ref_gpu_worker)."""
    if not os.path.exists(REF_GPU_LIB):
        return {"unavailable": "oracle/_ref/libref_tensor_cuda.so not built (needs the reference checkout)"}
    try:
        r = subprocess.run([sys.executable, os.path.abspath(__file__), "--ref-gpu-worker", "--steps", str(args.steps)],
                           capture_output=True, text=True, timeout=600)
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference GPU worker timed out"}
    for line in reversed(r.stdout.strip().splitlines()):
        if line.startswith("{"):
            d = json.loads(line)
            d["build"] = "src/tensor.c (-DVOXCPM_CUDA) + src/tensor_cuda.cu unchanged, nvcc sm_100, cuBLAS"
            return d
    return {"unavailable": f"reference GPU worker exited {r.returncode}: {r.stderr.strip()[-300:]}"}


ENGINE_BUILD = os.path.join(REPO, "voxcpm2-c_b200", "engine", "_build")
ENGINE_GOLDEN = os.path.join(REPO, "tests", "golden", "engine_c4_q8.json")


def _engine_run(exe, model, patches, env_extra, extra_args=()):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([os.path.join(ENGINE_BUILD, exe), "--model", model, "--patches", str(patches),
                        "--tokens", "64", "--token-seed", "1", *extra_args], env=env, capture_output=True,
                       text=True, timeout=3600)
    if r.returncode != 0:
        return {"unavailable": f"{exe} exited {r.returncode}: {r.stderr.strip()[-300:]}"}
    d = json.loads(r.stdout.strip().splitlines()[-1])
    d["per_patch_s"] = {k: round(v["s"] / patches, 5) for k, v in d["stages"].items()}
    return d


def _make_model(base=None):
    """Writes the seeded random-init model (make_model, seed 1) into a new folder under `base`;
    returns (folder, model path, make_model's summary) or raises."""
    import shutil
    import tempfile
    base = base or os.environ.get("VOXQ_MODEL_DIR") or tempfile.gettempdir()
    if shutil.disk_usage(base).free < 12e9:
        raise RuntimeError(f"less than 12 GB free in {base} for the 5 GB model")
    work = tempfile.mkdtemp(prefix="voxq_model_", dir=base)
    t0 = time.perf_counter()
    gen = json.loads(subprocess.run([os.path.join(ENGINE_BUILD, "make_model"), os.path.join(work, "rand"),
                                     "--seed", "1"], check=True, capture_output=True,
                                    text=True).stdout.strip().splitlines()[-1])
    gen["gen_s"] = round(time.perf_counter() - t0, 1)
    return work, os.path.join(work, "rand.vxcpm"), gen


C5_UTTERANCES_PER_GPU, C5_PATCHES = 16, 4


def measure_c5(model, gpu, utterances, workers_per_gpu):
    """BASELINE config 5 slice: independent utterances (token counts uniform in
    [32, 128], seeded ids), Q4, each synthesised by the unchanged engine on
    libvoxq; `workers_per_gpu` engine processes per GPU, utterances placed by
    LPT (voxq.serve).  Returns the serving summary without per-utterance rows."""
    sys.path.insert(0, os.path.join(REPO, "voxcpm2-c_b200"))
    from voxq import serve as S
    cmd = [os.path.join(ENGINE_BUILD, "voxq_engine_run_gpu"), "--model", model, "--gpu", "--serve",
           "--ralm-max-seq", "4096"]
    est = max(30.0, 4.0 * (1.0 + 0.6 * max(u["patches"] for u in utterances)))
    r = S.serve(cmd, utterances, gpus=[gpu], workers_per_gpu=workers_per_gpu,
                env=dict(os.environ, VOXCPM_QUANT="q4"), deadline_s=est)
    res = r.pop("results")
    r["patches"] = sum(int(x["patches"]) for x in res if "error" not in x)
    r["weight_bytes"] = sum(int(x.get("weight_bytes", 0)) for x in res if "error" not in x)
    r["weight_bytes_per_patch"] = round(r["weight_bytes"] / max(1, r["patches"]))
    r["generate_s_per_utterance"] = [round(float(x["generate_s"]), 3) for x in res if "error" not in x]
    return r


def c5_cpu_estimate(patches):
    """The reference CPU path's utterances/s for the C5 slice, estimated from the committed
    CPU engine run (tests/golden/engine_c4_q8.json, one host thread, 64 tokens): one process per
    core, 8 processes, prefill + patches x per-patch time; not measured on the GPU host."""
    if not os.path.exists(ENGINE_GOLDEN):
        return None
    g = json.load(open(ENGINE_GOLDEN))
    c = g["cpu_run"]
    pre = c["stages"]["tslm_forward"]["s"]
    per_patch = (c["generate_s"] - pre) / c["patches"]
    t_utt = pre + patches * per_patch
    return {"utt_per_s": round(8 / t_utt, 5), "processes": 8, "s_per_utterance": round(t_utt, 1),
            "basis": f"CPU engine run on the build host ({g.get('cpu', '?')}), 1 thread, 64 tokens, "
                     f"{c['patches']} patches: prefill {pre:.1f} s + {per_patch:.1f} s per patch; 8 processes "
                     "assumed to scale perfectly"}


def measure_c4(patches=4, workdir=None, cpu_patches=0, model=None):
    """one utterance through the unchanged reference engine
    (src/*.c compiled as they are) on the seeded random-init model: 64 token
    ids, `patches` patches (4 frames each), 10 Euler steps, CFG 2.0.  Three
    builds of the same engine: with libvoxq (VOXCPM_CUDA, VOXCPM_QUANT=q8),
    with the reference's own src/tensor_cuda.cu (cuBLAS FP32 on the stored
    fp16 weights), and, when cpu_patches > 0, without VOXCPM_CUDA (the CPU
    path, one host thread).  RTF = wall time of voxcpm_generate / audio
    seconds; per-stage times from the harness (voxq_engine_run.c)."""
    import shutil
    for exe in ("make_model", "voxq_engine_run_gpu"):
        if not os.path.exists(os.path.join(ENGINE_BUILD, exe)):
            return {"unavailable": f"{exe} not built (make -C voxcpm2-c_b200/engine REF=<reference checkout>)"}
    work = None
    try:
        if model is None:
            try:
                work, model, gen = _make_model(workdir)
            except RuntimeError as e:
                return {"unavailable": str(e)}
        else:
            gen = model[1]
            model = model[0]
        out = {"workload": f"BASELINE config 4 slice: unchanged engine, 64 token ids, {patches} patches, "
                           "10 Euler steps, CFG 2.0, random-init model (Q8-exact projection weights)",
               "model_gen_s": gen["gen_s"], "model_bytes": gen["model_bytes"] + gen["audiovae_bytes"]}
        out["ours"] = _engine_run("voxq_engine_run_gpu", model, patches, {"VOXCPM_QUANT": "q8"}, ["--gpu"])
        # the full config: 200 patches (max_new_tokens 800); the RALM cache (about 52 positions
        # per patch) set past the 2048 positions voxcpm_generate fixes (src/model.c:709), the one
        # engine deviation
        out["ours_200_patches"] = _engine_run("voxq_engine_run_gpu", model, 200, {"VOXCPM_QUANT": "q8"},
                                              ["--gpu", "--ralm-max-seq", "16384"])
        # the same build with only the tensor.h boundary in use: the engine's own blocks, sampler,
        # encoder and AudioVAE decoder on the host, their projections through tensor_matmul_nt_cuda
        out["ours_tensor_h_only"] = _engine_run("voxq_engine_run_gpu", model, patches,
                                                {"VOXCPM_QUANT": "q8", "VOXQ_ENGINE_BLOCK": "cpu",
                                                 "VOXQ_ENGINE_DIT": "cpu", "VOXQ_ENGINE_LOCENC": "cpu",
                                                 "VOXQ_ENGINE_VAE": "cpu"}, ["--gpu"])
        if os.path.exists(os.path.join(ENGINE_BUILD, "voxq_engine_run_refgpu")):
            out["reference_gpu"] = _engine_run("voxq_engine_run_refgpu", model, patches, {}, ["--gpu"])
        if cpu_patches > 0:
            out["reference_cpu"] = _engine_run("voxq_engine_run_cpu", model, cpu_patches, {})
        elif os.path.exists(ENGINE_GOLDEN):
            g = json.load(open(ENGINE_GOLDEN))
            c = g["cpu_run"]
            c["per_patch_s"] = {k: round(v["s"] / c["patches"], 5) for k, v in c["stages"].items()}
            c["measured_on"] = f"the build host ({g.get('cpu', '?')}), not this GPU host"
            out["reference_cpu"] = c
        return out
    finally:
        if work:
            shutil.rmtree(work, ignore_errors=True)


def engine_configs(args, dist, rank, world, local_rank):
    """Configs 4 and 5 on the unchanged engine.  One model file for both (rank 0 writes it;
    under torchrun the others use the same file).  C4 (one utterance) on 1 GPU only; C5 on every
    rank: 16 utterances per GPU (weak scaling), LPT-partitioned over the ranks, each rank's share
    served by its own engine workers; the aggregate is all answers over the slowest rank's time.
    Never fatal to the headline line: failures are reported as `unavailable`."""
    import shutil
    sys.path.insert(0, os.path.join(REPO, "voxcpm2-c_b200"))
    from voxq import serve as S
    from voxq.parallel import lpt_partition
    out = {}
    if not all(os.path.exists(os.path.join(ENGINE_BUILD, e)) for e in ("make_model", "voxq_engine_run_gpu")):
        return {"c5": {"unavailable": "engine not built (make -C voxcpm2-c_b200/engine REF=<reference checkout>)"}}
    made = [None]
    if rank == 0:
        try:
            made = [_make_model()]
        except Exception as e:  # reported, never fatal
            made = [f"{type(e).__name__}: {e}"[:300]]
    if world > 1:
        dist.broadcast_object_list(made, src=0)
    if isinstance(made[0], str) or made[0] is None:
        return {"c5": {"unavailable": made[0] or "model not written"}}
    work, model, gen = made[0]
    try:
        if world == 1:
            try:
                out["c4"] = measure_c4(args.c4_patches, model=(model, gen))
            except Exception as e:
                out["c4"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
        utts = S.workload(C5_UTTERANCES_PER_GPU * world, patches=C5_PATCHES, seed=5)
        mine = [utts[i] for i in lpt_partition([S.cost(u) for u in utts], world)[rank]]
        # one engine process per GPU: with the blocks and the AudioVAE on the device the work is
        # GPU-side, and further processes only time-slice the GPU between their contexts
        # (16 utterances, 1 / 2 / 4 / 8 workers on one B200: 5.2 / 3.3 / 3.3 / 2.9 utt/s)
        wpg = 1
        try:
            res = measure_c5(model, local_rank, mine, wpg)
        except Exception as e:
            res = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
        allres = [res]
        if world > 1:
            allres = [None] * world
            dist.all_gather_object(allres, res)
        if rank == 0:
            bad = [r for r in allres if "unavailable" in r]
            if bad:
                out["c5"] = {"unavailable": bad[0]["unavailable"]}
            else:
                wall = max(r["wall_s"] for r in allres)
                answered = sum(r["answered"] for r in allres)
                wb = sum(r["weight_bytes"] for r in allres)
                per_gpu = {}
                for r in allres:
                    per_gpu.update(r["per_gpu"])
                out["c5"] = {
                    "metric": "c5_utterances_per_s", "value": round(answered / wall, 4), "unit": "utt/s",
                    "workload": f"BASELINE config 5 slice: {len(utts)} utterances ({C5_UTTERANCES_PER_GPU} per GPU, "
                                f"token counts uniform in [32, 128], seeded ids), {C5_PATCHES} patches each, Q4, "
                                "unchanged engine on libvoxq (transformer blocks and AudioVAE on the device), LPT over GPUs",
                    "scaling": "weak", "n_gpus": world, "workers_per_gpu": wpg, "answered": answered,
                    "wall_s_max": wall, "per_rank_wall_s": [r["wall_s"] for r in allres],
                    "GBps_per_gpu": {g: v["GBps"] for g, v in per_gpu.items()},
                    "weight_bytes_per_patch": allres[0]["weight_bytes_per_patch"],
                    "rtf_aggregate": round(wall / sum(r["audio_s"] for r in allres), 4),
                    "load_s_max": max(r["load_s"] for r in allres),
                    "dead_workers": sum(len(r["dead_workers"]) for r in allres),
                    "weight_bytes": wb,
                    "cpu_estimate": c5_cpu_estimate(C5_PATCHES),
                    "per_rank": [{k: r[k] for k in ("answered", "wall_s", "utt_per_s", "load_s", "per_gpu")}
                                 for r in allres] if world > 1 else None,
                }
                if world == 1:
                    out["c5"]["generate_s_per_utterance"] = allres[0]["generate_s_per_utterance"]
    finally:
        if world > 1:
            dist.barrier()
        if rank == 0:
            shutil.rmtree(work, ignore_errors=True)
    return out


def run_c4(args):
    d = measure_c4(args.c4_patches, cpu_patches=args.c4_cpu_patches)
    ours = d.get("ours", {})
    line = {"metric": "c4_rtf", "value": ours.get("rtf"), "unit": "s/s", "higher_is_better": False,
            "n_gpus": 1, "config": {"workload": d.get("workload")}, "c4": d}
    print(json.dumps(line), flush=True)


def run_attn(args):
    """One transformer-block call (voxq_transformer_block_forward) at the LocDiT's shape at the
    last patch of the full C4 run: both CFG branches, 801 rows (5 + 4 x 199), hidden 1024, 16
    query heads over 2 kv heads of 128, FFN 4096, Q8 weights, a fresh cache filled whole.  The
    median wall time per call (upload, block, download) with the attention kernel that
    VOXQ_ATTN_MMA selects (unset or 1: tensor cores, 0: CUDA cores); everything else in the call
    is the same, so two runs, one per setting, differ by the attention alone."""
    import ctypes as C
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "voxcpm2-c_b200"))
    import voxq
    os.environ["VOXCPM_QUANT"] = "q8"
    L = voxq.lib()
    voxq.check(L.tensor_cuda_init(), "tensor_cuda_init")
    B, S, D, H, KVH, hd, F = 2, 801, 1024, 16, 2, 128, 4096
    rng = np.random.default_rng(5)

    def w(n, k):
        return (0.02 * rng.standard_normal((n, k))).astype(np.float32)

    W = {"wq": w(H * hd, D), "wk": w(KVH * hd, D), "wv": w(KVH * hd, D), "wo": w(D, H * hd), "w1": w(F, D),
         "w2": w(D, F), "w3": w(F, D), "n1": np.ones(D, np.float32), "n2": np.ones(D, np.float32)}
    T = {k: voxq.host_tensor(v) for k, v in W.items()}
    for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3"):
        voxq.check(L.tensor_to_cuda(T[k]), "tensor_to_cuda")
    n1, n2 = voxq.RmsNormDesc(T["n1"], 1e-6), voxq.RmsNormDesc(T["n2"], 1e-6)
    at = voxq.AttentionDesc(T["wq"], T["wk"], T["wv"], T["wo"], D, H, KVH, hd)
    ff = voxq.SwigluDesc(T["w1"], T["w2"], T["w3"], D, F)
    bd = voxq.BlockDesc(C.pointer(n1), C.pointer(at), C.pointer(n2), C.pointer(ff))
    x = voxq.host_tensor(rng.standard_normal((B, S, D)).astype(np.float32))
    out = voxq.host_tensor(np.zeros((B, S, D), np.float32))
    ck = voxq.host_tensor(np.zeros((B, KVH, S, hd), np.float32))
    cv = voxq.host_tensor(np.zeros((B, KVH, S, hd), np.float32))

    def call():
        voxq.check(L.voxq_transformer_block_forward(C.byref(bd), x, ck, cv, None, None, 0, out), "block")

    for _ in range(args.warmup):
        call()
    times = []
    for _ in range(max(1, min(args.steps, 200))):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    mma = os.environ.get("VOXQ_ATTN_MMA", "1")[:1] != "0"
    line = {"metric": "block_call_ms", "value": round(float(np.median(times)) * 1e3, 4), "unit": "ms",
            "higher_is_better": False, "steps": len(times), "warmup": args.warmup,
            "attention": "tensor cores (split TF32 mma.sync)" if mma else "CUDA cores (fp32 FMA)",
            "config": {"workload": "one transformer block, LocDiT shape at the last of 200 patches: B=2 (CFG), "
                                   "S=801, hidden 1024, heads 16/2 x 128, FFN 4096, Q8, fresh cache filled whole",
                       "attention_flops": 2 * 2 * B * H * S * S * hd},
            "min_ms": round(min(times) * 1e3, 4)}
    print(json.dumps(line), flush=True)
    L.voxq_block_cache_clear()
    L.tensor_cuda_shutdown()


def measure_sharded_c3(torch, voxq, dist, dev, st, rank, world, steps, warmup):
    """Config-3 GEMM column shards (no collective): rank r owns weight rows
    [r*N/G, (r+1)*N/G), quantized on its own GPU, and writes its column slice of
    out[M, N] from the full activation block.  Weak: N = 4096 per rank (the
    weight grows with the ranks); strong: N = 4096 in total.  Each rank's device
    time per call (CUDA-graph replay, rotated weights) is gathered; the
    aggregate TFLOP/s is all ranks' flops over the slowest rank's time."""
    M, K = 2048, 1024
    res = {}
    for kind, n_total in (("weak", 4096 * world), ("strong", 4096)):
        n_loc = n_total // world
        g = torch.Generator(device=dev).manual_seed(1000 + rank)
        copies = 8
        ws = [voxq.QWeight.from_float(torch.randn(n_loc, K, device=dev, generator=g) * 0.02, voxq.Q8)
              for _ in range(copies)]
        a = torch.randn(M, K, device=dev, generator=torch.Generator(device=dev).manual_seed(7))
        out = torch.empty(M, n_loc, device=dev)
        with torch.cuda.stream(st):
            for i in range(max(warmup, 3)):
                voxq.matmul_nt_q(a, ws[i % copies], out=out, stream=st)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        reps = 32
        with torch.cuda.graph(graph, stream=st):
            for i in range(reps):
                voxq.matmul_nt_q(a, ws[i % copies], out=out, stream=st)
        loops = max(2, steps // reps)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(st):
            graph.replay()
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(st):
            e0.record(st)
            for _ in range(loops):
                graph.replay()
            e1.record(st)
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) / (loops * reps) * 1e3
        del graph
        per_rank = [us]
        if dist is not None:
            t = torch.zeros(world, device=dev)
            t[rank] = us
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            per_rank = [round(float(v), 2) for v in t.tolist()]
        us_max = max(per_rank)
        flops = 2.0 * M * n_total * K
        res[kind] = {"M": M, "N_total": n_total, "N_per_rank": n_loc, "K": K, "qtype": "q8",
                     "us_max": round(us_max, 2), "TFLOPs": round(flops / (us_max * 1e-6) / 1e12, 1),
                     "per_rank_us": [round(v, 2) for v in per_rank],
                     "device_error": voxq.lib().voxq_device_error(1)}
        del ws
    return res


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
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "attn", "chain"],
                    help="c2: the headline decode step (default); c1: one Q8 GEMV; c3: GEMM sweep, one line per "
                         "shape; c4: the unchanged engine's RTF; attn: one transformer-block call at the LocDiT's "
                         "200-patch shape (VOXQ_ATTN_MMA picks the attention kernel); chain: the dependent C2 "
                         "decode step alone")
    ap.add_argument("--c4-patches", type=int, default=4)
    ap.add_argument("--c4-cpu-patches", type=int, default=0, help="c4: also time the CPU engine on this many patches")
    ap.add_argument("--no-configs", dest="configs", action="store_false",
                    help="c2 line without the configs object (C1, C3, chain, reference GPU)")
    ap.add_argument("--ref-gpu-worker", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.ref_gpu_worker:
        ref_gpu_worker(args)
        return
    if args.config in ("c1", "c3", "chain"):
        import torch
        {"c1": run_c1, "c3": run_c3, "chain": run_chain}[args.config](args, torch)
        return
    if args.config == "c4":
        run_c4(args)
        return
    if args.config == "attn":
        run_attn(args)
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
