"""Benchmark of the B200 INT8 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: x fp32 [1,2048] ~N(0,1), W int8 [6144,2048]
~U[-127,127], per-output-row fp32 scales ~U(0.001,0.02), seed 0;
y = x (W*s)^T.  One step = activation quantisation + INT8 GEMV.  64 distinct
weight copies (805 MB, > 6x the 126 MB L2) are rotated so every step streams
its weights from HBM.  Under torchrun every rank runs its own replica (the
path has no exchange step), so scaling is weak and the job value is the sum.

``--impl reference`` times the reference engine's own CPU kernel
(oracle/_ref, compiled from its sources) on this host's cores, same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GEMV_N, GEMV_K = 6144, 2048
GEMV_BYTES = GEMV_N * GEMV_K + 4 * GEMV_N + 4 * GEMV_K + 4 * GEMV_N   # W + scales + x + y
N_COPIES = 64
WORKLOAD = "config0_gemv_M1_N6144_K2048_rowwise"


def import_qvl():
    """Import the product package (directory qwen3-vl-2b-inference_b200) as `qvl_b200`."""
    import importlib.util
    if "qvl_b200" in sys.modules:
        return sys.modules["qvl_b200"]
    pkg = os.path.join(ROOT, "qwen3-vl-2b-inference_b200")
    spec = importlib.util.spec_from_file_location("qvl_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["qvl_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    def __init__(self, index=0):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                  "--format=csv,noheader,nounits", "-lms", "100"],
                                 stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        while not self._stop.is_set():
            line = p.stdout.readline()
            if not line:
                break
            self.samples.append([x.strip() for x in line.split(",")])
        p.terminate()

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=3)

    def summary(self):
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [num(s[0]) for s in self.samples if num(s[0]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 3 + i and s[3 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(self.samples[0][1]),
                "reasons": reasons, "samples": len(self.samples)}


def gemv_inputs(seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, GEMV_K), dtype=np.float32)
    w = rng.integers(-127, 128, size=(GEMV_N, GEMV_K), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, size=GEMV_N).astype(np.float32)
    return x, w, s


def cpu_gemv_rate(x, w, s, seconds=10.0, kind="reference"):
    """GB/s of the CPU GEMV on this host, bounded to ~`seconds`."""
    import oracle
    if kind == "reference":
        fn = lambda: oracle.ref_i8_kernel(x, w, s, GEMV_K)   # noqa: E731
    else:
        fn = lambda: oracle.linear_i8(x, w, s, GEMV_K)       # noqa: E731
    for _ in range(3):
        fn()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        fn()
        n += 1
    dt = (time.perf_counter() - t0) / n
    return GEMV_BYTES / dt / 1e9, n, dt


def profile_traffic(kernel_tag):
    """dram read+write bytes per launch from an ncu capture, read from the
    committed summary profiles/<kernel_tag>.md ("traffic_bytes_per_launch: N")."""
    p = os.path.join(ROOT, "profiles", kernel_tag + ".md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libqwen_ref.so not built"}))
        return
    x, w, s = gemv_inputs(0)
    cores = os.cpu_count()
    for _ in range(args.warmup):
        oracle.ref_i8_kernel(x, w, s, GEMV_K)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.ref_i8_kernel(x, w, s, GEMV_K)
    dt = (time.perf_counter() - t0) / args.steps
    gbs = GEMV_BYTES / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": "int8_gemv_hbm_gbs", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int16xint8->int32",
        "data": "synthetic (seed 0)",
        "config": {"workload": WORKLOAD, "l2": "CPU: one 12.6 MB weight copy, cache-warm"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "reference",
                         "sample": f"{args.steps} calls of f32a_i8f32sb_f32c_avx2_kernel (OpenMP, all cores)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def run_ours(args):
    import torch
    import torch.distributed as dist
    qvl = import_qvl()
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    x, w, s = gemv_inputs(0)
    xd = torch.from_numpy(x).to(dev)
    w0 = torch.from_numpy(w).to(dev)
    sd = torch.from_numpy(s).to(dev)
    wc = [w0] + [w0.clone() for _ in range(N_COPIES - 1)]   # same values, distinct HBM
    yd = torch.empty((1, GEMV_N), dtype=torch.float32, device=dev)
    work = qvl.Workspace(dev)
    work.get(qvl.load_library().qvl_linear_i8_workspace_bytes(1, GEMV_K, GEMV_K))
    q, qs = qvl.quantize_rows(xd, GEMV_K)
    stream = torch.cuda.Stream(dev)

    def step(i):        # the product call: quantise + GEMV
        qvl.linear(xd, wc[i % N_COPIES], sd, yd, group_quantized=False, workspace=work)

    def kstep(i):       # the GEMV kernel alone (roofline timing)
        qvl.linear_q16(q, qs, wc[i % N_COPIES], sd, GEMV_K, C=yd)

    def capture(fn, n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            for i in range(3):
                fn(i)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for i in range(n):
                    fn(i)
        return g

    g_step = capture(step, args.steps)
    g_kern = capture(kstep, args.steps)
    torch.cuda.synchronize()

    def timed(graph):
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                graph.replay()
            torch.cuda.synchronize()
            if ws > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if ws > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with ClockSampler(local) as clk:
        ms_total = timed(g_step)
        ms_kern = timed(g_kern)
    ms_step = ms_total / args.steps
    value = GEMV_BYTES * args.steps * ws / (ms_total / 1e3) / 1e9

    # e2e through the public API with host buffers: pinned x -> device, linear,
    # y -> pinned host; the host waits for each step's result.
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.empty((1, GEMV_N), dtype=torch.float32).pin_memory()
    graphs = []
    for c in range(N_COPIES):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                xd.copy_(xh, non_blocking=True)
                qvl.linear(xd, wc[c], sd, yd, group_quantized=False, workspace=work)
                yh.copy_(yd, non_blocking=True)
        graphs.append(g)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs[i % N_COPIES].replay()
            stream.synchronize()
        if ws > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            graphs[i % N_COPIES].replay()
            stream.synchronize()
        e2e_s = time.perf_counter() - t0
    if ws > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    y_check = yh.numpy().copy()
    e2e = GEMV_BYTES * args.steps * ws / e2e_s / 1e9

    if rank == 0:
        import oracle
        if not np.array_equal(oracle.linear_i8(x, w, s, GEMV_K), y_check):
            raise SystemExit("bench: GEMV output differs from the oracle")
        peak, peak_kind = load_peaks()
        achieved = GEMV_BYTES / (ms_kern / args.steps / 1e3) / 1e9
        cpu = None
        if args.cpu_seconds > 0:
            kind = "reference" if oracle.ref_available() else "port"
            gbs, n, dt = cpu_gemv_rate(x, w, s, args.cpu_seconds, kind)
            cpu = {"value": round(gbs, 3), "unit": "GB/s",
                   "cores": os.cpu_count() if kind == "reference" else 1, "kind": kind,
                   "sample": f"{n} GEMV calls ({dt * 1e3:.3f} ms each, weights cache-warm) over ~{args.cpu_seconds:.0f} s"}
        print(json.dumps({
            "metric": "int8_gemv_hbm_gbs", "value": round(value, 2), "unit": "GB/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int16xint8->int32", "data": "synthetic (seed 0)",
            "config": {"workload": WORKLOAD, "parallelism": f"replicas{ws}",
                       "l2": f"{N_COPIES} rotated weight copies ({N_COPIES * GEMV_N * GEMV_K / 1e6:.0f} MB > L2)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": profile_traffic("gemv_i8_config0"),
                         "kernel": "gemv_i8_fast_kernel<1,true,4>", "algorithmic_bytes_per_launch": GEMV_BYTES},
            "e2e": {"value": round(e2e, 3), "unit": "GB/s", "h2d_bytes_per_step": 4 * GEMV_K,
                    "d2h_bytes_per_step": 4 * GEMV_N},
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }))
    if ws > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=640)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
