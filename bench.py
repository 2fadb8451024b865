"""Benchmark of the B200 INT8 hot path (one JSON line on rank 0).

Headline (BASELINE metric "decode tokens/s (batch 1/32)"): decode tokens/s of
the Qwen3-VL-2B text decoder -- 28 layers, int8 per-row weights, tied
151936-row LM head, random-init (no checkpoint) -- at ``--batch`` requests
per GPU (default 1), after a 452-position prompt state (196 vision + 256 text
positions of BASELINE config 4; the KV contents are synthetic).  One step =
one generated token per request.  At batch 1 a step is ONE cooperative
launch (decode_persistent_kernel), captured in a CUDA graph; attention runs in
the reference's summation order by default (``--attn-order``), so the logits
are bit-identical to the reference's operators.  The same line carries
``batch32`` (32 requests on the tensor cores), ``gemv_config0`` (BASELINE
config 0, the INT8 GEMV alone), ``e2e`` (token ids through pinned host memory
every step), ``roofline`` and ``cpu_baseline``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|gemv|prefill|prefill_gemm|swiglu|attention]

Under torchrun every rank runs its own replica (decode requests are
independent; no collective on the data path), so scaling is weak and the job
value is the sum over ranks; time is the max over ranks.

``--impl reference`` times the reference engine's own CPU operators
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
    """The reference engine's own CPU operators (oracle/_ref) composed into
    forward_text, timed on this host: `steps` decode tokens after warm-up."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import oracle
    if not (oracle.ref_available() or oracle.ref_model_available()):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (the reference compiled from its sources) not built"}))
        return
    tps, n, dt = cpu_decode_rate(args, seconds=None, steps=args.steps, warmup=args.warmup)
    print(json.dumps({
        "impl": "reference", "metric": "decode_tokens_per_s", "value": round(tps, 3), "unit": "tokens/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int16xint8->int32",
        "data": "synthetic (random-init int8 weights, seed 0)", "config": decode_config(args, 1),
        "cpu_baseline": {"value": round(tps, 3), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "reference",
                         "sample": f"{n} decode tokens, batch 1 (the reference runs one request at a time): its own "
                                   f"init_model_weights + forward_text on a synthetic model file"},
        "e2e": {"value": round(tps, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


PROMPT_CTX = 452          # 196 vision tokens + 256 text tokens


def decode_config(args, ws):
    return {"workload": f"qwen3vl2b_text_decode_b{args.batch}", "layers": 28, "hidden": 2048,
            "intermediate": 6144, "heads": "16q/8kv x128", "vocab": 151936, "batch_per_gpu": args.batch,
            "prompt_ctx": PROMPT_CTX, "weights": "int8 per-row scales, norms int8 group 128",
            "parallelism": f"dp{ws} (independent replicas)", "l2": "1.72 GB of weights per step > L2"}


_cpu_state = {}


def _ref_model_file():
    """A synthetic model file in the exporter's layout (full-size text
    decoder, per-row INT8; a minimal vision tower, which forward_text does not
    touch) for the reference's own loader; written once per process."""
    path = _cpu_state.get("bin")
    if path is None:
        import tempfile
        import_qvl()
        import qvl_b200.modelfile as MF
        hdr = MF.qwen3vl_2b_header(vision_hidden_size=32, vision_intermediate_size=64, vision_num_heads=2)
        import atexit
        import shutil
        d = tempfile.mkdtemp(prefix="qvl_bench_")
        atexit.register(shutil.rmtree, d, True)
        path = os.path.join(d, "qwen3vl2b_text_rowwise.bin")
        MF.write_model_bin(path, hdr, MF.synthetic_text(hdr, seed=0))
        _cpu_state["bin"] = path
    return path


def cpu_decode_rate(args, seconds=None, steps=None, warmup=2):
    """Reference CPU decode on the same model shape, all host cores, bounded by
    `seconds` or `steps`: the reference's own loader and forward_text
    (oracle.RefModel, its FP32 KV cache) when that library is built, else its
    compiled operators composed in forward_text order (oracle/decode.py)."""
    import torch
    import oracle
    if oracle.ref_model_available():
        rm = oracle.RefModel(_ref_model_file(), fp16_kv=False)
        try:
            rng = np.random.default_rng(0)
            rm.k_cache[:, :, :PROMPT_CTX] = rng.standard_normal(rm.k_cache[:, :, :PROMPT_CTX].shape, dtype=np.float32)
            rm.v_cache[:, :, :PROMPT_CTX] = rng.standard_normal(rm.v_cache[:, :, :PROMPT_CTX].shape, dtype=np.float32)
            tok, pos = 5, PROMPT_CTX
            for _ in range(warmup):
                tok = oracle.argmax(rm.forward(tok, pos))
                pos += 1
            n, t0 = 0, time.perf_counter()
            while True:
                tok = oracle.argmax(rm.forward(tok, pos))
                pos += 1
                n += 1
                el = time.perf_counter() - t0
                if (steps is not None and n >= steps) or (seconds is not None and el >= seconds):
                    break
        finally:
            rm.close()
        dt = el / n
        return 1.0 / dt, n, dt
    from oracle.decode import CpuDecoder
    import_qvl()
    import qvl_b200.decoder as D
    cfg = D.TextConfig()
    w = _cpu_state.get("w")
    if w is None:
        dev = "cuda" if torch.cuda.is_available() else "cpu"
        w = D.TextWeights.random(cfg, seed=0, device=dev).numpy()
        _cpu_state["w"] = w
    cos, sin = D.rope_table(PROMPT_CTX + 1024, cfg.head_dim, cfg.rope_theta)
    backend = "ref" if oracle.ref_available() else "orc"
    dec = CpuDecoder(cfg, w, PROMPT_CTX + 1024, cos, sin, backend=backend)
    rng = np.random.default_rng(0)
    dec.kc[:, :, :PROMPT_CTX] = rng.standard_normal((cfg.layers, cfg.kv_heads, PROMPT_CTX, cfg.head_dim),
                                                    dtype=np.float32).astype(np.float16)
    dec.vc[:, :, :PROMPT_CTX] = rng.standard_normal((cfg.layers, cfg.kv_heads, PROMPT_CTX, cfg.head_dim),
                                                    dtype=np.float32).astype(np.float16)
    tok, pos = 5, PROMPT_CTX
    for _ in range(warmup):
        _, tok = dec.step(tok, pos)
        pos += 1
    n, t0 = 0, time.perf_counter()
    while True:
        _, tok = dec.step(tok, pos)
        pos += 1
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (seconds is not None and el >= seconds):
            break
    dt = el / n
    return 1.0 / dt, n, dt


def run_gemv(dev, steps=640, warmup=5):
    """BASELINE config 0 on this GPU: quantise + GEMV per step over rotated
    weight copies (inputs > L2).  Returns device-timed GB/s of the step and of
    the GEMV kernel alone."""
    import torch
    qvl = import_qvl()
    x, w, s = gemv_inputs(0)
    xd = torch.from_numpy(x).to(dev)
    w0 = torch.from_numpy(w).to(dev)
    sd = torch.from_numpy(s).to(dev)
    wc = [w0] + [w0.clone() for _ in range(N_COPIES - 1)]
    yd = torch.empty((1, GEMV_N), dtype=torch.float32, device=dev)
    work = qvl.Workspace(dev)
    work.get(qvl.load_library().qvl_linear_i8_workspace_bytes(1, GEMV_K, GEMV_K))
    q, qs = qvl.quantize_rows(xd, GEMV_K)
    stream = torch.cuda.Stream(dev)
    fns = {"step": lambda i: qvl.linear(xd, wc[i % N_COPIES], sd, yd, group_quantized=False, workspace=work),
           "kernel": lambda i: qvl.linear_q16(q, qs, wc[i % N_COPIES], sd, GEMV_K, C=yd)}
    out = {}
    for name, fn in fns.items():
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            for i in range(3):
                fn(i)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for i in range(steps):
                    fn(i)
            for _ in range(warmup):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        out[name] = GEMV_BYTES * steps / (e0.elapsed_time(e1) / 1e3) / 1e9
    import oracle
    if not np.array_equal(yd.cpu().numpy(), oracle.linear_i8(x, w, s, GEMV_K)):
        raise SystemExit("bench: config-0 GEMV output differs from the oracle")
    del wc
    return {"workload": WORKLOAD, "step_gbs": round(out["step"], 1), "kernel_gbs": round(out["kernel"], 1),
            "launches_per_step": 1, "step": "linear(): the activation quantisation inside the ring GEMV",
            "steps": steps}


def ctypes_byref(x):
    import ctypes
    return ctypes.byref(x)


def l2_flush_buffer(dev):
    import torch
    return torch.empty(256 << 20, dtype=torch.uint8, device=dev)    # 256 MB > the 126 MB L2


def time_cold(fn, stream, flush, steps, warmup):
    """Mean device time of fn() over `steps` launches, each preceded by an
    untimed L2 flush (a 256 MB write), CUDA events on `stream`."""
    import torch
    torch.cuda.synchronize()          # inputs were initialised on the default stream
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
    return total / steps / 1e3


def run_attention_line(args):
    """GQA decode attention over FP16 KV pages (16 q / 8 kv
    heads x 128), contexts {512, 4096, 32768} x decode batch {1, 8, 64}, one
    query per request at the last position.  HBM-bound: 4096 bytes of K+V per
    cached token per request.  L2 flushed before every timed launch."""
    import torch
    qvl = import_qvl()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, peak_kind = load_peaks()
    stream = torch.cuda.Stream(dev)
    flush = l2_flush_buffer(dev)
    sweep = []
    with ClockSampler(0) as clk:
        for ctx in (512, 4096, 32768):
            for B in (1, 8, 64):
                kv = qvl.PagedKV(B, ctx, 16, 8, 128, 64, max_pos=ctx, device=dev)
                kv.k.normal_()
                kv.v.normal_()
                q = torch.randn(B, 16, 128, device=dev)
                out = torch.empty_like(q)
                pos = torch.full((B,), ctx - 1, dtype=torch.int32, device=dev)
                seq = torch.arange(B, dtype=torch.int32, device=dev)
                work = qvl.Workspace(dev)
                work.get(qvl.load_library().qvl_attention_workspace_bytes(B, ctx, ctypes_byref(kv.dims)))
                fn = lambda: qvl.attention(q, kv, seq, pos, ctx, out=out, workspace=work)
                sec = time_cold(fn, stream, flush, args.steps, args.warmup)
                nbytes = 4096 * ctx * B + B * 16 * 128 * 4 * 2
                sweep.append({"ctx": ctx, "batch": B, "us": round(sec * 1e6, 2), "gbs": round(nbytes / sec / 1e9, 1),
                              "frac": round(nbytes / sec / 1e9 / peak, 4)})
                del kv, work
                torch.cuda.empty_cache()
    head = next(r for r in sweep if r["ctx"] == 32768 and r["batch"] == 64)
    print(json.dumps({
        "metric": "attention_decode_hbm_gbs", "value": head["gbs"], "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 KV, fp32 softmax", "data": "synthetic N(0,1)",
        "config": {"workload": "config3_gqa_decode_ctx32768_b64", "l2": "flushed before each launch"},
        "roofline": {"bound": "hbm", "achieved": head["gbs"], "peak": peak, "unit": "GB/s",
                     "frac": head["frac"], "peak_kind": peak_kind, "traffic": None,
                     "kernel": "attention (cluster kernel / split-K trio)"},
        "sweep": sweep, "clocks": clk.summary()}))


def int8_tensor_peak(dev):
    """Measured int8 dense tensor throughput on this GPU (cuBLASLt through
    torch._int_mm, 8192^3, best of 5), in TOPS (2*M*N*K)."""
    import torch
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev).t()
    try:
        torch._int_mm(a, b)
    except RuntimeError:
        return None
    torch.cuda.synchronize()
    best = 0.0
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = max(best, 2 * n ** 3 / (e0.elapsed_time(e1) / 1e3) / 1e12)
    return round(best, 1)


def run_swiglu_line(args):
    """the fused SwiGLU MLP down(silu(gate(x)) * up(x)),
    int8 gate/up [6144,2048] and down [2048,6144] with per-row scales, M in
    {1, 64, 512}; 8 rotated weight sets (302 MB > L2)."""
    import torch
    qvl = import_qvl()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, peak_kind = load_peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    H, I, NSET = 2048, 6144, 8
    sets = []
    for _ in range(NSET):
        mk = lambda n, k: torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g)
        sc = lambda n: torch.rand(n, device=dev, generator=g) * 0.019 + 0.001
        sets.append((mk(I, H), sc(I), mk(I, H), sc(I), mk(H, I), sc(H)))
    i8peak = int8_tensor_peak(dev)
    stream = torch.cuda.Stream(dev)
    sweep = []
    with ClockSampler(0) as clk:
        for M in (1, 64, 512):
            x = torch.randn(M, H, device=dev, generator=g)
            out = torch.empty(M, H, device=dev)
            work = qvl.Workspace(dev)
            sem = qvl.SEM_REFERENCE
            # group_size 0: per-row scales for all three products (down: group 6144)
            run = lambda i: qvl.swiglu_mlp(x, *sets[i % NSET], 0, out=out, semantics=sem, workspace=work)
            run(0)
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(gr, stream=stream):
                    for i in range(NSET):
                        run(i)
                for _ in range(args.warmup):
                    gr.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(args.steps):
                    gr.replay()
                e1.record(stream)
                torch.cuda.synchronize()
            sec = e0.elapsed_time(e1) / 1e3 / (args.steps * NSET)
            nbytes = 3 * H * I + 4 * (2 * I + H) + 4 * M * H * 2
            ops = 2 * M * 3 * H * I
            r = {"M": M, "us": round(sec * 1e6, 2), "gbs": round(nbytes / sec / 1e9, 1),
                 "tops": round(ops / sec / 1e12, 2), "hbm_frac": round(nbytes / sec / 1e9 / peak, 4)}
            if i8peak:
                r["tensor_frac"] = round(ops / sec / 1e12 / i8peak, 4)
            sweep.append(r)
    head = sweep[0]
    print(json.dumps({
        "metric": "swiglu_mlp_hbm_gbs", "value": head["gbs"], "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int16xint8->int32", "data": "synthetic (seed 0)",
        "config": {"workload": "config2_swiglu_mlp_M1", "inputs": f"{NSET} rotated weight sets (302 MB > L2)"},
        "roofline": {"bound": "hbm", "achieved": head["gbs"], "peak": peak, "unit": "GB/s",
                     "frac": head["hbm_frac"], "peak_kind": peak_kind, "traffic": None,
                     "kernel": "gate/up GEMV (SwiGLU pair) + quantise + down GEMV"},
        "int8_tensor_peak_tops": i8peak, "sweep": sweep, "clocks": clk.summary()}))


def run_gemv_line(args):
    """BASELINE config 0 alone (one GPU): the INT8 GEMV 6144x2048 with
    per-row scales, device-timed over rotated weight copies (> L2)."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with ClockSampler(0) as clk:
        r = run_gemv(dev, steps=args.steps * 5, warmup=args.warmup)
    peak, peak_kind = load_peaks()
    print(json.dumps({
        "metric": "int8_gemv_hbm_gbs", "value": r["kernel_gbs"], "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps * 5, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int16xint8->int32", "data": "synthetic (seed 0, BASELINE config 0)",
        "config": {"workload": WORKLOAD, "inputs": "64 rotated weight copies (805 MB > L2)"},
        "roofline": {"bound": "hbm", "achieved": r["kernel_gbs"], "peak": peak, "unit": "GB/s",
                     "frac": round(r["kernel_gbs"] / peak, 4), "peak_kind": peak_kind,
                     "traffic": profile_traffic("gemv_ring_config0"), "kernel": "gemv_ring_kernel"},
        "step_with_quantisation_gbs": r["step_gbs"], "clocks": clk.summary()}))


def decode_gemv_roofline(dec, steps=4):
    """Average GEMV launch of the decode step (q/k/v/o/gate/up/down x 28 +
    LM head), timed alone in a graph: algorithmic bytes / device time."""
    import torch
    qvl = import_qvl()
    cfg, t = dec.cfg, dec.w.t
    B = dec.B
    H, I = cfg.hidden, cfg.intermediate
    q_h, s_h = qvl.quantize_rows(torch.randn(B, H, device=dec.device), H)
    q_i, s_i = qvl.quantize_rows(torch.randn(B, I, device=dec.device), I)
    outs = {n: torch.empty((B, t[n].shape[-2]), device=dec.device) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")}
    logits = torch.empty((B, cfg.vocab), device=dec.device)
    nbytes = 0
    calls = []
    for l in range(cfg.layers):
        for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            W, S = t[n][l], t[n + "_s"][l]
            qq, ss = (q_i, s_i) if n == "wd" else (q_h, s_h)
            calls.append((qq, ss, W, S, outs[n]))
            nbytes += W.numel() + 4 * W.shape[0] + B * (2 * W.shape[1] + 4 * W.shape[0])
    calls.append((q_h, s_h, t["embed"], t["embed_s"], logits))
    nbytes += t["embed"].numel() + 4 * cfg.vocab + B * (2 * H + 4 * cfg.vocab)
    stream = torch.cuda.Stream(dec.device)
    g = torch.cuda.CUDAGraph()
    run = lambda: [qvl.linear_q16(a, b, c, d, a.shape[1], C=e, semantics=qvl.SEM_LANE8) for a, b, c, d, e in calls]
    with torch.cuda.stream(stream):
        run()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(steps):
                run()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3
    launches = len(calls) * steps * ((B + 7) // 8 if B > 4 else 1)
    return nbytes * steps / sec / 1e9, nbytes / len(calls), sec / (len(calls) * steps), launches


PREFILL_SHAPES = [(2048, 2048), (1024, 2048), (6144, 2048), (2048, 6144), (151936, 2048)]   # (N, K), config 1


def run_prefill_gemm(args):
    """batched INT8 GEMM at M=512 over the q/o, k/v,
    gate/up, down and LM-head shapes (per-row scales), one pass over all five
    shapes per step, through qvl.linear (quantise + hi/lo split + tcgen05)."""
    import torch
    import torch.distributed as dist
    qvl = import_qvl()
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    M = args.m
    g = torch.Generator(device=dev).manual_seed(rank)
    mats = []
    for N, K in PREFILL_SHAPES:
        W = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        S = torch.rand(N, device=dev, generator=g) * 0.019 + 0.001
        X = torch.randn(M, K, device=dev, generator=g)
        Y = torch.empty(M, N, device=dev)
        mats.append((X, W, S, Y))
    work = qvl.Workspace(dev)
    work.get(max(qvl.load_library().qvl_linear_i8_workspace_bytes(M, K, K) for _, K in PREFILL_SHAPES))
    stream = torch.cuda.Stream(dev)

    def step():
        for X, W, S, Y in mats:
            qvl.linear(X, W, S, Y, group_quantized=False, workspace=work)

    with torch.cuda.stream(stream):
        step()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            step()
        for _ in range(args.warmup):
            gr.replay()
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(args.steps):
                gr.replay()
            e1.record(stream)
            torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ops = sum(2 * M * N * K for N, K in PREFILL_SHAPES)
    tops = ops * args.steps * ws / (ms / 1e3) / 1e12
    if rank == 0:
        i8peak = int8_tensor_peak(dev)
        roofline_gemm = {"bound": "tensor", "achieved": round(tops / ws, 2), "peak": i8peak, "unit": "TOPS",
                         "frac": round(tops / ws / i8peak, 4) if i8peak else None,
                         "peak_kind": "measured (torch._int_mm int8, 8192^3, this GPU)", "traffic": None,
                         "kernel": "gemm_i8_tc (tcgen05 kind::i8; persistent for the LM head, split-K clusters for the rest; hi/lo planes: 2 MMAs per algorithmic one)"}
        import oracle
        X, W, S, Y = mats[0]
        ref = oracle.linear_i8(X[:2].cpu().numpy(), W.cpu().numpy(), S.cpu().numpy(), 2048, oracle.TILED)
        if not np.array_equal(Y[:2].cpu().numpy(), ref):
            raise SystemExit("bench: prefill GEMM differs from the oracle")
        print(json.dumps({
            "metric": "int8_prefill_gemm_tops", "value": round(tops, 2), "unit": "TOPS", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int16xint8->int32", "data": "synthetic",
            "config": {"workload": f"config1_gemm_M{M}", "shapes_NK": PREFILL_SHAPES,
                       "ops_per_step": ops, "note": "ops = 2*M*N*K (the hi/lo split doubles the MMA work)"},
            "roofline": roofline_gemm, "clocks": clk.summary(), "gpu_launches": 2 * len(PREFILL_SHAPES) * args.steps,
        }))
    if ws > 1:
        dist.destroy_process_group()


def run_prefill(args):
    """Prompt prefill (TTFT) of the text decoder: a 452-token prompt as one
    M=452 pass (tensor-core GEMMs, causal attention), graph-captured.  value =
    prompt tokens/s; the reference feeds prompts one token at a time."""
    import torch
    import torch.distributed as dist
    import_qvl()
    import qvl_b200.decoder as D
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    cfg = D.TextConfig()
    T = PROMPT_CTX
    tp = args.tp and ws > 1
    # tensor split: every rank holds the same weights and prompt and computes
    # its output columns of every product; replicas: one prompt per rank
    seed = 0 if tp else rank
    w = D.TextWeights.random(cfg, seed=seed, device=dev)
    dec = D.TextDecoder(w, max_batch=1, max_ctx=T + 8, device=dev, tp_group=dist.group.WORLD if tp else None)
    prompt = torch.randint(0, 151643, (T,), dtype=torch.int32, device=dev,
                           generator=torch.Generator(device=dev).manual_seed(seed))
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        dec.prefill(prompt)
        torch.cuda.synchronize()
        if tp:
            # the tensor-split pass runs eagerly (NCCL collectives are not
            # captured); one pass is ~600 launches, far below its 10+ ms
            class _Eager:
                def replay(self):
                    dec.prefill(prompt)
            g = _Eager()
        else:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                dec.prefill(prompt)
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            e0.record(stream)
            for _ in range(args.steps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ttft_ms = ms / args.steps
    if rank == 0:
        cpu = None
        if args.cpu_seconds > 0:
            del dec, g
            torch.cuda.empty_cache()
            tps, n, dt = cpu_decode_rate(args, seconds=args.cpu_seconds)
            cpu = {"value": round(tps, 3), "unit": "prompt tokens/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": f"{n} prompt tokens fed one at a time as the reference does ({dt * 1e3:.1f} ms each)"}
        prompts = 1 if tp else ws
        print(json.dumps({
            "metric": "prefill_tokens_per_s", "value": round(T * prompts * args.steps / (ms / 1e3), 1),
            "unit": "prompt tokens/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ttft_ms, "ttft_ms": ttft_ms, "higher_is_better": True,
            "scaling": "strong" if tp else "weak",
            "vs_baseline": None, "dtype": "int16xint8->int32", "data": "synthetic (random ids, random-init weights)",
            "config": {"workload": f"qwen3vl2b_text_prefill_T{T}", "order": "M=T tensor-core products (reference M>1 order)",
                       "parallelism": (f"tp{ws}: every product split by output column, NCCL all-gather"
                                       if tp else f"dp{ws} (one prompt per rank)")},
            "clocks": clk.summary(), "cpu_baseline": cpu,
        }))
    if ws > 1:
        dist.destroy_process_group()


def run_decode_batch(w, B, args, dev):
    """Decode tokens/s at B requests on this GPU (tensor-core products in the
    reference's M>1 order, one graph-captured step per token), for the
    "batch 32" half of the headline metric."""
    import torch
    import qvl_b200.decoder as D
    steps = args.batch32_steps
    max_ctx = PROMPT_CTX + args.warmup + steps + 8
    dec = D.TextDecoder(w, max_batch=B, max_ctx=max_ctx, device=dev, attn_order=args.attn_order)
    D.fill_kv_random(dec, PROMPT_CTX, seed=B)
    dec.tokens.copy_(torch.arange(B, dtype=torch.int32, device=dev) * 7919 % dec.cfg.vocab)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        dec.step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            dec.step()
        dec.positions.fill_(PROMPT_CTX)
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    w_bytes = sum(v.numel() * v.element_size() for v in w.t.values())
    out = {"tokens_per_s": round(B / (ms / 1e3), 1), "ms_per_step": round(ms, 4), "batch": B, "steps": steps,
           "order": "tiled (M=32 tcgen05 products, reference M>1 order)" if dec.use_tc else "lane8",
           "step_hbm_gbs": round(w_bytes / (ms / 1e3) / 1e9, 1)}
    del dec, g
    torch.cuda.empty_cache()
    return out


def run_config4(w, args, dev):
    """BASELINE config 4, one request end to end on this GPU: a synthetic
    448x448 image (host patches, pinned) and 256 text ids go to the device,
    the vision tower runs (784 patches -> 196 image tokens + deep stack),
    the 454-token prompt pass (tensor-core products, image embeddings and
    deep-stack rows in place), then N greedy tokens (one launch each), and
    the ids come back to the host.  Synthetic weights (text: the bench's
    decoder weights; vision: random fp16)."""
    import numpy as np
    import torch
    import qvl_b200.decoder as D
    import qvl_b200.modelfile as MF
    import qvl_b200.vision as V
    n_new = args.config4_tokens
    hdr = MF.qwen3vl_2b_header()
    rng = np.random.default_rng(4)
    img = rng.integers(0, 256, (448, 448, 3), dtype=np.uint8)
    patches, gh, gw = V.image_patches(img)
    enc = V.VisionEncoder.random(hdr, gh, gw, device=dev, seed=4)
    n_img = enc.D
    prompt = ([hdr["vision_start_token_id"]] + [hdr["image_token_id"]] * n_img + [hdr["vision_end_token_id"]] +
              rng.integers(0, 151643, 256).tolist())
    T = len(prompt)
    dec = D.TextDecoder(w, max_batch=1, max_ctx=T + n_new + 8, device=dev, persistent=True,
                        attn_order=args.attn_order)
    patches_h = torch.from_numpy(patches).pin_memory()
    prompt_h = torch.tensor(prompt, dtype=torch.int32).pin_memory()
    patches_d = torch.empty(patches.shape, dtype=torch.float32, device=dev)
    prompt_d = torch.empty(T, dtype=torch.int32, device=dev)
    ids_d = torch.empty(n_new, dtype=torch.int32, device=dev)
    ids_h = torch.empty(n_new, dtype=torch.int32).pin_memory()
    stream = torch.cuda.Stream(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]

    def request():
        with torch.cuda.stream(stream):
            ev[0].record(stream)
            patches_d.copy_(patches_h, non_blocking=True)
            prompt_d.copy_(prompt_h, non_blocking=True)
            emb, deep = enc.forward(patches_d)
            ev[1].record(stream)
            dec.prefill(prompt_d, image_embeds=emb, deepstack=deep)
            ev[2].record(stream)
            for i in range(n_new):
                dec.step()
                ids_d[i:i + 1].copy_(dec.tokens[:1])
            ev[3].record(stream)
            ids_h.copy_(ids_d, non_blocking=True)
            ev[4].record(stream)
        stream.synchronize()

    request()                                    # warm-up (kernel set-up, workspaces)
    t0 = time.perf_counter()
    request()
    wall = time.perf_counter() - t0
    out = {"workload": "config4: 448x448 image (196 image tokens) + 256 text ids -> "
                       f"{n_new} greedy tokens, batch 1, one request",
           "request_s": round(wall, 4), "generated_tokens_per_s": round(n_new / wall, 1),
           "vision_ms": round(ev[0].elapsed_time(ev[1]), 3), "prefill_ms": round(ev[1].elapsed_time(ev[2]), 3),
           "decode_tokens_per_s": round(n_new / (ev[2].elapsed_time(ev[3]) / 1e3), 1),
           "prompt_tokens": T, "h2d_bytes": int(patches.nbytes + 4 * T), "d2h_bytes": 4 * n_new}
    del dec, enc
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist
    qvl = import_qvl()
    import qvl_b200.decoder as D
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    cfg = D.TextConfig()
    B = args.batch
    max_ctx = PROMPT_CTX + args.warmup + args.steps + 8
    w = D.TextWeights.random(cfg, seed=rank, device=dev)
    persistent = args.engine == "persistent" or (args.engine == "auto" and B == 1 and max_ctx <= 8192)
    dec = D.TextDecoder(w, max_batch=B, max_ctx=max_ctx, device=dev, persistent=persistent,
                        attn_order=args.attn_order)
    D.fill_kv_random(dec, PROMPT_CTX, seed=rank)
    dec.tokens.copy_(torch.arange(B, dtype=torch.int32, device=dev) * 7919 % cfg.vocab)
    stream = torch.cuda.Stream(dev)
    # capture one decode token; replays advance positions on the device
    with torch.cuda.stream(stream):
        dec.step()                      # first call: kernel attribute set-up outside capture
        torch.cuda.synchronize()
        dec.positions.fill_(PROMPT_CTX)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            dec.step()
        torch.cuda.synchronize()
        dec.positions.fill_(PROMPT_CTX)

    def timed():
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                g.replay()
            torch.cuda.synchronize()
            if ws > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        per_rank = [ms]
        if ws > 1:
            t = torch.tensor([ms], device=dev)
            parts = [torch.empty_like(t) for _ in range(ws)]
            dist.all_gather(parts, t)
            per_rank = [float(p.item()) for p in parts]
            ms = max(per_rank)
        return ms, per_rank

    with ClockSampler(local) as clk:
        ms, per_rank_ms = timed()
    ms_step = ms / args.steps
    value = B * ws * args.steps / (ms / 1e3)
    # weights streamed per step + KV read per step (fp16, mean context)
    w_bytes = sum(v.numel() * v.element_size() for v in w.t.values())
    mean_ctx = PROMPT_CTX + args.warmup + args.steps / 2
    kv_bytes = B * cfg.layers * 2 * cfg.kv_heads * cfg.head_dim * 2 * mean_ctx
    step_gbs = (w_bytes + kv_bytes) / (ms_step / 1e3) / 1e9

    # e2e through the public API: pinned token ids -> device, one decode step,
    # greedy ids -> pinned host; the host waits for every token.
    tok_h = torch.zeros(B, dtype=torch.int32).pin_memory()
    out_h = torch.zeros(B, dtype=torch.int32).pin_memory()
    dec.positions.fill_(PROMPT_CTX)
    with torch.cuda.stream(stream):
        ge = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ge, stream=stream):
            dec.tokens.copy_(tok_h, non_blocking=True)
            dec.step()
            out_h.copy_(dec.tokens, non_blocking=True)
        torch.cuda.synchronize()
        dec.positions.fill_(PROMPT_CTX)
        for _ in range(args.warmup):
            ge.replay()
            stream.synchronize()
            tok_h.copy_(out_h)
        if ws > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ge.replay()
            stream.synchronize()
            tok_h.copy_(out_h)           # the host feeds back the generated ids
        e2e_s = time.perf_counter() - t0
    if ws > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = B * ws * args.steps / e2e_s

    gemv_gbs, gemv_bytes_per_launch, gemv_s_per_launch, _ = decode_gemv_roofline(dec)
    lib = qvl.load_library()
    tc_mode = dec.use_tc
    attn_k = 1 if max_ctx <= 8192 else 3          # cluster kernel / split-K trio
    if args.attn_order == "reference":
        attn_k = 2                                  # ordered scores + softmax/P.V
    if dec.use_tc:   # rmsnorm, split+3 GEMMs, rope, attention, quantize, split+GEMM, rmsnorm,
        # split+2 GEMMs+swiglu, quantize, split+GEMM
        per_layer, head = 1 + 4 + 1 + attn_k + 1 + 2 + 1 + 4 + 1 + 2, 1 + 1 + 2 + 1
    elif B == 1:  # qkv, rope, attention(+quantise tail), o(+norm tail), gate/up(+quant tail), down(+norm tail)
        per_layer, head = 5 + (1 if attn_k == 1 else attn_k + 1), 1 + 1 + 1 + 1  # embedding, first rmsnorm, LM head, argmax
    elif B <= 4:  # fast GEMV without the fused tails
        per_layer, head = 9 + attn_k, 1 + 2 + 1
    else:        # 8-row GEMV tiles, separate norms / swiglu
        tiles = (B + 7) // 8
        per_layer, head = 5 + attn_k + 7 * tiles, 1 + 1 + tiles + 1
    launches = args.steps * (cfg.layers * per_layer + head)
    if persistent:
        launches = args.steps * dec.kernels_per_step()
        aborted = qvl.text_decode_aborted(dec.pws)
        if aborted:
            raise RuntimeError("persistent decode: a grid barrier wait timed out")
    batch32 = None
    config4 = None
    if rank == 0 and args.batch == 1 and args.batch32_steps > 0:
        del g, ge
        batch32 = run_decode_batch(w, 32, args, dev)
    if rank == 0 and args.batch == 1 and args.config4_tokens > 0:
        config4 = run_config4(w, args, dev)
    gemv0 = run_gemv(dev) if rank == 0 else None
    if rank == 0:
        peak, peak_kind = load_peaks()
        gemv_roof = {"bound": "hbm", "achieved": round(gemv_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gemv_gbs / peak, 4), "peak_kind": peak_kind,
                     "traffic": profile_traffic("gemv_i8_decode"), "kernel": "gemv_i8 (decode GEMVs)",
                     "algorithmic_bytes_per_launch": round(gemv_bytes_per_launch),
                     "avg_launch_us": round(gemv_s_per_launch * 1e6, 3)}
        if persistent:
            # one launch per token: its algorithmic bytes are the step's
            # weights plus the KV rows read at the mean context
            roofline = {"bound": "hbm", "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(step_gbs / peak, 4), "peak_kind": peak_kind,
                        "traffic": profile_traffic("decode_persistent"),
                        "kernel": "decode_persistent (whole token, one cooperative launch)",
                        "algorithmic_bytes_per_launch": round(w_bytes + kv_bytes),
                        "avg_launch_us": round(ms_step * 1e3, 3), "gemv_chain": gemv_roof}
        else:
            roofline = gemv_roof
        cpu = None
        if args.cpu_seconds > 0:
            del dec
            torch.cuda.empty_cache()
            tps, n, dt = cpu_decode_rate(args, seconds=args.cpu_seconds)
            import oracle
            cpu = {"value": round(tps, 3), "unit": "tokens/s", "cores": os.cpu_count(),
                   "kind": "reference" if oracle.ref_available() else "port",
                   "sample": f"{n} decode tokens of one request ({dt * 1e3:.1f} ms each), same model shape: "
                             f"the reference's own loader + forward_text compiled from its sources (FP32 KV), "
                             f"OpenMP on all cores"}
        print(json.dumps({
            "metric": "decode_tokens_per_s", "value": round(value, 2), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int16xint8->int32", "data": "synthetic (random-init int8 weights, seed = rank)",
            "config": dict(decode_config(args, ws),
                           engine="persistent (one launch per token)" if persistent else "launch chain",
                           attn_order=("reference (the reference's summation order: logits bit-identical "
                                       "to its operators)") if args.attn_order == "reference"
                           else "fast (context split over CTAs)",
                           batch_order="tiled (M=B tcgen05, reference M>1 order)" if tc_mode
                           else "lane8 (each request in the reference M=1 order)"),
            "roofline": roofline,
            "step_hbm_gbs": round(step_gbs, 1),
            "per_rank_tokens_per_s": [round(B * args.steps / (m / 1e3), 1) for m in per_rank_ms],
            "e2e": {"value": round(e2e, 3), "unit": "tokens/s", "h2d_bytes_per_step": 4 * B,
                    "d2h_bytes_per_step": 4 * B},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "gemv_config0": gemv0,
            "batch32": batch32,
            "config4": config4,
        }))
    if ws > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--batch", type=int, default=1, help="decode requests per GPU")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "prefill_gemm", "gemv", "attention", "swiglu"])
    ap.add_argument("--attn-order", default="reference", choices=["reference", "fast"],
                    help="decode attention: the reference's summation order (bit-identical logits) or split context")
    ap.add_argument("--tp", action="store_true",
                    help="prefill: split every product of one prompt by output column over the ranks")
    ap.add_argument("--config4-tokens", type=int, default=128,
                    help="greedy tokens of the config-4 request in the bench line (0: skip)")
    ap.add_argument("--batch32-steps", type=int, default=32, help="steps of the batch-32 figure (0: skip)")
    ap.add_argument("--engine", default="auto", choices=["auto", "persistent", "chain"],
                    help="decode: one cooperative launch per token (batch 1) or the per-operator launch chain")
    ap.add_argument("--m", type=int, default=512, help="prefill_gemm: activation rows")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.cpu_seconds == 10.0:
        args.cpu_seconds = 15.0
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill_gemm":
        run_prefill_gemm(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "gemv":
        run_gemv_line(args)
    elif args.workload == "attention":
        run_attention_line(args)
    elif args.workload == "swiglu":
        run_swiglu_line(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
