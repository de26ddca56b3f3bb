"""Benchmark of the Polar Switch hot path on B200.

Default workload: the Qwen3-0.6B-shaped Muon orthogonalization step (BASELINE
config 4): 196 matrices (28 layers x q 2048x1024, k/v 1024x1024, o 1024x2048,
gate/up 3072x1024, down 1024x3072), N(0,1) fp32 from a fixed seed, method
PS2_55, sharded by FLOPs across the ranks with one NCCL all-gather of the FP16
updates. A step is one pass over all 196 matrices. `value` is the algorithmic
TFLOP/s of the whole job (PS2-55 FLOPs (6a+10)n^3 per matrix over the step
time, max over ranks).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload qwen|gemma|nanogpt|single]
    torchrun --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference ...     # the reference's CPU path, timed on host cores

Prints one JSON line (rank 0).
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "polar-switch_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

WORKLOADS = {
    "qwen": dict(desc="Qwen3-0.6B Muon step (BASELINE config 4)", method="PS2_55"),
    "gemma": dict(desc="Gemma-3-1B Muon step (BASELINE config 5)", method="PS3_55"),
    "nanogpt": dict(desc="Modded-NanoGPT Muon batch (BASELINE config 3)", method="PS3_55"),
    "single": dict(desc="single 8192x8192 matrix (BASELINE config 2, published heatmap point)",
                   method="PS2_55"),
    "stress": dict(desc="stress batch 4 x 8192 x 28672 (BASELINE config 5); on more GPUs than "
                        "matrices each matrix is split across ranks", method="PS3_55"),
}


def bank_shapes(workload):
    from polar_switch import distributed as pd
    if workload == "qwen":
        return pd.qwen3_0_6b_banks()
    if workload == "gemma":
        return pd.gemma3_1b_banks()
    if workload == "nanogpt":
        return pd.nanogpt_banks()
    if workload == "single":
        return [(1, 8192, 8192)]
    if workload == "stress":
        return [(4, 8192, 28672)]
    raise ValueError(workload)


def make_banks(shapes, device, seed=0, scale=1.0):
    """Seeded N(0, scale^2) fp32 banks, generated on the device (deterministic per seed)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return [torch.randn(L, r, c, generator=g, device=device, dtype=torch.float32) * scale
            for L, r, c in shapes]


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per matrix of a
# kernel class at one matrix size, from ncu captures of the current kernels:
# profiles/dram_traffic.json maps "<class>_n<n>" to {"bytes_per_matrix": B,
# "capture": "<what was captured>"}; a launch's traffic is B times the number
# of matrices it processes. Absent file or key: traffic is reported as null.
def load_traffic_table():
    try:
        with open(os.path.join(ROOT, "profiles", "dram_traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def roofline_entry(name, v, steps, n_dom, clocks, peaks, traffic_table):
    """Roofline of one kernel class from its profiled launches.

    achieved = algorithmic FLOPs (or bytes) per launch / mean launch time. The
    bound is taken from arithmetic intensity: FLOPs per DRAM byte (measured
    traffic when the table has it, else the algorithmic bytes) against the
    ridge point peak_flops / peak_bandwidth. The tensor peak is the measured
    burst figure when the run's SM clock median sat at its maximum (a kernel
    timed in bursts), else the sustained figure; the HBM peak is the measured
    copy bandwidth. Fallbacks (no MEASURED_PEAKS.json): 1590 / 1400 TFLOP/s and
    6650 GB/s.
    """
    burst = peaks.get("bf16_tflops")
    sustained = peaks.get("bf16_tflops_sustained")
    hbm = peaks.get("hbm_gbs")
    src = "measured (MEASURED_PEAKS.json)"
    if burst is None or sustained is None or hbm is None:
        burst, sustained, hbm, src = 1590.0, 1400.0, 6650.0, "fallback"
    at_max = (clocks.get("sm_mhz") and clocks.get("sm_max_mhz")
              and clocks["sm_mhz"] >= 0.97 * clocks["sm_max_mhz"])
    tpeak, tname = (burst, "burst") if at_max else (sustained, "sustained")
    launches = max(v["launches"], 1)
    sec = v["ms"] * 1e-3 / launches
    flops = v["flops"] / launches
    alg_bytes = v["bytes"] / launches
    traffic, traffic_src = None, None
    key = f"{name}_n{n_dom}"
    if key in traffic_table and flops:
        mats = flops / traffic_table[key].get("flops_per_matrix", float(n_dom) ** 3)
        traffic = traffic_table[key]["bytes_per_matrix"] * mats
        traffic_src = f"ncu dram read+write of {traffic_table[key]['capture']}, scaled to {mats:.0f} matrices"
    ai = flops / (traffic or alg_bytes) if (traffic or alg_bytes) else float("inf")
    ridge = tpeak * 1e12 / (hbm * 1e9)
    tensor = {"achieved": flops / sec / 1e12, "peak": tpeak, "frac": flops / sec / 1e12 / tpeak}
    mem = {"achieved": (traffic or alg_bytes) / sec / 1e9, "peak": hbm,
           "frac": (traffic or alg_bytes) / sec / 1e9 / hbm}
    bound = "hbm" if ai < ridge else "tensor"
    main = mem if bound == "hbm" else tensor
    label = "ps_circuit_pair_kernel (whole circuits)" if name == "circuit" else f"ps_gemm ({name})"
    return {"bound": bound, "kernel": label, "achieved": main["achieved"],
            "peak": main["peak"], "unit": "GB/s" if bound == "hbm" else "TFLOP/s", "frac": main["frac"],
            "peak_source": f"{src}: {'HBM copy' if bound == 'hbm' else 'bf16 ' + tname}",
            "traffic": traffic, "traffic_source": traffic_src,
            "arithmetic_intensity": ai, "ridge": ridge,
            "tensor_frac": tensor["frac"], "tensor_tflops": tensor["achieved"],
            "hbm_frac": mem["frac"], "hbm_gbs": mem["achieved"],
            "launches_per_step": v["launches"] / steps, "ms_per_launch": sec * 1e3}


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region: one
    `nvidia-smi -lms` process samples every `period_ms` until the block exits;
    entering waits (up to 5 s) for its first sample so the samples cover the
    region that follows."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index, period_ms=50):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.samples = []
        self._proc = None
        self._thread = None
        self._first = threading.Event()

    def _read(self):
        for line in self._proc.stdout:
            vals = [v.strip() for v in line.strip().split(",")]
            if len(vals) >= 9:
                self.samples.append(vals)
                self._first.set()

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", f"-lms={self.period_ms}"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return self
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        self._first.wait(5.0)
        self.samples.clear()  # keep only samples taken from here on
        return self

    def __exit__(self, *exc):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        smax = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(self.samples)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(value, world, device):
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_reference_sample(shapes, method, budget_s=12.0, max_layers=None):
    """Time the reference CPU path (a port: POLAR_EXPRESS via torch.bmm/baddbmm on
    FP16, reference polar_switch/__init__.py:48-63,180-182) on a bounded sample:
    whole layers (one matrix of each bank per layer), repeated until `budget_s`.
    Returns (seconds per full workload step extrapolated, sample description)."""
    sys.path.insert(0, ROOT)
    from oracle.reference_cpu import torch_pe
    from polar_switch import circuit_flops, coefficients
    layers = min(L for L, _, _ in shapes)
    per_layer = [(max(1, L // layers), r, c) for L, r, c in shapes]
    g = torch.Generator().manual_seed(1)
    mats = [torch.randn(k, r, c, generator=g) for k, r, c in per_layer]
    torch_pe(mats[0][:1, :64, :64])  # warm-up of the thread pool
    t0 = time.perf_counter()
    reps = 0
    while True:
        for M in mats:
            torch_pe(M)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or (max_layers and reps >= max_layers):
            break
    per_layer_s = el / reps
    step_s = per_layer_s * layers
    desc = (f"{reps} layer(s) of {sum(k for k, _, _ in per_layer)} matrices "
            f"({', '.join(f'{k}x{r}x{c}' for k, r, c in per_layer)}), {el:.1f} s, "
            f"extrapolated x{layers} layers; reference CPU path = POLAR_EXPRESS in torch FP16 bmm "
            f"(requested {method}); FLOPs counted as the requested {method} circuit")
    return step_s, desc


def run_reference(args, world, rank):
    """--impl reference: the reference CPU implementation on the host cores."""
    if rank != 0:
        return
    shapes = bank_shapes(args.workload)
    method = WORKLOADS[args.workload]["method"]
    from polar_switch import circuit_flops, coefficients
    table = getattr(coefficients, method)
    flops = sum(L * circuit_flops(table, r, c) for L, r, c in shapes)
    # torchrun sets OMP_NUM_THREADS=1 per rank; rank 0 runs alone here and
    # takes every core it may run on.
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    torch.set_num_threads(max(cores, 1))
    threads = torch.get_num_threads()
    times = []
    for i in range(args.warmup + args.steps):
        s, desc = cpu_reference_sample(shapes, method, budget_s=args.ref_budget, max_layers=1)
        if i >= args.warmup:
            times.append(s)
    step_s = statistics.median(times)
    value = flops / step_s / 1e12
    # Each "step" of this arm runs one layer of the workload (a bounded
    # sample); ms_per_step is that sample's time, and the full step's time is
    # the extrapolation over all layers, from which `value` is computed.
    layers = min(L for L, _, _ in shapes)
    line = {
        "impl": "reference", "metric": "muon_step_orthogonalize_tflops" if args.workload != "single"
        else "orthogonalize_tflops", "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3 / layers,
        "ms_per_full_step_extrapolated": step_s * 1e3, "sample_per_step": f"1 of {layers} layers",
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic", "config": config_dict(args, shapes, method),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(args, shapes, method):
    total = sum(L for L, _, _ in shapes)
    in_bytes = sum(L * r * c * 4 for L, r, c in shapes)
    return {"workload": f"{args.workload}: {WORKLOADS[args.workload]['desc']}", "method": method,
            "matrices": total, "banks": [list(s) for s in shapes], "input": "fp32 N(0,1), seed 0",
            "l2": f"inputs larger than L2 ({in_bytes / 1e9:.2f} GB per step vs 126 MB L2)",
            "parallelism": f"matrix-sharded x{args.gpus}, FP16 updates gathered over NVLink"}


def run_kernel(args):
    """--kernel: time one kernel class alone on the workload's batched shapes
    (also the small, self-contained command used for ncu captures)."""
    from polar_switch import cuda_ops
    from polar_switch import _native as nat
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    shapes = bank_shapes(args.workload)
    g = torch.Generator(device=device).manual_seed(0)
    if args.kernel == "circuit":
        # the whole-circuit kernel on the workload's banks (one launch per call)
        from polar_switch import make_polynomial_orthogonalizer
        L0 = args.L or None
        banks = [torch.randn(L0 or L, r, c, generator=g, device=device) for L, r, c in shapes]
        polar = make_polynomial_orthogonalizer(WORKLOADS[args.workload]["method"])
        nat.set_circuit_kernel(1)
        fn = lambda: polar.grouped(banks)  # noqa: E731
        desc = f"circuit ({WORKLOADS[args.workload]['method']}) banks {[tuple(b.shape) for b in banks]}"
    elif args.kernel == "chain":
        # all inner iterations of the workload's squares as the circuit runs
        # them: whole PS2-55 circuits on L square matrices of the bank's n
        from polar_switch import make_polynomial_orthogonalizer
        n = min(shapes[args.bank][1:])
        L = args.L or sum(Lg for Lg, r, c in shapes if min(r, c) == n)
        X = torch.randn(L, n, n, generator=g, device=device)
        Y = torch.empty_like(X)
        polar = make_polynomial_orthogonalizer("PS2_55")
        nat.set_circuit_kernel(0)  # per-stage launches: the chain runs the inner iterations
        fn = lambda: polar(X, out=Y)  # noqa: E731
        desc = f"chain (PS2_55 circuits) L={L} n={n}"
    elif args.kernel in ("muon_direction", "muon_update"):
        # Muon's elementwise kernels on one bank of the workload (BF16 parameters,
        # gradients and momentum; the stacked direction in BF16)
        from polar_switch import muon as pm
        L, r, c = shapes[args.bank]
        L = args.L or L
        grads = [torch.randn(r, c, generator=g, device=device).bfloat16() for _ in range(L)]
        moms = [torch.zeros(r, c, device=device, dtype=torch.bfloat16) for _ in range(L)]
        params = [torch.randn(r, c, generator=g, device=device).bfloat16() for _ in range(L)]
        upd = torch.randn(L, r, c, generator=g, device=device).bfloat16()
        fn = ((lambda: pm.muon_directions(grads, moms, 0.95, torch.bfloat16))
              if args.kernel == "muon_direction" else (lambda: pm.muon_update(params, upd, 0.999, -0.01)))
        desc = f"{args.kernel} L={L} {r}x{c} bf16"
    elif args.kernel in ("square", "sym_product"):
        n = min(shapes[args.bank][1:])
        L = args.L or sum(Lg for Lg, r, c in shapes if min(r, c) == n)
        X = torch.randn(L, n, 2 * n, generator=g, device=device)
        A = torch.empty(L, n, n, device=device, dtype=torch.float16)
        cuda_ops.gram(cuda_ops.normalize(X, 1e-7), False, A)
        C, out = A.clone(), torch.empty_like(A)
        P2 = A.clone()
        del X
        torch.cuda.empty_cache()
        fn = ((lambda: cuda_ops.square(A, C, out, 1.0, 0.5, 0.25)) if args.kernel == "square"
              else (lambda: cuda_ops.sym_product(A, P2, C, out, 1.0, 0.5, 0.25)))
        desc = f"{args.kernel} L={L} n={n}"
    else:
        L, r, c = shapes[args.bank]
        L = args.L or L
        X = cuda_ops.normalize(torch.randn(L, r, c, generator=g, device=device), 1e-7)
        n = min(r, c)
        B = torch.empty(L, n, n, device=device, dtype=torch.float16)
        cuda_ops.gram(X, r > c, B)
        if args.kernel == "gram":
            fn = lambda: cuda_ops.gram(X, r > c, B)  # noqa: E731
        elif args.kernel == "apply":
            Y = torch.empty_like(X)
            fn = lambda: cuda_ops.apply(X, B, r > c, 0.0, out=Y)  # noqa: E731
        else:
            X32 = torch.randn(L, r, c, generator=g, device=device)
            Xh = torch.empty(L, r, c, device=device, dtype=torch.float16)
            fn = lambda: cuda_ops.normalize(X32, 1e-7, out=Xh)  # noqa: E731
        desc = f"{args.kernel} L={L} {r}x{c}"
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    nat.profile_enable(True)
    for _ in range(args.steps):
        fn()
    prof = nat.profile_read()
    nat.profile_enable(False)
    kind = {"square": "square", "sym_product": "square", "chain": "square", "muon_direction": "other",
            "muon_update": "other"}.get(args.kernel, args.kernel)
    v = prof[kind]
    ms = v["ms"] / max(v["launches"], 1)
    print(json.dumps({"kernel": desc, "ms_per_launch": ms, "launches": v["launches"],
                      "tflops": v["flops"] / (v["ms"] * 1e-3) / 1e12 if v["flops"] else None,
                      "gbs": v["bytes"] / (v["ms"] * 1e-3) / 1e9}), flush=True)


# Published single-GPU medians (ms) of the reference on one B200 (its README's timing
# heatmap): shape (batch, rows, cols) -> {method: ms}.
PUBLISHED_MS = {
    (1, 8192, 8192): {"PS2_55": 7.47, "PS3_55": 7.47},
    (1, 16384, 16384): {"PS2_55": 55.7, "PS3_55": 56.0},
    (1, 14336, 4096): {"PS2_55": 1.87, "PS3_55": 1.86, "GNS": 2.24},
    (1, 28672, 8192): {"PS2_55": 13.9, "PS3_55": 14.0, "GNS": 16.3},
    (1, 53248, 16384): {"PS2_55": 102.0, "PS3_55": 103.0, "GNS": 120.0},
    (1, 4096, 14336): {"PS2_55": 1.86, "PS3_55": 1.88, "GNS": 2.25},
    (1, 8192, 28672): {"PS2_55": 13.9, "PS3_55": 13.9, "GNS": 16.3},
    (1, 16384, 53248): {"PS2_55": 102.0, "PS3_55": 103.0, "GNS": 119.0},
    (64, 4096, 4096): {"PS2_55": 59.8, "PS3_55": 59.4},
    (216, 7168, 2048): {"PS2_55": 55.7, "PS3_55": 55.0, "GNS": 65.9},
    (128, 8192, 1024): {"PS2_55": 9.70, "PS3_55": 9.42, "GNS": 10.9},
    (216, 2048, 7168): {"PS2_55": 55.9, "PS3_55": 54.1, "GNS": 65.6},
    (128, 1024, 8192): {"PS2_55": 9.72, "PS3_55": 9.34, "GNS": 10.8},
}


def time_other_configs(device, warmup, calls=10):
    """BASELINE configs 3 and 5 on one GPU, timed alongside the headline: the
    NanoGPT batch (48 x 768^2 + 12 x 768x3072 + 12 x 3072x768, N(0, 0.02^2))
    and the Gemma-3-1B step (26 layers), both PS3-55, each one grouped call
    into FP16 outputs, median of `calls` calls timed alone with CUDA events
    after a warm-up; FLOPs as the reference counts them."""
    from polar_switch import circuit_flops, coefficients, make_polynomial_orthogonalizer
    out = {}
    for name, scale in (("nanogpt", 0.02), ("gemma", 1.0)):
        shapes = bank_shapes(name)
        method = WORKLOADS[name]["method"]
        banks = make_banks(shapes, device, seed=0, scale=scale)
        outs = [torch.empty(b.shape, dtype=torch.float16, device=device) for b in banks]
        polar = make_polynomial_orthogonalizer(method)
        flops = sum(L * circuit_flops(getattr(coefficients, method), r, c) for L, r, c in shapes)
        for _ in range(max(warmup, 3)):
            polar.grouped(banks, outs=outs)
        torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        times = []
        for _ in range(calls):
            s.record()
            polar.grouped(banks, outs=outs)
            e.record()
            e.synchronize()
            times.append(s.elapsed_time(e))
        times.sort()
        ms = times[len(times) // 2]
        out[name] = {"workload": WORKLOADS[name]["desc"], "method": method,
                     "matrices": sum(L for L, _, _ in shapes), "median_ms": round(ms, 4),
                     "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "calls": calls}
        del banks, outs
    return out


def time_single_8192(device, warmup, calls=15):
    """The 8192 x 8192 PS2-55 circuit of the reference's published B200 heatmap
    (7.47 ms median, README.md:77-81), timed call by call with CUDA events on
    FP16 N(0, 1) input; median over `calls` after a warm-up."""
    from polar_switch import circuit_flops, coefficients, make_polynomial_orthogonalizer
    g = torch.Generator(device=device).manual_seed(0)
    X = torch.randn(8192, 8192, generator=g, device=device, dtype=torch.float16)
    polar = make_polynomial_orthogonalizer("PS2_55")
    Y = torch.empty_like(X)
    flops = circuit_flops(coefficients.PS2_55, 8192, 8192)
    for _ in range(max(warmup, 3)):
        polar(X, out=Y)
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    with ClockSampler(device.index or 0) as clocks:
        for _ in range(calls):
            s.record()
            polar(X, out=Y)
            e.record()
            e.synchronize()
            times.append(s.elapsed_time(e))
    times.sort()
    ms = times[len(times) // 2]
    del X, Y
    torch.cuda.empty_cache()
    return {"shape": [8192, 8192], "method": "PS2_55", "input": "fp16 N(0,1), seed 0",
            "calls": calls, "median_ms": ms, "min_ms": times[0], "tflops": flops / (ms * 1e-3) / 1e12,
            "published_ms": 7.47, "vs_published": 7.47 / ms, "clocks": clocks.summary()}


# Upper end of each method's published singular-value interval for inputs
# with sigma in [1e-3, 1] (reference README.md:64-73; GNS polar_switch/README.md).
DESIGN_TOP = {"PS2_55": 1.106236, "PS3_55": 1.080954, "GNS": 1.212979}


def sweep_output_check(Y, method, iters=30):
    """Cheap sanity check of a sweep output: finite, largest singular value (by
    power iteration on Y^T Y in FP32, per matrix) at most the method's design
    top plus 1e-2, and mean squared singular value in [0.5, 1.3]. A skipped or
    duplicated tile breaks at least one of these."""
    Yf = Y.float()
    finite = bool(torch.isfinite(Yf).all())
    n = min(Yf.shape[-2:])
    gen = torch.Generator(device=Y.device).manual_seed(5)
    v = torch.randn(Yf.shape[0], Yf.shape[-1], 1, device=Y.device, generator=gen)
    for _ in range(iters):
        v = Yf.mT @ (Yf @ v)
        v = v / v.norm(dim=(-2, -1), keepdim=True)
    smax = float((Yf @ v).norm(dim=(-2, -1)).max())
    fro2 = float((Yf.pow(2).sum(dim=(-2, -1)) / n).mean())
    ok = finite and smax <= DESIGN_TOP.get(method, 1.25) + 1e-2 and 0.5 <= fro2 <= 1.3
    return {"finite": finite, "sigma_max_est": round(smax, 5), "mean_sigma2": round(fro2, 4), "ok": ok}


def run_sweep(args):
    """--sweep: median latency of whole circuits on the shapes whose reference
    latency is published, one JSON line per (shape, method). Inputs are FP16
    N(0,1) (the kernels have no data-dependent paths); at least --steps timed
    calls each after --warmup, every call timed alone with CUDA events."""
    from polar_switch import circuit_flops, coefficients, make_polynomial_orthogonalizer
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device).manual_seed(0)
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    peak = peaks.get("bf16_tflops", 1590.0)
    for shape, pub in PUBLISHED_MS.items():
        X = torch.randn(shape, generator=g, device=device, dtype=torch.float16)
        for method in [m for m in ("PS2_55", "PS3_55", "GNS") if m in pub and m in args.methods]:
            polar = make_polynomial_orthogonalizer(method)
            if method == "GNS":  # the reference's count for GNS: (6a + 14) n^3
                n, m = min(shape[1:]), max(shape[1:])
                flops = shape[0] * (6 * m / n + 14) * n ** 3
            else:
                flops = shape[0] * circuit_flops(getattr(coefficients, method), shape[1], shape[2])
            # Warm up by time as well as by count: clocks take a while to settle
            # after the previous (possibly power-capped) shape.
            t_end = time.time() + 0.5
            for i in range(max(args.warmup, 1000)):
                polar(X)
                torch.cuda.synchronize()
                if i + 1 >= args.warmup and time.time() > t_end:
                    break
            times = []
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(0) as clocks:
                for _ in range(args.steps):
                    s.record()
                    polar(X)
                    e.record()
                    e.synchronize()
                    times.append(s.elapsed_time(e))
            times.sort()
            ms = times[len(times) // 2]
            check = sweep_output_check(polar(X), method)
            print(json.dumps({"shape": list(shape), "method": method, "median_ms": round(ms, 4),
                              "output_check": check,
                              "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                              "frac_of_measured_burst_peak": round(flops / (ms * 1e-3) / 1e12 / peak, 3),
                              "published_ms": pub[method],
                              "speedup_vs_published": round(pub[method] / ms, 3),
                              "clocks": clocks.summary()}), flush=True)
        del X
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="qwen", choices=sorted(WORKLOADS))
    ap.add_argument("--ref-budget", type=float, default=12.0, help="seconds of CPU work per reference sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--e2e-buckets", type=int, default=32,
                    help="1 GPU: buckets of the end-to-end host step (copies overlap the circuits bucket by bucket)")
    ap.add_argument("--no-single", dest="single", action="store_false",
                    help="skip the 8192 x 8192 PS2-55 point timed after the step at N = 1")
    ap.add_argument("--kernel", choices=["square", "sym_product", "gram", "apply", "normalize", "chain",
                                         "circuit", "muon_direction", "muon_update"],
                    help="time one kernel class alone (for profiling) instead of the whole step")
    ap.add_argument("--bank", type=int, default=0, help="bank of the workload used by --kernel")
    ap.add_argument("--L", type=int, default=0, help="--kernel: override the number of matrices")
    ap.add_argument("--buckets", default=None,
                    help="multi-GPU: bucket count, or comma-separated cost fractions, of the "
                         "gather/compute overlap (default: auto)")
    ap.add_argument("--gemm-ctas", type=int, default=None,
                    help="multi-GPU: cap on GEMM CTAs, leaving SMs to the all-gather")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="enqueue every step from the host instead of replaying a CUDA graph of it")
    ap.add_argument("--transport", default="auto", choices=["auto", "push", "overlap", "copy_engine", "collective"],
                    help="multi-GPU: result tiles stored into the peers' symmetric memory from inside "
                         "the circuit launch (push; auto when it fits), copy-engine pushes into "
                         "symmetric memory, or the NCCL all-gather")
    ap.add_argument("--sweep", action="store_true",
                    help="median circuit latency on every shape with a published reference latency")
    ap.add_argument("--methods", default="PS2_55,PS3_55,GNS", help="--sweep: methods to time")
    args = ap.parse_args()
    if args.sweep:
        run_sweep(args)
        return
    if args.kernel:
        run_kernel(args)
        return
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    from polar_switch import _native as nat
    from polar_switch.distributed import ShardedOrthogonalizer, make_sharded_orthogonalizer

    shapes = bank_shapes(args.workload)
    method = WORKLOADS[args.workload]["method"]
    banks = make_banks(shapes, device, seed=0)
    buckets = args.buckets
    if buckets is not None:
        buckets = [float(f) for f in buckets.split(",")] if "," in buckets else int(buckets)
    step = make_sharded_orthogonalizer(shapes, method=method, group=None, device=device,
                                       world_size=world, rank=rank, buckets=buckets,
                                       gemm_ctas=args.gemm_ctas, transport=args.transport)
    flops = step.flops_total

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for _ in range(args.warmup):
        step(banks)
    barrier()
    run_step = lambda: step(banks)  # noqa: E731
    launches_per_step = None
    if args.graph:
        n0 = nat.launch_count()
        step.capture(banks, warmup=0)
        launches_per_step = nat.launch_count() - n0
        run_step = step.replay
        barrier()

    stream = torch.cuda.current_stream(device)
    t_start, t_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = nat.launch_count()
    with ClockSampler(local) as clocks:
        barrier()
        h0 = time.perf_counter()
        t_start.record(stream)
        for _ in range(args.steps):
            run_step()
        t_stop.record(stream)
        host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
        barrier()
    launches = nat.launch_count() - launches0
    if launches_per_step is not None:
        launches = launches_per_step * args.steps  # graph replays launch the captured kernels
    ms = t_start.elapsed_time(t_stop) / args.steps
    ms = max_over_ranks(ms, world, device)
    value = flops / (ms * 1e-3) / 1e12

    # Per-kernel-class device time from CUDA events around each launch, over
    # a second pass of the same steps (kept out of the headline timing).
    nat.profile_enable(True)
    barrier()
    for _ in range(args.steps):
        step(banks)
    barrier()
    prof = nat.profile_read()
    nat.profile_enable(False)

    # End-to-end through the public API with host buffers (step_host): each
    # rank uploads its own slices from pinned memory bucket by bucket, computes
    # each bucket as its inputs land and downloads the full gathered FP16
    # update set, the transfers overlapping the circuits. With one GPU the
    # host path uses its own plan of --e2e-buckets buckets (the device-resident step above
    # needs none).
    host_banks = [b.cpu().pin_memory() for b in banks]
    host_step = step
    if world == 1:
        host_step = ShardedOrthogonalizer(shapes, method=method, group=None, device=device,
                                          world_size=1, rank=0, buckets=args.e2e_buckets)
    host_out = torch.empty(host_step.recv.numel(), dtype=torch.float16).pin_memory()
    ranges = host_step.local_ranges()
    h2d = sum(count * shapes[g][1] * shapes[g][2] * 4 for g, _, count in ranges)

    def e2e_step():
        host_step.step_host(host_banks, host_out)

    e2e_step()
    barrier()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e_stop.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_stop) / args.e2e_steps, world, device)
    d2h = host_out.numel() * 2
    if host_step is not step:
        host_step.close()

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        step_s, desc = cpu_reference_sample(shapes, method, budget_s=args.ref_budget)
        cpu_baseline = {"value": flops / step_s / 1e12, "unit": "TFLOP/s",
                        "cores": torch.get_num_threads(), "kind": "port", "sample": desc}

    single = others = None
    if world == 1 and args.single and args.workload != "single":
        single = time_single_8192(device, args.warmup)
    if world == 1 and args.single and args.workload == "qwen":
        try:
            others = time_other_configs(device, args.warmup)
        except Exception as e:  # an auxiliary measurement: report it, keep the headline line
            others = {"error": f"{type(e).__name__}: {e}"}

    if rank == 0:
        peaks = load_peaks()
        clock_summary = clocks.summary()
        gemm_kinds = {k: v for k, v in prof.items()
                      if k in ("gram", "square", "apply", "circuit") and v["launches"]}
        dom_name, dom = max(gemm_kinds.items(), key=lambda kv: kv[1]["ms"])
        n_dom = min(min(r, c) for _, r, c in shapes)
        roofline = roofline_entry(dom_name, dom, args.steps, n_dom, clock_summary, peaks, load_traffic_table())
        breakdown = {k: {"ms_per_step": v["ms"] / args.steps, "launches_per_step": v["launches"] / args.steps,
                         "tflops": (v["flops"] / (v["ms"] * 1e-3) / 1e12) if v["ms"] and v["flops"] else None,
                         "gbs": (v["bytes"] / (v["ms"] * 1e-3) / 1e9) if v["ms"] else None}
                     for k, v in prof.items() if v["launches"]}
        line = {
            "metric": "muon_step_orthogonalize_tflops" if args.workload != "single" else "orthogonalize_tflops",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": config_dict(args, shapes, method),
            "roofline": roofline,
            "kernels": breakdown,
            "cpu_baseline": cpu_baseline,
            "clocks": clock_summary,
            "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "host_enqueue_ms_per_step": host_ms,
        }
        if single is not None:
            line["single_8192"] = single
        if others is not None:
            line["other_configs"] = others
        # how the step ran (kept out of `config`, which names the workload and
        # matches the reference arm's)
        line["run"] = {"cuda_graph": bool(args.graph)}
        if world > 1:
            line["run"]["gather"] = {"transport": step.transport, "buckets": len(step.plans),
                                        "phases": getattr(step, "phase_fractions", None),
                                        "split_matrices": type(step).__name__ == "SplitOrthogonalizer",
                                        "gemm_ctas": args.gemm_ctas,
                                        "bucket_matrices": [sum(c for _, _, c in p["pieces"]) for p in step.plans],
                                        "bytes_per_step": step.recv.numel() * 2}
        if args.workload == "single":
            # the reference's published 7.47 ms for one 8192 x 8192 PS2-55 call on a B200
            # (README.md:77-81, figures/fp16_timing_heatmaps.png): 16 * 8192^3 / 7.47 ms = 1177 TFLOP/s
            line["vs_baseline"] = value / 1177.0
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize(device)
        step.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
