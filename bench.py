"""Benchmark of the B200 path on BASELINE.json's metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (the metric's configs[1]): the fused map
y = sin(x^2+3x) plus its calculus-pass derivative dy = cos(x^2+3x)(2x+3),
f32, 2^28 elements per GPU (weak scaling: each rank owns a contiguous 2^28
element shard of an N*2^28 element problem; no data-path collective). One
step = one pass of the hot path over one shard; value = whole-job HBM GB/s
at 12 algorithmic bytes per element. The other BASELINE configs (1, 3, 4,
4', 5) are measured the same way and reported under "configs", with a
`chain` row: the generic chain path (compiled at run time) on the derivative
chain the reference's calculus passes emit for config 2.

Timing: W warm-up steps, then K steps bracketed by a barrier and a device
synchronise, CUDA events on the launching stream, max over ranks. Inputs
(1 GiB per shard) exceed the 126 MB L2, so no flush is needed. nvidia-smi
clocks are sampled during the timed region. `e2e` is the same metric through
the C-ABI host entry (mlkb_module_run_host) on the module the reference's own
compiler emits for config 2 (its Tier-1 pipeline output for y and for the
calculus passes' dy, committed in tests/golden/pipeline.npz, at 2^28
elements), from pinned host buffers, with the H2D copy of x and the D2H copy
of y and dy inside every one of the K steps.

With N > 1 ranks a strong-scaling pass follows: each fixed BASELINE problem
(2^24 / 2^28 elements, 65536 rows, M = 8192, 256 batches) is split over the
N ranks and timed the same way, plus the NCCL all-gather that assembles the
config-2 result. Config 1's shard (a few microseconds of kernel at N = 8) is
timed as one CUDA graph of the K steps over input/output pairs rotated past
twice the L2's size, since an eager loop would time the host's launch cost.

The line is kept short (the full record goes to --detail PATH): the driver
keeps the end of stdout, so `configs` and `strong` come last, in short keys:
v = value, u = unit, ms = ms per step, f = roofline fraction (burst, of the
measured peak), fs = the same after 1.5 s of continuous running, ok = parity.

--impl reference times the reference's own CPU executor (oracle/_ref, built
from the reference sources; the C restatement when absent) on rank 0 with
all host threads, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEED = 0x4D4C4B2B
BYTES_PER_ELEM_MAP2 = 12  # x read + y, dy written (f32)
# A burst starts from an idle GPU; its warm-up lasts at least this long as well
# as W steps, so a kernel of a few microseconds (config 1: ~23 us) is not timed
# while the GPU is still leaving its idle state. 10 ms is far below the tens of
# milliseconds a full-power kernel runs before the power limit engages.
# --min-warm-s 0 (profiling runs) drops it with the other time-based warm-ups.
BURST_WARM_S = 0.010


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic():
    """Per-launch DRAM traffic of each config's dominant kernel, from the
    committed ncu summaries (profiles/traffic.json), if captured."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi sampling during the timed region (every 200 ms)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sms)}


def cpu_reference_map2(n_sample: int, steps: int, default_threads: bool = False):
    """The reference's own executor (or the C port) on a bounded sample of
    the config-2 workload, all host threads (or, with default_threads, the
    executor's own default of at most 4 threads, kernel_buffers.cpp:183-199).
    Returns (GB/s, kind, cores, secs)."""
    import numpy as np

    import oracle
    from mlk2_b200 import kir

    cores = os.cpu_count() or 1
    x = oracle.fill_uniform_f32(n_sample, SEED, 2, -8.0, 8.0).astype(np.float64)
    chains = [kir.SIN_CHAIN, kir.DSIN_CHAIN]
    if oracle.ref_available():
        ex, kind = oracle.ref(), "reference"
        if default_threads:
            cores = min(cores, 4)
        thr = 0 if default_threads else cores
        run = lambda: ex.chain(chains, x, threads=thr)  # noqa: E731
    else:
        ex, kind, cores = oracle.port(), "port", 1
        run = lambda: ex.chain(chains, x)  # noqa: E731
    run()
    times = []
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return n_sample * BYTES_PER_ELEM_MAP2 / t / 1e9, kind, cores, t


def cpu_reference_configs(reps: int = 3):
    """The reference's executor (or the C port) on bounded samples of configs
    1, 3, 4, 4' and 5, timed on this host beside the GPU numbers. Bytes are
    counted at the GPU path's storage width, as the GPU rows are."""
    import numpy as np

    import oracle
    from mlk2_b200 import kir

    cores = os.cpu_count() or 1
    have_ref = oracle.ref_available()
    ex, kind = (oracle.ref(), "reference") if have_ref else (oracle.port(), "port")
    thr = cores if have_ref else 1

    def timed(fn):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    rng = np.random.default_rng(SEED)
    out = {}
    # config 1: the whole workload (2^24 elements)
    n1 = 1 << 24
    x1 = oracle.fill_uniform_f32(n1, SEED, 1, -4.0, 4.0).astype(np.float64)
    t = timed(lambda: ex.chain([kir.SIN_CHAIN], x1, threads=thr))
    out["map1"] = {"value": n1 * 8 / t / 1e9, "unit": "GB/s", "cores": thr, "kind": kind,
                   "sample": "the full 2^24-element config 1, f64 arithmetic, bytes at f32 "
                             "width (8 B/element)"}
    # the generic chain row: the pipeline's derivative chain on 2^24 of 2^28
    import json as _json

    pipe = np.load(os.path.join(ROOT, "tests", "golden", "pipeline.npz"))
    dchain = kir.chains_of(_json.loads(str(pipe["dsin_json"])))[-1]
    xc = oracle.fill_uniform_f32(n1, SEED, 7, -8.0, 8.0).astype(np.float64)
    t = timed(lambda: ex.chain([dchain], xc, threads=thr))
    out["chain"] = {"value": n1 * 8 / t / 1e9, "unit": "GB/s", "cores": thr, "kind": kind,
                    "sample": "2^24 of the 2^28 elements, the pipeline's derivative chain, "
                              "f64 arithmetic, bytes at f32 width (8 B/element)"}
    del xc
    # config 3: 1024 of the 65536 rows (Call(Softmax) is single-threaded)
    xs = (rng.standard_normal((1024, 4096)) * 4.0).astype(np.float32).astype(np.float64)
    t = timed(lambda: ex.softmax(xs))
    out["softmax"] = {"value": xs.size * 8 / t / 1e9, "unit": "GB/s", "cores": 1,
                      "kind": kind, "sample": "1024 rows x 4096 of config 3 (the reference's "
                                              "softmax runs on one thread), bytes at 8 B/elem"}
    # config 4: a 64-row M sample of the 8192^3 GEMM, extrapolated linearly in M
    a = (rng.standard_normal((64, 8192), dtype=np.float32) / 90.50966799187809)
    b = (rng.standard_normal((8192, 8192), dtype=np.float32) / 90.50966799187809)
    a = a.astype(np.float16).astype(np.float64)
    b = b.astype(np.float16).astype(np.float64)
    t = timed(lambda: ex.matmul(a, b, threads=thr)) if reps else 0.0
    out["gemm_f16"] = {"value": 2.0 * 64 * 8192 * 8192 / t / 1e12, "unit": "TFLOP/s",
                       "cores": thr, "kind": kind,
                       "sample": "64 of 8192 rows of A (f16 values widened to f64), full B; "
                                 "TFLOP/s extrapolated linearly in M"}
    del b
    # config 4': the whole 1024^3 f32 GEMM (in f64)
    a = rng.standard_normal((1024, 1024)).astype(np.float32).astype(np.float64) / 32
    b = rng.standard_normal((1024, 1024)).astype(np.float32).astype(np.float64) / 32
    t = timed(lambda: ex.matmul(a, b, threads=thr))
    out["gemm_f32_1024"] = {"value": 2.0 * 1024 ** 3 / t / 1e12, "unit": "TFLOP/s",
                            "cores": thr, "kind": kind, "sample": "the full 1024^3 GEMM"}
    # config 5: one 128-row band of one batch (MatMul -> scale map -> Softmax)
    q = rng.standard_normal((128, 128)).astype(np.float16).astype(np.float64)
    kt = rng.standard_normal((2048, 128)).astype(np.float16).astype(np.float64).T.copy()
    mul = kir.chain(kir.E("mul", kir.A, kir.C(128 ** -0.5)))

    def qk_band():
        sc = ex.matmul(q, kt, threads=thr)
        (sv,) = ex.chain([mul], sc.ravel(), threads=thr)
        ex.softmax(sv.reshape(sc.shape))
    t = timed(qk_band)
    band_bytes = (2 * 256 * 2048 * 128 * 2 + 256 * 2048 * 2048 * 4) / (256 * 16)
    out["qk_softmax"] = {"value": band_bytes / t / 1e9, "unit": "GB/s", "cores": thr,
                         "kind": kind, "sample": "one 128-row band of one batch (K^T "
                                                 "materialised, as the reference requires); "
                                                 "GB/s at the GPU path's bytes per band"}
    return out


def run_reference_arm(args, rank):
    if rank != 0:
        return
    n_sample = 1 << 24
    value, kind, cores, t = cpu_reference_map2(n_sample, args.steps)
    line = {
        "metric": "HBM GB/s (map/softmax) & GEMM TFLOP/s vs B200 peak at 1/2/4/8 GPUs",
        "impl": "reference", "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": "config2: y=sin(x^2+3x), dy=cos(x^2+3x)(2x+3), f32 inputs, "
                               f"sample {n_sample} elements per step (of 2^28)",
                   "elements_per_step": n_sample},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": f"{n_sample} elements of config 2 per step, f64 arithmetic, "
                                   "bytes counted at f32 width (12 B/element)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _ulp_f32(torch, got, ref64):
    """Ordered-bits ULP distance between f32 results and f64 references
    rounded to f32 (NaN pairs count 0, +0 and -0 equal)."""
    g = got.float().contiguous().view(torch.int32).to(torch.int64)
    r = ref64.float().contiguous().view(torch.int32).to(torch.int64)
    g = torch.where(g < 0, -2147483648 - g, g)
    r = torch.where(r < 0, -2147483648 - r, r)
    d = (g - r).abs()
    both_nan = torch.isnan(got.float()) & torch.isnan(ref64)
    return torch.where(both_nan, torch.zeros_like(d), d)


def parity_gate(torch, name, got, ref64, ulp_bound=None, rel_bound=None, abs_floor=0.0):
    """Checks a sample of a config's output against a torch f64 recomputation
    (the CUDA result is what is checked; torch only recomputes the formula)."""
    if ulp_bound is not None:
        worst = int(_ulp_f32(torch, got, ref64).max().item())
        return {"check": f"{name}: <= {ulp_bound} ULP vs f64", "worst_ulp": worst,
                "pass": worst <= ulp_bound}
    err = ((got.double() - ref64).abs() / (ref64.abs() + abs_floor)).max().item()
    return {"check": f"{name}: rel err <= {rel_bound}", "worst_rel": err, "pass": err <= rel_bound}


def time_device(torch, fn, warmup, steps, dist, world, min_warm_s=0.0, stats=None):
    """W untimed steps (continued until min_warm_s has passed, so clock samples
    see the same steady load), then K steps between barrier+sync; CUDA events
    on the current stream; max over ranks. Returns seconds per step.

    With a `stats` dict, K more steps follow, each bracketed by its own pair
    of events, and `stats` receives this rank's median / min / max step time
    (the reference's reporting: median of reps with min and max). That pass
    is separate because events between steps would break the back-to-back
    launch overlap the timed region measures."""
    t0 = time.perf_counter()
    done = 0
    while done < warmup or time.perf_counter() - t0 < min_warm_s:
        fn()
        done += 1
        if done % 16 == 0:
            torch.cuda.synchronize()
    # Barrier, then synchronize: the barrier's collective queues behind the
    # last warm-up steps instead of leaving the GPU idle for its length right
    # before the timed region.
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if stats is not None:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for e0, e1 in ev:
            e0.record()
            fn()
            e1.record()
        torch.cuda.synchronize()
        each = sorted(e0.elapsed_time(e1) for e0, e1 in ev)
        stats.update({"median_ms": statistics.median(each), "min_ms": each[0],
                      "max_ms": each[-1], "reps": steps,
                      "how": "separate pass, one event pair per step (this rank)"})
    return ms / 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--headline-only", action="store_true")
    ap.add_argument("--min-warm-s", type=float, default=1.5,
                    help="headline warm-up continues at least this long (clock samples); "
                         "also the run-in of each config's sustained figure; 0: neither, "
                         "and bursts warm up for W steps only (profiling runs)")
    ap.add_argument("--case", default=None,
                    choices=["map1", "map2", "chain", "softmax", "gemm", "gemm_f32", "qk", "qk_kt"],
                    help="run one kernel W+K times (profiling target), no JSON line")
    ap.add_argument("--detail", default=None,
                    help="also write the full (verbose) record as JSON to this path")
    ap.add_argument("--size", type=int, default=0,
                    help="--case size: elements (maps), rows (softmax), M=N=K (gemm), batch (qk)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.case:
        run_case(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    import numpy as np
    import torch
    import torch.distributed as dist

    import mlk2_b200 as mb
    from mlk2_b200 import api, kir

    from mlk2_b200 import dist as mdist

    torch.cuda.set_device(local)
    if world > 1:
        mdist.init("nccl", local, timeout_s=120.0)
    peaks = load_peaks()
    traffic = load_traffic()

    # ---- headline: config 2, map + derivative, 2^28 f32 per GPU ----------------
    n = 1 << 28
    x = torch.empty(n, dtype=torch.float32, device="cuda")
    api.fill(x, SEED, 2 + 256 * rank, "uniform", -8.0, 8.0)
    y = torch.empty_like(x)
    dy = torch.empty_like(x)
    step = lambda: api.map_sin_dsin(x, y, dy)  # noqa: E731
    step()  # parity gate before timing: every 4096th element against f64
    xs_, us_ = x[::4096].double(), None
    us_ = xs_ * xs_ + 3.0 * xs_
    gate = {"y": parity_gate(torch, "sin(x^2+3x)", y[::4096], torch.sin(us_), ulp_bound=2),
            "dy": parity_gate(torch, "cos(x^2+3x)(2x+3)", dy[::4096],
                              torch.cos(us_) * (2.0 * xs_ + 3.0), ulp_bound=2)}
    del xs_, us_
    step_ms = {}
    with ClockSampler(local) as clk:
        sec = time_device(torch, step, args.warmup, args.steps, dist, world,
                          min_warm_s=args.min_warm_s, stats=step_ms)
    clocks = clk.summary()
    alg_bytes = n * BYTES_PER_ELEM_MAP2
    achieved = alg_bytes / sec / 1e9
    value = world * alg_bytes / sec / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"],
                "kernel": "map_vec_kernel<SinDsinOp>",
                "traffic": traffic.get("map2", {}).get("bytes_per_launch")}

    # ---- optional assembly of the sharded result (the only collective) ----------
    gather = None
    if world > 1:
        for _ in range(2):
            full = mdist.all_gather_shards(y, dist)
            del full
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        full = mdist.all_gather_shards(y, dist)
        g1.record()
        torch.cuda.synchronize()
        gms = mdist.max_over_ranks(g0.elapsed_time(g1), dist, device="cuda")
        out_bytes = full.numel() * 4
        gather = {"what": "NCCL all_gather_into_tensor of y (f32) onto every rank",
                  "bytes_out_per_rank": out_bytes, "ms": gms,
                  "busbw_gbs": out_bytes * (world - 1) / world / (gms / 1e3) / 1e9,
                  "note": "reported separately; not part of value"}
        del full
        torch.cuda.empty_cache()

    # ---- e2e through the C-ABI host entry ---------------------------------------
    # The module is the reference compiler's own output for config 2 (Tier-1
    # pipeline, y and the calculus passes' dy), stretched to 2^28 elements.
    del y, dy
    import numpy as _np

    pipe = _np.load(os.path.join(ROOT, "tests", "golden", "pipeline.npz"))
    module_doc = kir.with_static_length(json.loads(str(pipe["both_json"])), n)
    module = api.Module(module_doc)
    plan = module.plan([mb.F32] * 3)
    # device-timed run of the same module through mlkb_module_run_dev
    ym, dym = torch.empty_like(x), torch.empty_like(x)
    msec = time_device(torch, lambda: module.run_dev([x, ym, dym], n=n, device=local), args.warmup,
                       args.steps, dist, world)
    module_dev = {"plan": plan, "ms": msec * 1e3,
                  "f": alg_bytes / msec / 1e9 / peaks["hbm_gbs"]}
    del ym, dym
    xh = torch.empty(n, dtype=torch.float32).pin_memory()
    yh = torch.empty(n, dtype=torch.float32).pin_memory()
    dyh = torch.empty(n, dtype=torch.float32).pin_memory()
    xh.copy_(x.cpu())
    del x
    torch.cuda.empty_cache()
    bufs = [xh, yh, dyh]
    module.run_host(bufs, n=n, n_gpus=1)  # warm the device buffer cache
    e2e_steps = args.steps
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        module.run_host(bufs, n=n, n_gpus=1)
    e2e_sec = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_sec], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_sec = float(t.item())
    e2e = {"value": round(world * alg_bytes / e2e_sec / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": n * 4, "d2h_bytes_per_step": n * 8,
           "ms_per_step": round(e2e_sec * 1e3, 3), "steps": e2e_steps,
           "api": "mlkb_module_run_host, reference-compiled module, pinned host f32"}
    del xh, yh, dyh, bufs, module
    torch.cuda.empty_cache()

    # ---- the other BASELINE configs ---------------------------------------------
    configs = {}
    if not args.headline_only:
        configs = other_configs(torch, api, args, dist, world, rank, peaks, traffic)

    # ---- strong scaling: each fixed problem split over the ranks -------------------
    strong = None
    if world > 1 and not args.headline_only:
        strong = strong_configs(torch, api, mdist, args, dist, world, rank, peaks)

    # ---- CPU baseline (rank 0, N = 1 only) ----------------------------------------
    cpu = None
    if rank == 0 and world == 1:
        v, kind, cores, t = cpu_reference_map2(1 << 24, 3)
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": kind,
               "sample": "2^24 of the 2^28 config-2 elements, f64, bytes at f32 width"}
        if kind == "reference":
            vd, _, cd, _ = cpu_reference_map2(1 << 24, 3, default_threads=True)
            cpu["default_executor"] = {"value": round(vd, 3), "cores": cd}
        if configs:
            for name, base in cpu_reference_configs().items():
                if name in configs:
                    configs[name]["cpu_baseline"] = base

    if rank == 0:
        launches = args.steps * 2 + sum(c.get("gpu_launches", 0) for c in configs.values())
        if strong:
            launches += sum(c.get("gpu_launches", 0) for c in strong.values() if isinstance(c, dict))
        detail = {
            "metric": "HBM GB/s (map/softmax) & GEMM TFLOP/s vs B200 peak at 1/2/4/8 GPUs",
            "value": value, "roofline": roofline, "parity": gate, "cpu_baseline": cpu,
            "e2e": e2e, "gather": gather, "module_dev": module_dev, "clocks": clocks,
            "step_ms": step_ms, "configs": configs, "strong": strong, "library": mb.version(),
        }
        if args.detail:
            with open(args.detail, "w") as f:
                json.dump(detail, f, indent=1)

        def r(v, k=4):
            return None if v is None else float(f"{v:.{k}g}")

        def short(c):
            d = {"v": r(c["value"]), "u": c["unit"], "ms": r(c["ms_per_step"]),
                 "f": r(c["roofline"]["frac"], 3)}
            if "sustained" in c:
                d["fs"] = r(c["sustained"]["frac"], 3)
            if "parity" in c:
                d["ok"] = bool(c["parity"]["pass"])
            if c.get("cpu_baseline"):
                d["cpu"] = r(c["cpu_baseline"]["value"], 3)
            return d

        line = {
            "metric": "HBM GB/s (map/softmax) & GEMM TFLOP/s vs B200 peak at 1/2/4/8 GPUs",
            "value": r(value, 6), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r(sec * 1e3, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic, seeded U(-8,8), generated on the device",
            "config": {"workload": "config2 y=sin(x^2+3x), dy=cos(x^2+3x)(2x+3), f32, "
                                   "one fused kernel", "elements_per_gpu": n,
                       "parallelism": f"dp{world}", "l2": "1 GiB inputs > L2, no flush"},
            "roofline": {"bound": "hbm", "achieved": r(achieved, 5), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": r(roofline["frac"], 4),
                         "traffic": roofline["traffic"]},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": {"sm_mhz": clocks["sm_mhz"], "sm_max_mhz": clocks["sm_max_mhz"],
                       "reasons": clocks["reasons"]},
            "parity_ok": bool(gate["y"]["pass"] and gate["dy"]["pass"]),
            "module": {"plan": module_dev["plan"], "ms": r(module_dev["ms"]),
                       "f": r(module_dev["f"], 3)},
        }
        if gather is not None:
            line["gather"] = {"ms": r(gather["ms"]), "busbw": r(gather["busbw_gbs"])}
        line["configs"] = {k: short(c) for k, c in configs.items()}
        if strong:
            line["strong"] = {k: ({"v": r(c["value"]), "ms": r(c["ms"]), "f": r(c["frac"], 3)}
                                  if "value" in c else {"ms": r(c["ms"]), "busbw": r(c["busbw"])})
                              for k, c in strong.items()}
        print(json.dumps(line, separators=(",", ":")), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def rotation_pairs(pair_bytes, steps, l2_bytes):
    """How many input/output pairs a rotating config-1 loop uses: the smallest
    count d that divides K (so the rotation also holds across replays of a
    graph of the K steps) and puts at least twice the L2's size of other
    pairs' traffic, (d - 1) * pair_bytes, between two uses of one pair; K when
    no divisor does."""
    need = -(-2 * l2_bytes // pair_bytes) + 1
    return next((d for d in range(max(need, 1), steps + 1) if steps % d == 0), steps)


def graph_of_steps(torch, fn, steps):
    """`steps` calls of fn captured into one CUDA graph on a side stream (fn
    launches on the current stream, which the capture makes the side one)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side, capture_error_mode="thread_local"):
            for _ in range(steps):
                fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    return g


def strong_configs(torch, api, mdist, args, dist, world, rank, peaks):
    """Each fixed BASELINE problem split over the ranks (contiguous element,
    row, M-block and batch shards; B replicated for the GEMM). value = the
    whole problem's work / the slowest rank's step time."""
    out = {}
    hbm, tc = peaks["hbm_gbs"], peaks["bf16_tflops"]

    def rec(name, fn, work, unit, peak, graph=False):
        time.sleep(1.0)  # from an idle GPU, like the weak-scaling configs (a burst)
        warm_s = BURST_WARM_S if args.min_warm_s > 0 else 0.0
        if graph:
            # The K steps as one CUDA graph, timed as one replay (W replays of
            # warm-up first): for kernels shorter than the host's ~10 us to
            # issue a launch, which an eager loop would time instead.
            for _ in range(args.warmup):
                fn()  # first-use set-up stays outside the capture
            torch.cuda.synchronize()
            g = graph_of_steps(torch, fn, args.steps)
            sec = time_device(torch, g.replay, args.warmup, 1, dist, world,
                              min_warm_s=warm_s) / args.steps
        else:
            sec = time_device(torch, fn, args.warmup, args.steps, dist, world, min_warm_s=warm_s)
        scale = 1e9 if unit == "GB/s" else 1e12
        out[name] = {"value": work / sec / scale, "unit": unit, "ms": sec * 1e3,
                     "frac": work / sec / scale / (world * peak), "gpu_launches": args.steps}
        if graph:
            out[name]["timed"] = "cuda graph"

    def part(total):
        return total * (rank + 1) // world - total * rank // world

    # config 1 (2^24) and config 2 (2^28) element shards. A config-1 shard is
    # 16-128 MB, so steps rotate over input/output pairs (rotation_pairs).
    n1 = part(1 << 24)
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    pairs = rotation_pairs(n1 * 8, args.steps, l2)
    x1s = [torch.empty(n1, device="cuda") for _ in range(pairs)]
    y1s = [torch.empty_like(x1s[0]) for _ in range(pairs)]
    for x in x1s:
        api.fill(x, SEED, 1 + 256 * rank, "uniform", -4.0, 4.0)
    turn = [0]

    def step1():
        i = turn[0] % pairs
        turn[0] += 1
        api.map_sin(x1s[i], y1s[i])
    rec("map1", step1, (1 << 24) * 8, "GB/s", hbm, graph=True)
    out["map1"]["pairs"] = pairs
    del x1s, y1s
    n2 = part(1 << 28)
    x2 = torch.empty(n2, device="cuda")
    api.fill(x2, SEED, 2 + 256 * rank, "uniform", -8.0, 8.0)
    y2, dy2 = torch.empty_like(x2), torch.empty_like(x2)
    rec("map2", lambda: api.map_sin_dsin(x2, y2, dy2), (1 << 28) * 12, "GB/s", hbm)
    # assembling y on every rank: NCCL all-gather (the only collective)
    if (1 << 28) % world == 0:
        for _ in range(2):
            del_full = mdist.all_gather_shards(y2, dist)
            del del_full
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        full = mdist.all_gather_shards(y2, dist)
        g1.record()
        torch.cuda.synchronize()
        gms = mdist.max_over_ranks(g0.elapsed_time(g1), dist, device="cuda")
        nbytes = full.numel() * 4
        out["gather_map2_y"] = {"ms": gms, "busbw": nbytes * (world - 1) / world / (gms / 1e3) / 1e9}
        del full
    del x2, y2, dy2
    torch.cuda.empty_cache()
    # config 3: row shards of 65536 x 4096
    r3 = part(65536)
    xs = torch.empty((r3, 4096), device="cuda")
    api.fill(xs, SEED, 3 + 256 * rank, "normal", 0.0, 4.0)
    ys = torch.empty_like(xs)
    rec("softmax", lambda: api.softmax(xs, ys), 2 * 4 * 65536 * 4096, "GB/s", hbm)
    del xs, ys
    # config 4: M-block shards of the 8192^3 GEMM, B on every rank
    m4 = part(8192)
    a = torch.empty((m4, 8192), dtype=torch.float16, device="cuda")
    b = torch.empty((8192, 8192), dtype=torch.float16, device="cuda")
    api.fill(a, SEED, 41 + 256 * rank, "normal", 0.0, 8192 ** -0.5)
    api.fill(b, SEED, 42, "normal", 0.0, 8192 ** -0.5)
    c = torch.empty((m4, 8192), device="cuda")
    rec("gemm_f16", lambda: api.gemm(a, b, c), 2.0 * 8192 ** 3, "TFLOP/s", tc)
    del a, b, c
    # config 5: batch shards of 256 x [2048 x 2048]
    bq = part(256)
    q = torch.empty((bq, 2048, 128), dtype=torch.float16, device="cuda")
    k = torch.empty((bq, 2048, 128), dtype=torch.float16, device="cuda")
    api.fill(q, SEED, 51 + 256 * rank, "normal", 0.0, 1.0)
    api.fill(k, SEED, 52 + 256 * rank, "normal", 0.0, 1.0)
    yq = torch.empty((bq, 2048, 2048), device="cuda")
    rec("qk_softmax", lambda: api.qk_softmax(q, k, yq, 128 ** -0.5),
        2 * 256 * 2048 * 128 * 2 + 256 * 2048 * 2048 * 4, "GB/s", hbm)
    del q, k, yq
    torch.cuda.empty_cache()
    return out


def run_case(args):
    """One kernel, W + K launches, default stream; prints ms per launch."""
    import torch

    from mlk2_b200 import api

    torch.cuda.set_device(0)
    c, sz = args.case, args.size
    if c in ("map1", "map2"):
        n = sz or (1 << 26)
        x = torch.empty(n, device="cuda")
        api.fill(x, SEED, 2, "uniform", -8.0, 8.0)
        y, dy = torch.empty_like(x), torch.empty_like(x)
        fn = (lambda: api.map_sin_dsin(x, y, dy)) if c == "map2" else (lambda: api.map_sin(x, y))
    elif c == "chain":  # the pipeline's derivative chain through the compiled chain path
        import numpy as np

        from mlk2_b200 import kir

        pipe = np.load(os.path.join(ROOT, "tests", "golden", "pipeline.npz"))
        dchain = kir.chains_of(json.loads(str(pipe["dsin_json"])))[-1]
        n = sz or (1 << 26)
        x = torch.empty(n, device="cuda")
        api.fill(x, SEED, 7, "uniform", -8.0, 8.0)
        y = torch.empty_like(x)
        fn = lambda: api.map_chain(dchain, x, y)  # noqa: E731
    elif c == "softmax":
        rows = sz or 16384
        x = torch.empty((rows, 4096), device="cuda")
        api.fill(x, SEED, 3, "normal", 0.0, 4.0)
        y = torch.empty_like(x)
        fn = lambda: api.softmax(x, y)  # noqa: E731
    elif c in ("gemm", "gemm_f32"):
        n = sz or 8192
        dt = torch.float16 if c == "gemm" else torch.float32
        a = torch.empty((n, n), dtype=dt, device="cuda")
        b = torch.empty((n, n), dtype=dt, device="cuda")
        a.normal_(0, n ** -0.5)
        b.normal_(0, n ** -0.5)
        cc = torch.empty((n, n), device="cuda")
        fn = lambda: api.gemm(a, b, cc)  # noqa: E731
    else:
        bq = sz or 32
        q = torch.empty((bq, 2048, 128), dtype=torch.float16, device="cuda")
        k = torch.empty((bq, 2048, 128), dtype=torch.float16, device="cuda")
        q.normal_()
        k.normal_()
        yq = torch.empty((bq, 2048, 2048), device="cuda")
        if c == "qk":
            fn = lambda: api.qk_softmax(q, k, yq, 128 ** -0.5)  # noqa: E731
        else:  # K given as the reference's MatMul B operand, Kt [batch, d, s]
            kt = k.transpose(1, 2).contiguous()
            fn = lambda: api.qk_softmax_kt(q, kt, yq, 128 ** -0.5)  # noqa: E731
    sec = time_device(torch, fn, args.warmup, args.steps, None, 1)
    print(json.dumps({"case": c, "size": sz, "ms_per_launch": sec * 1e3}), flush=True)


def other_configs(torch, api, args, dist, world, rank, peaks, traffic):
    out = {}
    steps, warm = args.steps, args.warmup
    last = {}  # per-step statistics and the sustained time of the latest measure()

    def measure(fn):
        """Seconds per step of a burst: each config starts from an idle GPU (1 s
        pause), so its number does not depend on the heat the previous config
        left under the 1 kW power limit, and warms up for at least W steps and
        BURST_WARM_S; then the same steps once more after
        --min-warm-s (default 1.5 s) of continuous running, reported beside it
        as `sustained` (skipped with --min-warm-s 0)."""
        time.sleep(1.0)
        warm_s = BURST_WARM_S if args.min_warm_s > 0 else 0.0
        sec = time_device(torch, fn, warm, steps, dist, world, min_warm_s=warm_s, stats=last)
        if args.min_warm_s > 0:
            sus = time_device(torch, fn, 0, steps, dist, world, min_warm_s=args.min_warm_s)
            last["sustained_ms_per_step"] = sus * 1e3
        return sec

    def rec(name, sec, work, unit, bound, peak, launches, extra=None):
        achieved = work / sec / (1e9 if unit == "GB/s" else 1e12)
        d = {"value": world * achieved, "unit": unit, "ms_per_step": sec * 1e3,
             "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                          "frac": achieved / peak,
                          "traffic": traffic.get(name, {}).get("bytes_per_launch")},
             "gpu_launches": launches * steps}
        sus = last.pop("sustained_ms_per_step", None)
        d["step_ms"] = dict(last)
        if sus is not None:
            per_gpu = work / (sus / 1e3) / (1e9 if unit == "GB/s" else 1e12)
            # a long-running GEMM is judged against the measured sustained cuBLAS rate
            sus_peak = (peaks.get("bf16_tflops_sustained") or peak) if bound == "tensor" else peak
            d["sustained"] = {"ms_per_step": sus, "value": world * per_gpu, "peak": sus_peak,
                              "frac": per_gpu / sus_peak,
                              "note": f"same steps after {args.min_warm_s} s of continuous running"}
        last.clear()
        if extra:
            d.update(extra)
        out[name] = d

    # config 1: y = sin(x^2+3x), 2^24 f32 (128 MiB touched per step). Steps
    # rotate over 8 input/output pairs (1 GiB), so the pair a step uses was
    # last touched 7 steps (896 MiB of traffic) earlier and is not in L2.
    n1, nsets = 1 << 24, 8
    xs1 = [torch.empty(n1, device="cuda") for _ in range(nsets)]
    ys1 = [torch.empty_like(xs1[0]) for _ in range(nsets)]
    for x in xs1:
        api.fill(x, SEED, 1 + 256 * rank, "uniform", -4.0, 4.0)
    turn = [0]

    def step1():
        i = turn[0] % nsets
        turn[0] += 1
        api.map_sin(xs1[i], ys1[i])
    api.map_sin(xs1[0], ys1[0])
    x64 = xs1[0][::1024].double()
    g1 = parity_gate(torch, "sin(x^2+3x)", ys1[0][::1024], torch.sin(x64 * x64 + 3.0 * x64),
                     ulp_bound=2)
    sec = measure(step1)
    rec("map1", sec, n1 * 8, "GB/s", "hbm", peaks["hbm_gbs"], 1,
        {"note": "steps rotate over 8 input/output pairs (1 GiB > L2), no flush",
         "parity": g1})
    del xs1, ys1

    # the generic chain path (every scalar-realisable chain): the derivative chain the
    # reference's calculus passes emit for config 2 (Tier-1 output committed in
    # tests/golden/pipeline.npz), 2^28 f32 through mlkb_map_chain, which runs
    # it as a chain kernel compiled at run time (no dedicated kernel applies
    # on this entry). 8 B per element; 2 GiB touched per step (> L2).
    import numpy as _np

    from mlk2_b200 import kir

    pipe = _np.load(os.path.join(ROOT, "tests", "golden", "pipeline.npz"))
    dchain = kir.chains_of(json.loads(str(pipe["dsin_json"])))[-1]
    nc = 1 << 28
    xc = torch.empty(nc, device="cuda")
    api.fill(xc, SEED, 7 + 256 * rank, "uniform", -8.0, 8.0)
    yc = torch.empty_like(xc)
    _, _, launched0 = api.chain_compile(-1)
    api.map_chain(dchain, xc, yc)
    xs64 = xc[::4096].double()
    gc = parity_gate(torch, "pipeline d/dx sin(x^2+3x) via the generic chain", yc[::4096],
                     torch.cos(xs64 * xs64 + 3.0 * xs64) * (2.0 * xs64 + 3.0), ulp_bound=2)
    active, _, launched1 = api.chain_compile(-1)
    sec = measure(lambda: api.map_chain(dchain, xc, yc))
    rec("chain", sec, nc * 8, "GB/s", "hbm", peaks["hbm_gbs"], 1,
        {"parity": gc, "path": "compiled" if active and launched1 > launched0 else "interpreted",
         "kernel": "mlkb_chain_kernel (NVRTC, run time)"})
    del xc, yc

    # config 3: softmax [65536 x 4096] f32 per GPU
    xs = torch.empty((65536, 4096), device="cuda")
    api.fill(xs, SEED, 3 + 256 * rank, "normal", 0.0, 4.0)
    ys = torch.empty_like(xs)
    api.softmax(xs, ys)
    g3 = parity_gate(torch, "softmax rows", ys[::1024],
                     torch.softmax(xs[::1024].double(), dim=1), ulp_bound=2)
    sec = measure(lambda: api.softmax(xs, ys))
    rec("softmax", sec, 2 * 4 * 65536 * 4096, "GB/s", "hbm", peaks["hbm_gbs"], 1,
        {"parity": g3})
    del xs, ys

    # config 4: GEMM 8192^3 f16 -> f32 (M-block shard per GPU in weak scaling)
    n4 = 8192
    a = torch.empty((n4, n4), dtype=torch.float16, device="cuda")
    b = torch.empty((n4, n4), dtype=torch.float16, device="cuda")
    api.fill(a, SEED, 41 + 256 * rank, "normal", 0.0, n4 ** -0.5)
    api.fill(b, SEED, 42, "normal", 0.0, n4 ** -0.5)
    c = torch.empty((n4, n4), device="cuda")
    api.gemm(a, b, c)
    rows = slice(0, n4, 128)
    ref4 = a[rows].double() @ b.double()
    mag4 = a[rows].double().abs() @ b.double().abs()
    err4 = ((c[rows].double() - ref4).abs() / mag4).max().item()
    g4 = {"check": "f16 GEMM: |C - C_f64| <= 2^-12 sum|a b| (every 128th row)",
          "worst": err4, "pass": err4 <= 2.0 ** -12}
    del ref4, mag4
    sec = measure(lambda: api.gemm(a, b, c))
    rec("gemm_f16", sec, 2.0 * n4 ** 3, "TFLOP/s", "tensor", peaks["bf16_tflops"], 1,
        {"peak_note": "peak = measured cuBLAS bf16 dense burst (f16 has the same rate)",
         "parity": g4})
    del a, b, c

    # config 4': GEMM 1024^3 f32 (SIMT FMA)
    a = torch.randn((1024, 1024), device="cuda") / 32
    b = torch.randn((1024, 1024), device="cuda") / 32
    c = torch.empty((1024, 1024), device="cuda")
    api.gemm(a, b, c)
    err5 = ((c.double() - a.double() @ b.double()).abs() /
            (a.double().abs() @ b.double().abs())).max().item()
    g5 = {"check": "f32 GEMM: |C - C_f64| <= 2^-14 sum|a b|", "worst": err5,
          "pass": err5 <= 2.0 ** -14}
    sec = measure(lambda: api.gemm(a, b, c))
    rec("gemm_f32_1024", sec, 2.0 * 1024 ** 3, "TFLOP/s", "fp32-simt", 80.0, 1,
        {"peak_note": "nominal FP32 SIMT 80 TFLOP/s (context only)", "parity": g5})
    del a, b, c

    # config 5: batched Q K^T * s + softmax, 256 x [2048 x 2048], d = 128
    bq, s, d = 256, 2048, 128
    q = torch.empty((bq, s, d), dtype=torch.float16, device="cuda")
    k = torch.empty((bq, s, d), dtype=torch.float16, device="cuda")
    api.fill(q, SEED, 51 + 256 * rank, "normal", 0.0, 1.0)
    api.fill(k, SEED, 52 + 256 * rank, "normal", 0.0, 1.0)
    yq = torch.empty((bq, s, s), device="cuda")
    api.qk_softmax(q, k, yq, d ** -0.5)
    ref6 = torch.softmax((q[bq - 1, ::16].double() @ k[bq - 1].double().T) * d ** -0.5, dim=1)
    g6 = parity_gate(torch, "softmax(Q K^T / sqrt(d)) (batch 255, every 16th row)",
                     yq[bq - 1, ::16], ref6, rel_bound=2.0 ** -16, abs_floor=2.0 ** -14)
    del ref6
    sec = measure(lambda: api.qk_softmax(q, k, yq, d ** -0.5))
    alg = 2 * bq * s * d * 2 + bq * s * s * 4
    rec("qk_softmax", sec, alg, "GB/s", "hbm", peaks["hbm_gbs"], 1,
        {"tflops": 2.0 * bq * s * s * d / sec / 1e12, "parity": g6})
    del q, k, yq
    torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    main()
