"""Benchmark of the B200 reduce/scan path (BASELINE.json metric: achieved HBM
GB/s for reduce/scan).

Default workload: u32 exclusive prefix scan over
2^28 elements per GPU, values h & 15 from seed 1 (SplitMix64 stream, generated
on the device).  At N>1 GPUs config 2 runs as replicas (every rank scans its own
2^28 elements, weak scaling); with --partitioned every rank owns 2^28 elements of
one global N*2^28-element buffer and the step is the partitioned scan: local total
-> NCCL all-gather of the totals -> carry -> seeded scan.  Config 5 is the 1-D
partitioned case: 2^32 i32 split over the ranks (strong scaling), its scan and
i64 sum fused so that one pass over each slice feeds both exchanges.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--config 1|2|3|4|5|6|7]

Prints ONE JSON line on rank 0.  `value` is whole-job algorithmic bytes per
second with inputs resident in HBM (CUDA events on the compute stream, max
over ranks); `e2e` is the same metric through the public API with pinned host
buffers and the host<->device copies inside the timed region; `roofline`
compares the dominant kernel's algorithmic bytes per launch / its event-timed
duration against the measured HBM copy bandwidth (MEASURED_PEAKS.json);
`cpu_baseline` is the oracle restatement of the reference's host semantics
timed on this box's cores on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "achieved HBM GB/s (and % of ~8 TB/s) for reduce/scan at 1/2/4/8 B200"
L2_BYTES = 126 * 2**20

CONFIGS = {
    1: dict(workload="f32 full sum reduction over 2^20 elements, uniform[-1,1) seed 0 "
                     "(64 rotating buffers, 256 MiB > L2, submitted as one prepared batch per step: the batch's 64 "
                     "reductions run as one fused launch)", n=1 << 20, dtype="f32",
            kernel="reduce_fused_kernel", bytes_per_elem=4),
    2: dict(workload="u32 exclusive prefix scan over 2^28 elements per GPU, h&15 seed 1",
            n=1 << 28, dtype="u32", kernel="scan_chunked_kernel", bytes_per_elem=8),
    3: dict(workload="f32 row-wise max + argmax over [65536 x 4096] row-major, N(0,1) seed 2, "
                     "~1% injected exact ties", rows=65536, cols=4096, dtype="f32",
            kernel="row_reduce_kernel"),
    4: dict(workload="f64 column-wise (axis=0) sum over [4096 x 65536] row-major, U[0,1) seed 3",
            rows=4096, cols=65536, dtype="f64", kernel="col_reduce_kernel"),
    5: dict(workload="i32 inclusive scan + i64-accumulated sum over 2^32 elements (16 GiB) "
                     "U{-1000..1000} seed 4, partitioned 1-D across the GPUs",
            n=1 << 32, dtype="i32", kernel="scan_chunked_kernel"),
    # Gapped N-D views (the reference stages these through a contiguous copy
    # first): a sub-block of a larger row-major matrix.
    6: dict(workload="f32 full sum over the [16384 x 16000] sub-block (row stride 16384, offset 64) of a "
                     "[16384 x 16384] matrix, U[-1,1) seed 0; 16-byte-aligned rows",
            rows=16384, cols=16000, ld=16384, offset=64, dtype="f32", kernel="reduce_walk_kernel"),
    7: dict(workload="f32 full sum over the [16384 x 15999] sub-block (row stride 16387, offset 1) of a "
                     "16384 x 16387 matrix, U[-1,1) seed 0; rows not 16-byte aligned",
            rows=16384, cols=15999, ld=16387, offset=1, dtype="f32", kernel="reduce_runs_kernel"),
    # Axis scan of a matrix (ScanOps::scan_axis_into on a rank-2 view, axis 1):
    # many long lines, each a look-back chain of 32 tiles.
    8: dict(workload="u32 inclusive scan along the rows (axis 1) of a [1024 x 262144] row-major matrix, "
                     "h&15 seed 1", rows=1024, cols=262144, dtype="u32", kernel="scan_lookback_kernel"),
    # A few long lines: all of them in one launch of the chunked kernel.
    9: dict(workload="u32 inclusive scan along the rows (axis 1) of a [16 x 2^24] row-major matrix, "
                     "h&15 seed 1", rows=16, cols=1 << 24, dtype="u32", kernel="scan_chunked_kernel"),
    # One large dense full reduction (the shared-memory-staged kernel).
    10: dict(workload="f32 full sum reduction over 2^28 elements (1 GiB), uniform[-1,1) seed 0",
             n=1 << 28, dtype="f32", kernel="reduce_bulk_kernel", bytes_per_elem=4),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=5)
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end measurement")
    ap.add_argument("--published", action="store_true",
                    help="time the reference's own published reduce/scan cases (benchmark_results.md) instead")
    ap.add_argument("--partitioned", action="store_true",
                    help="config 2 at N>1: one global scan partitioned over the ranks instead of replicas")
    ap.add_argument("--misalign", type=int, default=0,
                    help="configs 3/4: the same-shape view at element offset K of a row-padded matrix "
                         "(rows not 16-byte aligned)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-check", action="store_true",
                    help="config 5: skip the element-by-element check of the results after the timed region")
    ap.add_argument("--shape", default=None,
                    help="configs 8/9: ROWSxCOLS instead of the configured matrix (e.g. 64x4194304)")
    ap.add_argument("--n", type=int, default=None,
                    help="override the element count of configs 1, 2 and 5 (small profiling cases)")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(kernel: str, config: int):
    """dram bytes per launch recorded from an ncu capture (profiles/*.md line
    `traffic[<config>] <kernel>: <bytes>`), or None."""
    pat = re.compile(rf"traffic\[{config}\]\s+{re.escape(kernel)}:\s*([0-9.eE+]+)")
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for f in sorted(os.listdir(pdir)):
        if f.endswith((".md", ".txt")):
            m = pat.search(open(os.path.join(pdir, f)).read())
            if m:
                return float(m.group(1))
    return None


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------- reference arm


_CPU_DATA = {}


def cpu_workload(cfg_id: int, cfg: dict, oracle, threads: int):
    """The configured workload at its full size on the host: (one pass, its
    algorithmic bytes, description).  Inputs are generated once per process
    by the oracle's generator (the device's SplitMix64 stream)."""
    mt = f"{threads} threads" if threads > 1 else "one thread"

    def data(key, make):
        if key not in _CPU_DATA:
            _CPU_DATA[key] = make()
        return _CPU_DATA[key]

    if cfg_id in (2, 5):
        n = cfg["n"]
        dt = np.uint32 if cfg_id == 2 else np.int32
        kind = oracle.GEN_U32_LOW4 if cfg_id == 2 else oracle.GEN_I32_PM1000
        x = data(("x", cfg_id, n), lambda: oracle.generate(kind, 1 if cfg_id == 2 else 4, n))
        out = data(("y", cfg_id, n), lambda: np.empty(n, dt))
        if cfg_id == 2:
            return (lambda: oracle.exclusive_scan_u32_mt(x, out, 0, threads)), 8 * n, \
                f"u32 exclusive scan of {n} elements ({mt})"

        def step5():
            oracle.inclusive_scan_i32_mt(x, out, 0, threads)
            oracle.sum_i32_to_i64_mt(x, threads)
        return step5, 12 * n, f"i32 inclusive scan + i64 sum of {n} elements ({mt})"
    if cfg_id in (1, 10):
        n = cfg["n"]
        x = data(("x", 1, n), lambda: oracle.generate(oracle.GEN_F32_UNIFORM_PM1, 0, n))
        return (lambda: oracle.sum_f32_mt(x, threads)), 4 * n, f"f32 sum of {n} elements ({mt})"
    if cfg_id == 3:
        rows, cols = cfg["rows"], cfg["cols"]
        x = data(("x", 3), lambda: oracle.generate(oracle.GEN_F32_NORMAL, 2, rows * cols))
        return (lambda: oracle.row_argmax_f32_mt(x, rows, cols, threads)), 4 * rows * cols + 8 * rows, \
            f"row max + argmax of [{rows} x {cols}] f32 ({mt})"
    if cfg_id == 4:
        rows, cols = cfg["rows"], cfg["cols"]
        x = data(("x", 4), lambda: oracle.generate(oracle.GEN_F64_UNIT, 3, rows * cols))
        return (lambda: oracle.col_sum_f64_mt(x, rows, cols, threads)), 8 * rows * cols + 8 * cols, \
            f"column sum of [{rows} x {cols}] f64 ({mt})"
    if cfg_id in (6, 7):
        rows, cols, ld, off = cfg["rows"], cfg["cols"], cfg["ld"], cfg["offset"]
        x = data(("x", cfg_id), lambda: oracle.generate(oracle.GEN_F32_UNIFORM_PM1, 0, rows * ld + off))
        return (lambda: oracle.reduce_full(x, [rows, cols], [ld, 1], off)), 4 * rows * cols, \
            f"f32 sum of the [{rows} x {cols}] sub-block (row stride {ld}) (one thread: sequential strided fold)"
    rows, cols = cfg["rows"], cfg["cols"]  # configs 8 and 9
    x = data(("x", cfg_id, rows, cols), lambda: oracle.generate(oracle.GEN_U32_LOW4, 1, rows * cols))
    out = data(("y", cfg_id, rows, cols), lambda: np.empty_like(x))
    return (lambda: oracle.scan_axis(x, [rows, cols], 1, out_storage=out)), 8 * rows * cols, \
        f"u32 row scan of [{rows} x {cols}] (one thread: sequential per-line fold)"


def cpu_threads_used(cfg_id: int, threads: int) -> int:
    return 1 if cfg_id in (6, 7, 8, 9) else threads


def cpu_sample(cfg_id: int, cfg: dict, oracle, seconds: float = 10.0, threads: int = 0):
    """Time the oracle restatement on the FULL configured workload, repeated
    until `seconds` have passed (at least one pass).  Returns (GB/s, cores,
    description).  threads=0 means every host core this process may run on:
    the count is passed to the oracle explicitly, so torchrun's
    OMP_NUM_THREADS=1 does not shrink the sample."""
    threads = threads or len(os.sched_getaffinity(0))
    fn, nbytes, desc = cpu_workload(cfg_id, cfg, oracle, threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt_s = (time.perf_counter() - t0) / reps
    return nbytes / dt_s / 1e9, cpu_threads_used(cfg_id, threads), f"{desc} x {reps} passes"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, cfg):
    """The reference arm: the oracle restatement of the reference's host
    device timed on this box's cores, on the same configured workload and
    with the same `config` as the GPU arm.  Rank 0 alone runs under torchrun.
    Each step is one or more full passes over the workload (at least ~1 s);
    `value` uses every host core, and the single-threaded figure -- the
    reference's host device is single-threaded -- is reported beside it as
    `single_thread_value`."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    sys.path.insert(0, ROOT)
    from oracle import host_ref as oracle
    oracle.build()
    shrink = cpu_fit(args.config, cfg)
    if shrink:
        cfg = dict(cfg, n=shrink)
    vals = []
    desc, cores = "", 0
    t_run = time.perf_counter()
    steps_run = 0
    for i in range(args.warmup + args.steps):
        v, cores, desc = cpu_sample(args.config, cfg, oracle, seconds=1.0)
        if i >= args.warmup:
            vals.append(v)
            steps_run += 1
        # keep the whole arm within a few minutes on slow hosts
        if time.perf_counter() - t_run > 240 and vals:
            break
    value = statistics.median(vals)
    if cores == 1:
        single, single_desc = value, desc
    else:
        single, _, single_desc = cpu_sample(args.config, cfg, oracle, seconds=0.0, threads=1)
    sample = desc + " per step (oracle restatement of the host reference semantics)"
    if shrink:
        sample += f"; host memory allows {shrink} of the {CONFIGS[args.config]['n']} elements"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "steps_run": steps_run, "warmup": args.warmup,
        "higher_is_better": True, "scaling": scaling_kind(args.config),
        "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic",
        "config": config_dict(args, cfg, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample,
                         "single_thread_value": round(single, 3), "single_thread_sample": single_desc,
                         "primary": "single_thread_value (the reference's host device is single-threaded)",
                         "nproc": os.cpu_count(), "cpu_model": cpu_model()},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def cpu_fit(cfg_id: int, cfg: dict):
    """Config 5 holds 2 x 16 GiB on the host.  Returns None when the host has
    room for it (with 8 GiB to spare), else the largest power-of-two element
    count that fits."""
    if cfg_id != 5:
        return None
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        return None
    need = 8 * cfg["n"] + (8 << 30)
    if avail >= need:
        return None
    n = 1 << 26
    while 8 * (2 * n) + (8 << 30) <= avail and 2 * n < cfg["n"]:
        n *= 2
    return n


def scaling_kind(cfg_id: int) -> str:
    return "strong" if cfg_id == 5 else "weak"


def config_dict(args, cfg: dict, world: int) -> dict:
    """The `config` object, identical in both arms for the same flags."""
    if cfg.get("n") is not None and args.config == 5:
        per = (cfg["n"] + world - 1) // world
        total = cfg["n"]
    elif cfg.get("n") is not None:
        per = cfg["n"]
        total = per * world
    else:
        per = cfg["rows"] * cfg["cols"]
        total = per * world
    if args.config == 5:
        par = f"partitioned1d{world}" if world > 1 else "single"
    elif args.config == 2 and args.partitioned and world > 1:
        par = f"partitioned1d{world}"
    else:
        par = f"replicas{world}" if world > 1 else "single"
    return {"workload": cfg["workload"], "config_index": args.config,
            "elements_total": total, "elements_per_gpu": per,
            "l2": "64 rotating 4 MiB inputs (256 MiB > L2)" if args.config == 1 else "inputs larger than L2",
            "parallelism": par}


# --------------------------------------------------------------------- b200 arm


# The reference's published reduce/scan/map cases (benchmark_results.md:151-181,
# WGPU on a GeForce RTX 5080): name, its GPU time in us.
PUBLISHED = [
    ("sum f32 N=2^20 (prepared)", 42.70),
    ("axis-0 sum 256x256 f32 (prepared)", 22.14),
    ("axis-0 min 256x256 f32 (prepared)", 20.73),
    ("axis-0 max 256x256 f32 (prepared)", 11.78),
    ("axis-0 mean 256x256 f32 (prepared)", 18.05),
    ("cumsum 256x256 f32 axis 1", 46.53),
    ("dot f32 N=65536", 97.42),
    ("trace 256x256 f32", 42.72),
    ("norm L1 f32 N=65536", 78.14),
    ("norm L2 f32 N=65536", 162.24),
    ("norm max f32 N=65536", 89.88),
]


def run_published(args):
    """Times the reference's published small cases through this library on
    one B200: device_us = CUDA-event time of one call queued behind a short
    spin (the events bracket the device work, not the host's issue time);
    host_us = wall time of one call + synchronisation (+ the 1-element
    read-back for the cases that return a scalar), Python/ctypes included."""
    import torch
    sys.path.insert(0, ROOT)
    import hephaestus_b200 as H
    import hephaestus_b200.seams as S
    from hephaestus_b200.core import CumSumOp, Layout, MaxOp, MinOp, StridedView, SumOp
    from hephaestus_b200 import _native as N

    dev = H.CudaDevice(0)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    rng = np.random.default_rng(0)
    one = Layout.c_contiguous([1])

    def up(shape):
        return dev.upload(rng.uniform(-1, 1, size=int(np.prod(shape))).astype(np.float32))

    v20, m256, v64k, w64k = up([1 << 20]), up([256, 256]), up([65536]), up([65536])
    out1 = dev.alloc_zeroed(np.float32, 1)
    row = dev.alloc_zeroed(np.float32, 256)
    scanned = dev.alloc_zeroed(np.float32, 256 * 256)
    fops, aops, sops = H.CudaFullReductionOps(), H.CudaAxisReductionOps(), H.CudaScanOps()
    ml, rl = Layout.c_contiguous([256, 256]), Layout.c_contiguous([1, 256])
    p_sum = fops.prepare_reduce_full(SumOp, dev, StridedView(v20, Layout.c_contiguous([1 << 20])), StridedView(out1, one))
    p_axis = {name: aops.prepare_reduce_axis_into(op, dev, StridedView(m256, ml), 0, StridedView(row, rl))
              for name, op in (("sum", SumOp), ("min", MinOp), ("max", MaxOp))}
    p_mean = S.prepare_mean_axis_into(dev, StridedView(m256, ml), 0, StridedView(row, rl))
    p_scan = sops.prepare_scan_axis(CumSumOp, dev, StridedView(m256, ml), 1, N.FORWARD, StridedView(scanned, ml))
    p_dot = S.prepare_dot(dev, StridedView(v64k, Layout.c_contiguous([65536])),
                          StridedView(w64k, Layout.c_contiguous([65536])))
    diag = StridedView(m256, Layout.try_new([256], [257], 0))
    maps = {kind: S.PreparedMap(dev, kind, StridedView(v64k, Layout.c_contiguous([65536])))
            for kind in (N.MAP_NORM_L1, N.MAP_NORM_L2, N.MAP_NORM_MAX)}
    p_trace = S.PreparedMap(dev, N.MAP_SUM, diag)
    cases = {
        "sum f32 N=2^20 (prepared)": (lambda: fops.dispatch_full(dev, p_sum, stream=sp), out1),
        "axis-0 sum 256x256 f32 (prepared)": (lambda: aops.dispatch_prepared(dev, p_axis["sum"], stream=sp), None),
        "axis-0 min 256x256 f32 (prepared)": (lambda: aops.dispatch_prepared(dev, p_axis["min"], stream=sp), None),
        "axis-0 max 256x256 f32 (prepared)": (lambda: aops.dispatch_prepared(dev, p_axis["max"], stream=sp), None),
        "axis-0 mean 256x256 f32 (prepared)": (lambda: aops.dispatch_prepared(dev, p_mean, stream=sp), None),
        "cumsum 256x256 f32 axis 1": (lambda: sops.dispatch_scan(dev, p_scan, stream=sp), None),
        "dot f32 N=65536": (lambda: p_dot.dispatch(stream=sp), p_dot.output()),
        "trace 256x256 f32": (lambda: p_trace.dispatch(stream=sp), p_trace.output()),
        "norm L1 f32 N=65536": (lambda: maps[N.MAP_NORM_L1].dispatch(stream=sp), maps[N.MAP_NORM_L1].output()),
        "norm L2 f32 N=65536": (lambda: maps[N.MAP_NORM_L2].dispatch(stream=sp), maps[N.MAP_NORM_L2].output()),
        "norm max f32 N=65536": (lambda: maps[N.MAP_NORM_MAX].dispatch(stream=sp), maps[N.MAP_NORM_MAX].output()),
    }
    results = []
    host = np.empty(1, np.float32)
    for name, ref_us in PUBLISHED:
        fn, scalar = cases[name]
        with torch.cuda.stream(stream):
            for _ in range(5):
                fn()
            dev.synchronize_stream(sp)
            ds = []
            for _ in range(30):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda._sleep(50_000)
                a.record(stream)
                fn()
                b.record(stream)
                b.synchronize()
                ds.append(a.elapsed_time(b) * 1e3)
            hs = []
            for _ in range(30):
                t0 = time.perf_counter()
                fn()
                dev.synchronize_stream(sp)
                if scalar is not None:
                    dev.download(scalar, host)  # the value a caller reads back
                hs.append((time.perf_counter() - t0) * 1e6)
        results.append({"case": name, "reference_wgpu_rtx5080_us": ref_us,
                        "device_us": round(statistics.median(ds), 2), "host_us": round(statistics.median(hs), 2)})
    print(json.dumps({"mode": "published_cases", "gpu": torch.cuda.get_device_name(0), "cases": results}),
          flush=True)
    return 0


def main():
    args = parse()
    if args.published:
        return run_published(args)
    cfg = dict(CONFIGS[args.config])
    if args.misalign:
        if args.config not in (3, 4):
            raise SystemExit("--misalign applies to configs 3 and 4")
        cfg["workload"] += f" [view at element offset {args.misalign} of a row-padded matrix: rows not 16-byte aligned]"
    if args.n is not None and "n" in cfg:
        cfg["n"] = int(args.n)
        cfg["workload"] += f" [reduced to {args.n} elements]"
    elif args.n is not None and args.config in (6, 7):
        cfg["rows"] = int(args.n)
        cfg["workload"] += f" [reduced to {args.n} rows]"
    if args.shape and args.config in (8, 9):
        r, c = (int(v) for v in args.shape.lower().split("x"))
        cfg["rows"], cfg["cols"] = r, c
        cfg["workload"] = cfg["workload"].split(" of a [")[0] + f" of a [{r} x {c}] row-major matrix, h&15 seed 1"
    if args.impl == "reference":
        return run_reference(args, cfg)

    import torch
    sys.path.insert(0, ROOT)
    import hephaestus_b200 as H
    import hephaestus_b200.seams as S
    from hephaestus_b200.core import CumSumOp, Layout, StridedView, SumOp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = H.CudaDevice(local)
    stream = torch.cuda.Stream(device=local)
    sp = stream.cuda_stream
    peak, peak_kind = peaks()

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    comm = None
    # Config 2 runs as replicas at N>1 (every rank scans its own 2^28
    # elements; the 1-D partitioned case is config 5); --partitioned makes it
    # one global scan over all ranks' slices instead.
    if world > 1 and (args.config == 5 or (args.config == 2 and args.partitioned)):
        from hephaestus_b200.dist import Communicator
        comm = Communicator.from_torch(dev)

    # ---------------- workload set-up (inputs generated on the device) -------------
    launches_per_step = 1
    e2e_fn = None
    if args.config == 2:
        n = cfg["n"]
        x = dev.alloc_uninitialized(np.uint32, n)
        S.synth_fill(dev, x, S.SYNTH_U32_LOW4, seed=1, index_base=rank * n if comm else 0, stream=sp)
        y = dev.alloc_uninitialized(np.uint32, n)
        lay = Layout.c_contiguous([n])
        bytes_per_step = 8 * n
        if comm:
            def step():
                comm.scan_into(CumSumOp, StridedView(x, lay), StridedView(y, lay), exclusive=True, stream=sp)
            launches_per_step = 4  # reduce, fold, scan + (NCCL all-gather, not ours)
        else:
            ops = H.CudaScanOps()

            def step():
                ops.scan_axis_into(CumSumOp, dev, StridedView(x, lay), 0, 0, StridedView(y, lay),
                                   exclusive=True, stream=sp)
        kernel_bytes = 8 * n
        kernel_step = None if not comm else (lambda: H.CudaScanOps().scan_axis_into(
            CumSumOp, dev, StridedView(x, lay), 0, 0, StridedView(y, lay), exclusive=True, stream=sp))
        units = n
    elif args.config == 1:
        n = cfg["n"]
        nbuf = 64
        bufs = []
        for b in range(nbuf):
            xb = dev.alloc_uninitialized(np.float32, n)
            S.synth_fill(dev, xb, S.SYNTH_F32_UNIFORM_PM1, seed=0, stream=sp)
            bufs.append(xb)
        out = dev.alloc_zeroed(np.float32, nbuf)
        lay = Layout.c_contiguous([n])
        ops = H.CudaFullReductionOps()
        # Throughput mode: the 64 prepared reductions over 64 rotating 4 MiB
        # buffers (256 MiB > L2) submitted as one batch (heph_batch_*), which
        # fuses them into one kernel recorded in a CUDA graph; a step replays it.
        prepared = [ops.prepare_reduce_full(SumOp, dev, StridedView(bufs[b], lay),
                                            StridedView(out, Layout.try_new([1], [1], b))) for b in range(nbuf)]
        batch = S.Batch(dev, prepared)

        def step():
            batch.launch(stream=sp)
        launches_per_step = 1
        bytes_per_step = 4 * n * nbuf
        kernel_bytes = 4 * n * nbuf  # one replay: one fused launch over the 64 buffers
        kernel_step = None
        units = n * nbuf
    elif args.config == 3:
        rows, cols = cfg["rows"], cfg["cols"]
        k = args.misalign
        ld = cols + k  # k > 0: every row starts at a different 16-byte misalignment
        x = dev.alloc_uninitialized(np.float32, rows * ld + k)
        S.synth_fill(dev, x, S.SYNTH_F32_NORMAL, seed=2, stream=sp)
        if k == 0:
            S.synth_inject_row_ties(dev, x, rows, cols, seed=2, stream=sp)
        vals = dev.alloc_zeroed(np.float32, rows)
        idx = dev.alloc_zeroed(np.uint32, rows)
        ops = H.CudaAxisReductionOps()
        il, ol = Layout.try_new([rows, cols], [ld, 1], k), Layout.c_contiguous([rows, 1])

        def step():
            ops.argmax_axis_into(dev, StridedView(x, il), 1, StridedView(vals, ol), StridedView(idx, ol),
                                 stream=sp)
        bytes_per_step = 4 * rows * cols + 8 * rows
        kernel_bytes = bytes_per_step
        kernel_step = None
        units = rows * cols
    elif args.config == 4:
        rows, cols = cfg["rows"], cfg["cols"]
        k = args.misalign
        ld = cols + (2 if k else 0)  # row stride stays a 16-byte multiple; the view starts k elements in
        x = dev.alloc_uninitialized(np.float64, rows * ld + k)
        S.synth_fill(dev, x, S.SYNTH_F64_UNIT, seed=3, stream=sp)
        out = dev.alloc_zeroed(np.float64, cols)
        ops = H.CudaAxisReductionOps()
        il, ol = Layout.try_new([rows, cols], [ld, 1], k), Layout.c_contiguous([1, cols])

        def step():
            ops.reduce_axis_into(SumOp, dev, StridedView(x, il), 0, StridedView(out, ol), stream=sp)
        bytes_per_step = 8 * rows * cols + 8 * cols
        kernel_bytes = bytes_per_step
        launches_per_step = 2  # column slices + slice finalize
        kernel_step = None
        units = rows * cols
    elif args.config == 10:
        n = cfg["n"]
        x = dev.alloc_uninitialized(np.float32, n)
        S.synth_fill(dev, x, S.SYNTH_F32_UNIFORM_PM1, seed=0, stream=sp)
        out = dev.alloc_zeroed(np.float32, 1)
        ops = H.CudaFullReductionOps()
        lay10 = Layout.c_contiguous([n])

        def step():
            ops.reduce_full_into(SumOp, dev, StridedView(x, lay10), StridedView(out, Layout.c_contiguous([1])),
                                 stream=sp)
        bytes_per_step = 4 * n
        kernel_bytes = bytes_per_step
        kernel_step = None
        units = n
    elif args.config in (6, 7):
        rows, cols, ld, off = cfg["rows"], cfg["cols"], cfg["ld"], cfg["offset"]
        x = dev.alloc_uninitialized(np.float32, rows * ld + off)
        S.synth_fill(dev, x, S.SYNTH_F32_UNIFORM_PM1, seed=0, stream=sp)
        out = dev.alloc_zeroed(np.float32, 1)
        view = Layout.try_new([rows, cols], [ld, 1], off)
        ops = H.CudaFullReductionOps()

        def step():
            ops.reduce_full_into(SumOp, dev, StridedView(x, view), StridedView(out, Layout.c_contiguous([1])),
                                 stream=sp)
        bytes_per_step = 4 * rows * cols
        kernel_bytes = bytes_per_step
        kernel_step = None
        units = rows * cols
    elif args.config in (8, 9):
        rows, cols = cfg["rows"], cfg["cols"]
        x = dev.alloc_uninitialized(np.uint32, rows * cols)
        S.synth_fill(dev, x, S.SYNTH_U32_LOW4, seed=1, stream=sp)
        y = dev.alloc_uninitialized(np.uint32, rows * cols)
        lay = Layout.c_contiguous([rows, cols])
        ops = H.CudaScanOps()

        def step():
            ops.scan_axis_into(CumSumOp, dev, StridedView(x, lay), 1, 0, StridedView(y, lay), stream=sp)
        bytes_per_step = 8 * rows * cols
        kernel_bytes = bytes_per_step
        kernel_step = None
        units = rows * cols
    else:  # config 5: strong scaling of 2^32 i32 over the ranks
        total = cfg["n"]
        n = (total + world - 1) // world
        n = min(n, total - rank * n)
        x = dev.alloc_uninitialized(np.int32, n)
        S.synth_fill(dev, x, S.SYNTH_I32_PM1000, seed=4, index_base=rank * ((total + world - 1) // world),
                     stream=sp)
        y = dev.alloc_uninitialized(np.int32, n)
        s64 = dev.alloc_zeroed(np.int64, 1)
        lay = Layout.c_contiguous([n])
        one = Layout.c_contiguous([1])
        if comm:
            # One pass over the slice yields both the scan's carry total and
            # the sum's partial; one all-gather exchanges both.
            def step():
                comm.scan_reduce_into(CumSumOp, StridedView(x, lay), StridedView(y, lay), SumOp,
                                      StridedView(s64, one), stream=sp)
            launches_per_step = 3  # dual reduction, rank fold, scan (+ the NCCL all-gather)
        else:
            sops, fops = H.CudaScanOps(), H.CudaFullReductionOps()

            def step():
                sops.scan_axis_into(CumSumOp, dev, StridedView(x, lay), 0, 0, StridedView(y, lay), stream=sp)
                fops.reduce_full_into(SumOp, dev, StridedView(x, lay), StridedView(s64, one), stream=sp)
            launches_per_step = 2
        bytes_per_step = 8 * n + 4 * n  # scan r+w, then the widening sum reads again
        kernel_bytes = 8 * n
        kernel_step = lambda: H.CudaScanOps().scan_axis_into(  # noqa: E731
            CumSumOp, dev, StridedView(x, lay), 0, 0, StridedView(y, lay), stream=sp)
        units = n
        slice_lo = rank * ((total + world - 1) // world)
    dev.synchronize_stream(sp)
    total_units = units * world

    # ---------------- warm-up, then exactly K timed steps -------------
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    dev.synchronize_stream(sp)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    with ClockSampler(local) as clocks:
        time.sleep(0.3)
        barrier()
        t_all0 = torch.cuda.Event(enable_timing=True)
        t_all1 = torch.cuda.Event(enable_timing=True)
        t_all0.record(stream)
        for k in range(args.steps):
            starts[k].record(stream)
            step()
            ends[k].record(stream)
        t_all1.record(stream)
        dev.synchronize_stream(sp)
        barrier()
    total_ms_local = t_all0.elapsed_time(t_all1)
    total_ms = max_over_ranks(total_ms_local)
    per_launch_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms_per_step = total_ms / args.steps
    value = bytes_per_step * world * args.steps / (total_ms / 1e3) / 1e9

    # ---------------- correctness of the timed results (config 5) -------------
    check_result = None
    if args.config == 5 and not args.no_check:
        check_result = check_config5(dev, x, y, s64, n, slice_lo, cfg["n"], rank, world, dist, local)

    # ---------------- dominant kernel roofline -------------
    if kernel_step is not None:
        ks, ke = [], []
        with torch.cuda.stream(stream):
            for _ in range(3):
                kernel_step()
            for _ in range(10):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                kernel_step()
                b.record(stream)
                ks.append(a)
                ke.append(b)
        dev.synchronize_stream(sp)
        kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in zip(ks, ke))
    else:
        kernel_ms = statistics.mean(per_launch_ms)
    achieved = kernel_bytes / (kernel_ms / 1e3) / 1e9
    traffic = profiled_traffic(cfg["kernel"], args.config)

    latency = None
    if args.config == 1:
        # Latency mode: single 4 MiB reductions (reduce_dense_kernel), each its
        # own call over rotating buffers.  (a) back to back: 64 calls queued
        # behind a spin, so the events time the device and not the host's
        # issue: device time per call; (b) one call on its own, bracketed by
        # events behind a replay of the batch (median of 20).
        with torch.cuda.stream(stream):
            per_call = []
            for rep in range(5):
                torch.cuda._sleep(10_000_000)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for k in range(nbuf):
                    ops.reduce_full_into(SumOp, dev, StridedView(bufs[k], lay),
                                         StridedView(out, Layout.try_new([1], [1], k)), stream=sp)
                b.record(stream)
                per_call.append((a, b))
            ls, le = [], []
            for k in range(23):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                batch.launch(stream=sp)
                a.record(stream)
                ops.reduce_full_into(SumOp, dev, StridedView(bufs[k % nbuf], lay),
                                     StridedView(out, Layout.try_new([1], [1], k % nbuf)), stream=sp)
                b.record(stream)
                ls.append(a)
                le.append(b)
        dev.synchronize_stream(sp)
        us = statistics.median(a.elapsed_time(b) * 1e3 / nbuf for a, b in per_call)
        single = statistics.median(a.elapsed_time(b) * 1e3 for a, b in list(zip(ls, le))[3:])
        latency = {"us_per_reduction": round(us, 3), "mode": "64 separate calls back to back, per call",
                   "single_call_us": round(single, 3), "kernel": "reduce_dense_kernel",
                   "gbs": round(4 * n / (us / 1e6) / 1e9, 2)}

    # ---------------- end to end through the public API with host buffers -------------
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, cfg, dev, stream, sp, world, rank, comm, max_over_ranks, barrier)

    # ---------------- CPU baseline (rank 0, N=1 only) -------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        # The reference arm in a fresh process (no CUDA / torch runtime in it),
        # so the baseline is measured exactly as the reference line is.
        env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
        res = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference", "--config",
                              str(args.config), "--steps", "2", "--warmup", "1"],
                             capture_output=True, text=True, env=env, timeout=600)
        try:
            ref = json.loads(res.stdout.strip().splitlines()[-1])
            cpu = dict(ref["cpu_baseline"])
        except Exception:
            cpu = {"value": None, "unit": "GB/s", "cores": None, "kind": "port",
                   "sample": "reference arm failed: " + res.stderr[-200:]}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6),
            "higher_is_better": True, "scaling": "weak" if args.config != 5 else "strong",
            "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic",
            "config": config_dict(args, cfg, world),
            "elements_per_s": round(total_units / (ms_per_step / 1e3), 1),
            "fraction_of_hbm_peak": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": cfg["kernel"], "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": kernel_bytes,
                         "launch_ms": round(kernel_ms, 6)},
            "cpu_baseline": cpu,
            "e2e": e2e,
            **({"latency_mode": latency} if latency else {}),
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * args.steps,
            **({"check": check_result["status"], "check_detail": check_result["detail"]} if check_result else {}),
            **({"exchange": "peer memory (one kernel)" if comm.peer_exchange else "ncclAllGather"} if comm else {}),
        }
        print(json.dumps(line), flush=True)
    if comm:
        comm.destroy()
    if dist:
        dist.destroy_process_group()
    return 0 if check_result is None or check_result["status"] == "ok" else 1


def check_config5(dev, x, y, s64, n, lo, total, rank, world, dist, local):
    """Element-by-element check of the timed step's results with numpy (not
    the oracle: the product's own bench checks itself independently).  Each
    rank downloads its slice in 1 GiB pieces and checks y = carry + the
    wrapping running sum of x, where carry is read off y[0] - x[0]; the ranks
    then exchange their slice sums and carries: every carry must be the
    wrapped sum of the lower ranks' slices, and the i64 result on every rank
    the sum of all slices."""
    import torch

    def wrap32(v):
        return (v + (1 << 31)) % (1 << 32) - (1 << 31)

    piece = 1 << 28
    xs, ys = np.empty(min(piece, n), np.int32), np.empty(min(piece, n), np.int32)
    local_sum, carry, running, bad = 0, None, 0, -1
    t0 = time.perf_counter()
    for off in range(0, n, piece):
        m = min(piece, n - off)
        dev.download_sub_buffer(x, off, xs[:m])
        dev.download_sub_buffer(y, off, ys[:m])
        if carry is None:
            carry = wrap32(int(ys[0]) - int(xs[0]))
            running = carry
        want = np.cumsum(xs[:m], dtype=np.int32)
        want += np.int32(running)  # wraps, as the scan does
        if bad < 0 and not np.array_equal(want, ys[:m]):
            bad = off + int(np.argmax(want != ys[:m]))
        running = int(want[-1])
        local_sum += int(xs[:m].sum(dtype=np.int64))
    got_sum = int(dev.download_owned(s64)[0])
    mine = torch.tensor([local_sum, carry, got_sum, bad], dtype=torch.int64, device=f"cuda:{local}")
    if dist:
        every = torch.empty(world * 4, dtype=torch.int64, device=f"cuda:{local}")
        dist.all_gather_into_tensor(every, mine)
        rows = every.view(world, 4).cpu().tolist()
    else:
        rows = [mine.cpu().tolist()]
    grand = sum(r[0] for r in rows)
    problems = []
    for r, (ls, c, gs, b) in enumerate(rows):
        if b >= 0:
            problems.append(f"rank {r}: scan differs from element {b} of its slice")
        if c != wrap32(sum(q[0] for q in rows[:r])):
            problems.append(f"rank {r}: carry {c} is not the wrapped sum of the lower slices")
        if gs != grand:
            problems.append(f"rank {r}: i64 sum {gs} != {grand}")
    detail = (f"{total} elements on {world} rank(s): every scan output against a numpy wrapping cumsum of the "
              f"downloaded input seeded with the rank's carry, carries against the lower slices' sums, the "
              f"i64 sum ({grand}) against numpy; {time.perf_counter() - t0:.1f} s")
    if problems:
        return {"status": "failed", "detail": "; ".join(problems[:4])}
    return {"status": "ok", "detail": detail}


def run_e2e(args, cfg, dev, stream, sp, world, rank, comm, max_over_ranks, barrier):
    """Same metric through the public API: pinned host input uploaded, the path
    run, the result read back, every step inside the timed region."""
    import ctypes

    import torch

    import hephaestus_b200 as H
    from hephaestus_b200 import _native as N
    from hephaestus_b200.core import CumSumOp, Layout, StridedView, SumOp, check

    pins = []

    def pinned(nbytes):
        p = ctypes.c_void_p()
        check(N.lib.heph_host_alloc_pinned(nbytes, ctypes.byref(p)))
        pins.append(p)
        return p

    if args.config == 2:
        n = cfg["n"]
        hin, hout = pinned(4 * n), pinned(4 * n)
        x = dev.alloc_uninitialized(np.uint32, n)
        y = dev.alloc_uninitialized(np.uint32, n)
        lay = Layout.c_contiguous([n])

        if comm is None:
            # One call through the public host-buffer entry point: chunked
            # copies and scans overlapped on both copy engines.
            def e2e_step():
                check(N.lib.heph_scan_host(dev.handle, N.SUM, 1, N.U32, hin, hout, n, 0))
        else:
            def e2e_step():
                check(N.lib.heph_buffer_upload_async(dev.handle, x.handle, 0, hin, n, ctypes.c_void_p(sp)))
                comm.scan_into(CumSumOp, StridedView(x, lay), StridedView(y, lay), exclusive=True, stream=sp)
                check(N.lib.heph_buffer_download_async(dev.handle, y.handle, 0, hout, n, ctypes.c_void_p(sp)))
        bytes_step, h2d, d2h = 8 * n, 4 * n, 4 * n
    elif args.config == 5:
        total = cfg["n"]
        per = (total + world - 1) // world
        n = min(per, total - rank * per)
        hin, hout, hsum = pinned(4 * n), pinned(4 * n), pinned(8)
        x = dev.alloc_uninitialized(np.int32, n)
        y = dev.alloc_uninitialized(np.int32, n)
        s64 = dev.alloc_zeroed(np.int64, 1)
        lay, one = Layout.c_contiguous([n]), Layout.c_contiguous([1])
        if comm is None:
            # One call through the public host-buffer entry point: the slice
            # flows through device slots in chunks, uploads, scans + sums and
            # downloads overlapped on both copy engines.
            def e2e_step():
                check(N.lib.heph_scan_reduce_host(dev.handle, N.SUM, 0, N.I32, hin, hout, n, N.SUM, N.I64, hsum, 0))
        else:
            # The carry needs every rank's total first, so the slice is
            # uploaded whole, then scanned + summed, then downloaded.
            def e2e_step():
                check(N.lib.heph_buffer_upload_async(dev.handle, x.handle, 0, hin, n, ctypes.c_void_p(sp)))
                comm.scan_reduce_into(CumSumOp, StridedView(x, lay), StridedView(y, lay), SumOp,
                                      StridedView(s64, one), stream=sp)
                check(N.lib.heph_buffer_download_async(dev.handle, y.handle, 0, hout, n, ctypes.c_void_p(sp)))
                check(N.lib.heph_buffer_download_async(dev.handle, s64.handle, 0, hsum, 1, ctypes.c_void_p(sp)))
        bytes_step, h2d, d2h = 12 * n, 4 * n, 4 * n + 8
    elif args.config in (1, 10):
        n = cfg["n"]
        hin = pinned(4 * n)
        hout = pinned(4)
        x = dev.alloc_uninitialized(np.float32, n)
        out = dev.alloc_zeroed(np.float32, 1)
        lay = Layout.c_contiguous([n])
        ops = H.CudaFullReductionOps()

        def e2e_step():
            check(N.lib.heph_buffer_upload_async(dev.handle, x.handle, 0, hin, n, ctypes.c_void_p(sp)))
            ops.reduce_full_into(SumOp, dev, StridedView(x, lay), StridedView(out, Layout.c_contiguous([1])),
                                 stream=sp)
            check(N.lib.heph_buffer_download_async(dev.handle, out.handle, 0, hout, 1, ctypes.c_void_p(sp)))
        bytes_step, h2d, d2h = 4 * n, 4 * n, 4
    elif args.config == 3:
        rows, cols = cfg["rows"], cfg["cols"]
        hin, hv, hi = pinned(4 * rows * cols), pinned(4 * rows), pinned(4 * rows)
        x = dev.alloc_uninitialized(np.float32, rows * cols)
        vals, idx = dev.alloc_zeroed(np.float32, rows), dev.alloc_zeroed(np.uint32, rows)
        ops = H.CudaAxisReductionOps()
        il, ol = Layout.c_contiguous([rows, cols]), Layout.c_contiguous([rows, 1])

        def e2e_step():
            check(N.lib.heph_buffer_upload_async(dev.handle, x.handle, 0, hin, rows * cols, ctypes.c_void_p(sp)))
            ops.argmax_axis_into(dev, StridedView(x, il), 1, StridedView(vals, ol), StridedView(idx, ol), stream=sp)
            check(N.lib.heph_buffer_download_async(dev.handle, vals.handle, 0, hv, rows, ctypes.c_void_p(sp)))
            check(N.lib.heph_buffer_download_async(dev.handle, idx.handle, 0, hi, rows, ctypes.c_void_p(sp)))
        bytes_step, h2d, d2h = 4 * rows * cols + 8 * rows, 4 * rows * cols, 8 * rows
    elif args.config in (6, 7):
        rows, cols, ld, off = cfg["rows"], cfg["cols"], cfg["ld"], cfg["offset"]
        total = rows * ld + off
        hin, ho = pinned(4 * total), pinned(4)
        x = dev.alloc_uninitialized(np.float32, total)
        out = dev.alloc_zeroed(np.float32, 1)
        view = Layout.try_new([rows, cols], [ld, 1], off)
        ops = H.CudaFullReductionOps()

        def e2e_step():
            check(N.lib.heph_buffer_upload_async(dev.handle, x.handle, 0, hin, total, ctypes.c_void_p(sp)))
            ops.reduce_full_into(SumOp, dev, StridedView(x, view), StridedView(out, Layout.c_contiguous([1])),
                                 stream=sp)
            check(N.lib.heph_buffer_download_async(dev.handle, out.handle, 0, ho, 1, ctypes.c_void_p(sp)))
        bytes_step, h2d, d2h = 4 * rows * cols, 4 * total, 4
    elif args.config in (8, 9):
        rows, cols = cfg["rows"], cfg["cols"]
        n = rows * cols
        hin, ho = pinned(4 * n), pinned(4 * n)
        x, y = dev.alloc_uninitialized(np.uint32, n), dev.alloc_uninitialized(np.uint32, n)
        lay = Layout.c_contiguous([rows, cols])
        ops = H.CudaScanOps()

        def e2e_step():
            check(N.lib.heph_buffer_upload_async(dev.handle, x.handle, 0, hin, n, ctypes.c_void_p(sp)))
            ops.scan_axis_into(CumSumOp, dev, StridedView(x, lay), 1, 0, StridedView(y, lay), stream=sp)
            check(N.lib.heph_buffer_download_async(dev.handle, y.handle, 0, ho, n, ctypes.c_void_p(sp)))
        bytes_step, h2d, d2h = 8 * n, 4 * n, 4 * n
    else:
        rows, cols = cfg["rows"], cfg["cols"]
        hin, ho = pinned(8 * rows * cols), pinned(8 * cols)
        x = dev.alloc_uninitialized(np.float64, rows * cols)
        out = dev.alloc_zeroed(np.float64, cols)
        ops = H.CudaAxisReductionOps()
        il, ol = Layout.c_contiguous([rows, cols]), Layout.c_contiguous([1, cols])

        def e2e_step():
            check(N.lib.heph_buffer_upload_async(dev.handle, x.handle, 0, hin, rows * cols, ctypes.c_void_p(sp)))
            ops.reduce_axis_into(SumOp, dev, StridedView(x, il), 0, StridedView(out, ol), stream=sp)
            check(N.lib.heph_buffer_download_async(dev.handle, out.handle, 0, ho, cols, ctypes.c_void_p(sp)))
        bytes_step, h2d, d2h = 8 * rows * cols + 8 * cols, 8 * rows * cols, 8 * cols

    steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    dev.synchronize_stream(sp)
    dev.synchronize()
    barrier()
    # Host clock around fully synchronised steps: the copies of the pipelined
    # entry point run on its own streams, and every step ends with the result
    # in host memory.
    t0 = time.perf_counter()
    for _ in range(steps):
        e2e_step()
        dev.synchronize_stream(sp)
    ms = max_over_ranks((time.perf_counter() - t0) * 1e3) / steps
    for p in pins:  # the host memory goes back before the CPU baseline runs
        check(N.lib.heph_host_free_pinned(p))
    return {"value": round(bytes_step * world / (ms / 1e3) / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 4),
            "steps": steps}


if __name__ == "__main__":
    sys.exit(main())
