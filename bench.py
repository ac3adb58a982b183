#!/usr/bin/env python3
"""Benchmark: bf16 weight rows -> GGML blocks on B200, the reference's headline metric.

Workload (the metric's quoted config that fits one GPU):
Q4_K with imatrix (--pure) over eight bf16 tensors, 4 x (4096 x 4096) and 4 x (14336 x 4096),
N(0, 0.02) with 0.1 % N(0, 0.5) outliers, per-column imatrix lognormal(0, 1.5). Synthetic
data generated on the device from fixed seeds; 302 M values = 604 MB of bf16 per step, larger
than the 126 MB L2, so no L2 flush is needed between steps.

One step = quantize all eight tensors (eight kernel launches). N GPUs: one process per GPU,
each quantizes its own tensor set (weak scaling, no collective on the data path; NCCL is used
only for the barrier and the max-over-ranks of the timings).

  value  input GB/s with inputs resident in HBM (whole job, all ranks)
  e2e    the same metric through the public API from pinned host buffers: per step every
         tensor is copied host->device, quantized and its blocks copied back to host, in
         row chunks with the copies and kernels overlapped on three streams; beside it the
         same copies with no kernels, on every rank at once (`copy_ceiling`)
  roofline  the Q4_K kernel against the FP32 lane-op ceiling (148 SMs x 128 lanes x SM clock):
         algorithmic ops = 655 per value (37 x 17 per candidate step + 11 initial + 3 sums
         + 5 weights + 7 requant/pack); plus the HBM view of the same launches, and ncu's
         DRAM bytes and thread instructions per value of one launch (profiles/traffic_*.json)
  config1 / config3  (one GPU) BASELINE configs[0] (Q4_0 of one 4096 x 4096 tensor, against
         HBM) and configs[2] (IQ2_XXS set + the 151936 x 2560 embedding as Q4_0)
cpu_baseline  the CPU restatement of the reference's algorithm (oracle/) on all host cores over
         a bounded sample of the workload; the same sample is quantized on the GPU and
         `identical_blocks` is the fraction of blocks that match; `vs_reference`: the GPU
         output on the configs[1] rows of tests/golden/config_parity.json against the
         reference's own outputs there (identical-block fraction vs the shipped reference)
--impl reference: the CPU restatement of the reference's algorithm (oracle/) on all host
cores over a bounded sample of the same workload (the reference's eager code is Python and
oracle/ is its bit-exact C port, about 10x faster than it); beside it, the reference itself
from its copy in baseline/_ref: its torch CPU path on all host cores (`reference_torch_cpu`)
and its GPU path (torch + Triton) on the same B200 and workload (`reference_gpu`).
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "quant-studio_b200"))
sys.path.insert(0, str(ROOT))

SHAPES_C2 = [(4096, 4096)] * 4 + [(14336, 4096)] * 4
NAMES_C2 = [f"blk.{i}.attn_q.weight" for i in range(4)] + [f"blk.{i}.ffn_up.weight" for i in range(4)]
# algorithmic FP32 lane ops per value for each (type, imatrix) the bench can time
ALG_OPS = {("q4_k", True): 655, ("q4_k", False): 21 * 17 + 11 + 3 + 4 + 7,
           # Q5_K / Q2_K with imatrix: the same make_qkx search (37 steps x 17 lane ops per value)
           ("q5_k", True): 655, ("q2_k", True): 655,
           ("q6_k", False): 19 * 9 + 20, ("q6_k", True): 19 * 9 + 18, ("q4_0", False): 10, ("q4_0", True): 10,
           # IQ lattice searches, counted on the benchmark distribution (off-grid problems and
           # neighbour-list lengths from an instrumented run): candidates per value x (4 ops per
           # position + 1 compare) + sweep steps x 12 (levels, accept sums) + 15 (weights,
           # signs) [+ 110 for IQ2_XXS's initial make_qp fit]; candidates per value 39.1 /
           # 93.3 / 13.3 / 50.8 / 38.9
           ("iq2_xxs", True): round(39.1 * 33) + 14 * 12 + 15 + 110, ("iq2_xs", True): round(93.3 * 33) + 20 * 12 + 15,
           ("iq2_s", True): round(13.3 * 33) + 20 * 12 + 15, ("iq3_xxs", True): round(50.8 * 17) + 32 * 12 + 15,
           ("iq3_s", True): round(38.9 * 17) + 20 * 12 + 15,
           # the 32-value block formats: block max/min, one scale, 3-4 ops per value
           ("q4_1", False): 10, ("q5_0", False): 10, ("q5_1", False): 10, ("q8_0", False): 8,
           # Q3_K: with imatrix the make_qx search of Q6_K (nmax 4); without, make_q3_quants: the
           # initial fit (9 per value), 5 greedy passes x 19 (both sums' updates, the division,
           # round, clamps, the comparison), the superblock-scale fit and packing (19)
           ("q3_k", True): 19 * 9 + 18, ("q3_k", False): 9 + 5 * 19 + 19,
           # IQ4_XS: 16 candidate scales x 14 (id x, the 4-step bracket and midpoint compare of
           # the non-linear grid, two weighted products and sums) + 18 (weights, requantize, pack)
           ("iq4_xs", True): 16 * 14 + 18, ("iq4_xs", False): 16 * 14 + 18}
ALG_BYTES_OUT = {"q4_0": 18 / 32, "q2_k": 84 / 256, "q3_k": 110 / 256, "q4_k": 144 / 256,
                 "q5_k": 176 / 256, "q6_k": 210 / 256, "iq4_xs": 136 / 256, "iq2_xxs": 66 / 256,
                 "iq2_xs": 74 / 256, "iq2_s": 82 / 256, "iq3_xxs": 98 / 256, "iq3_s": 110 / 256,
                 "q4_1": 20 / 32, "q5_0": 22 / 32, "q5_1": 24 / 32, "q8_0": 34 / 32}
TYPE_IDS = {"q4_0": 2, "q4_1": 3, "q5_0": 6, "q5_1": 7, "q8_0": 8, "q2_k": 10, "q3_k": 11, "q4_k": 12,
            "q5_k": 13, "q6_k": 14, "iq2_xxs": 16, "iq2_xs": 17, "iq3_xxs": 18, "iq3_s": 21, "iq2_s": 22,
            "iq4_xs": 23}
IMATRIX_FREE = ("q4_0", "q4_1", "q5_0", "q5_1", "q8_0")  # formats that ignore importance weights


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if not self.rows:
            return None
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def max_over_ranks(dist, value: float, device) -> float:
    """The slowest rank's time: every rank takes the same all_reduce(MAX) step."""
    if dist is None:
        return value
    import torch
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(torch, device, seed: int, shapes):
    """Seeded synthetic bf16 weights + lognormal imatrix, generated on the device."""
    g = torch.Generator(device=device)
    xs, qws = [], []
    for i, (r, c) in enumerate(shapes):
        g.manual_seed(seed * 1000 + i)
        x = torch.empty((r, c), dtype=torch.float32, device=device).normal_(0.0, 0.02, generator=g)
        out = torch.rand((r, c), device=device, generator=g) < 0.001
        x[out] = torch.empty(int(out.sum()), device=device).normal_(0.0, 0.5, generator=g)
        xs.append(x.to(torch.bfloat16))
        del x, out
        qws.append(torch.empty(c, device=device).log_normal_(0.0, 1.5, generator=g))
    return xs, qws


REF_DIR = ROOT / "baseline" / "_ref" / "quant-studio"
# the reference's entry point per type: (module, function) in its kernels package
REF_FUNCS = {"q4_0": ("q4_0", "quantize_q4_0"), "q2_k": ("q2_k", "quantize_q2_k"), "q3_k": ("q3_k", "quantize_q3_k"),
             "q4_k": ("q4_k", "quantize_q4_k"), "q5_k": ("q5_k", "quantize_q5_k"), "q6_k": ("q6_k", "quantize_q6_k"),
             "iq4_xs": ("iq4_xs", "quantize_iq4_xs"), "iq2_xxs": ("iq2", "quantize_iq2_xxs"),
             "iq2_xs": ("iq2_xs", "quantize_iq2_xs"), "iq2_s": ("iq2_s", "quantize_iq2_s"),
             "iq3_xxs": ("iq3_xxs", "quantize_iq3_xxs"), "iq3_s": ("iq3_s", "quantize_iq3_s")}


def reference_quantizer(qtype: str):
    """The reference's own quantize_<type>, imported unmodified from its copy in baseline/_ref
    (its GPU path: torch ops on CUDA plus its Triton kernels; its CPU path: torch eager). pip
    gguf 0.19 lacks two enum members the reference's policy module names (GGMLQuantizationType
    .Q2_0, LlamaFileType.MOSTLY_Q2_0); they are added first, as placeholders, so that its
    package imports. Returns None when the copy is absent."""
    if not REF_DIR.exists() or qtype not in REF_FUNCS:
        return None
    from gguf import GGMLQuantizationType as GT
    from gguf.constants import LlamaFileType as FT

    def add(cls, name, value):
        if hasattr(cls, name):
            return
        m = int.__new__(cls, value)
        m._name_, m._value_ = name, value
        type.__setattr__(cls, name, m)
        cls._member_map_[name] = m
        cls._value2member_map_[value] = m
        cls._member_names_.append(name)

    add(FT, "MOSTLY_Q2_0", 1000)
    add(GT, "Q2_0", 1000)
    sys.dont_write_bytecode = True
    sys.path[:] = [p for p in sys.path if not p.rstrip("/").endswith("quant-studio_b200")]
    sys.path.insert(0, str(REF_DIR))
    import importlib
    mod, fn = REF_FUNCS[qtype]
    return getattr(importlib.import_module(f"kernels.{mod}"), fn)


def reference_torch_cpu(args, fn, qw_np, sample) -> dict:
    """The reference's own CPU path (torch eager, all host threads) on a bounded sample."""
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    qw = None if qw_np is None else torch.from_numpy(qw_np)

    def call(a):
        xt = torch.from_numpy(a)
        return fn(xt) if args.qtype == "q4_0" else fn(xt, qw)

    call(sample(8))
    probe = sample(64)
    t0 = time.perf_counter()
    call(probe)
    rate = probe.size / max(time.perf_counter() - t0, 1e-6)
    rows = int(min(4096, max(64, rate * 4.0 / probe.shape[1])))
    x = sample(rows)
    t0 = time.perf_counter()
    call(x)
    dt = time.perf_counter() - t0
    return {"value": round(x.size * 2 / dt / 1e9, 6), "unit": "GB/s", "cores": cores,
            "torch_threads": torch.get_num_threads(), "kind": "reference (torch eager CPU path, unmodified)",
            "sample": f"{rows} rows x {x.shape[1]} values ({x.size * 2 / 1e6:.1f} MB bf16), {dt:.2f} s"}


def reference_gpu(args, fn) -> dict:
    """The reference's own GPU path (torch ops on CUDA + its Triton kernels), unmodified, on the
    same workload and device as the qsb200 arm: device-resident bf16 tensors, upcast to float32
    as its pipeline does (quant-studio.py:197), then quant_fn; CUDA events around each step."""
    import torch
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    xs, qws = make_inputs(torch, device, seed=0, shapes=SHAPES_C2)
    if not args.imatrix or args.qtype == "q4_0":
        qws = [None] * len(xs)

    def step():
        outs = []
        for x, q in zip(xs, qws):
            xf = x.to(torch.float32)
            outs.append(fn(xf) if args.qtype == "q4_0" else fn(xf, q))
        return outs

    t0 = time.perf_counter()
    step()                               # Triton JIT compiles here
    torch.cuda.synchronize()
    compile_s = time.perf_counter() - t0
    for _ in range(max(1, args.warmup - 1)):
        step()
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    n = sum(r * c for r, c in SHAPES_C2)
    return {"value": round(2 * n / (ms * 1e-3) / 1e9, 4), "unit": "GB/s", "ms_per_step": round(ms, 3),
            "steps": steps, "first_step_s": round(compile_s, 2),
            "kind": "reference GPU path (torch + Triton, unmodified), same B200, device-resident bf16 inputs "
                    "upcast to f32 as its pipeline does", "device": torch.cuda.get_device_name(device)}


def run_reference(args, config: dict) -> None:
    """The reference arm: the CPU port of the reference algorithm on all host threads, with the
    reference's own CPU path and its GPU path on the same box beside it."""
    import oracle

    cores = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    k = 4096
    qw = rng.lognormal(0.0, 1.5, k).astype(np.float32)

    def sample(rows):
        a = rng.normal(0.0, 0.02, (rows, k))
        m = rng.random(a.shape) < 0.001
        a[m] = rng.normal(0.0, 0.5, int(m.sum()))
        # bf16-representable values, as the bf16 weights are
        return ((a.astype(np.float32).view(np.uint32) + 0x8000) & 0xFFFF0000).view(np.float32)

    oracle.quantize(args.qtype, sample(8), qw, nthreads=1)  # one-time table set-up
    probe = sample(256)
    t0 = time.perf_counter()
    oracle.quantize(args.qtype, probe, qw if args.imatrix else None, nthreads=cores)
    rate = probe.size / max(time.perf_counter() - t0, 1e-6)
    rows = int(min(8192, max(64, rate * args.ref_seconds / k)))
    x = sample(rows)
    for _ in range(args.warmup):
        oracle.quantize(args.qtype, x[:64], qw if args.imatrix else None, nthreads=cores)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.quantize(args.qtype, x, qw if args.imatrix else None, nthreads=cores)
        times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    gbs = x.size * 2 / dt / 1e9
    extra = {}
    ref_fn = None
    try:
        ref_fn = reference_quantizer(args.qtype)
    except Exception as e:  # the unmodified reference failed to import
        extra["reference_import_error"] = f"{type(e).__name__}: {e}"[:300]
    if ref_fn is not None:
        try:
            extra["reference_torch_cpu"] = reference_torch_cpu(args, ref_fn, qw if args.imatrix else None, sample)
        except Exception as e:
            extra["reference_torch_cpu"] = {"error": f"{type(e).__name__}: {e}"[:300]}
        if args.ref_gpu:
            try:
                extra["reference_gpu"] = reference_gpu(args, ref_fn)
            except Exception as e:
                extra["reference_gpu"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    elif "reference_import_error" not in extra:
        extra["reference_torch_cpu"] = {"unavailable": f"no copy of the reference at {REF_DIR.relative_to(ROOT)}"}
    line = {"impl": "reference", "value": round(gbs, 6),
            "metric": f"input GB/s quantized (bf16->{args.qtype}{', imatrix' if args.imatrix else ''})",
            "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(gbs, 6), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"{rows} rows x {k} bf16 values per step ({x.size * 2 / 1e6:.1f} MB) "
                                       f"of the benchmark distribution, median of {args.steps} steps"},
            "e2e": {"value": round(gbs, 6), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    line.update(extra)
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="qsb200", choices=["qsb200", "reference"])
    ap.add_argument("--qtype", default="q4_k")
    ap.add_argument("--no-imatrix", dest="imatrix", action="store_false")
    ap.add_argument("--ref-seconds", type=float, default=1.0, help="CPU seconds per reference step")
    ap.add_argument("--no-ref-gpu", dest="ref_gpu", action="store_false",
                    help="--impl reference: skip timing the reference's own GPU path")
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--op", default="quantize", choices=["quantize", "dequantize", "tensor_error", "cli"],
                    help="quantize (the headline line); or time the block decode / the decode-error sum "
                         "over the blocks of the same workload (HBM-bound, one GPU); or `cli`: the drop-in "
                         "CLI on a whole synthetic model (BASELINE configs 4 / 5), sharded over --gpus")
    ap.add_argument("--model", default="4b", choices=["4b", "8b"], help="--op cli: synthetic model class")
    ap.add_argument("--scheme", default=None, help="--op cli: scheme (default Q4_K_M for 4b, IQ3_XXS for 8b)")
    ap.add_argument("--model-dir", default=None, help="--op cli: directory for the synthetic model and output")
    ap.add_argument("--mem", default="4G", help="--op cli: the CLI's --mem")
    ap.add_argument("--no-configs", dest="configs", action="store_false",
                    help="skip the config-1 / config-3 keys of the default line")
    args = ap.parse_args()
    if args.op == "cli":
        bench_cli(args)
        return
    args.warmup = max(args.warmup, 3)
    if args.qtype in IMATRIX_FREE:
        args.imatrix = False

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n_elem = sum(r * c for r, c in SHAPES_C2)
    config = {"workload": f"BASELINE configs[1]: {args.qtype}{' + imatrix' if args.imatrix else ''} --pure over "
                          f"4 x 4096x4096 + 4 x 14336x4096 bf16 tensors per GPU",
              "tensors": len(SHAPES_C2), "values_per_gpu": n_elem, "input_bytes_per_gpu": 2 * n_elem,
              "l2": "inputs 604 MB/GPU > 126 MB L2: no flush needed", "parallelism": f"shard{world}"}

    if args.impl == "reference":
        if rank == 0:
            run_reference(args, config)
        return

    import torch

    from kernels import _native

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    gt = TYPE_IDS[args.qtype]
    xs, qws = make_inputs(torch, device, seed=rank, shapes=SHAPES_C2)
    if not args.imatrix:
        qws = [None] * len(xs)
    outs = [torch.empty((x.shape[0], _native.row_bytes(gt, x.shape[1])), dtype=torch.uint8, device=device)
            for x in xs]
    stream = torch.cuda.Stream(device)
    if args.op != "quantize":
        bench_decode_op(torch, _native, gt, xs, qws, outs, stream, device, args, config, n_elem)
        return

    def step(evs=None):
        for i, (x, q, o) in enumerate(zip(xs, qws, outs)):
            if evs is not None:
                evs[i][0].record(stream)
            _native.quantize_into(gt, x, q, o, stream)
            if evs is not None:
                evs[i][1].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    kev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in xs]
           for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        t_start.record(stream)
        for s in range(args.steps):
            step(kev[s])
        t_end.record(stream)
        stream.synchronize()
        barrier()
    ms_total = t_start.elapsed_time(t_end)
    kern_ms = [[a.elapsed_time(b) for a, b in ev] for ev in kev]
    launch_ms = sum(sum(k) for k in kern_ms) / (args.steps * len(xs))

    def allmax(v: float) -> float:
        return max_over_ranks(dist, v, device)

    ms_total = allmax(ms_total)
    ms_step = ms_total / args.steps
    value = world * 2 * n_elem / (ms_step * 1e-3) / 1e9

    # roofline of the quantize kernel: lane ops (compute bound) and bytes (HBM view)
    clocks = clk.summary()
    peaks = measured_peaks()
    sm_count = torch.cuda.get_device_properties(device).multi_processor_count
    sm_mhz = (clocks or {}).get("sm_mhz") or peaks.get("clocks_under_load", {}).get("sm_mhz_median") or 1965.0
    ops = ALG_OPS.get((args.qtype, args.imatrix))
    elems_per_launch = n_elem / len(xs)
    peak_info = {"sm_count": sm_count, "sm_mhz": sm_mhz, "peaks": peaks}
    alg_bytes = elems_per_launch * (2 + ALG_BYTES_OUT[args.qtype])
    hbm = {"bound": "hbm", "achieved": round(alg_bytes / (launch_ms * 1e-3) / 1e9, 2), "peak": peaks["hbm_gbs"],
           "unit": "GB/s", "peak_source": "MEASURED_PEAKS.json hbm_gbs" if not peaks.get("fallback") else "fallback"}
    hbm["frac"] = round(hbm["achieved"] / hbm["peak"], 4)
    # the binding roofline is the slower of the two bounds: bytes at HBM bandwidth and
    # algorithmic lane ops at the FP32 lane peak; the other one is reported inside it
    lane_peak = sm_count * 128 * sm_mhz * 1e6 / 1e12
    if ops is not None and ops / (lane_peak * 1e12) > (2 + ALG_BYTES_OUT[args.qtype]) / (peaks["hbm_gbs"] * 1e9):
        roof = {"bound": "fp32-lane", "achieved": round(ops * elems_per_launch / (launch_ms * 1e-3) / 1e12, 3),
                "peak": round(lane_peak, 3), "unit": "Tops/s",
                "peak_source": f"{sm_count} SMs x 128 FP32 lanes x {sm_mhz:.0f} MHz median SM clock in the timed region",
                "ops_per_value": ops, "hbm": hbm, "traffic": None}
        roof["frac"] = round(roof["achieved"] / roof["peak"], 4)
    else:
        roof = dict(hbm, traffic=None)
        if ops is not None:
            lane_ach = ops * elems_per_launch / (launch_ms * 1e-3) / 1e12
            roof["fp32_lane"] = {"achieved": round(lane_ach, 3), "peak": round(lane_peak, 3), "unit": "Tops/s",
                                 "ops_per_value": ops, "frac": round(lane_ach / lane_peak, 4)}
    prof = ROOT / "profiles" / f"traffic_{args.qtype}{'_imat' if args.imatrix else ''}.json"
    if prof.exists():
        counters = json.loads(prof.read_text())
        roof["traffic"] = counters.get("bytes_per_value_launch")
        if roof["traffic"] is not None:
            roof["traffic"] = round(roof["traffic"] * elems_per_launch)
        # executed work beside the frozen algorithmic count: ncu's thread instructions per value
        # on one 14336 x 4096 launch of this kernel (profiles/traffic_<type>.json)
        if counters.get("thread_inst_per_value") is not None:
            roof["inst_per_value_ncu"] = counters["thread_inst_per_value"]

    # end to end through the public API from pinned host memory
    e2e = None
    if args.e2e:
        e2e = e2e_bench(torch, _native, gt, xs, qws, outs, device, args, dist, allmax, world, n_elem)

    line = {"metric": f"input GB/s quantized (bf16->{args.qtype}{', imatrix' if args.imatrix else ''})",
            "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded, generated on device; random-init weights of the config shapes)",
            "config": config, "roofline": roof, "clocks": clocks, "gpu_launches": args.steps * len(xs),
            "kernel_ms_per_launch": round(launch_ms, 4),
            "kernel_ms_by_shape": {f"{r}x{c}": round(statistics.median(k[i] for k in kern_ms), 4)
                                   for i, (r, c) in enumerate(SHAPES_C2) if i in (0, len(SHAPES_C2) - 1)},
            "e2e": e2e}
    if world == 1 and args.op == "quantize" and args.qtype == "q4_k" and args.configs:
        # the north star's other single-GPU configs, on the same device, after the headline
        del xs, outs
        torch.cuda.empty_cache()
        line["config1"] = bench_config1(torch, _native, device, args, peak_info)
        line["config3"] = bench_config3(torch, _native, device, args, peak_info)
    if rank == 0 and world == 1 and args.cpu_baseline:
        def gpu_quantize(a, qw):
            xd = torch.from_numpy(a).to(device).to(torch.bfloat16)  # a holds bf16-representable values
            q = None if qw is None else torch.from_numpy(qw).to(device)
            return _native.quantize(gt, xd, q).cpu().numpy()
        line["cpu_baseline"] = cpu_baseline(args, gpu_quantize)
        pv = parity_vs_reference(args, gpu_quantize)
        if pv is not None:
            line["cpu_baseline"]["vs_reference"] = pv
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def graph_of(torch, stream, fn):
    """fn() captured into a CUDA graph on `stream` (after one eager run), so that a batch of
    short launches is timed without the host's per-call overhead between them."""
    with torch.cuda.stream(stream):
        fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
        fn()
    return g


def bench_config1(torch, _native, device, args, info) -> dict:
    """Q4_0 (no imatrix) of one bf16 4096 x 4096 tensor, N(0, 0.02) with
    0.1 % N(0, 0.5) outliers. One launch moves 43 MB, which fits the 126 MB L2, so the launches
    rotate over R copies of the tensor (R x 43 MB > 3 x L2): a copy is evicted by the time it is
    quantized again. Time = a CUDA graph of R launches, replayed, divided by R (launch gaps
    included)."""
    rows = cols = 4096
    R = 9
    xs, _ = make_inputs(torch, device, seed=7, shapes=[(rows, cols)])
    x0 = xs[0]
    copies = [x0] + [x0.clone() for _ in range(R - 1)]
    rb = _native.row_bytes(2, cols)
    outs = [torch.empty((rows, rb), dtype=torch.uint8, device=device) for _ in range(R)]
    stream = torch.cuda.Stream(device)

    def batch():
        for x, o in zip(copies, outs):
            _native.quantize_into(2, x, None, o, stream)

    g = graph_of(torch, stream, batch)
    reps = max(args.steps, 10)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # replay() launches on the current stream
        for _ in range(args.warmup):
            g.replay()
        stream.synchronize()
        with ClockSampler(device.index) as clk:
            torch.cuda.synchronize()
            t0.record(stream)
            for _ in range(reps):
                g.replay()
            t1.record(stream)
            stream.synchronize()
    us = t0.elapsed_time(t1) * 1e3 / (reps * R)
    alg = rows * cols * (2 + 18 / 32)
    peaks = info["peaks"]
    ach = alg / (us * 1e-6) / 1e9
    ok = all(torch.equal(o, outs[0]) for o in outs[1:])
    del g
    counters = ROOT / "profiles" / "traffic_q4_0.json"
    traffic = inst = None
    if counters.exists():  # ncu DRAM bytes per value of one 14336 x 4096 launch, scaled to this one
        c = json.loads(counters.read_text())
        traffic = round(c["bytes_per_value_launch"] * rows * cols)
        inst = c.get("thread_inst_per_value")
    return {"workload": "BASELINE configs[0]: Q4_0, no imatrix, one 4096x4096 bf16 tensor (43.0 MB per launch); "
                        f"launches rotate over {R} copies (L2 cold for every launch)",
            "metric": "input GB/s quantized (bf16->q4_0)", "value": round(2 * rows * cols / (us * 1e-6) / 1e9, 2),
            "unit": "GB/s", "us_per_launch": round(us, 3), "launches": reps * R,
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(ach / peaks["hbm_gbs"], 4), "bytes_per_value": 2 + 18 / 32,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if not peaks.get("fallback") else "fallback",
                         "traffic": traffic, "traffic_note": "ncu DRAM bytes per value of a 14336 x 4096 launch x the "
                                                             "values of this launch", "inst_per_value_ncu": inst},
            "copies_identical": ok, "clocks": clk.summary()}


def bench_config3(torch, _native, device, args, info) -> dict:
    """IQ2_XXS with imatrix over the configs[1] tensor set, plus the
    151936 x 2560 token embedding as Q4_0 (--token-embedding-type q4_0). One step = the nine
    launches; inputs (1.38 GB) are larger than L2."""
    shapes = SHAPES_C2 + [(151936, 2560)]
    xs, qws = make_inputs(torch, device, seed=3, shapes=shapes)
    types = [16] * len(SHAPES_C2) + [2]
    qws[-1] = None
    outs = [torch.empty((x.shape[0], _native.row_bytes(t, x.shape[1])), dtype=torch.uint8, device=device)
            for x, t in zip(xs, types)]
    stream = torch.cuda.Stream(device)
    steps = max(3, min(args.steps, 10))
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in xs]
          for _ in range(steps)]

    def step(e=None):
        for i, (x, q, o, t) in enumerate(zip(xs, qws, outs, types)):
            if e is not None:
                e[i][0].record(stream)
            _native.quantize_into(t, x, q, o, stream)
            if e is not None:
                e[i][1].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clk:
        torch.cuda.synchronize()
        t0.record(stream)
        for s in range(steps):
            step(ev[s])
        t1.record(stream)
        stream.synchronize()
    ms = t0.elapsed_time(t1) / steps
    n_iq = sum(r * c for r, c in SHAPES_C2)
    n_emb = 151936 * 2560
    iq_ms = statistics.median(sum(a.elapsed_time(b) for a, b in e[:-1]) for e in ev)
    emb_ms = statistics.median(e[-1][0].elapsed_time(e[-1][1]) for e in ev)
    lane_peak = info["sm_count"] * 128 * info["sm_mhz"] * 1e6 / 1e12
    ops = ALG_OPS[("iq2_xxs", True)]
    iq_ach = ops * n_iq / (iq_ms * 1e-3) / 1e12
    emb_ach = n_emb * (2 + 18 / 32) / (emb_ms * 1e-3) / 1e9
    peaks = info["peaks"]
    del xs, outs
    return {"workload": "BASELINE configs[2]: IQ2_XXS + imatrix over 4 x 4096x4096 + 4 x 14336x4096 bf16, "
                        "plus a 151936x2560 bf16 token embedding to Q4_0",
            "metric": "input GB/s quantized (bf16->iq2_xxs mix)", "value": round(2 * (n_iq + n_emb) / (ms * 1e-3) / 1e9, 3),
            "unit": "GB/s", "ms_per_step": round(ms, 3), "steps": steps,
            "iq2_xxs": {"ms_per_step": round(iq_ms, 3), "value": round(2 * n_iq / (iq_ms * 1e-3) / 1e9, 3),
                        "roofline": {"bound": "fp32-lane", "achieved": round(iq_ach, 3), "peak": round(lane_peak, 3),
                                     "unit": "Tops/s", "ops_per_value": ops, "frac": round(iq_ach / lane_peak, 4)}},
            "q4_0_embedding": {"ms": round(emb_ms, 4), "roofline": {"bound": "hbm", "achieved": round(emb_ach, 1),
                                                                    "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                                                    "frac": round(emb_ach / peaks["hbm_gbs"], 4)}},
            "clocks": clk.summary()}


def bench_decode_op(torch, _native, gt, xs, qws, outs, stream, device, args, config, n_elem):
    """Time qs_dequantize or qs_tensor_error over the blocks of the workload (one GPU)."""
    with torch.cuda.stream(stream):
        for x, q, o in zip(xs, qws, outs):
            _native.quantize_into(gt, x, q, o, stream)
        if args.op == "dequantize":
            fouts = [torch.empty(x.shape, dtype=torch.float32, device=device) for x in xs]
            L = _native.lib()

            def one(i):
                _native.check(L.qs_dequantize(gt, outs[i].data_ptr(), outs[i].stride(0), xs[i].shape[0],
                                              xs[i].shape[1], fouts[i].data_ptr(), fouts[i].stride(0),
                                              stream.cuda_stream))
            bytes_per_value = ALG_BYTES_OUT[args.qtype] + 4.0
            launches_per_call = 1
        else:
            res = torch.empty(2, dtype=torch.float64, device=device)
            L = _native.lib()

            def one(i):
                q = qws[i]
                _native.check(L.qs_tensor_error(gt, outs[i].data_ptr(), outs[i].stride(0), xs[i].data_ptr(), 30,
                                                xs[i].shape[0], xs[i].shape[1], None if q is None else q.data_ptr(),
                                                res.data_ptr(), stream.cuda_stream))
            bytes_per_value = ALG_BYTES_OUT[args.qtype] + 2.0
            launches_per_call = 2
        for _ in range(args.warmup):
            for i in range(len(xs)):
                one(i)
    stream.synchronize()
    kev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in xs]
           for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clk:
        torch.cuda.synchronize()
        t0.record(stream)
        for s in range(args.steps):
            for i in range(len(xs)):
                kev[s][i][0].record(stream)
                one(i)
                kev[s][i][1].record(stream)
        t1.record(stream)
        stream.synchronize()
    ms_step = t0.elapsed_time(t1) / args.steps
    launch_ms = statistics.mean(a.elapsed_time(b) for ev in kev for a, b in ev)
    peaks = measured_peaks()
    alg_bytes = n_elem / len(xs) * bytes_per_value
    achieved = alg_bytes / (launch_ms * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None, "bytes_per_value": round(bytes_per_value, 4),
            "peak_source": "MEASURED_PEAKS.json hbm_gbs" if not peaks.get("fallback") else "fallback"}
    what = "packed blocks in + f32 values out" if args.op == "dequantize" else "packed blocks + bf16 rows in"
    line = {"metric": f"{args.op} GB/s ({args.qtype}: {what})", "value": round(n_elem * bytes_per_value / (ms_step * 1e-3) / 1e9, 3),
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32" if args.op == "dequantize" else "f64",
            "data": "synthetic (blocks quantized on device from the seeded workload)",
            "config": dict(config, op=args.op), "roofline": roof, "clocks": clk.summary(),
            "gpu_launches": args.steps * len(xs) * launches_per_call, "kernel_ms_per_call": round(launch_ms, 4)}
    print(json.dumps(line), flush=True)


def bench_cli(args) -> None:
    """Whole-model quantization through the drop-in CLI (quant-studio.py) on a synthetic
    bf16 model of BASELINE's config 4 (4B-class, Q4_K_M + imatrix) or 5 (8B-class, IQ3_XXS /
    IQ2_M + imatrix): one process, row chunks sharded over --gpus, blocks written with pwrite.
    value = bf16 tensor bytes / the CLI's quantization time (reading the mapped model, copies,
    kernels, copies back, writes); the CLI's process wall time (startup, planning, fsync) is
    reported beside it. --warmup runs are untimed (page cache, CUDA start-up)."""
    import re
    import tempfile

    sys.path.insert(0, str(ROOT / "quant-studio_b200"))
    import synth_model

    scheme = args.scheme or ("Q4_K_M" if args.model == "4b" else "IQ3_XXS")
    d = Path(args.model_dir or Path(tempfile.gettempdir()) / "qsb200_synth")
    d.mkdir(parents=True, exist_ok=True)
    model, imat = d / f"synth-{args.model}.gguf", d / f"synth-{args.model}.imatrix.gguf"
    gen_s = None
    if not (model.exists() and imat.exists()):
        t0 = time.time()
        cols = synth_model.write_model(model, args.model)
        synth_model.write_imatrix(imat, cols)
        gen_s = round(time.time() - t0, 2)
    cfg = synth_model.MODELS[args.model]
    n_w = sum(r * c for _, (r, c), w in ((n, s, w) for n, s, w in synth_model.tensor_list(cfg) if w))
    out = d / f"out-{args.model}-{scheme}.gguf"
    cmd = [sys.executable, str(ROOT / "quant-studio_b200" / "quant-studio.py"), str(model), str(out), scheme,
           "--imatrix", str(imat), "--gpus", str(args.gpus), "--mem", args.mem]
    runs = []
    for i in range(args.warmup + args.steps):
        t0 = time.time()
        r = subprocess.run(cmd, capture_output=True, text=True)
        wall = time.time() - t0
        if r.returncode != 0:
            raise SystemExit(f"CLI failed ({r.returncode}): {r.stderr[-2000:]}")
        m = re.search(r"done in ([0-9.]+)s", r.stdout)
        phases = dict((k, float(v)) for k, v in re.findall(r"(\w+) ([0-9.]+)", r.stdout.split("pipeline seconds", 1)[-1].split("\n", 1)[0].split(":", 1)[-1]))
        w = re.search(r"waited ([0-9.]+)s for device start-up", r.stdout)
        if w:
            phases["startup_wait"] = float(w.group(1))
        if i >= args.warmup:
            runs.append((float(m.group(1)), wall, phases))
    q_s = statistics.median(x for x, _, _ in runs)
    wall_s = statistics.median(y for _, y, _ in runs)
    line = {"metric": f"CLI input GB/s (synthetic {args.model.upper()}-class bf16 GGUF -> {scheme}, imatrix)",
            "value": round(2 * n_w / q_s / 1e9, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(q_s * 1e3, 1), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 in", "data": "synthetic (BASELINE config architecture, random-init weights)",
            "config": {"workload": f"BASELINE configs[{3 if args.model == '4b' else 4}]: {args.model} model, {scheme} + imatrix, "
                                   f"--gpus {args.gpus}, --mem {args.mem}", "weight_values": n_w,
                       "model_bytes": model.stat().st_size, "output_bytes": out.stat().st_size},
            "quantize_s": round(q_s, 3), "cli_wall_s": round(wall_s, 2), "generate_s": gen_s,
            "pipeline_phase_s": runs[-1][2]}
    print(json.dumps(line), flush=True)


def e2e_bench(torch, _native, gt, xs, qws, outs, device, args, dist, allmax, world, n_elem):
    """Host-buffer pipeline: chunks of rows go H2D on one stream, are quantized and copied
    back on another; events order the two so copies overlap the kernels. Chunks of 64 MB of
    source rows: measured on a B200 over PCIe, 16 / 32 / 64 / 112 MB chunks reached 46 / 49 /
    52 / 46 GB/s against 55.6 GB/s for a lone pinned H2D copy (about 48.5 per direction with
    the blocks copied back at the same time)."""
    kmax = max(x.shape[1] for x in xs)
    chunk_rows = max(1, (64 << 20) // (kmax * xs[0].element_size()))
    h_in = [torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for x in xs]
    for h, x in zip(h_in, xs):
        h.copy_(x)
    h_out = [torch.empty(o.shape, dtype=torch.uint8, pin_memory=True) for o in outs]
    s_h2d, s_comp, s_d2h = (torch.cuda.Stream(device) for _ in range(3))
    nbuf = 3
    d_in = [torch.empty((chunk_rows, kmax), dtype=torch.bfloat16, device=device) for _ in range(nbuf)]
    d_out = [torch.empty((chunk_rows, max(o.shape[1] for o in outs)), dtype=torch.uint8, device=device)
             for _ in range(nbuf)]
    h2d_done, kern_done, d2h_done = ([torch.cuda.Event() for _ in range(nbuf)] for _ in range(3))
    launches = [0]

    def one_step(kernels=True):
        slot = 0
        for x_h, q, o_h in zip(h_in, qws, h_out):
            n, k = x_h.shape
            rb = o_h.shape[1]
            for r0 in range(0, n, chunk_rows):
                r = min(chunk_rows, n - r0)
                din = d_in[slot][:r, :k]
                dout = d_out[slot][:r, :rb]
                s_h2d.wait_event(kern_done[slot])       # the slot's previous kernel has read d_in
                with torch.cuda.stream(s_h2d):
                    din.copy_(x_h[r0:r0 + r], non_blocking=True)
                h2d_done[slot].record(s_h2d)
                s_comp.wait_event(h2d_done[slot])
                s_comp.wait_event(d2h_done[slot])       # the slot's previous blocks are on the host
                if kernels:
                    _native.quantize_into(gt, din, q, dout, s_comp)
                    launches[0] += 1
                kern_done[slot].record(s_comp)
                s_d2h.wait_event(kern_done[slot])
                with torch.cuda.stream(s_d2h):
                    o_h[r0:r0 + r].copy_(dout, non_blocking=True)
                d2h_done[slot].record(s_d2h)
                slot = (slot + 1) % nbuf

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    launches[0] = 0
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_h2d)
    for _ in range(args.steps):
        one_step()
    s_h2d.wait_stream(s_comp)
    s_h2d.wait_stream(s_d2h)
    t1.record(s_h2d)
    torch.cuda.synchronize()
    ms = allmax(t0.elapsed_time(t1)) / args.steps
    ok = all(torch.equal(o_h.to(device), o) for o_h, o in zip(h_out, outs))
    # the same copies with the kernels left out, on every rank at once: the host<->device
    # ceiling of this pipeline on this box (PCIe and host memory shared by all ranks)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(s_h2d)
    for _ in range(args.steps):
        one_step(kernels=False)
    s_h2d.wait_stream(s_comp)
    s_h2d.wait_stream(s_d2h)
    c1.record(s_h2d)
    torch.cuda.synchronize()
    ms_copy = allmax(c0.elapsed_time(c1)) / args.steps
    value = world * 2 * n_elem / (ms * 1e-3) / 1e9
    ceiling = world * 2 * n_elem / (ms_copy * 1e-3) / 1e9
    return {"value": round(value, 3), "unit": "GB/s",
            "h2d_bytes_per_step": int(sum(x.numel() * x.element_size() for x in xs)),
            "d2h_bytes_per_step": int(sum(o.numel() for o in outs)), "ms_per_step": round(ms, 3),
            "gpu_launches": launches[0], "pipeline": f"{chunk_rows}-row chunks, {nbuf} device slots, H2D / kernel / D2H streams",
            "matches_device_resident_output": ok,
            "copy_ceiling": {"value": round(ceiling, 3), "unit": "GB/s", "ms_per_step": round(ms_copy, 3),
                             "what": "the same H2D / D2H copies and chunking with no kernels, all ranks at once"},
            "frac_of_copy_ceiling": round(value / ceiling, 4)}


def parity_vs_reference(args, gpu_quantize) -> dict | None:
    """Identical-block fraction of the GPU output against the reference as shipped on the
    configs[1] row subsets of tests/golden/config_parity.json (the reference's own outputs):
    the GPU bytes must hash like the reference with a correctly rounded sqrt; the shipped
    reference then differs exactly in the blocks the fixture lists."""
    import hashlib
    fix_path = ROOT / "tests" / "golden" / "config_parity.json"
    if not fix_path.exists():
        return None
    sys.path.insert(0, str(ROOT / "tests" / "golden"))
    import config_rows
    cases = [c for c in json.loads(fix_path.read_text())["cases"].values()
             if c["type"] == args.qtype and c["case"] in ("c2_a", "c2_b") and c["imatrix"] == args.imatrix]
    if not cases:
        return None
    blocks = differ = 0
    exact = True
    for c in cases:
        x = config_rows.rows_f32(c["case"])
        got = gpu_quantize(x, config_rows.imatrix(x.shape[1]) if c["imatrix"] else None)
        exact &= hashlib.sha256(got.tobytes()).hexdigest() == c["sha_ieee"]
        blocks += c["blocks"]
        differ += len(c["diff"])
    return {"identical_blocks_vs_reference": round(1.0 - differ / blocks, 6) if exact else None,
            "bit_exact_vs_ieee_sqrt_reference": exact, "blocks_compared": blocks,
            "sample": "first rows of the configs[1] tensors (tests/golden/config_parity.json)"}


def cpu_baseline(args, gpu_quantize=None) -> dict:
    """The oracle (C port of the reference algorithm) on this host's cores, bounded sample; with
    gpu_quantize, the same sample is also quantized on the GPU and the fraction of identical
    blocks reported (the identical-block part of the metric)."""
    import oracle

    cores = os.cpu_count() or 1
    rng = np.random.default_rng(2)
    k = 4096
    qw = rng.lognormal(0.0, 1.5, k).astype(np.float32) if args.imatrix else None
    oracle.quantize(args.qtype, rng.normal(0.0, 0.02, (8, k)).astype(np.float32), qw, nthreads=1)
    a = rng.normal(0.0, 0.02, (256, k)).astype(np.float32)
    t0 = time.perf_counter()
    oracle.quantize(args.qtype, a, qw, nthreads=cores)
    rate = a.size / max(time.perf_counter() - t0, 1e-6)
    rows = int(min(16384, max(64, rate * 10.0 / k)))
    a = rng.normal(0.0, 0.02, (rows, k))
    m = rng.random(a.shape) < 0.001
    a[m] = rng.normal(0.0, 0.5, int(m.sum()))
    a = ((a.astype(np.float32).view(np.uint32) + 0x8000) & 0xFFFF0000).view(np.float32)
    t0 = time.perf_counter()
    ref = oracle.quantize(args.qtype, a, qw, nthreads=cores)
    dt = time.perf_counter() - t0
    out = {"value": round(a.size * 2 / dt / 1e9, 6), "unit": "GB/s", "cores": cores, "kind": "port",
           "sample": f"{rows} rows x {k} values ({a.size * 2 / 1e6:.1f} MB bf16) of the benchmark distribution, "
                     f"{dt:.1f} s on {cores} threads"}
    if gpu_quantize is not None:
        got = gpu_quantize(a, qw)
        bb = ref.shape[1] // (k // (32 if args.qtype == "q4_0" else 256))
        same = (got.reshape(-1, bb) == ref.reshape(-1, bb)).all(1)
        out["identical_blocks"] = round(float(same.mean()), 6)
        out["blocks_compared"] = int(same.size)
    return out


if __name__ == "__main__":
    main()
