#!/usr/bin/env python3
"""INT8 convolution throughput on B200: effective TOPS and roofline fraction.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: BASELINE config 5a, the batch-scaled stress conv (N=256, H=W=56,
C=K=256, 3x3, stride 1, pad 1), int8 uniform on [-128,127], int32 bias on
[-65536,65536], seeded.  With N GPUs (one process per GPU under torchrun) the
batch is split evenly: rank r convolves images [r*256/N, (r+1)*256/N); no
collective is on the data path (NCCL only gathers outputs for verification,
outside the timed region).  A step is one convolution of the whole batch.

Printed (rank 0, one JSON line):
  value     whole-job effective TOPS = 2*N*P*Q*K*C*R*S*steps / max-over-ranks
            device time (CUDA events on the launching stream, inputs resident)
  e2e       same metric through the public API with pinned host buffers:
            host->device copy of each step's input shard, filter and bias,
            the launch, and the device->host copy of the NHWK output
  roofline  the conv kernel's achieved TOPS vs the B200 dense INT8 peak
            (4.5 POPS), with 2x the measured bf16 cuBLAS burst as a second figure
  sustained the same launches back to back for --sustained-seconds under the
            power cap, with the clocks of that loop
  cpu_baseline  the CPU oracle on the host cores (N=1 only), on whole images
            of the same workload
  verified  the timed launches' own output against the CPU oracle: at N=1
            image 0 and the cpu_baseline images, at N>1 (NCCL gather to rank 0)
            the first and last image of every rank's shard plus a seeded
            sample; the host-buffer (e2e) output separately
--impl reference times the reference's own CPU implementation of the path
(reference_value of src/conv_lab.cu:39-66, built from the reference sources
into oracle/_ref) on the host cores instead; that arm loads nothing of this
package (shapes and inputs are computed here in plain Python).
"""
from __future__ import annotations

import argparse
import csv
import ctypes
import datetime
import io
import json
import math
import os
import shutil
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "INT8 conv TOPS & % of B200 INT8 tensor peak at 1/2/4/8 GPUs vs host-CPU oracle"
DEFAULT_WORKLOAD = "cfg5a_stress_3x3"
NOMINAL_INT8_TOPS = 4500.0
WORKLOADS_CSV = ROOT / "int8_kernel_lab_b200" / "workloads.csv"
REFERENCE_SEED = 20260925
SHAPE_FIELDS = ("n", "h", "w", "c", "k", "r", "s", "pad_h", "pad_w", "stride_h", "stride_w",
                "dilation_h", "dilation_w")
# The same statement in both arms (the GPU arm's actual set count is under "run").
L2_POLICY = ("inputs larger than L2: the GPU arm's input + output set is >= 2x the 126 MB L2, "
             "or enough sets rotate that consecutive steps never share one")


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--batch", type=int, default=0,
                    help="override the workload's batch N (a measurement aid: one GPU "
                         "running N/G images reproduces one rank of a G-GPU job)")
    ap.add_argument("--strategy", default="auto")
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="image groups the host-buffer path overlaps copies over")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--sustained-seconds", type=float, default=2.0,
                    help="length of the back-to-back loop under the power cap (0: skip)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def int8_peak():
    """Roofline denominator of the conv kernel: B200's dense INT8 tensor peak,
    4.5 POPS nominal.  The int8 tensor pipe itself (lib/mma_ceiling:
    back-to-back kind::i8 MMAs, no memory traffic) retires 16 384 ops per
    clock per SM: 4.59 POPS at 1.9 GHz with zero operands, 3.88 POPS at
    1.61 GHz with random ones held for 115 ms, so the nominal figure is the
    tighter of the two."""
    return NOMINAL_INT8_TOPS, ("B200 dense INT8 nominal 4.5 POPS (the int8 tensor pipe "
                               "retires 16384 ops/clk/SM: 4.59 POPS at 1.9 GHz, zero "
                               "operands; 3.88 POPS at 1.61 GHz, random operands)")


def bf16_peaks():
    """2x the measured cuBLAS bf16 dense figures of MEASURED_PEAKS.json (burst,
    sustained): B200's dense INT8 rate is 2x its bf16 rate."""
    try:
        data = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return 2.0 * float(data["bf16_tflops"]), 2.0 * float(data["bf16_tflops_sustained"])
    except (OSError, KeyError, ValueError):
        return 2.0 * 1590.0, 2.0 * 1400.0


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region.

    The sampler starts before the warm-up and `wait_ready` blocks until its
    first sample, so a short timed region is not missed while nvidia-smi
    starts.  Every sample carries nvidia-smi's timestamp; `mark_start` /
    `mark_stop` bracket the timed region on the host clock, and `stop` keeps
    the samples inside it, or, for a region shorter than the sampling period,
    the nearest sample on each side of it."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 20
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_id: str):
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None
        if shutil.which("nvidia-smi"):
            fd, self.path = tempfile.mkstemp(prefix="bench_clocks_", suffix=".csv")
            with os.fdopen(fd, "w") as sink:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                     "-i", gpu_id, "-lms", str(self.PERIOD_MS)],
                    stdout=sink, stderr=subprocess.DEVNULL)

    def _rows(self):
        """(host seconds, row) of every complete sample written so far."""
        with open(self.path) as f:
            text = f.read()
        out = []
        for r in csv.reader(io.StringIO(text)):
            if len(r) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                continue
            out.append((ts, [c.strip() for c in r]))
        return out

    def _wait_for(self, pred, timeout_s: float):
        deadline = time.time() + timeout_s
        while time.time() < deadline:
            if self.proc.poll() is not None or pred(self._rows()):
                return
            time.sleep(0.005)

    def wait_ready(self, timeout_s: float = 5.0):
        if self.proc is not None:
            self._wait_for(lambda rows: len(rows) > 0, timeout_s)

    def mark_start(self):
        self.t0 = time.time()

    def mark_stop(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return None
        try:
            if self.t1 is not None:
                # One sample at or after the end of the region closes the bracket.
                self._wait_for(lambda rows: any(ts >= self.t1 for ts, _ in rows),
                               10 * self.PERIOD_MS / 1e3)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            rows = self._rows()
        finally:
            os.unlink(self.path)
        if not rows:
            return None
        t0 = self.t0 if self.t0 is not None else rows[0][0]
        t1 = self.t1 if self.t1 is not None else rows[-1][0]
        inside = [r for ts, r in rows if t0 <= ts <= t1]
        chosen = inside
        if not chosen:
            # Region shorter than the period: the nearest sample on each side.
            before = [r for ts, r in rows if ts < t0]
            after = [r for ts, r in rows if ts > t1]
            chosen = before[-1:] + after[:1]
        sm = sorted(float(r[2]) for r in chosen if r[2].replace(".", "").isdigit())
        reasons = sorted({self.REASONS[i] for r in chosen for i in range(4)
                          if "Active" in r[6 + i] and "Not" not in r[6 + i]})
        max_mhz = next((float(r[3]) for r in chosen if r[3].replace(".", "").isdigit()), None)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max_mhz,
                "reasons": reasons, "samples": len(chosen), "samples_inside": len(inside),
                "region_ms": round((t1 - t0) * 1e3, 3), "period_ms": self.PERIOD_MS}


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------

class PlainShape:
    """A workloads.csv row with the shape algebra of conv_shape.cuh:22-32 (C++
    truncating division in out_h/out_w), for the reference arm, which loads
    nothing of this package."""

    def __init__(self, **fields):
        for f in SHAPE_FIELDS:
            setattr(self, f, int(fields[f]))
        self.out_h = int((self.h + 2 * self.pad_h - self.dilation_h * (self.r - 1) - 1)
                         / self.stride_h) + 1
        self.out_w = int((self.w + 2 * self.pad_w - self.dilation_w * (self.s - 1) - 1)
                         / self.stride_w) + 1
        self.gemm_m = self.n * self.out_h * self.out_w
        self.gemm_k = self.r * self.s * self.c
        self.input_elements = self.n * self.h * self.w * self.c
        self.filter_elements = self.k * self.r * self.s * self.c
        self.output_elements = self.gemm_m * self.k
        self.ops = 2 * self.gemm_m * self.k * self.gemm_k


def plain_workload(name: str) -> PlainShape:
    with open(WORKLOADS_CSV, newline="") as stream:
        for row in csv.DictReader(stream):
            if row["name"] == name:
                return PlainShape(**row)
    raise SystemExit(f"unknown workload {name}")


def plain_inputs(shape: PlainShape, seed: int = REFERENCE_SEED):
    """The benchmark's seeded inputs: the same MT19937 draws, in the same
    order, as the GPU arm's make_inputs (int8 uniform [-128,127], bias uniform
    [-65536,65536])."""
    import numpy as np
    rng = np.random.RandomState(seed)
    x = rng.randint(-128, 128, size=shape.input_elements, dtype=np.int16).astype(np.int8)
    w = rng.randint(-128, 128, size=shape.filter_elements, dtype=np.int16).astype(np.int8)
    b = rng.randint(-65536, 65537, size=shape.k, dtype=np.int64).astype(np.int32)
    return x, w, b


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0  # only rank 0 runs and prints the reference arm
    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle  # noqa: E402  (test infrastructure: the reference leg only)

    shape = plain_workload(args.workload)
    if args.batch > 0:
        shape = PlainShape(**dict({f: getattr(shape, f) for f in SHAPE_FIELDS}, n=args.batch))
    x, w, b = plain_inputs(shape)
    threads = os.cpu_count() or 1
    binary = pyoracle.ref_binary(args.workload) if args.batch <= 0 else None
    rows_per_image = shape.out_h * shape.out_w
    # Size each step so warmup + steps fit in about two minutes.
    budget_s = 120.0 / max(1, args.steps + args.warmup)
    probe_rows = min(64, shape.gemm_m)
    if binary is not None:
        kind = "reference"
        _, t = pyoracle.ref_cpu_rows(args.workload, x, w, b, 0, probe_rows, threads)
    else:
        kind = "port"
        t0 = time.perf_counter()
        pyoracle.conv_rows(shape, x, w, b, 0, probe_rows, threads)
        t = time.perf_counter() - t0
    rows = int(max(1, min(shape.gemm_m, probe_rows * budget_s / max(t, 1e-6))))
    total_steps = args.steps + args.warmup
    if kind == "reference":
        with tempfile.TemporaryDirectory() as tmp:
            paths = [os.path.join(tmp, n) for n in ("x.bin", "w.bin", "b.bin", "y.bin")]
            x.tofile(paths[0]); w.tofile(paths[1]); b.tofile(paths[2])
            proc = subprocess.run([str(binary), "cpu", *paths, "0", str(rows), str(threads),
                                   str(total_steps)], check=True, capture_output=True, text=True)
            res = json.loads(proc.stdout.strip().splitlines()[-1])
            step_s = res["step_seconds"][args.warmup:]
    else:
        step_s = []
        for i in range(total_steps):
            t0 = time.perf_counter()
            pyoracle.conv_rows(shape, x, w, b, 0, rows, threads)
            if i >= args.warmup:
                step_s.append(time.perf_counter() - t0)
    sec = sum(step_s) / len(step_s)
    ops = 2.0 * rows * shape.k * shape.gemm_k
    value = ops / sec / 1e12
    sample = (f"output rows [0, {rows}) of {args.workload} ({rows / rows_per_image:.3f} "
              f"images of {shape.n}, all {shape.k} channels) per step, {threads} threads")
    line = {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "TOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": workload_config(shape, args, args.gpus),
        "run": {"reference_binary": str(binary.relative_to(ROOT)) if binary else None},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(shape, args, world):
    return {
        "workload": args.workload,
        "shape": {f: getattr(shape, f) for f in ("n", "h", "w", "c", "k", "r", "s", "pad_h",
                                                 "pad_w", "stride_h", "stride_w", "dilation_h",
                                                 "dilation_w")},
        "out_hw": [shape.out_h, shape.out_w],
        "ops_per_step": shape.ops,
        "parallelism": f"batch-sharded x{world} (no data-path collective)",
        "values": "int8 uniform [-128,127], bias int32 uniform [-65536,65536], seed 20260925",
        "l2": L2_POLICY,
    }


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args):
    import numpy as np
    import torch

    import int8_kernel_lab_b200 as m
    from int8_kernel_lab_b200 import _abi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        # stdout carries exactly one JSON line: NCCL's own log lines (its
        # version banner, NCCL_DEBUG output) go to stderr instead.
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    full = m.load_workloads()[args.workload]
    if args.batch > 0:
        full = full.with_batch(args.batch)
    from int8_kernel_lab_b200.sharding import shard_range
    lo, hi = shard_range(full.n, rank, world)
    local_shape = full.with_batch(hi - lo)
    x, w, b = m.make_inputs(full)
    per_image_in = full.h * full.w * full.c
    x_local = x[lo * per_image_in:hi * per_image_in]
    strategy = local_shape.select() if args.strategy == "auto" else args.strategy
    code = _abi.STRATEGIES[strategy]
    cshape = local_shape.c_struct()

    # Device buffers.  Enough input/output sets rotate that a step never finds
    # its operands in L2 (working set >= 2x L2 across consecutive steps).
    props = torch.cuda.get_device_properties(local)
    l2 = int(getattr(props, "L2_cache_size", 126 * 2**20))
    per_set = x_local.nbytes + 4 * local_shape.output_elements
    sets = max(1, math.ceil(2 * l2 / per_set)) if per_set < 2 * l2 else 1
    dw = torch.from_numpy(w).cuda()
    db = torch.from_numpy(b).cuda()
    dxs = [torch.from_numpy(x_local).cuda() for _ in range(sets)]
    dys = [torch.empty(local_shape.output_elements, dtype=torch.int32, device="cuda")
           for _ in range(sets)]
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    launch = _abi.lib.int8conv_launch
    args_per_set = [(code, cshape, dxs[i].data_ptr(), dw.data_ptr(), db.data_ptr(),
                     dys[i].data_ptr(), None, 0, sptr) for i in range(sets)]

    def step(i):
        st = launch(*args_per_set[i % sets])
        if st != _abi.OK:
            raise _abi.Int8ConvError(st, "bench launch")

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    gpu_uuid = "GPU-" + str(props.uuid) if hasattr(props, "uuid") else str(local)
    sampler = ClockSampler(gpu_uuid)  # every rank records its own GPU's clocks
    if sampler:
        sampler.wait_ready()
    for i in range(args.warmup):
        step(i)
    barrier()
    launches0 = m.launch_count()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    if sampler:
        sampler.mark_start()
    start.record(stream)
    for i in range(args.steps):
        step(i)
    stop.record(stream)
    torch.cuda.synchronize()
    if sampler:
        sampler.mark_stop()
    launches = m.launch_count() - launches0
    clocks = sampler.stop() if sampler else None
    elapsed_ms = start.elapsed_time(stop)
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    if m.device_status() != _abi.OK:
        raise SystemExit("device status not OK after the timed region")
    ms_per_step = max_ms / args.steps
    value = full.ops / (ms_per_step * 1e-3) / 1e12
    local_launch_ms = elapsed_ms / args.steps  # one kernel per step on this stream
    achieved = local_shape.ops / (local_launch_ms * 1e-3) / 1e12
    peak, peak_src = int8_peak()
    bf16_burst, bf16_sustained = bf16_peaks()
    # The last timed launch's output, kept aside for verification before any
    # later launch reuses its buffer.
    y_timed = dys[(args.steps - 1) % sets].clone()

    # ---- the same launches back to back under the power cap ----
    sustained = None
    if args.sustained_seconds > 0:
        sustained = sustained_loop(step, local_shape, full, args, stream, sampler_factory=(
            (lambda: ClockSampler(gpu_uuid)) if rank == 0 else None), barrier=barrier,
            dist=dist, bf16_sustained=bf16_sustained)

    # ---- end to end through the public API, host buffers ----
    # Its own device buffers: the timed launches' output stays for verification.
    hx = torch.from_numpy(x_local).pin_memory()
    hw = torch.from_numpy(w).pin_memory()
    hb = torch.from_numpy(b).pin_memory()
    hy = torch.empty(local_shape.output_elements, dtype=torch.int32).pin_memory()
    ex = torch.empty_like(dxs[0])
    ew = torch.empty_like(dw)
    eb = torch.empty_like(db)
    ey = torch.empty(local_shape.output_elements, dtype=torch.int32, device="cuda")

    chunks = max(1, min(args.e2e_chunks, local_shape.n))

    def e2e_step():
        # int8conv_launch_host: H2D of image groups, kernels and D2H overlap.
        m.launch_host(strategy, local_shape, hx, hw, hb, hy, ex, ew, eb, ey, chunks=chunks,
                      stream=stream)

    e2e_step()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = float(te.item()) / args.e2e_steps
    h2d = int(hx.numel() + hw.numel() + 4 * hb.numel()) * world
    d2h = int(4 * hy.numel()) * world
    if m.device_status() != _abi.OK:
        raise SystemExit("device status not OK after the end-to-end steps")

    # ---- verification against the CPU oracle / CPU baseline ----
    cpu = None
    verified = None
    if world == 1:
        if rank == 0:
            cpu, verified = verify_single(full, x, w, b, y_timed.cpu().numpy(), hy.numpy(), args)
    else:
        verified = verify_sharded(full, x, w, b, y_timed, hy, dist, rank, world, clocks)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": workload_config(full, args, world),
            "run": {"strategy": strategy, "images_per_rank": hi - lo, "rotating_sets": sets,
                    "set_mb": round(per_set / 1e6, 1), "l2_mb": round(l2 / 1e6, 1)},
            "e2e": {"value": full.ops / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms, "api": "int8conv_launch_host",
                    "chunks": chunks},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TOPS", "frac": achieved / peak, "peak_source": peak_src,
                         "frac_of_2x_measured_bf16_burst": achieved / bf16_burst,
                         "kernel": f"conv_kernel ({strategy})",
                         "launch_ms": local_launch_ms,
                         "traffic": traffic_per_launch(args, local_shape),
                         "traffic_source": "DRAM bytes per launch from the committed ncu "
                                           "capture profiles/traffic.json, scaled by images; "
                                           "not measured in this run"},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "verified": verified,
        }
        if sustained is not None:
            line["sustained"] = sustained
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if world > 1 and verified is not None:
            line["clocks_per_rank"] = verified.pop("clocks_per_rank")
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def sustained_loop(step, local_shape, full, args, stream, sampler_factory, barrier, dist,
                   bf16_sustained):
    """The timed launches back to back for about --sustained-seconds, long
    enough for the 1 kW power cap to set the clock: TOPS and the clocks of
    that loop, next to the burst figure of the main timed region."""
    import torch

    # Launches per second from a short probe, then one bracketed loop.
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(4):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    per_ms = max(t0.elapsed_time(t1) / 4, 1e-3)
    n = torch.tensor([max(8, int(args.sustained_seconds * 1e3 / per_ms))], device="cuda")
    if dist is not None:
        dist.all_reduce(n, op=dist.ReduceOp.MAX)  # every rank runs the same count
    n = int(n.item())
    sampler = sampler_factory() if sampler_factory else None
    if sampler:
        sampler.wait_ready()
    barrier()
    if sampler:
        sampler.mark_start()
    t0.record(stream)
    for i in range(n):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    if sampler:
        sampler.mark_stop()
    clocks = sampler.stop() if sampler else None
    tt = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item()) / n
    achieved = local_shape.ops / (t0.elapsed_time(t1) / n * 1e-3) / 1e12
    return {"value": full.ops / (ms * 1e-3) / 1e12, "unit": "TOPS", "steps": n,
            "seconds": round(float(tt.item()) / 1e3, 3), "ms_per_step": ms,
            "frac_of_nominal_4500": achieved / NOMINAL_INT8_TOPS,
            "frac_of_2x_measured_bf16_sustained": achieved / bf16_sustained,
            "clocks": clocks}


def traffic_per_launch(args, local_shape):
    """DRAM bytes per launch from the committed ncu capture of this kernel
    (profiles/traffic.json), scaled by images, or None if not captured."""
    path = ROOT / "profiles" / "traffic.json"
    try:
        data = json.loads(path.read_text())[args.workload]
        return data["bytes_per_image"] * local_shape.n
    except (OSError, KeyError, ValueError):
        return None


def verify_single(shape, x, w, b, y_timed, y_e2e, args):
    """N = 1: times the oracle port (oracle/conv_oracle.c) on whole images of
    the workload with all host threads (the cpu_baseline), and checks image 0
    and those images of the timed launches' output and of the host-buffer
    output against it, bit-exactly."""
    import numpy as np
    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle  # noqa: E402  (test infrastructure: the cpu_baseline leg only)

    threads = os.cpu_count() or 1
    rows = shape.out_h * shape.out_w
    first = pyoracle.conv_rows(shape, x, w, b, 0, rows, threads)  # warm
    t0 = time.perf_counter()
    first = pyoracle.conv_rows(shape, x, w, b, 0, rows, threads)
    t1 = time.perf_counter() - t0
    if args.no_cpu_baseline:
        images = 0
    else:
        images = int(max(1, min(shape.n - 1, args.cpu_seconds / max(t1, 1e-6) - 1)))
    # images [n - images, n): the end of the batch
    lo = shape.n - images
    k = shape.k
    ok_timed = bool(np.array_equal(y_timed[:rows * k], first))
    ok_e2e = bool(np.array_equal(y_e2e[:rows * k], first))
    cpu = None
    if images > 0:
        t0 = time.perf_counter()
        tail = pyoracle.conv_rows(shape, x, w, b, lo * rows, shape.n * rows, threads)
        sec = time.perf_counter() - t0
        ops = 2.0 * images * rows * shape.k * shape.gemm_k
        ok_timed = ok_timed and bool(np.array_equal(y_timed[lo * rows * k:], tail))
        ok_e2e = ok_e2e and bool(np.array_equal(y_e2e[lo * rows * k:], tail))
        cpu = {"value": ops / sec / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
               "sample": f"{images} whole image(s) of {args.workload} (images {lo}.."
                         f"{shape.n - 1}), {ops / 1e9:.1f} Gop in {sec:.2f} s"}
    verified = {"timed_output": ok_timed, "e2e_output": ok_e2e, "against": "CPU oracle",
                "images": f"0 and {lo}..{shape.n - 1}" if images else "0"}
    return cpu, verified


def verify_sharded(full, x, w, b, y_timed, y_e2e, dist, rank, world, clocks):
    """N > 1: NCCL gathers every rank's NHWK slice of the timed launches'
    output (and of the host-buffer output) to rank 0, which checks the first
    and last image of every rank's shard plus a seeded sample of all outputs
    against the CPU oracle, bit-exactly (outside the timed region).  Rank 0
    also collects every rank's clock record."""
    import numpy as np
    import torch

    from int8_kernel_lab_b200.sharding import gather_outputs, shard_range
    gathered = gather_outputs(y_timed, full, rank, world, dist)
    gathered_e2e = gather_outputs(y_e2e.to(y_timed.device), full, rank, world, dist)
    records = [None] * world
    dist.all_gather_object(records, clocks)
    if rank != 0:
        return None
    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle  # noqa: E402  (test infrastructure: the verification leg only)

    threads = os.cpu_count() or 1
    y = gathered.cpu().numpy()
    y2 = gathered_e2e.cpu().numpy()
    rows = full.out_h * full.out_w
    k = full.k
    ok = ok2 = True
    checked = []
    for r in range(world):
        lo, hi = shard_range(full.n, r, world)
        for img in sorted({lo, hi - 1}):
            want = pyoracle.conv_rows(full, x, w, b, img * rows, (img + 1) * rows, threads)
            span = slice(img * rows * k, (img + 1) * rows * k)
            ok = ok and bool(np.array_equal(y[span], want))
            ok2 = ok2 and bool(np.array_equal(y2[span], want))
            checked.append(img)
    rng = np.random.RandomState(world)
    idx = rng.randint(0, full.output_elements, size=200_000, dtype=np.int64)
    want = pyoracle.values(full, x, w, b, idx, threads)
    ok = ok and bool(np.array_equal(y[idx], want))
    ok2 = ok2 and bool(np.array_equal(y2[idx], want))
    return {"timed_output": ok, "e2e_output": ok2, "against": "CPU oracle",
            "images": checked, "sampled_outputs": int(idx.size),
            "clocks_per_rank": records}


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
