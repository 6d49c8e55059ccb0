#!/usr/bin/env python3
"""Measure a set of workloads with the conv_lab CLI and write one CSV row each.

B200 counterpart of the reference's scripts/sweep.py (same flags where they
apply: --configs, --cases, --output, --iterations).  Shapes are runtime
arguments of one conv_lab binary, so there is no per-case rebuild (the
reference ran `make CASE=...` per case, sweep.py:35-38).  Every eligible
family is run (--strategy all); rows are written incrementally after each case
(sweep.py:58-61), so an interrupted sweep keeps what it measured.  The CSV is
conv_lab's: the reference's 16 columns, then the appended ones.

--arch keeps the reference's flag; the library is built for sm_100a only, so
any other value is an error.  --with-cudnn keeps the reference's merge columns
(sweep.py:44-56: dispatch_ms, cudnn_ms, cudnn_over_dispatch,
comparison_contract).  cuDNN is not part of this engine, so cudnn_ms stays
empty and the contract reads "cudnn_not_built"; dispatch_ms maps the winner of
all four families to its time (the reference's mapping, sweep.py:48, knows
only strip and generic).

    python -m int8_kernel_lab_b200.sweep --cases cfg2_mid_3x3,big_3x3_s1 \\
        --output build/dispatch_measurements.csv
"""
import argparse
import csv
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent


def dispatch_ms(row: dict) -> str:
    """The winner's per-launch time, for any of the four families."""
    column = {"generic": "generic_ms", "strip": "strip_ms", "halo": "halo_ms",
              "splitk": "splitk_ms"}.get(row["winner"])
    return row[column] if column else ""


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--configs", default=str(PKG / "workloads.csv"), type=Path)
    ap.add_argument("--cases", help="comma-separated case names; default all")
    ap.add_argument("--output", default="build/dispatch_measurements.csv", type=Path)
    ap.add_argument("--iterations", type=int, default=101)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--strategy", default="all")
    ap.add_argument("--values", default="full", choices=("full", "reference"))
    ap.add_argument("--pairing", default="auto", choices=("auto", "single", "pair"))
    ap.add_argument("--full-validate-ops", type=float, default=2e11,
                    help="shapes with more ops validate 200000 sampled outputs, not all")
    ap.add_argument("--conv-lab", default=str(PKG / "lib" / "conv_lab"))
    ap.add_argument("--arch", default="sm_100a")
    ap.add_argument("--with-cudnn", action="store_true")
    ap.add_argument("--cudnn-root", default="")
    args = ap.parse_args(argv)
    if args.arch not in ("sm_100a", "sm_100"):
        raise SystemExit(f"--arch {args.arch}: this engine is built for sm_100a only")
    with open(args.configs, newline="") as stream:
        rows = list(csv.DictReader(stream))
    requested = args.cases.split(",") if args.cases else [r["name"] for r in rows]
    unknown = sorted(set(requested) - {r["name"] for r in rows})
    if unknown:
        raise SystemExit(f"unknown cases: {', '.join(unknown)}")
    args.output.parent.mkdir(parents=True, exist_ok=True)
    measurements = []
    status = 0
    shapes = {r["name"]: r for r in rows}
    for case in requested:
        r = shapes[case]
        oh = int((int(r["h"]) + 2 * int(r["pad_h"]) - int(r["dilation_h"]) * (int(r["r"]) - 1) - 1)
                 / int(r["stride_h"])) + 1
        ow = int((int(r["w"]) + 2 * int(r["pad_w"]) - int(r["dilation_w"]) * (int(r["s"]) - 1) - 1)
                 / int(r["stride_w"])) + 1
        ops = 2.0 * int(r["n"]) * oh * ow * int(r["k"]) * int(r["c"]) * int(r["r"]) * int(r["s"])
        extra = ["--validate-samples", "200000"] if ops > args.full_validate_ops else []
        result = subprocess.run(
            [args.conv_lab, "--case", case, "--config", str(args.configs), "--strategy",
             args.strategy, "--iterations", str(args.iterations), "--warmup", str(args.warmup),
             "--values", args.values, "--pairing", args.pairing, "--csv"] + extra,
            text=True, capture_output=True)
        if result.returncode != 0:
            status = 1
            sys.stderr.write(result.stderr)
        lines = result.stdout.strip().splitlines()
        if len(lines) < 2:
            print(f"{case}: conv_lab failed (exit {result.returncode})", file=sys.stderr)
            continue
        measurement = next(csv.DictReader(lines))
        if args.with_cudnn:
            measurement.update(dispatch_ms=dispatch_ms(measurement), cudnn_ms="",
                               cudnn_over_dispatch="", comparison_contract="cudnn_not_built")
        measurements.append(measurement)
        with open(args.output, "w", newline="") as stream:
            writer = csv.DictWriter(stream, fieldnames=measurements[0].keys())
            writer.writeheader()
            writer.writerows(measurements)
        print(f"{case}: wrote {args.output}", flush=True)
    return status


if __name__ == "__main__":
    sys.exit(main())
