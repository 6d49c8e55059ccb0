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

--repeat N runs the case list N times, interleaved (every case once, then
again), and writes the per-family means: launch-time medians drift by a few
tenths of a microsecond between runs on one box, and interleaving spreads
that drift over all cases alike.  A family counts as correct only if every
repetition validated; the winner, tops and roofline_frac follow the means,
and a `repeats` column is appended.

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


FAMILIES = ("generic", "strip", "halo", "splitk")


def _ms(value: str) -> float:
    try:
        return float(value)
    except (TypeError, ValueError):
        return -1.0


def merge_repeats(rows: list, expected: int = 0) -> dict:
    """One row from several conv_lab rows of the same case: mean launch times
    (-1 unless every repetition timed the family), correctness only if every
    repetition validated and all `expected` repetitions returned a row,
    winner / tops / roofline_frac from the means.  graph_ms is the winner's
    graph time in each row, so it is averaged over the repetitions whose
    winner is the merged winner only (-1 if none)."""
    merged = dict(rows[0])
    for column in [f + "_ms" for f in FAMILIES]:
        if column not in merged:
            continue
        values = [_ms(r.get(column)) for r in rows]
        merged[column] = ("%.6g" % (sum(values) / len(values))
                          if all(v >= 0 for v in values) else "-1")
    complete = len(rows) >= expected
    for f in FAMILIES:
        column = f + "_correct"
        if column in merged:
            merged[column] = ("1" if complete and all(r.get(column) == "1" for r in rows)
                              else "0")
    timed = {f: _ms(merged[f + "_ms"]) for f in FAMILIES if f + "_ms" in merged}
    timed = {f: v for f, v in timed.items() if v >= 0}
    if "winner" in merged:
        old_winner = rows[0].get("winner")
        merged["winner"] = min(timed, key=timed.get) if timed else "none"
        first_ms = _ms(rows[0].get(old_winner + "_ms", "")) if old_winner in FAMILIES else -1.0
        if timed and first_ms > 0:
            # tops and roofline_frac scale with the winner's time.
            scale = first_ms / timed[merged["winner"]]
            for column in ("tops", "roofline_frac"):
                if _ms(merged.get(column)) >= 0:
                    merged[column] = "%.6g" % (_ms(merged[column]) * scale)
    if "graph_ms" in merged:
        same = [_ms(r.get("graph_ms")) for r in rows if r.get("winner") == merged.get("winner")]
        same = [v for v in same if v >= 0]
        merged["graph_ms"] = "%.6g" % (sum(same) / len(same)) if same else "-1"
    merged["repeats"] = str(len(rows))
    return merged


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
    ap.add_argument("--repeat", type=int, default=1,
                    help="run the case list this many times, interleaved, and write means")
    ap.add_argument("--rotate-l2", action="store_true",
                    help="time every launch on rotating buffer sets (L2-cold)")
    args = ap.parse_args(argv)
    if args.repeat < 1:
        raise SystemExit("--repeat must be at least 1")
    if args.arch not in ("sm_100a", "sm_100"):
        raise SystemExit(f"--arch {args.arch}: this engine is built for sm_100a only")
    with open(args.configs, newline="") as stream:
        rows = list(csv.DictReader(stream))
    requested = args.cases.split(",") if args.cases else [r["name"] for r in rows]
    unknown = sorted(set(requested) - {r["name"] for r in rows})
    if unknown:
        raise SystemExit(f"unknown cases: {', '.join(unknown)}")
    args.output.parent.mkdir(parents=True, exist_ok=True)
    runs = {}  # case -> list of conv_lab rows, one per repetition
    attempts = {}  # case -> repetitions run so far (a failed run returns no row)
    status = 0
    shapes = {r["name"]: r for r in rows}
    for rep in range(args.repeat):
        for case in requested:
            attempts[case] = attempts.get(case, 0) + 1
            r = shapes[case]
            oh = int((int(r["h"]) + 2 * int(r["pad_h"]) -
                      int(r["dilation_h"]) * (int(r["r"]) - 1) - 1) / int(r["stride_h"])) + 1
            ow = int((int(r["w"]) + 2 * int(r["pad_w"]) -
                      int(r["dilation_w"]) * (int(r["s"]) - 1) - 1) / int(r["stride_w"])) + 1
            ops = (2.0 * int(r["n"]) * oh * ow * int(r["k"]) * int(r["c"]) * int(r["r"]) *
                   int(r["s"]))
            extra = ["--validate-samples", "200000"] if ops > args.full_validate_ops else []
            if args.rotate_l2:
                extra.append("--rotate-l2")
            result = subprocess.run(
                [args.conv_lab, "--case", case, "--config", str(args.configs), "--strategy",
                 args.strategy, "--iterations", str(args.iterations), "--warmup",
                 str(args.warmup), "--values", args.values, "--pairing", args.pairing,
                 "--csv"] + extra,
                text=True, capture_output=True)
            if result.returncode != 0:
                status = 1
                sys.stderr.write(result.stderr)
            lines = result.stdout.strip().splitlines()
            if len(lines) < 2:
                print(f"{case}: conv_lab failed (exit {result.returncode})", file=sys.stderr)
                continue
            runs.setdefault(case, []).append(next(csv.DictReader(lines)))
            measurements = []
            for name in requested:
                if name not in runs:
                    continue
                m = (merge_repeats(runs[name], attempts[name]) if args.repeat > 1
                     else dict(runs[name][0]))
                if args.with_cudnn:
                    m.update(dispatch_ms=dispatch_ms(m), cudnn_ms="", cudnn_over_dispatch="",
                             comparison_contract="cudnn_not_built")
                measurements.append(m)
            with open(args.output, "w", newline="") as stream:
                writer = csv.DictWriter(stream, fieldnames=measurements[0].keys())
                writer.writeheader()
                writer.writerows(measurements)
            suffix = f" (repetition {rep + 1}/{args.repeat})" if args.repeat > 1 else ""
            print(f"{case}: wrote {args.output}{suffix}", flush=True)
    return status


if __name__ == "__main__":
    sys.exit(main())
