#!/usr/bin/env python3
"""Generates tests/golden/*.npz from the reference's OWN CPU oracle.

Run where the reference sources exist (the GPU box has none):
    python tests/golden/make_golden.py [--reference PATH_TO_INT8_KERNEL_LAB]
The reference checkout defaults to $INT8_KERNEL_LAB_REFERENCE, else a
directory named `reference` beside this repository.

For every row of golden_cases.csv it builds oracle/_ref/ref_<case> with
oracle/Makefile (the reference's src/conv_lab.cu compiled unchanged, its
scripts/gen_case.py writing the case header), feeds it seeded inputs and
stores inputs + the reference's outputs.  The committed fixtures pin the C
restatement in oracle/conv_oracle.c and the GPU kernels.
"""
import argparse
import csv
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "oracle"))
import pyoracle  # noqa: E402

FIELDS = pyoracle.FIELDS


class Shape:
    def __init__(self, row):
        for f in FIELDS:
            setattr(self, f, int(row[f]))
        oh = int((self.h + 2 * self.pad_h - self.dilation_h * (self.r - 1) - 1) / self.stride_h) + 1
        ow = int((self.w + 2 * self.pad_w - self.dilation_w * (self.s - 1) - 1) / self.stride_w) + 1
        self.gemm_m = self.n * oh * ow
        self.output_elements = self.gemm_m * self.k


def inputs(name, shape, seed):
    rng = np.random.RandomState(seed)
    nx = shape.n * shape.h * shape.w * shape.c
    nw = shape.k * shape.r * shape.s * shape.c
    if name == "g_extreme":
        # maximum-magnitude products: every term is (-128) * (-128)
        return (np.full(nx, -128, np.int8), np.full(nw, -128, np.int8),
                np.full(shape.k, 65536, np.int32))
    x = rng.randint(-128, 128, size=nx).astype(np.int8)
    w = rng.randint(-128, 128, size=nw).astype(np.int8)
    b = rng.randint(-65536, 65537, size=shape.k).astype(np.int32)
    return x, w, b


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("INT8_KERNEL_LAB_REFERENCE",
                                                          str(ROOT.parent / "reference")))
    args = ap.parse_args()
    table = HERE / "golden_cases.csv"
    rows = list(csv.DictReader(open(table, newline="")))
    names = [r["name"] for r in rows]
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "ref", f"REFERENCE={args.reference}",
                    f"WORKLOADS={table}", "REF_CASES=" + " ".join(names), "-j8"], check=True)
    for i, row in enumerate(rows):
        name = row["name"]
        shape = Shape(row)
        x, w, b = inputs(name, shape, 1000 + i)
        y, _ = pyoracle.ref_cpu_rows(name, x, w, b, 0, shape.gemm_m, 1)
        assert y.size == shape.output_elements
        np.savez_compressed(HERE / f"{name}.npz", shape=np.array([int(row[f]) for f in FIELDS]),
                            x=x, w=w, b=b, y=y)
        print(f"{name}: {y.size} outputs")


if __name__ == "__main__":
    main()
