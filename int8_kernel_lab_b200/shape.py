"""Runtime convolution shape: the 13 fields of the reference's ConvShape.

Mirrors include/conv_shape.cuh:5-36 (fields, derived out_h/out_w, GEMM sizes,
element counts, and the c % 16 == 0 / non-empty-output checks).  Derivations
are computed by the C ABI (int8conv_shape_dims) so Python and C agree.
"""
from __future__ import annotations

import csv
import dataclasses
from pathlib import Path
from typing import Dict, Iterable

from . import _abi

WORKLOADS_CSV = Path(__file__).resolve().parent / "workloads.csv"


@dataclasses.dataclass(frozen=True)
class ConvShape:
    n: int
    h: int
    w: int
    c: int
    k: int
    r: int
    s: int
    pad_h: int = 0
    pad_w: int = 0
    stride_h: int = 1
    stride_w: int = 1
    dilation_h: int = 1
    dilation_w: int = 1

    # ---- C interop -------------------------------------------------------
    def c_struct(self) -> _abi.CShape:
        return _abi.CShape(*[int(getattr(self, f)) for f in _abi.SHAPE_FIELDS])

    def as_tuple(self):
        return tuple(getattr(self, f) for f in _abi.SHAPE_FIELDS)

    # ---- conv_shape.cuh:22-35 ---------------------------------------------
    @property
    def valid(self) -> bool:
        return bool(_abi.lib.int8conv_shape_valid(self.c_struct()))

    def dims(self) -> _abi.CDims:
        d = _abi.CDims()
        _abi.check(_abi.lib.int8conv_shape_dims(self.c_struct(), d), f"shape {self}")
        return d

    @property
    def out_h(self) -> int:
        # C++ integer division truncates toward zero (conv_shape.cuh:22-23).
        return int((self.h + 2 * self.pad_h - self.dilation_h * (self.r - 1) - 1) / self.stride_h) + 1

    @property
    def out_w(self) -> int:
        return int((self.w + 2 * self.pad_w - self.dilation_w * (self.s - 1) - 1) / self.stride_w) + 1

    @property
    def gemm_m(self) -> int:
        return self.n * self.out_h * self.out_w

    @property
    def gemm_n(self) -> int:
        return self.k

    @property
    def gemm_k(self) -> int:
        return self.r * self.s * self.c

    @property
    def input_elements(self) -> int:
        return self.n * self.h * self.w * self.c

    @property
    def filter_elements(self) -> int:
        return self.k * self.r * self.s * self.c

    @property
    def output_elements(self) -> int:
        return self.gemm_m * self.gemm_n

    # ---- throughput accounting ---------------------------------------------
    @property
    def ops(self) -> int:
        """Effective INT8 ops: 2*N*P*Q*K*C*R*S (padded taps count)."""
        return 2 * self.gemm_m * self.gemm_n * self.gemm_k

    @property
    def compulsory_bytes(self) -> int:
        """N*H*W*C + K*R*S*C + 4K + 4*N*P*Q*K: every input byte read once,
        every output byte written once."""
        return self.input_elements + self.filter_elements + 4 * self.k + 4 * self.output_elements

    # ---- predicates -------------------------------------------------------
    def eligible(self, strategy: str) -> bool:
        return bool(_abi.lib.int8conv_eligible(self.c_struct(), _abi.STRATEGIES[strategy]))

    def select(self) -> str:
        return _abi.lib.int8conv_strategy_name(_abi.lib.int8conv_select(self.c_struct())).decode()

    def with_batch(self, n: int) -> "ConvShape":
        return dataclasses.replace(self, n=n)


def load_workloads(path: Path | str = WORKLOADS_CSV) -> Dict[str, ConvShape]:
    """Named shapes of a workloads CSV (the reference's column layout,
    workloads.csv:1 of pthodima/int8_kernel_lab)."""
    with open(path, newline="") as stream:
        rows = list(csv.DictReader(stream))
    missing = [f for f in ("name",) + _abi.SHAPE_FIELDS if rows and f not in rows[0]]
    if missing:
        raise ValueError(f"{path} is missing columns: {', '.join(missing)}")
    return {row["name"]: ConvShape(*[int(row[f]) for f in _abi.SHAPE_FIELDS]) for row in rows}


# The five BASELINE configurations (ten shapes).
BASELINE_CASES = (
    "cfg1_smoke", "cfg2_mid_3x3", "cfg3a_down_3x3_s2", "cfg3b_pointwise",
    "cfg4a_deep_1x1", "cfg4b_small_3x3", "cfg4c_tail_k100",
    "cfg5a_stress_3x3", "cfg5b_dilated_3x3", "cfg5c_1x7",
)


def baseline_shapes() -> Dict[str, ConvShape]:
    table = load_workloads()
    return {name: table[name] for name in BASELINE_CASES}


def iter_reference_workloads() -> Iterable[tuple]:
    """The 41 workloads of the reference table (everything but cfg* rows)."""
    for name, shape in load_workloads().items():
        if not name.startswith("cfg"):
            yield name, shape
