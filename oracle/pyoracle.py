"""Python binding of the CPU oracle.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module; it is the checker and the timed CPU baseline,
never part of the product path.

`liboracle.so` is the C restatement (conv_oracle.c) of reference_value<Shape>
(src/conv_lab.cu:39-66 of pthodima/int8_kernel_lab).  `ref_binary()` returns
the reference's own oracle built from its sources (oracle/_ref), when present.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"

FIELDS = ("n", "h", "w", "c", "k", "r", "s", "pad_h", "pad_w",
          "stride_h", "stride_w", "dilation_h", "dilation_w")


class _Shape(ctypes.Structure):
    _fields_ = [(f, ctypes.c_int32) for f in FIELDS]


def build() -> None:
    subprocess.run(["make", "-s", "-C", os.fspath(HERE)], check=True)


def _lib() -> ctypes.CDLL:
    if not LIB.exists():
        build()
    lib = ctypes.CDLL(os.fspath(LIB))
    P = ctypes.c_void_p
    SP = ctypes.POINTER(_Shape)
    lib.oracle_conv.argtypes = [SP, P, P, P, P, ctypes.c_int]
    lib.oracle_conv_rows.argtypes = [SP, P, P, P, ctypes.c_int64, ctypes.c_int64, P, ctypes.c_int]
    lib.oracle_values.argtypes = [SP, P, P, P, P, ctypes.c_int64, P, ctypes.c_int]
    lib.oracle_value.argtypes = [SP, P, P, P, ctypes.c_int64]
    lib.oracle_value.restype = ctypes.c_int32
    lib.oracle_out_h.argtypes = [SP]
    lib.oracle_out_w.argtypes = [SP]
    lib.oracle_max_threads.restype = ctypes.c_int
    lib.oracle_requant.argtypes = [P, ctypes.c_int64, ctypes.c_int32, P, P, ctypes.c_int32,
                                   ctypes.c_int32, P, ctypes.c_int]
    lib.oracle_requant_value.argtypes = [ctypes.c_int32] * 5
    lib.oracle_requant_value.restype = ctypes.c_int32
    return lib


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = _lib()
    return _LIB


def _cshape(shape) -> _Shape:
    return _Shape(*[int(getattr(shape, f)) for f in FIELDS])


def _arrays(x, w, b):
    return (np.ascontiguousarray(x, dtype=np.int8), np.ascontiguousarray(w, dtype=np.int8),
            np.ascontiguousarray(b, dtype=np.int32))


def conv(shape, x, w, b, threads: int = 0) -> np.ndarray:
    """Full NHWK int32 output."""
    x, w, b = _arrays(x, w, b)
    out = np.empty(shape.output_elements, dtype=np.int32)
    lib().oracle_conv(_cshape(shape), x.ctypes.data, w.ctypes.data, b.ctypes.data,
                      out.ctypes.data, int(threads))
    return out


def conv_rows(shape, x, w, b, m_begin: int, m_end: int, threads: int = 0) -> np.ndarray:
    """Output rows [m_begin, m_end), all K channels each."""
    x, w, b = _arrays(x, w, b)
    out = np.empty((m_end - m_begin) * shape.k, dtype=np.int32)
    lib().oracle_conv_rows(_cshape(shape), x.ctypes.data, w.ctypes.data, b.ctypes.data,
                           int(m_begin), int(m_end), out.ctypes.data, int(threads))
    return out


def values(shape, x, w, b, indices, threads: int = 0) -> np.ndarray:
    """Selected output elements (flat NHWK indices)."""
    x, w, b = _arrays(x, w, b)
    idx = np.ascontiguousarray(indices, dtype=np.int64)
    out = np.empty(idx.size, dtype=np.int32)
    lib().oracle_values(_cshape(shape), x.ctypes.data, w.ctypes.data, b.ctypes.data,
                        idx.ctypes.data, int(idx.size), out.ctypes.data, int(threads))
    return out


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def ref_binary(case: str) -> Path | None:
    """oracle/_ref/ref_<case>: the reference's own code for that workloads.csv case."""
    path = REF_DIR / f"ref_{case}"
    return path if path.exists() else None


def ref_cpu_rows(case: str, x, w, b, m_begin: int, m_end: int, threads: int):
    """Runs reference_value<Shape> (src/conv_lab.cu:39-66) over rows
    [m_begin, m_end) in the reference-built binary.  Returns (rows, seconds)."""
    binary = ref_binary(case)
    if binary is None:
        raise FileNotFoundError(f"no reference build for {case} under {REF_DIR}")
    x, w, b = _arrays(x, w, b)
    with tempfile.TemporaryDirectory() as tmp:
        paths = [os.path.join(tmp, n) for n in ("x.bin", "w.bin", "b.bin", "y.bin")]
        x.tofile(paths[0])
        w.tofile(paths[1])
        b.tofile(paths[2])
        proc = subprocess.run(
            [os.fspath(binary), "cpu", *paths, str(m_begin), str(m_end), str(threads)],
            check=True, capture_output=True, text=True)
        result = json.loads(proc.stdout.strip().splitlines()[-1])
        rows = np.fromfile(paths[3], dtype=np.int32)
    return rows, float(result["seconds"])


# ---- requantised int8 output (no reference counterpart) ----------------------

def requant(acc, k: int, multiplier, exponent, zero_point: int = 0, relu: bool = False,
            threads: int = 0) -> np.ndarray:
    """NHWK int32 (conv() output) -> NHWK int8 by the C restatement."""
    acc = np.ascontiguousarray(acc, dtype=np.int32).reshape(-1)
    mult = np.ascontiguousarray(multiplier, dtype=np.int32)
    expo = np.ascontiguousarray(exponent, dtype=np.int32)
    assert acc.size % k == 0 and mult.size == k and expo.size == k
    out = np.empty(acc.size, dtype=np.int8)
    lib().oracle_requant(acc.ctypes.data, acc.size // k, int(k), mult.ctypes.data,
                         expo.ctypes.data, int(zero_point), int(bool(relu)), out.ctypes.data,
                         int(threads))
    return out


def requant_value(t: int, multiplier: int, exponent: int, zero_point: int = 0,
                  relu: bool = False) -> int:
    return int(lib().oracle_requant_value(int(t), int(multiplier), int(exponent),
                                          int(zero_point), int(bool(relu))))


def requant_value_py(t: int, multiplier: int, exponent: int, zero_point: int = 0,
                     relu: bool = False) -> int:
    """Third restatement of the same rule with Python's unbounded integers:
    the rounding steps written as exact rational rounding."""
    e = max(-31, min(31, exponent))
    if e > 0:
        t = max(-2**31, min(2**31 - 1, t * 2**e))
    if t == -2**31 and multiplier == -2**31:
        u = 2**31 - 1
    else:
        ab = t * multiplier
        num = ab + (2**30 if ab >= 0 else 1 - 2**30)
        u = abs(num) // 2**31 * (1 if num >= 0 else -1)      # truncating division
    if e < 0:
        d = 2**-e
        q, r = divmod(abs(u), d)                               # |u| = q*d + r
        q += 1 if 2 * r >= d else 0                            # half away from zero
        u = q if u >= 0 else -q
    y = u + zero_point
    y = max(zero_point if relu else -128, y)
    return min(127, y)


def to_nchw_vect_c(y_nhwk: np.ndarray, n: int, out_h: int, out_w: int, k: int) -> np.ndarray:
    """NHWK int8 -> cuDNN INT8x32 NCHW_VECT_C [N][K/32][P][Q][32] (flat)."""
    assert k % 32 == 0
    y = np.asarray(y_nhwk).reshape(n, out_h, out_w, k // 32, 32)
    return np.ascontiguousarray(y.transpose(0, 3, 1, 2, 4)).reshape(-1)
