"""ctypes binding of the C ABI in include/int8conv.h (libint8conv.so).

The library is built in-tree (``make -C int8_kernel_lab_b200/csrc``).  There is
no fallback: if the shared object is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libint8conv.so"

SHAPE_FIELDS = (
    "n", "h", "w", "c", "k", "r", "s", "pad_h", "pad_w",
    "stride_h", "stride_w", "dilation_h", "dilation_w",
)

# int8conv_status
OK = 0
NOT_ELIGIBLE = 1
BAD_SHAPE = 2
BAD_POINTER = 3
CUDA_ERROR = 4
DEVICE_TIMEOUT = 5
WORKSPACE_TOO_SMALL = 6
UNSUPPORTED_DEVICE = 7
BAD_ARGUMENT = 8

# int8conv_strategy
GENERIC = 0
STRIP = 1
HALO = 2
SPLITK = 3
AUTO = 100
STRATEGIES = {"generic": GENERIC, "strip": STRIP, "halo": HALO, "splitk": SPLITK, "auto": AUTO}


# int8conv_layout
LAYOUT_NHWC = 0
LAYOUT_NCHW_VECT_C = 1
LAYOUTS = {"nhwc": LAYOUT_NHWC, "nchw_vect_c": LAYOUT_NCHW_VECT_C}


class CRequant(ctypes.Structure):
    _fields_ = [("multiplier", ctypes.c_void_p), ("exponent", ctypes.c_void_p),
                ("zero_point", ctypes.c_int32), ("relu", ctypes.c_int32),
                ("layout", ctypes.c_int32)]


class CShape(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in SHAPE_FIELDS]


class CDims(ctypes.Structure):
    _fields_ = [
        ("out_h", ctypes.c_int32), ("out_w", ctypes.c_int32),
        ("gemm_m", ctypes.c_int64), ("gemm_n", ctypes.c_int64), ("gemm_k", ctypes.c_int64),
        ("input_elements", ctypes.c_int64), ("filter_elements", ctypes.c_int64),
        ("output_elements", ctypes.c_int64),
    ]


# (name, restype, argtypes) for every symbol the header declares.
_P = ctypes.c_void_p
_SP = ctypes.POINTER(CShape)
SIGNATURES = {
    "int8conv_abi_version": (ctypes.c_int, []),
    "int8conv_shape_valid": (ctypes.c_int, [_SP]),
    "int8conv_shape_dims": (ctypes.c_int, [_SP, ctypes.POINTER(CDims)]),
    "int8conv_eligible": (ctypes.c_int, [_SP, ctypes.c_int]),
    "int8conv_select": (ctypes.c_int, [_SP]),
    "int8conv_workspace_bytes": (ctypes.c_size_t, [_SP, ctypes.c_int]),
    "int8conv_strategy_name": (ctypes.c_char_p, [ctypes.c_int]),
    "int8conv_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "int8conv_launch": (ctypes.c_int, [ctypes.c_int, _SP, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "int8conv_launch_generic": (ctypes.c_int, [_SP, _P, _P, _P, _P, _P]),
    "int8conv_launch_spatial_strip": (ctypes.c_int, [_SP, _P, _P, _P, _P, _P]),
    "int8conv_launch_halo": (ctypes.c_int, [_SP, _P, _P, _P, _P, _P]),
    "int8conv_launch_splitk": (ctypes.c_int, [_SP, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]),
    "int8conv_launch_host": (ctypes.c_int, [ctypes.c_int, _SP] + [_P] * 8 + [ctypes.c_int, _P]),
    "int8conv_launch_requant": (ctypes.c_int, [ctypes.c_int, _SP, _P, _P, _P,
                                               ctypes.POINTER(CRequant), _P, _P, ctypes.c_size_t,
                                               _P]),
    "int8conv_device_status": (ctypes.c_int, []),
    "int8conv_set_wait_limit_ns": (None, [ctypes.c_uint64]),
    "int8conv_debug_starve_producer": (None, [ctypes.c_int]),
    "int8conv_launch_count": (ctypes.c_uint64, []),
    "int8conv_set_cta_pairing": (ctypes.c_int, [ctypes.c_int]),
    "int8conv_set_generic_staging": (ctypes.c_int, [ctypes.c_int]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C {LIB_PATH.parent.parent / 'csrc'}` "
            "(or __graft_entry__.build()); there is no non-CUDA fallback")
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


class Int8ConvError(RuntimeError):
    """A non-OK int8conv_status."""

    def __init__(self, status: int, what: str = ""):
        self.status = status
        text = lib.int8conv_status_string(status).decode()
        super().__init__(f"{what}: {text} (status {status})" if what else text)


def check(status: int, what: str = "") -> None:
    if status != OK:
        raise Int8ConvError(status, what)
