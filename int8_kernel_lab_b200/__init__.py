"""int8_kernel_lab_b200 - B200-native (sm_100a) INT8 implicit-GEMM convolution.

A drop-in for the conv path of pthodima/int8_kernel_lab: NHWC int8 input, KRSC
int8 filter, K int32 bias, NHWK int32 output, the conv_shape descriptor and
per-family eligibility predicates.  All compute runs in libint8conv.so
(hand-written tcgen05 / TMA kernels) behind the C ABI of include/int8conv.h.
"""
from ._abi import (AUTO, GENERIC, HALO, SPLITK, STRIP, STRATEGIES, Int8ConvError,  # noqa: F401
                   LIB_PATH)
from .api import (conv2d, debug_starve_producer, device_status, launch,  # noqa: F401
                  launch_count, launch_host, launch_generic, launch_generic_sm80, launch_requant,
                  launch_spatial_strip,
                  set_cta_pairing, set_generic_staging, set_wait_limit_ns,
                  spatial_strip_eligible, workspace_bytes)
from .data import REFERENCE_SEED, make_inputs  # noqa: F401
from .shape import (BASELINE_CASES, ConvShape, baseline_shapes, load_workloads)  # noqa: F401

__all__ = [
    "ConvShape", "load_workloads", "baseline_shapes", "BASELINE_CASES", "make_inputs",
    "launch", "launch_host", "launch_requant", "launch_generic", "launch_generic_sm80", "launch_spatial_strip",
    "spatial_strip_eligible", "conv2d", "workspace_bytes", "device_status", "launch_count",
    "Int8ConvError", "STRATEGIES",
]
