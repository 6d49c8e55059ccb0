"""Host-side mirror of the reference's launcher interface, on device buffers.

Reference interface (header-only templates, compile-time Shape):
    launch_generic<Shape>(input, filter, bias, output, stream = 0)
        include/generic_implicit_gemm.cuh:155-165 (and launch_generic_sm80, :229-238)
    launch_spatial_strip<Shape>(input, filter, bias, output, stream = 0)
        include/spatial_strip.cuh:289-301
    kSpatialStripEligible<Shape>
        include/spatial_strip.cuh:11-15
Here Shape is a runtime ConvShape and the buffers are CUDA tensors (or raw
device pointers).  The caller owns every buffer; launches are asynchronous on
the stream; nothing allocates.  Where the reference fails to compile
(static_assert on an ineligible shape) these raise Int8ConvError with
status NOT_ELIGIBLE.
"""
from __future__ import annotations

from typing import Optional

from . import _abi
from .shape import ConvShape


def _ptr(buf) -> int:
    if buf is None:
        return 0
    if isinstance(buf, int):
        return buf
    return int(buf.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        import torch

        return int(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def _check_device(*tensors) -> None:
    """Every launch runs on the current CUDA device.  A buffer that lives on
    another GPU would be dereferenced there through a foreign address (an
    illegal-address fault without peer access), so it is refused here."""
    import torch

    current = None
    for t in tensors:
        if t is None or isinstance(t, int) or not getattr(t, "is_cuda", False):
            continue
        if current is None:
            current = torch.cuda.current_device()
        if t.device.index != current:
            raise ValueError(
                f"buffer on {t.device}, but the current CUDA device is cuda:{current}: "
                f"launch under torch.cuda.device({t.device.index}) or move the buffers")


def _check_tensors(shape: ConvShape, x, w, b, y) -> None:
    import torch

    for name, t, dtype, count in (
        ("input", x, torch.int8, shape.input_elements),
        ("filter", w, torch.int8, shape.filter_elements),
        ("bias", b, torch.int32, shape.k),
        ("output", y, torch.int32, shape.output_elements),
    ):
        if t is None or isinstance(t, int):
            continue
        if not t.is_cuda or t.dtype != dtype or not t.is_contiguous() or t.numel() != count:
            raise ValueError(
                f"{name}: expected a contiguous CUDA {dtype} tensor of {count} elements, "
                f"got {t.dtype} {tuple(t.shape)} on {t.device}")
    _check_device(x, w, b, y)


def launch(strategy: str, shape: ConvShape, x, w, b, y, *, workspace=None,
           workspace_bytes: int = 0, stream=None) -> None:
    """int8conv_launch: one family ('generic', 'strip', 'halo', 'splitk') or 'auto'."""
    _check_tensors(shape, x, w, b, y)
    status = _abi.lib.int8conv_launch(
        _abi.STRATEGIES[strategy], shape.c_struct(), _ptr(x), _ptr(w), _ptr(b), _ptr(y),
        _ptr(workspace), int(workspace_bytes), _stream(stream))
    _abi.check(status, f"{strategy} launch of {shape}")


def launch_generic(shape: ConvShape, x, w, b, y, stream=None) -> None:
    _check_tensors(shape, x, w, b, y)
    _abi.check(_abi.lib.int8conv_launch_generic(shape.c_struct(), _ptr(x), _ptr(w), _ptr(b),
                                                _ptr(y), _stream(stream)), "launch_generic")


# The reference's SM80 generic launcher has the same contract (one B200 kernel
# serves both names).
launch_generic_sm80 = launch_generic


def launch_spatial_strip(shape: ConvShape, x, w, b, y, stream=None) -> None:
    _check_tensors(shape, x, w, b, y)
    _abi.check(_abi.lib.int8conv_launch_spatial_strip(shape.c_struct(), _ptr(x), _ptr(w), _ptr(b),
                                                      _ptr(y), _stream(stream)),
               "launch_spatial_strip")


def spatial_strip_eligible(shape: ConvShape) -> bool:
    """kSpatialStripEligible<Shape> for the B200 strip kernel."""
    return shape.eligible("strip")


def workspace_bytes(shape: ConvShape, strategy: str) -> int:
    return int(_abi.lib.int8conv_workspace_bytes(shape.c_struct(), _abi.STRATEGIES[strategy]))


def conv2d(shape: ConvShape, x, w, b, strategy: str = "auto", stream=None):
    """Allocate the NHWK int32 output and launch.  Convenience for callers that
    own no output buffer; returns the output tensor."""
    import torch

    y = torch.empty(shape.output_elements, dtype=torch.int32, device=x.device)
    ws = None
    nbytes = workspace_bytes(shape, strategy) if strategy != "auto" else workspace_bytes(
        shape, shape.select())
    if nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    launch(strategy, shape, x, w, b, y, workspace=ws, workspace_bytes=nbytes, stream=stream)
    return y


def launch_host(strategy: str, shape: ConvShape, hx, hw, hb, hy, dx, dw, db, dy, *,
                chunks: int = 8, stream=None) -> None:
    """int8conv_launch_host: convolve HOST tensors (pinned CPU tensors for
    overlap) through caller-owned device buffers, streaming the batch in
    `chunks` groups of images so the PCIe copies in both directions overlap the
    kernels.  Asynchronous on `stream`; synchronise it before reading `hy`."""
    import torch

    for name, t, dev in (("hx", hx, False), ("hw", hw, False), ("hb", hb, False),
                         ("hy", hy, False), ("dx", dx, True), ("dw", dw, True),
                         ("db", db, True), ("dy", dy, True)):
        if t.is_cuda != dev or not t.is_contiguous():
            where = "CUDA" if dev else "host"
            raise ValueError(f"{name}: expected a contiguous {where} tensor")
    _check_tensors(shape, dx, dw, db, dy)
    if (hx.numel() != shape.input_elements or hw.numel() != shape.filter_elements
            or hb.numel() != shape.k or hy.numel() != shape.output_elements):
        raise ValueError("host tensor sizes do not match the shape")
    status = _abi.lib.int8conv_launch_host(
        _abi.STRATEGIES[strategy], shape.c_struct(), _ptr(hx), _ptr(hw), _ptr(hb), _ptr(hy),
        _ptr(dx), _ptr(dw), _ptr(db), _ptr(dy), int(chunks), _stream(stream))
    _abi.check(status, f"{strategy} host launch of {shape}")


def launch_requant(strategy: str, shape: ConvShape, x, w, b, multiplier, exponent, y, *,
                   zero_point: int = 0, relu: bool = False, layout: str = "nhwc",
                   workspace=None, workspace_bytes: int = 0, stream=None) -> None:
    """int8conv_launch_requant: the convolution with an int8 epilogue.

    `multiplier` and `exponent` are K-entry int32 CUDA tensors (Q31 multiplier
    and power-of-two exponent per output channel); `y` is an int8 CUDA tensor
    of N*out_h*out_w*K elements in `layout` ('nhwc' or 'nchw_vect_c', cuDNN's
    INT8x32).  No reference counterpart: the reference's kernels write int32."""
    import torch

    _check_tensors(shape, x, w, b, None)
    for name, t, dtype, count in (("multiplier", multiplier, torch.int32, shape.k),
                                  ("exponent", exponent, torch.int32, shape.k),
                                  ("output", y, torch.int8, shape.output_elements)):
        if isinstance(t, int):
            continue
        if not t.is_cuda or t.dtype != dtype or not t.is_contiguous() or t.numel() != count:
            raise ValueError(
                f"{name}: expected a contiguous CUDA {dtype} tensor of {count} elements, "
                f"got {t.dtype} {tuple(t.shape)} on {t.device}")
    _check_device(x, multiplier, exponent, y)
    rq = _abi.CRequant(_ptr(multiplier), _ptr(exponent), int(zero_point), 1 if relu else 0,
                       _abi.LAYOUTS[layout])
    status = _abi.lib.int8conv_launch_requant(
        _abi.STRATEGIES[strategy], shape.c_struct(), _ptr(x), _ptr(w), _ptr(b), rq, _ptr(y),
        _ptr(workspace), int(workspace_bytes), _stream(stream))
    _abi.check(status, f"{strategy} requantised launch of {shape}")


def device_status() -> int:
    """int8conv_device_status(): synchronises; DEVICE_TIMEOUT if a bounded wait ran out."""
    return int(_abi.lib.int8conv_device_status())


def launch_count() -> int:
    return int(_abi.lib.int8conv_launch_count())


def set_wait_limit_ns(ns: int) -> None:
    _abi.lib.int8conv_set_wait_limit_ns(int(ns))


PAIRING = {"auto": 0, "single": 1, "pair": 2}


def set_cta_pairing(mode: str) -> None:
    """'auto' | 'single' | 'pair': how the GENERIC/STRIP kernels group CTAs."""
    _abi.check(_abi.lib.int8conv_set_cta_pairing(PAIRING[mode]), "set_cta_pairing")


STAGING = {"auto": 0, "gather": 1}


def set_generic_staging(mode: str) -> None:
    """'auto' | 'gather': how GENERIC stages activations ('auto' uses the TMA
    im2col map wherever it can encode the shape; 'gather' uses the gather warp
    for every shape)."""
    _abi.check(_abi.lib.int8conv_set_generic_staging(STAGING[mode]), "set_generic_staging")


def debug_starve_producer(on: bool) -> None:
    _abi.lib.int8conv_debug_starve_producer(1 if on else 0)
