"""The C-ABI library without a GPU: loads, exports every declared symbol, and
answers the host-only questions (shape algebra, predicates, status codes)."""
import ctypes
import re
from pathlib import Path

import pytest

import int8_kernel_lab_b200 as m
from int8_kernel_lab_b200 import _abi

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "int8conv.h").read_text()
    return sorted(set(re.findall(r"\b(int8conv_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert set(declared_symbols()) == set(_abi.SIGNATURES)


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports_declared_symbol(name):
    lib = ctypes.CDLL(str(_abi.LIB_PATH))
    assert hasattr(lib, name)


def test_abi_version():
    assert _abi.lib.int8conv_abi_version() == 1


def test_shape_dims_match_reference_formulas():
    # conv_shape.cuh:22-32 on BASELINE config 5a and a strided case.
    s = m.ConvShape(256, 56, 56, 256, 256, 3, 3, 1, 1, 1, 1, 1, 1)
    d = s.dims()
    assert (d.out_h, d.out_w) == (56, 56)
    assert d.gemm_m == 256 * 56 * 56 and d.gemm_n == 256 and d.gemm_k == 2304
    assert d.output_elements == 256 * 56 * 56 * 256
    s2 = m.ConvShape(1, 224, 224, 32, 64, 7, 7, 3, 3, 2, 2, 1, 1)
    assert s2.dims().out_h == 112 and s2.out_h == 112


def test_out_size_uses_truncating_division():
    # (2 + 0 - 2 - 1) / 2 + 1 == 1 in C++ (truncation), not 0 (floor).
    s = m.ConvShape(1, 2, 2, 16, 4, 3, 3, 0, 0, 2, 2, 1, 1)
    assert s.valid and s.dims().out_h == 1 and s.out_h == 1


@pytest.mark.parametrize("bad", [
    dict(c=24),            # conv_shape.cuh:34  c % 16
    dict(h=1, r=3),        # conv_shape.cuh:35  empty output
    dict(n=0), dict(k=0), dict(stride_h=0), dict(dilation_w=0), dict(pad_h=-1),
])
def test_invalid_shapes_rejected(bad):
    base = dict(n=1, h=8, w=8, c=32, k=8, r=3, s=3, pad_h=0, pad_w=0)
    base.update(bad)
    s = m.ConvShape(**base)
    assert not s.valid
    assert _abi.lib.int8conv_shape_dims(s.c_struct(), _abi.CDims()) == _abi.BAD_SHAPE
    for fam in ("generic", "strip", "halo", "splitk"):
        assert not s.eligible(fam)


def test_launch_status_codes_without_gpu():
    s = m.load_workloads()["cfg1_smoke"]
    lib = _abi.lib
    bad = m.ConvShape(1, 8, 8, 24, 8, 3, 3)
    assert lib.int8conv_launch_generic(bad.c_struct(), 16, 16, 16, 16, None) == _abi.BAD_SHAPE
    assert lib.int8conv_launch_generic(s.c_struct(), None, 16, 16, 16, None) == _abi.BAD_POINTER
    assert lib.int8conv_launch_generic(s.c_struct(), 17, 16, 16, 16, None) == _abi.BAD_POINTER
    assert lib.int8conv_launch(7, s.c_struct(), 16, 16, 16, 16, None, 0, None) == _abi.BAD_ARGUMENT
    # A well-formed call on a machine without a GPU is a CUDA error, never a
    # silent success or a CPU fallback.
    assert lib.int8conv_launch_generic(s.c_struct(), 16, 16, 16, 16, None) in (
        _abi.CUDA_ERROR, _abi.UNSUPPORTED_DEVICE)


def test_status_and_strategy_strings():
    assert _abi.lib.int8conv_status_string(_abi.NOT_ELIGIBLE) == b"shape not eligible for this strategy"
    for name, code in _abi.STRATEGIES.items():
        assert _abi.lib.int8conv_strategy_name(code).decode() == name


def test_select_returns_an_eligible_family():
    for name, s in m.load_workloads().items():
        fam = s.select()
        assert s.eligible(fam), name


def test_row_count_bound_leaves_a_tile_of_slack():
    # The kernels index rows as int32 and run up to one 256-row tile past the
    # last row, so N*P*Q must stay below 2^31 - 512.
    ok = m.ConvShape(1, 256, 8388605, 16, 16, 1, 1, 0, 0, 1, 1, 1, 1)
    assert ok.n * ok.out_h * ok.out_w == 2**31 - 768 and ok.valid
    for w in (8388606, 8388607):  # 2^31 - 512, 2^31 - 256 rows
        big = m.ConvShape(1, 256, w, 16, 16, 1, 1, 0, 0, 1, 1, 1, 1)
        assert big.n * big.h * big.w < 2**31 and not big.valid


class _FakeCudaTensor:
    """Stands in for a CUDA tensor on another GPU (no GPU needed)."""

    def __init__(self, dtype, count, index):
        import torch

        self.is_cuda = True
        self.dtype = dtype
        self.shape = (count,)
        self.device = torch.device("cuda", index)
        self._count = count

    def is_contiguous(self):
        return True

    def numel(self):
        return self._count

    def data_ptr(self):
        return 1 << 20


def test_buffers_on_another_device_are_refused(monkeypatch):
    # The launch would run on the current device with pointers into another
    # GPU's memory; the Python mirror refuses it before calling the library.
    import torch

    from int8_kernel_lab_b200 import api

    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    s = m.load_workloads()["cfg1_smoke"]
    x = _FakeCudaTensor(torch.int8, s.input_elements, 1)
    w = _FakeCudaTensor(torch.int8, s.filter_elements, 1)
    b = _FakeCudaTensor(torch.int32, s.k, 1)
    y = _FakeCudaTensor(torch.int32, s.output_elements, 1)
    with pytest.raises(ValueError, match="current CUDA device is cuda:0"):
        api.launch("generic", s, x, w, b, y)
    with pytest.raises(ValueError, match="current CUDA device"):
        api.launch_generic(s, x, w, b, y)
    # Same device: the check passes (the launch itself is not reached here).
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 1)
    api._check_tensors(s, x, w, b, y)
