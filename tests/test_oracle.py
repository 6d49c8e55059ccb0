"""The CPU oracle against the reference's own outputs and hand-computed answers."""
import numpy as np
import pytest

import pyoracle
from conftest import golden_cases, load_golden

import int8_kernel_lab_b200 as m


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_reference_golden(name):
    # Fixtures were produced by reference_value<Shape> (src/conv_lab.cu:39-66)
    # built from the reference sources (tests/golden/make_golden.py).
    shape, x, w, b, y = load_golden(name)
    assert np.array_equal(pyoracle.conv(shape, x, w, b), y)


def _shape(**kw):
    base = dict(n=1, h=5, w=5, c=16, k=4, r=3, s=3, pad_h=1, pad_w=1)
    base.update(kw)
    return m.ConvShape(**base)


def test_identity_1x1_filter():
    s = _shape(r=1, s=1, pad_h=0, pad_w=0, k=16)
    rng = np.random.RandomState(0)
    x = rng.randint(-128, 128, s.input_elements).astype(np.int8)
    w = np.eye(16, dtype=np.int8).reshape(-1)
    b = np.arange(16, dtype=np.int32) * 1000
    y = pyoracle.conv(s, x, w, b).reshape(-1, 16)
    assert np.array_equal(y, x.reshape(-1, 16).astype(np.int32) + b)


@pytest.mark.parametrize("tap", [(fy, fx) for fy in range(3) for fx in range(3)])
def test_delta_filter_per_tap_shifts_input(tap):
    fy, fx = tap
    s = _shape(k=16)
    rng = np.random.RandomState(1)
    x = rng.randint(-128, 128, s.input_elements).astype(np.int8)
    w = np.zeros((16, 3, 3, 16), np.int8)
    for k in range(16):
        w[k, fy, fx, k] = 1
    b = np.zeros(16, np.int32)
    y = pyoracle.conv(s, x, w.reshape(-1), b).reshape(5, 5, 16)
    xp = np.pad(x.reshape(5, 5, 16).astype(np.int32), ((1, 1), (1, 1), (0, 0)))
    assert np.array_equal(y, xp[fy:fy + 5, fx:fx + 5, :])


def test_padding_corner_sees_only_four_taps():
    s = _shape(k=1)
    x = np.ones(s.input_elements, np.int8)
    w = np.ones(s.filter_elements, np.int8)
    y = pyoracle.conv(s, x, w, np.zeros(1, np.int32)).reshape(5, 5)
    assert y[0, 0] == 4 * 16 and y[0, 2] == 6 * 16 and y[2, 2] == 9 * 16


def test_max_magnitude_no_overflow():
    s = m.ConvShape(1, 7, 7, 512, 2, 3, 3, 1, 1)  # BASELINE config 4b's reduction
    x = np.full(s.input_elements, -128, np.int8)
    w = np.full(s.filter_elements, -128, np.int8)
    b = np.full(2, 65536, np.int32)
    y = pyoracle.conv(s, x, w, b).reshape(7, 7, 2)
    assert y[3, 3, 0] == 9 * 512 * 16384 + 65536  # 75,563,008 < 2**31


def test_values_and_rows_agree_with_full():
    shape, x, w, b, y = load_golden("g_c48_k100")
    idx = np.array([0, 1, 99, 100, y.size - 1, 12345 % y.size])
    assert np.array_equal(pyoracle.values(shape, x, w, b, idx), y[idx])
    rows = pyoracle.conv_rows(shape, x, w, b, 3, 9)
    assert np.array_equal(rows, y[3 * shape.k:9 * shape.k])


@pytest.mark.parametrize("threads", [1, 3])
def test_thread_count_does_not_change_result(threads):
    shape, x, w, b, y = load_golden("g_k63")
    assert np.array_equal(pyoracle.conv(shape, x, w, b, threads=threads), y)


def test_reference_binary_agrees_when_present():
    # oracle/_ref exists where the reference was built (this container and
    # the GPU box, which receives the built binaries).
    if pyoracle.ref_binary("cfg1_smoke") is None:
        pytest.skip("reference oracle not built")
    s = m.load_workloads()["cfg1_smoke"]
    x, w, b = m.make_inputs(s)
    rows, _ = pyoracle.ref_cpu_rows("cfg1_smoke", x, w, b, 0, s.gemm_m, 2)
    assert np.array_equal(rows, pyoracle.conv(s, x, w, b))
