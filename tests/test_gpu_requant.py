"""GPU parity of the requantised int8 epilogue (int8conv_launch_requant).

Every eligible family, both output layouts, with and without the fused ReLU,
against the CPU oracle: the int32 convolution (src/conv_lab.cu:39-66 of the
reference, restated in oracle/conv_oracle.c) followed by the oracle's
restatement of the gemmlowp requantisation.  Bit-exact.
"""
import functools

import numpy as np
import pytest

import pyoracle

import int8_kernel_lab_b200 as m
from int8_kernel_lab_b200 import _abi

pytestmark = pytest.mark.gpu

FAMILIES = ("generic", "strip", "halo", "splitk")
GUARD = 4096  # bytes after the output that must stay untouched


def _shapes():
    wl = m.load_workloads()
    return {
        "cfg1_smoke": wl["cfg1_smoke"],                    # K=64, split-K, TMA int8 store
        "cfg2_mid_3x3": wl["cfg2_mid_3x3"],                # K=128
        "cfg4a_deep_1x1": wl["cfg4a_deep_1x1"],            # K=512: two 256-wide N tiles
        "cfg4c_tail_k100": wl["cfg4c_tail_k100"],          # K=100: no TMA store, no VECT_C
        "nonmultiple8_k63": wl["nonmultiple8_k63"],        # odd K
        "k288": m.ConvShape(2, 14, 14, 64, 288, 3, 3, 1, 1, 1, 1, 1, 1),  # bn 144 / 160
        "cfg5b_n2": wl["cfg5b_dilated_3x3"].with_batch(2),
        "cfg5a_n2": wl["cfg5a_stress_3x3"].with_batch(2),  # 256-wide tiles, pairs when asked
    }


SHAPES = _shapes()


def _params(shape, seed):
    """Per-channel Q31 multipliers and exponents that spread full-range
    accumulators over the int8 range (with some saturation)."""
    rng = np.random.RandomState(seed)
    mult = rng.randint(1 << 30, (1 << 31) - 1, shape.k, dtype=np.int64).astype(np.int32)
    expo = rng.randint(-13, -7, shape.k).astype(np.int32)
    return mult, expo


def _run(torch, strategy, shape, x, w, b, mult, expo, zp, relu, layout):
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (x, w, b, mult, expo)]
    buf = torch.full((shape.output_elements + GUARD,), 0x5A, dtype=torch.int8, device="cuda")
    y = buf[:shape.output_elements]
    m.launch_requant(strategy, shape, dev[0], dev[1], dev[2], dev[3], dev[4], y,
                     zero_point=zp, relu=relu, layout=layout)
    assert m.device_status() == _abi.OK
    host = buf.cpu().numpy()
    assert np.all(host[shape.output_elements:] == 0x5A), "write past the end of the output"
    return host[:shape.output_elements]


def _want(shape, acc, mult, expo, zp, relu, layout):
    y = pyoracle.requant(acc, shape.k, mult, expo, zero_point=zp, relu=relu)
    if layout == "nchw_vect_c":
        y = pyoracle.to_nchw_vect_c(y, shape.n, shape.out_h, shape.out_w, shape.k)
    return y


@functools.lru_cache(maxsize=None)
def _case(name):
    shape = SHAPES[name]
    x, w, b = m.make_inputs(shape)
    return shape, x, w, b, pyoracle.conv(shape, x, w, b)


@pytest.fixture(params=["single", "pair"])
def pairing(request):
    m.set_cta_pairing(request.param)
    yield request.param
    m.set_cta_pairing("auto")


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_requant_all_families_and_layouts(cuda, pairing, name):
    shape, x, w, b, acc = _case(name)
    mult, expo = _params(shape, 11)
    layouts = ["nhwc"] + (["nchw_vect_c"] if shape.k % 32 == 0 else [])
    for fam in [f for f in FAMILIES if shape.eligible(f)]:
        for layout in layouts:
            for zp, relu in ((0, False), (-7, True)):
                got = _run(cuda, fam, shape, x, w, b, mult, expo, zp, relu, layout)
                want = _want(shape, acc, mult, expo, zp, relu, layout)
                bad = np.count_nonzero(got != want)
                assert bad == 0, f"{fam} {layout} zp={zp} relu={relu} on {name}: {bad} mismatches"


def test_unit_scale_is_the_saturating_cast(cuda):
    # multiplier 2^30, exponent 1: y = clamp(int32 output, -128, 127), the int8
    # output of cuDNN INT8x32 with alpha = 1 (include/cudnn_legacy.cuh:51-55).
    shape = SHAPES["cfg2_mid_3x3"]
    x, w, b = m.make_inputs(shape, values="reference")
    mult = np.full(shape.k, 1 << 30, dtype=np.int32)
    expo = np.ones(shape.k, dtype=np.int32)
    dx, dw, db = (cuda.from_numpy(a).cuda() for a in (x, w, b))
    y32 = cuda.empty(shape.output_elements, dtype=cuda.int32, device="cuda")
    m.launch("generic", shape, dx, dw, db, y32)
    got = _run(cuda, "auto", shape, x, w, b, mult, expo, 0, False, "nhwc")
    assert np.array_equal(got, np.clip(y32.cpu().numpy(), -128, 127).astype(np.int8))


def test_requant_stream_and_auto(cuda):
    shape = SHAPES["cfg4c_tail_k100"]
    x, w, b = m.make_inputs(shape, seed=5)
    mult, expo = _params(shape, 5)
    s = cuda.cuda.Stream()
    dev = [cuda.from_numpy(a).cuda() for a in (x, w, b, mult, expo)]
    y = cuda.zeros(shape.output_elements, dtype=cuda.int8, device="cuda")
    s.wait_stream(cuda.cuda.current_stream())  # the buffers' copies and fill
    with cuda.cuda.stream(s):
        m.launch_requant("auto", shape, *dev, y, zero_point=3, relu=True, stream=s)
    s.synchronize()
    want = _want(shape, pyoracle.conv(shape, x, w, b), mult, expo, 3, True, "nhwc")
    assert np.array_equal(y.cpu().numpy(), want)


I32 = (-(1 << 31), (1 << 31) - 1)
EDGE_T = [I32[0], I32[1], 0, 1, -1, 2, -2, 3, -3, 5, -5, 1 << 30, -(1 << 30), 65537, -65537,
          (1 << 24) + 1, 127, 128, -128, -129, 1000003, -999999]
EDGE_M = [I32[0], I32[1], 1 << 30, 0, 1, -7, 1518500250, (1 << 29) + 12345, -(1 << 30)]
EDGE_E = [-40, -31, -30, -13, -1, 0, 1, 2, 30, 31, 40]


@pytest.mark.parametrize("layout", ["nhwc", "nchw_vect_c"])
def test_requant_edge_values_on_device(cuda, layout):
    # A zero filter makes every output t = bias[k] exactly, so the device's
    # requantisation meets chosen edge values of t, multiplier and exponent.
    shape = m.ConvShape(1, 4, 4, 16, 256, 3, 3, 1, 1, 1, 1, 1, 1)
    rng = np.random.RandomState(23)
    x = rng.randint(-128, 128, shape.input_elements).astype(np.int8)
    w = np.zeros(shape.filter_elements, dtype=np.int8)
    for trial in range(6):
        b = np.array([EDGE_T[(k + 7 * trial) % len(EDGE_T)] for k in range(shape.k)], np.int64)
        mult = np.array([EDGE_M[(k // 3 + trial) % len(EDGE_M)] for k in range(shape.k)], np.int64)
        expo = np.array([EDGE_E[(k // 5 + 2 * trial) % len(EDGE_E)] for k in range(shape.k)])
        b, mult, expo = b.astype(np.int32), mult.astype(np.int32), expo.astype(np.int32)
        acc = np.tile(b, shape.out_h * shape.out_w)
        for zp, relu in ((0, False), (-128, False), (127, True), (-9, True)):
            want = _want(shape, acc, mult, expo, zp, relu, layout)
            for fam in ("generic", "splitk"):
                got = _run(cuda, fam, shape, x, w, b, mult, expo, zp, relu, layout)
                bad = np.flatnonzero(got != want)
                assert bad.size == 0, (fam, trial, zp, relu, bad[:5], got[bad[:5]], want[bad[:5]])


def test_device_meets_hand_derived_known_answers(cuda):
    # The published rule's known answers (derived by hand, not by the oracle):
    # INT32_MIN * INT32_MIN, saturating left shifts, ties at every exponent of
    # the rounding divide.  A zero filter makes t = bias[k]; each channel
    # carries one (t, multiplier, exponent) row, and rows sharing a zero
    # point and ReLU flag run in one launch.
    from test_requant_cpu import Q30, TIES, known_answer_table

    rows = known_answer_table() + [
        (sign * (2 * k + 1) * 2 ** n, Q30, -n, 0, 0, sign * (k + 1)) for n, k, sign in TIES]
    groups = {}
    for row in rows:
        groups.setdefault((row[3], row[4]), []).append(row)
    for (zp, relu), group in groups.items():
        k = len(group)
        shape = m.ConvShape(1, 2, 3, 16, k, 1, 1, 0, 0, 1, 1, 1, 1)
        x = np.zeros(shape.input_elements, np.int8)
        w = np.ones(shape.filter_elements, np.int8)
        b = np.array([r[0] for r in group], np.int64).astype(np.int32)
        mult = np.array([r[1] for r in group], np.int64).astype(np.int32)
        expo = np.array([r[2] for r in group], np.int32)
        want = np.tile(np.array([r[5] for r in group], np.int8), shape.out_h * shape.out_w)
        for fam in ("generic", "auto"):
            got = _run(cuda, fam, shape, x, w, b, mult, expo, zp, bool(relu), "nhwc")
            bad = np.flatnonzero(got != want)
            assert bad.size == 0, (fam, zp, relu, [group[i % k] for i in bad[:4]], got[bad[:4]])
