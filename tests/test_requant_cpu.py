"""Requantised int8 output: the oracle's restatement and the ABI's argument
checks, without a GPU.

The rule (include/int8conv.h, int8conv_requant) is gemmlowp / TensorFlow Lite
fixed-point requantisation.  The reference has no int8 epilogue of its own;
its cuDNN comparison writes int8 with alpha = 1 (include/cudnn_legacy.cuh:51-55),
which is the multiplier 2^30, exponent 1 case.  The known answers below follow
from the rule's definition by hand.
"""
import ctypes
import itertools

import numpy as np
import pytest

import pyoracle

import int8_kernel_lab_b200 as m
from int8_kernel_lab_b200 import _abi

Q30 = 1 << 30
I32_MIN, I32_MAX = -(1 << 31), (1 << 31) - 1


@pytest.mark.parametrize("t, mult, e, zp, relu, want", [
    # multiplier 2^30, exponent 1: the saturating cast of cuDNN's alpha = 1.
    (5, Q30, 1, 0, 0, 5), (-5, Q30, 1, 0, 0, -5), (127, Q30, 1, 0, 0, 127),
    (128, Q30, 1, 0, 0, 127), (-129, Q30, 1, 0, 0, -128), (I32_MAX, Q30, 1, 0, 0, 127),
    (I32_MIN, Q30, 1, 0, 0, -128),
    # exponent 0: x / 2 with the doubling-high-multiply nudge (ties toward +inf).
    (5, Q30, 0, 0, 0, 3), (-5, Q30, 0, 0, 0, -2), (3, Q30, 0, 0, 0, 2), (-3, Q30, 0, 0, 0, -1),
    (4, Q30, 0, 0, 0, 2), (-4, Q30, 0, 0, 0, -2),
    # exponent -1 after an exact halving: rounding divide, ties away from zero.
    (6, Q30, -1, 0, 0, 2), (-6, Q30, -1, 0, 0, -2), (10, Q30, -1, 0, 0, 3),
    (-10, Q30, -1, 0, 0, -3), (8, Q30, -1, 0, 0, 2), (-8, Q30, -1, 0, 0, -2),
    # zero point and fused ReLU (clamp below at the zero point).
    (-50, Q30, 1, 10, 0, -40), (-50, Q30, 1, 10, 1, 10), (50, Q30, 1, 10, 1, 60),
    (200, Q30, 1, -20, 0, 127), (-200, Q30, 1, 100, 1, 100),
    # saturation: INT32_MIN * INT32_MIN, and a saturating left shift.
    (I32_MIN, I32_MIN, 0, 0, 0, 127), (2, Q30, 31, 0, 0, 127), (-2, Q30, 31, 0, 0, -128),
    # exponents outside [-31, 31] are clamped (-40 acts as -31: (2^31 - 2) / 2^31
    # rounds to 1); a zero multiplier gives the zero point.
    (I32_MAX, Q30, 40, 0, 0, 127), (I32_MAX, I32_MAX, -40, 0, 0, 1), (12345, 0, 0, 7, 0, 7),
    # a realistic scale, 0.0123 = Q31 multiplier 0.7872 times 2^-6:
    # 10000 * 0.7872 = 7872.3 -> 7872, / 64 = 123.0 -> 123.
    (10000, 1690543995, -6, 0, 0, 123), (-10000, 1690543995, -6, 0, 0, -123),
])
def test_requant_known_answers(t, mult, e, zp, relu, want):
    assert pyoracle.requant_value(t, mult, e, zp, relu) == want
    assert pyoracle.requant_value_py(t, mult, e, zp, relu) == want


def test_requant_restatements_agree():
    # The C oracle (integer division) and the Python restatement (exact
    # rational rounding) on edge and random values.
    edges = [0, 1, -1, 2, -2, 3, -3, 5, -5, 2**30, -2**30, I32_MAX, I32_MIN, 65537, -65537]
    mults = [Q30, I32_MAX, I32_MIN, 1, 0, -7, 1518500250, 2**29 + 12345]
    exps = [-31, -30, -7, -1, 0, 1, 2, 31, 40, -40]
    for t, mult, e in itertools.product(edges, mults, exps):
        for zp, relu in ((0, 0), (-5, 1), (17, 0), (127, 1), (-128, 0)):
            assert (pyoracle.requant_value(t, mult, e, zp, relu)
                    == pyoracle.requant_value_py(t, mult, e, zp, relu)), (t, mult, e, zp, relu)
    rng = np.random.RandomState(7)
    for _ in range(20000):
        t, mult = (int(v) for v in rng.randint(I32_MIN, I32_MAX, 2, dtype=np.int64))
        e, zp, relu = int(rng.randint(-35, 36)), int(rng.randint(-128, 128)), int(rng.randint(2))
        assert (pyoracle.requant_value(t, mult, e, zp, relu)
                == pyoracle.requant_value_py(t, mult, e, zp, relu))


def test_requant_array_is_per_channel():
    rng = np.random.RandomState(3)
    k = 24
    acc = rng.randint(-2**20, 2**20, 10 * k).astype(np.int32)
    mult = rng.randint(Q30, I32_MAX, k).astype(np.int32)
    expo = rng.randint(-14, 2, k).astype(np.int32)
    y = pyoracle.requant(acc, k, mult, expo, zero_point=-3, relu=True)
    want = [pyoracle.requant_value_py(int(acc[i]), int(mult[i % k]), int(expo[i % k]), -3, True)
            for i in range(acc.size)]
    assert y.dtype == np.int8 and y.tolist() == want


def test_vect_c_layout():
    # cuDNN NCHW_VECT_C INT8x32: element (n, k, y, x) at
    # ((n*K/32 + k/32)*P + y)*Q + x)*32 + k%32.
    n, p, q, k = 2, 3, 5, 64
    y = np.arange(n * p * q * k, dtype=np.int64).astype(np.int8)
    v = pyoracle.to_nchw_vect_c(y, n, p, q, k)
    nhwk = y.reshape(n, p, q, k)
    for (bn, bk, by, bx) in [(0, 0, 0, 0), (1, 33, 2, 4), (0, 63, 1, 3), (1, 31, 0, 1)]:
        assert v[(((bn * (k // 32) + bk // 32) * p + by) * q + bx) * 32 + bk % 32] == \
            nhwk[bn, by, bx, bk]


def _launch_args(shape, rq):
    # Aligned fake device addresses: argument checks come before any device use.
    fake = 1 << 20
    return (_abi.GENERIC, shape.c_struct(), fake, fake, fake, ctypes.byref(rq), fake, None, 0,
            None)


@pytest.mark.parametrize("field, value", [("zero_point", 128), ("zero_point", -129),
                                          ("relu", 2), ("layout", 2), ("layout", -1)])
def test_requant_bad_arguments(field, value):
    shape = m.load_workloads()["cfg2_mid_3x3"]
    rq = _abi.CRequant(1 << 20, 1 << 20, 0, 0, 0)
    setattr(rq, field, value)
    assert _abi.lib.int8conv_launch_requant(*_launch_args(shape, rq)) == _abi.BAD_ARGUMENT


def test_requant_null_and_misaligned_parameters():
    shape = m.load_workloads()["cfg2_mid_3x3"]
    for mult, expo in ((None, 1 << 20), (1 << 20, None), ((1 << 20) + 4, 1 << 20)):
        rq = _abi.CRequant(mult, expo, 0, 0, 0)
        assert _abi.lib.int8conv_launch_requant(*_launch_args(shape, rq)) == _abi.BAD_POINTER
    args = list(_launch_args(shape, _abi.CRequant(1 << 20, 1 << 20, 0, 0, 0)))
    args[5] = None
    assert _abi.lib.int8conv_launch_requant(*args) == _abi.BAD_ARGUMENT


def test_vect_c_needs_k_multiple_of_32():
    shape = m.load_workloads()["cfg4c_tail_k100"]
    rq = _abi.CRequant(1 << 20, 1 << 20, 0, 0, _abi.LAYOUT_NCHW_VECT_C)
    assert _abi.lib.int8conv_launch_requant(*_launch_args(shape, rq)) == _abi.NOT_ELIGIBLE


# Ties at every exponent of the rounding divide.  With the multiplier 2^30 the
# doubling high multiply halves an even t exactly, so u = t / 2; the divide by
# 2^n then sees u = +-(2k+1) * 2^(n-1), exactly half way, and the published
# rule (gemmlowp RoundingDivideByPOT) rounds it away from zero to +-(k+1).
TIES = [(n, k, sign) for n in range(1, 31) for k in (0, 1, 2) for sign in (1, -1)
        if (2 * k + 1) * 2 ** n <= I32_MAX]


@pytest.mark.parametrize("n, k, sign", TIES)
def test_requant_ties_round_away_from_zero_at_every_exponent(n, k, sign):
    t = sign * (2 * k + 1) * 2 ** n
    want = sign * (k + 1)
    assert pyoracle.requant_value(t, Q30, -n, 0, 0) == want
    assert pyoracle.requant_value_py(t, Q30, -n, 0, 0) == want
    # one below the tie in magnitude rounds toward zero instead
    assert pyoracle.requant_value(t - sign * 2, Q30, -n, 0, 0) == sign * k


def known_answer_table():
    """(t, multiplier, exponent, zero_point, relu, want) rows derived by hand
    from the rule in include/int8conv.h; shared with the GPU test."""
    rows = [
        # doubling high multiply of INT32_MIN by itself saturates to INT32_MAX,
        # then / 2^31 rounds (2^31 - 1) / 2^31 up to 1
        (I32_MIN, I32_MIN, 0, 0, 0, 127), (I32_MIN, I32_MIN, -31, 0, 0, 1),
        (I32_MIN, I32_MIN, -31, -7, 0, -6),
        # saturating left shift: -3e8 * 8 is below INT32_MIN and saturates there
        # (a wrapping shift would give +1.89e9 and 127); * 0.5 -> -2^30 -> -128
        (-300000000, Q30, 3, 0, 0, -128), (300000000, Q30, 3, 0, 0, 127),
        # the left shift alone, inside int32: 40 * 2^2 * 0.5 = 80
        (40, Q30, 2, 0, 0, 80), (-40, Q30, 2, 0, 0, -80),
        # negative ties at exponent -1 .. -3 through a full multiplier
        (-6, Q30, -1, 0, 0, -2), (-12, Q30, -2, 0, 0, -2), (-24, Q30, -3, 0, 0, -2),
        (6, Q30, -1, 0, 0, 2), (12, Q30, -2, 0, 0, 2), (24, Q30, -3, 0, 0, 2),
        # ReLU clamps at the zero point, after the zero point is added
        (-6, Q30, -1, 5, 1, 5), (60, Q30, -1, 5, 1, 20),
    ]
    return rows


@pytest.mark.parametrize("row", known_answer_table())
def test_requant_published_rule_known_answers(row):
    t, mult, e, zp, relu, want = row
    assert pyoracle.requant_value(t, mult, e, zp, relu) == want
    assert pyoracle.requant_value_py(t, mult, e, zp, relu) == want
