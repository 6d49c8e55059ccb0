"""GPU parity of GENERIC's gather staging, bit-exact against the CPU oracle.

The reference's generic kernel computes every shape with c % 16 == 0 and a
non-empty output: its gather (generic_implicit_gemm.cuh:46-69 of the reference)
takes any stride, pad and dilation.  Shapes beyond the TMA im2col map
(stride > 8, pad > 127, (R-1)*dilation > 127, a bounding-box corner out of
range) run GENERIC with a gather warp staging the same swizzled tiles.  These
tests cover those shapes (golden fixtures produced by the reference's own
reference_value, seeded random shapes, realistic patch embeds) and, with the
gather forced on every shape, cross-check it against the im2col staging.
"""
import numpy as np
import pytest

import pyoracle
from conftest import load_golden
from test_shape_rules import BEYOND_IM2COL, im2col_encodable

import int8_kernel_lab_b200 as m
from int8_kernel_lab_b200 import _abi

pytestmark = pytest.mark.gpu

GATHER_GOLDENS = ["g_patch16_s16", "g_patch32_s32", "g_stride9", "g_stride12", "g_pad130",
                  "g_span140", "g_gather_c48_k100"]


@pytest.fixture
def forced_gather():
    m.set_generic_staging("gather")
    yield
    m.set_generic_staging("auto")


def _dev(torch, *arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrays]


def _run(torch, strategy, shape, x, w, b):
    dx, dw, db = _dev(torch, x, w, b)
    dy = torch.full((shape.output_elements,), -123456789, dtype=torch.int32, device="cuda")
    m.launch(strategy, shape, dx, dw, db, dy)
    assert m.device_status() == _abi.OK
    return dy.cpu().numpy()


@pytest.mark.parametrize("name", GATHER_GOLDENS)
def test_gather_goldens_generic_and_auto(cuda, name):
    shape, x, w, b, y = load_golden(name)
    assert not im2col_encodable(shape), name
    for strategy in ("generic", "auto"):
        got = _run(cuda, strategy, shape, x, w, b)
        bad = np.count_nonzero(got != y)
        assert bad == 0, f"{strategy} on {name}: {bad} outputs differ from the reference"


def test_every_golden_with_forced_gather(cuda, forced_gather):
    from conftest import golden_cases

    for name in golden_cases():
        shape, x, w, b, y = load_golden(name)
        got = _run(cuda, "generic", shape, x, w, b)
        assert np.array_equal(got, y), f"gather staging differs from the reference on {name}"


def _beyond_shapes(count, seed=909):
    """Seeded shapes past the im2col limits: strides to 24, pads to 200,
    dilations to 70, taps to 33, ragged C and K, several images."""
    rng = np.random.RandomState(seed)
    out = []
    while len(out) < count:
        sh = m.ConvShape(
            n=int(rng.randint(1, 4)), h=int(rng.randint(1, 90)), w=int(rng.randint(1, 90)),
            c=int(16 * rng.randint(1, 20)), k=int(rng.randint(1, 400)),
            r=int(rng.randint(1, 34)), s=int(rng.randint(1, 34)),
            pad_h=int(rng.choice([0, 1, 3, 40, 130, 200])),
            pad_w=int(rng.choice([0, 2, 5, 64, 128, 160])),
            stride_h=int(rng.randint(1, 25)), stride_w=int(rng.randint(1, 25)),
            dilation_h=int(rng.randint(1, 8)), dilation_w=int(rng.randint(1, 8)))
        if sh.valid and not im2col_encodable(sh) and sh.ops <= 3e9 and sh.output_elements <= 4e6:
            out.append(sh)
    return out


BEYOND = _beyond_shapes(30)


@pytest.mark.parametrize("idx", range(len(BEYOND)))
def test_random_shapes_beyond_im2col(cuda, idx):
    shape = BEYOND[idx]
    x, w, b = m.make_inputs(shape, seed=300 + idx)
    want = pyoracle.conv(shape, x, w, b)
    for strategy in ("generic", "auto"):
        got = _run(cuda, strategy, shape, x, w, b)
        bad = np.count_nonzero(got != want)
        assert bad == 0, f"{strategy} on {shape}: {bad} mismatches"
    # The int8 epilogue through the gather staging, in each layout it allows.
    rng = np.random.RandomState(idx)
    mult = rng.randint(1 << 30, (1 << 31) - 1, shape.k, dtype=np.int64).astype(np.int32)
    expo = rng.randint(-14, -4, shape.k).astype(np.int32)
    dev = _dev(cuda, x, w, b, mult, expo)
    for layout in ["nhwc"] + (["nchw_vect_c"] if shape.k % 32 == 0 else []):
        y8 = cuda.zeros(shape.output_elements, dtype=cuda.int8, device="cuda")
        m.launch_requant("generic", shape, *dev, y8, zero_point=-3, relu=bool(idx % 2),
                         layout=layout)
        assert m.device_status() == _abi.OK
        want8 = pyoracle.requant(want, shape.k, mult, expo, zero_point=-3, relu=bool(idx % 2))
        if layout == "nchw_vect_c":
            want8 = pyoracle.to_nchw_vect_c(want8, shape.n, shape.out_h, shape.out_w, shape.k)
        assert np.array_equal(y8.cpu().numpy(), want8), f"requant {layout} on {shape}"


@pytest.mark.parametrize("name", sorted(BEYOND_IM2COL))
def test_named_shapes_beyond_im2col(cuda, name):
    # Realistic sizes (ViT-B/16 patch embed on 8 images: 9.9 Gop; a 32 x 32
    # stride-32 embed; pad 130; tap span 140; a corner-only case): every
    # output of the first and last image plus a seeded sample.
    shape = BEYOND_IM2COL[name]
    x, w, b = m.make_inputs(shape, seed=41)
    got = _run(cuda, "auto", shape, x, w, b)
    per_image = shape.out_h * shape.out_w
    for img in (0, shape.n - 1):
        rows = pyoracle.conv_rows(shape, x, w, b, img * per_image, (img + 1) * per_image)
        lo = img * per_image * shape.k
        assert np.array_equal(got[lo:lo + rows.size], rows), f"{name}: image {img} differs"
    rng = np.random.RandomState(3)
    idx = rng.randint(0, shape.output_elements, size=min(100_000, shape.output_elements))
    assert np.array_equal(got[idx], pyoracle.values(shape, x, w, b, idx)), name


@pytest.mark.parametrize("case", ["cfg5a_stress_3x3", "cfg5c_1x7", "cfg4c_tail_k100",
                                  "cfg3a_down_3x3_s2", "cfg5b_dilated_3x3"])
def test_forced_gather_matches_im2col_staging(cuda, case):
    # Size-independent property at full BASELINE size: the two stagings of
    # GENERIC (im2col tensor map, gather warp) give the same integers, and
    # the gather's result matches the oracle on a sample.
    shape = m.load_workloads()[case]
    x, w, b = m.make_inputs(shape, seed=8)
    m.set_cta_pairing("single")
    try:
        tma = _run(cuda, "generic", shape, x, w, b)
        m.set_generic_staging("gather")
        gathered = _run(cuda, "generic", shape, x, w, b)
    finally:
        m.set_generic_staging("auto")
        m.set_cta_pairing("auto")
    assert np.array_equal(gathered, tma), case
    rng = np.random.RandomState(1)
    idx = rng.randint(0, shape.output_elements, size=50_000)
    assert np.array_equal(gathered[idx], pyoracle.values(shape, x, w, b, idx)), case


GUARD_WORDS = 1024


@pytest.mark.parametrize("shape", [
    m.ConvShape(3, 40, 40, 48, 100, 5, 5, 3, 3, 9, 9, 2, 2),     # K % 4 == 0: TMA stores
    m.ConvShape(2, 33, 35, 32, 63, 4, 3, 130, 2, 11, 10, 1, 1),  # odd K: row-segment stores
], ids=["k100", "k63"])
def test_gather_writes_nothing_outside_the_output(cuda, shape):
    torch = cuda
    assert not im2col_encodable(shape)
    x, w, b = m.make_inputs(shape, seed=12)
    dx, dw, db = _dev(torch, x, w, b)
    g = GUARD_WORDS
    buf = torch.full((shape.output_elements + 2 * g,), 0x5A5A5A5A, dtype=torch.int32,
                     device="cuda")
    m.launch("generic", shape, dx, dw, db, buf[g:g + shape.output_elements])
    assert m.device_status() == _abi.OK
    host = buf.cpu().numpy()
    assert np.all(host[:g] == 0x5A5A5A5A) and np.all(host[-g:] == 0x5A5A5A5A)
    assert np.array_equal(host[g:-g], pyoracle.conv(shape, x, w, b))


def test_gather_wait_timeout_is_reported_and_context_survives(cuda):
    # The starve hook in the gather staging: no copies and no arrivals, every
    # consumer wait runs out, the kernel unwinds, the host reads the status.
    torch = cuda
    shape = BEYOND_IM2COL["stride9"]
    x, w, b = m.make_inputs(shape, seed=2)
    dx, dw, db = _dev(torch, x, w, b)
    dy = torch.zeros(shape.output_elements, dtype=torch.int32, device="cuda")
    m.set_wait_limit_ns(20_000_000)
    m.debug_starve_producer(True)
    try:
        m.launch("generic", shape, dx, dw, db, dy)
        assert m.device_status() == _abi.DEVICE_TIMEOUT
    finally:
        m.debug_starve_producer(False)
        m.set_wait_limit_ns(0)
    assert m.device_status() == _abi.OK
    m.launch("generic", shape, dx, dw, db, dy)
    assert m.device_status() == _abi.OK
    assert np.array_equal(dy.cpu().numpy(), pyoracle.conv(shape, x, w, b))


def test_gather_through_host_buffers(cuda):
    torch = cuda
    shape = m.ConvShape(6, 64, 64, 32, 96, 16, 16, 0, 0, 16, 16, 1, 1)
    x, w, b = m.make_inputs(shape, seed=6)
    hx, hw, hb = (torch.from_numpy(a).pin_memory() for a in (x, w, b))
    hy = torch.full((shape.output_elements,), -1, dtype=torch.int32).pin_memory()
    dx = torch.empty(shape.input_elements, dtype=torch.int8, device="cuda")
    dw = torch.empty(shape.filter_elements, dtype=torch.int8, device="cuda")
    db = torch.empty(shape.k, dtype=torch.int32, device="cuda")
    dy = torch.empty(shape.output_elements, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    m.launch_host("auto", shape, hx, hw, hb, hy, dx, dw, db, dy, chunks=3, stream=s)
    s.synchronize()
    assert m.device_status() == _abi.OK
    assert np.array_equal(hy.numpy(), pyoracle.conv(shape, x, w, b))


def _channel_block(c):
    """Host copy of i8c_channel_block (include/int8conv_rules.h)."""
    best, best_cost, best_pad = 32, -1, 0
    cb = 128
    while cb >= 32:
        blocks = -(-c // cb)
        cost, pad = blocks * (cb + 128), blocks * cb - c
        if best_cost < 0 or cost < best_cost or (cost == best_cost and pad < best_pad):
            best, best_cost, best_pad = cb, cost, pad
        cb //= 2
    return best


def _stages_filter_rows(shape):
    """True where the gather stages 128-byte k-blocks of a filter row's S*C
    span instead of per-tap channel blocks (unit horizontal dilation, no more
    bytes staged than per-tap blocks)."""
    cb = _channel_block(shape.c)
    rows = shape.r * -(-(shape.s * shape.c) // 128) * 128
    taps = shape.r * shape.s * -(-shape.c // cb) * cb
    return shape.dilation_w == 1 and rows <= taps


ROW_BLOCK_SHAPES = {
    # S*C = 80: one 128-byte block per filter row, 48 bytes of it past the row.
    "c16_5x5": m.ConvShape(4, 30, 31, 16, 72, 5, 5, 2, 2, 1, 1, 1, 1),
    # S*C = 336: three blocks per row, the last one ragged; vertical dilation.
    "c48_7x7_dh2": m.ConvShape(2, 41, 37, 48, 100, 7, 7, 5, 3, 2, 1, 2, 1),
    # S*C = 240 with C = 80 (32-byte channel blocks per tap would pad to 96).
    "c80_3x3": m.ConvShape(3, 19, 23, 80, 63, 3, 3, 1, 1, 1, 1, 1, 1),
    # Patch embed, S*C = 256: two full blocks per row.
    "patch16_c16": m.ConvShape(3, 96, 80, 16, 192, 16, 16, 0, 0, 16, 16, 1, 1),
    # Taps straddle the right edge and the padding on both sides.
    "c16_11x11_s9": m.ConvShape(2, 50, 47, 16, 40, 11, 11, 6, 9, 9, 9, 1, 1),
}


@pytest.mark.parametrize("name", sorted(ROW_BLOCK_SHAPES))
def test_filter_row_blocks_match_oracle(cuda, forced_gather, name):
    shape = ROW_BLOCK_SHAPES[name]
    assert _stages_filter_rows(shape), name
    x, w, b = m.make_inputs(shape, seed=71)
    want = pyoracle.conv(shape, x, w, b)
    got = _run(cuda, "generic", shape, x, w, b)
    bad = np.count_nonzero(got != want)
    assert bad == 0, f"{name}: {bad} mismatches"
