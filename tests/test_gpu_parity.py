"""GPU parity: every family against the CPU oracle, bit-exact, through the C ABI.

Sizes are chosen so the oracle finishes in seconds; full-size BASELINE shapes
are checked on every output of a few whole images plus a seeded random sample
of all others (the oracle restates src/conv_lab.cu:39-66 of the reference).
"""
import numpy as np
import pytest

import pyoracle
from conftest import golden_cases, load_golden

import int8_kernel_lab_b200 as m
from int8_kernel_lab_b200 import _abi

pytestmark = pytest.mark.gpu

FAMILIES = ("generic", "strip", "halo", "splitk")


def _run(torch, strategy, shape, x, w, b):
    dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    dw = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    db = torch.from_numpy(np.ascontiguousarray(b)).cuda()
    # Poison the output so unwritten elements cannot pass by accident.
    dy = torch.full((shape.output_elements,), -123456789, dtype=torch.int32, device="cuda")
    nbytes = m.workspace_bytes(shape, strategy) if strategy != "auto" else 0
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda") if nbytes else None
    m.launch(strategy, shape, dx, dw, db, dy, workspace=ws, workspace_bytes=nbytes)
    assert m.device_status() == _abi.OK
    return dy.cpu().numpy()


def _families(shape):
    return [f for f in FAMILIES if shape.eligible(f)]


@pytest.fixture(params=["single", "pair"])
def pairing(request):
    # GENERIC and STRIP run as single CTAs (cta_group::1) or CTA pairs
    # (cta_group::2); both must give the oracle's integers.
    m.set_cta_pairing(request.param)
    yield request.param
    m.set_cta_pairing("auto")


@pytest.mark.parametrize("name", golden_cases())
def test_golden_fixtures_all_families(cuda, pairing, name):
    shape, x, w, b, y = load_golden(name)
    fams = _families(shape)
    assert "generic" in fams
    for fam in fams:
        got = _run(cuda, fam, shape, x, w, b)
        assert np.array_equal(got, y), f"{fam} differs from the reference on {name}"


def _reduced(shape, max_ops=3e10):
    if shape.ops <= max_ops:
        return shape
    return shape.with_batch(max(1, int(shape.n * max_ops / shape.ops)))


@pytest.mark.parametrize("case", m.BASELINE_CASES)
def test_baseline_configs_full_compare(cuda, pairing, case):
    shape = _reduced(m.load_workloads()[case])
    x, w, b = m.make_inputs(shape)
    want = pyoracle.conv(shape, x, w, b)
    for fam in _families(shape):
        got = _run(cuda, fam, shape, x, w, b)
        bad = np.count_nonzero(got != want)
        assert bad == 0, f"{fam} on {case} (n={shape.n}): {bad} mismatches"


def _sampled_check(shape, x, w, b, got, seed=7, samples=200_000, whole_images=(0, -1)):
    """Every output of the listed images plus a random sample of all outputs."""
    per_image = shape.out_h * shape.out_w
    for img in whole_images:
        img = img % shape.n
        rows = pyoracle.conv_rows(shape, x, w, b, img * per_image, (img + 1) * per_image)
        lo = img * per_image * shape.k
        assert np.array_equal(got[lo:lo + rows.size], rows), f"image {img} differs"
    rng = np.random.RandomState(seed)
    idx = rng.randint(0, shape.output_elements, size=min(samples, shape.output_elements))
    assert np.array_equal(got[idx], pyoracle.values(shape, x, w, b, idx))


@pytest.mark.parametrize("case", ["cfg5a_stress_3x3", "cfg5b_dilated_3x3", "cfg5c_1x7",
                                  "cfg2_mid_3x3", "cfg3b_pointwise"])
def test_baseline_full_size_sampled(cuda, case):
    shape = m.load_workloads()[case]
    x, w, b = m.make_inputs(shape)
    for fam in _families(shape):
        got = _run(cuda, fam, shape, x, w, b)
        _sampled_check(shape, x, w, b, got)


def test_families_agree_bitwise_full_size(cuda):
    # Size-independent property: every eligible family computes the same
    # integers (order of the int32 reduction cannot matter: no overflow).
    shape = m.load_workloads()["cfg5a_stress_3x3"]
    x, w, b = m.make_inputs(shape, seed=99)
    fams = _families(shape)
    outs = [_run(cuda, f, shape, x, w, b) for f in fams]
    for f, o in zip(fams[1:], outs[1:]):
        assert np.array_equal(o, outs[0]), f"{f} != {fams[0]}"


def test_linearity_in_bias(cuda):
    # y(b + d) - y(b) == d broadcast over channels, at full size.
    shape = m.load_workloads()["cfg5b_dilated_3x3"]
    x, w, b = m.make_inputs(shape, seed=5)
    y0 = _run(cuda, "auto", shape, x, w, b).reshape(-1, shape.k)
    d = np.arange(shape.k, dtype=np.int32) * 7 - 300
    y1 = _run(cuda, "auto", shape, x, w, b + d).reshape(-1, shape.k)
    assert np.array_equal(y1 - y0, np.broadcast_to(d, y0.shape))


REFERENCE_WORKLOADS = [name for name, _ in m.shape.iter_reference_workloads()]


@pytest.mark.parametrize("name", REFERENCE_WORKLOADS)
def test_reference_workloads(cuda, name):
    shape = m.load_workloads()[name]
    x, w, b = m.make_inputs(shape, values="full")
    small = _reduced(shape, 2e9)
    for fam in _families(shape):
        if small is shape:
            got = _run(cuda, fam, shape, x, w, b)
            assert np.array_equal(got, pyoracle.conv(shape, x, w, b)), fam
        else:
            got = _run(cuda, fam, shape, x, w, b)
            _sampled_check(shape, x, w, b, got, samples=50_000, whole_images=(0,))


def _random_wide_shapes(count, seed=77):
    """Wider parameters: pads to 7, strides to 8, dilations to 6, taps to
    11 x 11, C to 512, K to 700 (kept to oracle-friendly sizes)."""
    rng = np.random.RandomState(seed)
    out = []
    while len(out) < count:
        sh = m.ConvShape(
            n=int(rng.randint(1, 3)), h=int(rng.randint(4, 48)), w=int(rng.randint(4, 48)),
            c=int(16 * rng.randint(1, 33)), k=int(rng.randint(1, 701)),
            r=int(rng.randint(1, 12)), s=int(rng.randint(1, 12)),
            pad_h=int(rng.randint(0, 8)), pad_w=int(rng.randint(0, 8)),
            stride_h=int(rng.randint(1, 9)), stride_w=int(rng.randint(1, 9)),
            dilation_h=int(rng.randint(1, 7)), dilation_w=int(rng.randint(1, 7)))
        if sh.valid and sh.eligible("generic") and sh.ops <= 4e9:
            out.append(sh)
    return out


WIDE_SHAPES = _random_wide_shapes(24)


@pytest.mark.parametrize("idx", range(len(WIDE_SHAPES)))
def test_random_wide_shapes(cuda, idx):
    shape = WIDE_SHAPES[idx]
    x, w, b = m.make_inputs(shape, seed=100 + idx)
    want = pyoracle.conv(shape, x, w, b)
    for fam in _families(shape):
        got = _run(cuda, fam, shape, x, w, b)
        bad = np.count_nonzero(got != want)
        assert bad == 0, f"{fam} on {shape}: {bad} mismatches"
    # The int8 epilogue on the same shape, in each layout it allows.
    rng = np.random.RandomState(idx)
    mult = rng.randint(1 << 30, (1 << 31) - 1, shape.k, dtype=np.int64).astype(np.int32)
    expo = rng.randint(-14, -4, shape.k).astype(np.int32)
    dev = [cuda.from_numpy(a).cuda() for a in (x, w, b, mult, expo)]
    for layout in ["nhwc"] + (["nchw_vect_c"] if shape.k % 32 == 0 else []):
        y8 = cuda.zeros(shape.output_elements, dtype=cuda.int8, device="cuda")
        m.launch_requant("auto", shape, *dev, y8, zero_point=4, relu=True, layout=layout)
        assert m.device_status() == _abi.OK
        want8 = pyoracle.requant(want, shape.k, mult, expo, zero_point=4, relu=True)
        if layout == "nchw_vect_c":
            want8 = pyoracle.to_nchw_vect_c(want8, shape.n, shape.out_h, shape.out_w, shape.k)
        assert np.array_equal(y8.cpu().numpy(), want8), f"requant {layout} on {shape}"


def _random_shapes(count, seed=2026):
    rng = np.random.RandomState(seed)
    out = []
    while len(out) < count:
        r, s = rng.randint(1, 6), rng.randint(1, 6)
        sh = m.ConvShape(
            n=int(rng.randint(1, 4)), h=int(rng.randint(1, 24)), w=int(rng.randint(1, 24)),
            c=int(16 * rng.randint(1, 12)), k=int(rng.randint(1, 300)), r=int(r), s=int(s),
            pad_h=int(rng.randint(0, 3)), pad_w=int(rng.randint(0, 3)),
            stride_h=int(rng.randint(1, 4)), stride_w=int(rng.randint(1, 4)),
            dilation_h=int(rng.randint(1, 3)), dilation_w=int(rng.randint(1, 3)))
        if sh.valid and sh.eligible("generic"):
            out.append(sh)
    return out


@pytest.mark.parametrize("idx,shape", list(enumerate(_random_shapes(40))))
def test_random_shapes(cuda, pairing, idx, shape):
    x, w, b = m.make_inputs(shape, seed=idx)
    want = pyoracle.conv(shape, x, w, b)
    for fam in _families(shape):
        got = _run(cuda, fam, shape, x, w, b)
        assert np.array_equal(got, want), f"{fam} on {shape}"


def test_reference_value_range(cuda):
    # The reference's own value distribution ([-4,4], bias [-31,31]).
    shape = m.load_workloads()["resnet_s3_3x3"]
    x, w, b = m.make_inputs(shape, values="reference")
    got = _run(cuda, "auto", shape, x, w, b)
    assert np.array_equal(got, pyoracle.conv(shape, x, w, b))


def test_stream_argument_and_async(cuda):
    torch = cuda
    shape = m.load_workloads()["cfg2_mid_3x3"]
    x, w, b = m.make_inputs(shape)
    dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
    dy = torch.zeros(shape.output_elements, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # the buffers' copies and fill
    with torch.cuda.stream(s):
        m.launch_generic(shape, dx, dw, db, dy, stream=s)
    s.synchronize()
    assert np.array_equal(dy.cpu().numpy(), pyoracle.conv(shape, x, w, b))


def test_ineligible_and_bad_pointer_statuses(cuda):
    torch = cuda
    shape = m.load_workloads()["cfg3a_down_3x3_s2"]  # stride 2: strip-ineligible
    assert not shape.eligible("strip")
    x = torch.zeros(shape.input_elements, dtype=torch.int8, device="cuda")
    w = torch.zeros(shape.filter_elements, dtype=torch.int8, device="cuda")
    b = torch.zeros(shape.k, dtype=torch.int32, device="cuda")
    y = torch.zeros(shape.output_elements, dtype=torch.int32, device="cuda")
    with pytest.raises(m.Int8ConvError) as err:
        m.launch_spatial_strip(shape, x, w, b, y)
    assert err.value.status == _abi.NOT_ELIGIBLE
    st = _abi.lib.int8conv_launch_generic(shape.c_struct(), x.data_ptr() + 1, w.data_ptr(),
                                          b.data_ptr(), y.data_ptr(), None)
    assert st == _abi.BAD_POINTER


def test_device_wait_timeout_is_reported_and_context_survives(cuda, pairing):
    # Failure detection without a GPU fault: the producer is told to issue no
    # copies, every consumer wait runs out after 20 ms, the kernel unwinds
    # (TMEM released, nothing in flight) and the host reads DEVICE_TIMEOUT.
    torch = cuda
    shape = m.load_workloads()["cfg1_smoke"]
    x, w, b = m.make_inputs(shape)
    dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
    dy = torch.zeros(shape.output_elements, dtype=torch.int32, device="cuda")
    m.set_wait_limit_ns(20_000_000)
    m.debug_starve_producer(True)
    try:
        m.launch("generic", shape, dx, dw, db, dy)
        assert m.device_status() == _abi.DEVICE_TIMEOUT
    finally:
        m.debug_starve_producer(False)
        m.set_wait_limit_ns(0)
    assert m.device_status() == _abi.OK  # flag cleared
    m.launch("generic", shape, dx, dw, db, dy)
    assert m.device_status() == _abi.OK
    assert np.array_equal(dy.cpu().numpy(), pyoracle.conv(shape, x, w, b))


@pytest.mark.parametrize("family", ["generic", "splitk"])
def test_cached_plan_replays_and_follows_run_controls(cuda, family):
    # A repeated launch (same shape, buffers, family, pairing) replays the
    # thread's cached launch plan.  The replay must give the same integers,
    # honour the starve hook and wait limit set since it was cached, and keep
    # working after they are cleared.
    torch = cuda
    shape = m.load_workloads()["cfg4b_small_3x3"]
    x, w, b = m.make_inputs(shape, seed=11)
    dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
    dy = torch.zeros(shape.output_elements, dtype=torch.int32, device="cuda")
    want = pyoracle.conv(shape, x, w, b)
    for _ in range(3):
        dy.zero_()
        m.launch(family, shape, dx, dw, db, dy)
        assert m.device_status() == _abi.OK
        assert np.array_equal(dy.cpu().numpy(), want)
    m.set_wait_limit_ns(20_000_000)
    m.debug_starve_producer(True)
    try:
        m.launch(family, shape, dx, dw, db, dy)
        assert m.device_status() == _abi.DEVICE_TIMEOUT
    finally:
        m.debug_starve_producer(False)
        m.set_wait_limit_ns(0)
    dy.zero_()
    m.launch(family, shape, dx, dw, db, dy)
    assert m.device_status() == _abi.OK
    assert np.array_equal(dy.cpu().numpy(), want)
    # Other buffers with the same shape: a different plan, not the cached one.
    dy2 = torch.zeros_like(dy)
    m.launch(family, shape, dx, dw, db, dy2)
    assert m.device_status() == _abi.OK
    assert np.array_equal(dy2.cpu().numpy(), want)


@pytest.mark.parametrize("chunks", [1, 3, 64])
def test_host_buffer_pipeline(cuda, chunks):
    # int8conv_launch_host: pinned host buffers in, host output back, with the
    # copies of image groups overlapped with the kernels.
    torch = cuda
    shape = m.load_workloads()["cfg2_mid_3x3"].with_batch(7)
    x, w, b = m.make_inputs(shape, seed=3)
    hx = torch.from_numpy(x).pin_memory()
    hw = torch.from_numpy(w).pin_memory()
    hb = torch.from_numpy(b).pin_memory()
    hy = torch.full((shape.output_elements,), -1, dtype=torch.int32).pin_memory()
    dx = torch.empty(shape.input_elements, dtype=torch.int8, device="cuda")
    dw = torch.empty(shape.filter_elements, dtype=torch.int8, device="cuda")
    db = torch.empty(shape.k, dtype=torch.int32, device="cuda")
    dy = torch.empty(shape.output_elements, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    m.launch_host("auto", shape, hx, hw, hb, hy, dx, dw, db, dy, chunks=chunks, stream=s)
    s.synchronize()
    assert m.device_status() == _abi.OK
    assert np.array_equal(hy.numpy(), pyoracle.conv(shape, x, w, b))


@pytest.mark.parametrize("chunks", [2, 3, 5])
def test_host_buffer_pipeline_unaligned_image_outputs(cuda, chunks):
    # out_h*out_w*K odd (7 x 7 output, K = 63): an image's output is not a
    # whole number of 16-byte groups, so group boundaries must fall on every
    # fourth image for the kernels' 16-byte alignment rule.
    torch = cuda
    shape = m.ConvShape(9, 7, 7, 32, 63, 3, 3, 1, 1, 1, 1, 1, 1)
    x, w, b = m.make_inputs(shape, seed=chunks)
    hx, hw, hb = (torch.from_numpy(a).pin_memory() for a in (x, w, b))
    hy = torch.full((shape.output_elements,), -1, dtype=torch.int32).pin_memory()
    dx = torch.empty(shape.input_elements, dtype=torch.int8, device="cuda")
    dw = torch.empty(shape.filter_elements, dtype=torch.int8, device="cuda")
    db = torch.empty(shape.k, dtype=torch.int32, device="cuda")
    dy = torch.empty(shape.output_elements, dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    for strategy in ("auto", "generic", "splitk"):
        hy.fill_(-1)
        m.launch_host(strategy, shape, hx, hw, hb, hy, dx, dw, db, dy, chunks=chunks, stream=s)
        s.synchronize()
        assert m.device_status() == _abi.OK
        assert np.array_equal(hy.numpy(), pyoracle.conv(shape, x, w, b)), strategy


def test_output_beyond_2g_elements(cuda):
    # Maximum-size indexing: 2^21 output rows x 1040 channels = 2.18e9 int32
    # outputs (8.7 GB), past 2^31 elements, with five 208-wide N tiles.  The
    # first and last output rows and a seeded sample are checked.
    torch = cuda
    shape = m.ConvShape(2, 1024, 1024, 16, 1040, 3, 3, 1, 1, 1, 1, 1, 1)
    assert shape.output_elements > (1 << 31)
    x, w, b = m.make_inputs(shape, seed=17)
    dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
    dy = torch.empty(shape.output_elements, dtype=torch.int32, device="cuda")
    rng = np.random.RandomState(5)
    rows = shape.n * shape.out_h * shape.out_w
    idx = np.concatenate([np.arange(shape.k), (rows - 1) * shape.k + np.arange(shape.k),
                          rng.randint(0, shape.output_elements, 100_000, dtype=np.int64)])
    want = pyoracle.values(shape, x, w, b, idx)
    for fam in ("generic", "auto"):
        dy.fill_(-7)
        m.launch(fam, shape, dx, dw, db, dy)
        assert m.device_status() == _abi.OK
        got = dy[torch.from_numpy(idx).cuda()].cpu().numpy()
        assert np.array_equal(got, want), f"{fam}: {np.count_nonzero(got != want)} mismatches"
    del dy
    torch.cuda.empty_cache()


GUARD_BYTES = 4096


@pytest.mark.parametrize("name", ["cfg4c_tail_k100", "nonmultiple8_k63", "cfg1_smoke", "k288",
                                  "cfg2_n3"])
def test_no_writes_outside_the_output(cuda, pairing, name):
    # Stand-in for a sanitizer (closed on this pool): the output sits between
    # two poisoned 4 KB guard bands, and no family may touch them.
    torch = cuda
    table = m.load_workloads()
    shape = {"k288": m.ConvShape(2, 14, 14, 64, 288, 3, 3, 1, 1, 1, 1, 1, 1),
             "cfg2_n3": table["cfg2_mid_3x3"].with_batch(3)}.get(name) or table[name]
    x, w, b = m.make_inputs(shape, seed=29)
    dx, dw, db = (torch.from_numpy(a).cuda() for a in (x, w, b))
    g = GUARD_BYTES // 4
    want = pyoracle.conv(shape, x, w, b)
    for fam in _families(shape):
        buf = torch.full((shape.output_elements + 2 * g,), 0x5A5A5A5A, dtype=torch.int32,
                         device="cuda")
        m.launch(fam, shape, dx, dw, db, buf[g:g + shape.output_elements])
        assert m.device_status() == _abi.OK
        host = buf.cpu().numpy()
        assert np.all(host[:g] == 0x5A5A5A5A), f"{fam} wrote before the output"
        assert np.all(host[g + shape.output_elements:] == 0x5A5A5A5A), f"{fam} wrote past it"
        assert np.array_equal(host[g:g + shape.output_elements], want), fam


# STRIP's int32 epilogue stores each block of 32 padded positions as its valid
# rows, compacted, through the output map whose box has that many rows; the
# planner counts the dropped positions per block in closed form when a row
# has at least 32 outputs and by scanning the block starts otherwise, and
# falls back to 16-byte stores when more than eight maps would be needed or
# a block (the grid's tail) holds fewer valid rows than any map.
STRIP_STORE_SHAPES = {
    "closed_form_q40": m.ConvShape(3, 9, 40, 32, 64, 3, 3, 1, 1),      # Q = 40, 2 dropped per row
    "scan_q20": m.ConvShape(5, 7, 20, 32, 96, 3, 3, 1, 1),            # Q = 20, Wp = 22
    "fallback_q12_s5": m.ConvShape(4, 6, 12, 32, 64, 5, 5, 2, 2),     # Wp = 16: 8 dropped of 32
    "tail_q33_k36": m.ConvShape(1, 5, 33, 48, 36, 3, 3, 1, 1),        # Mp not a multiple of 32
    "wide_q70_s7": m.ConvShape(2, 4, 70, 16, 128, 1, 7, 0, 3),        # 6 dropped per row
}


@pytest.mark.parametrize("name", sorted(STRIP_STORE_SHAPES))
def test_strip_compacted_stores(cuda, pairing, name):
    shape = STRIP_STORE_SHAPES[name]
    assert shape.eligible("strip"), name
    x, w, b = m.make_inputs(shape)
    want = pyoracle.conv(shape, x, w, b)
    got = _run(cuda, "strip", shape, x, w, b)
    assert np.array_equal(got, want), f"strip differs from the oracle on {name}"
