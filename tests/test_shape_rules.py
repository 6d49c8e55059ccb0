"""Eligibility predicates and the workloads table (host only)."""
from pathlib import Path

import numpy as np
import pytest

import int8_kernel_lab_b200 as m

ROOT = Path(__file__).resolve().parent.parent


def reference_strip_predicate(s):
    # include/spatial_strip.cuh:11-15 of the reference.
    return (s.r == 3 and s.s == 3 and s.stride_w == 1 and s.dilation_w == 1 and s.c % 64 == 0
            and s.k % 64 == 0 and s.out_w % 128 == 0)


def test_workloads_table_has_reference_rows_and_baseline():
    table = m.load_workloads()
    ref = dict(m.shape.iter_reference_workloads())
    assert len(ref) == 41
    for name in m.BASELINE_CASES:
        assert name in table
    assert table["big_3x3_s1"] == m.ConvShape(16, 256, 256, 256, 256, 3, 3, 1, 1, 1, 1, 1, 1)


def test_every_workload_is_generic_eligible():
    for name, s in m.load_workloads().items():
        assert s.valid and s.eligible("generic"), name


def test_reference_strip_shapes_stay_strip_eligible():
    # Drop-in property: whatever the reference could run as strip, the B200
    # strip family accepts too (only big_3x3_s1 in the table).
    ref_strip = [n for n, s in m.load_workloads().items() if reference_strip_predicate(s)]
    assert ref_strip == ["big_3x3_s1"]
    for name in ref_strip:
        assert m.load_workloads()[name].eligible("strip")


@pytest.mark.parametrize("name,expect", [
    ("cfg2_mid_3x3", True), ("cfg5a_stress_3x3", True), ("cfg5c_1x7", True),
    ("cfg5b_dilated_3x3", False),   # dilation_w 2
    ("cfg3a_down_3x3_s2", False),   # stride_w 2
    ("cfg3b_pointwise", False),     # s == 1: nothing to reuse
])
def test_strip_predicate(name, expect):
    assert m.load_workloads()[name].eligible("strip") is expect


def test_ops_and_bytes_accounting():
    s = m.load_workloads()["cfg5a_stress_3x3"]
    assert s.ops == 2 * 256 * 56 * 56 * 256 * 256 * 9
    assert s.compulsory_bytes == (256 * 56 * 56 * 256 + 256 * 9 * 256 + 4 * 256
                                  + 4 * 256 * 56 * 56 * 256)


@pytest.mark.parametrize("name,expect", [
    ("cfg4b_small_3x3", True), ("cfg4c_tail_k100", True), ("cfg2_mid_3x3", True),
    ("cfg5b_dilated_3x3", True),    # dilation is a larger shift of the same tile
    ("cfg3a_down_3x3_s2", False),   # stride 2
    ("big_3x3_s1", False),          # 256-wide rows: the staged tile would exceed 512 pixels
])
def test_halo_predicate(name, expect):
    assert m.load_workloads()[name].eligible("halo") is expect


def test_splitk_needs_two_kblocks():
    assert not m.ConvShape(1, 8, 8, 32, 8, 1, 1).eligible("splitk")     # one k-block
    assert m.ConvShape(1, 8, 8, 256, 8, 1, 1).eligible("splitk")       # two 128-channel blocks
    assert m.ConvShape(1, 8, 8, 32, 8, 3, 3, 1, 1).eligible("splitk")  # nine taps


def test_dispatch_policy_on_baseline():
    want = {"cfg4b_small_3x3": "splitk", "cfg4c_tail_k100": "halo",
            "cfg5a_stress_3x3": "generic", "cfg5b_dilated_3x3": "generic",
            "cfg3b_pointwise": "generic"}
    table = m.load_workloads()
    for name, fam in want.items():
        assert table[name].select() == fam, name


def test_narrow_generic_tiles_take_the_small_odd_k_layer():
    # GENERIC runs narrow N tiles where its tiles fill less than one wave
    # and bn is not a multiple of 64 (int8conv_rules.h, i8c_generic_bn); of
    # the 51 workloads only 4c (K = 100, bn 112 -> four 32-column tiles)
    # qualifies.  There GENERIC beat SPLITK on B200 (13.4-13.8 against
    # 15.1-15.2 us per launch) and HALO, which stages each row tile's taps
    # once instead of once per narrow tile, beat GENERIC (6.1 against 7.0 us
    # per launch in graph replay), so such a layer runs HALO where HALO is
    # eligible and GENERIC elsewhere.
    # smoke (K = 32, nine k-blocks) takes GENERIC by the k-block threshold
    # of split-K instead (test_splitk_needs_ten_kblocks).
    table = m.load_workloads()
    small_odd = {name for name, s in table.items()
                 if s.select() in ("generic", "halo") and s.eligible("splitk") and s.k % 64 != 0
                 and (s.n * s.out_h * s.out_w + 127) // 128 < 148}
    assert small_odd == {"cfg4c_tail_k100", "smoke"}
    assert table["cfg4c_tail_k100"].select() == "halo"
    assert table["smoke"].select() == "generic"
    # Without HALO (a stride of 2) the same narrow-tile layer stays GENERIC.
    s = table["cfg4c_tail_k100"]
    strided = m.ConvShape(s.n, 2 * s.h, 2 * s.w, s.c, s.k, s.r, s.s, s.pad_h, s.pad_w, 2, 2)
    assert not strided.eligible("halo") and strided.select() == "generic"


def test_splitk_needs_ten_kblocks():
    # Split-K only with at least ten k-blocks (tap x channel block): with 8 or
    # 9, GENERIC's tail-balanced column parts were as fast or faster on B200
    # (darknet_res_13_reduce 13.6 vs 15.0 us, dilated_3x3 13.6 vs 15.0).
    table = m.load_workloads()
    for name in ("darknet_res_13_reduce", "darknet_detect_13_padded", "dilated_3x3",
                 "cfg1_smoke", "resnet_s3_3x3"):
        assert table[name].select() == "generic", name
    for name in ("cfg4a_deep_1x1", "cfg4b_small_3x3", "resnet_s5_3x3", "resnet_s4_down"):
        assert table[name].select() == "splitk", name


def test_dispatch_needs_a_single_wave_split():
    # Split-K only where its clusters fit in one wave of resident clusters
    # (B200: 74 pairs, 45 triples, ..., 15 clusters of 7 or 8).  batch8_3x3 has
    # 98 split tiles (two waves even as pairs) and lost to GENERIC 28.8 vs
    # 18.2 us; darknet_down_52 (24 tiles) fits as clusters of 5.
    table = m.load_workloads()
    assert table["batch8_3x3"].select() == "generic"
    for name in ("darknet_down_52", "cfg4a_deep_1x1", "darknet_head_13", "resnet_s4_3x3"):
        assert table[name].select() == "splitk", name


def test_channel_block_choices(tmp_path):
    # The k-block width each C gets (int8conv_rules.h, i8c_channel_block):
    # cheapest blocks x (width + 128-byte fixed cost), ties to less padding.
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no gcc")
    src = tmp_path / "cb.c"
    src.write_text('#include <stdio.h>\n#include "int8conv_rules.h"\n'
                   'int main(void){int cs[]={16,32,48,64,80,96,128,160,192,256,320,512};'
                   'for(int i=0;i<12;++i) printf("%d %d\\n", cs[i], i8c_channel_block(cs[i]));'
                   'return 0;}\n')
    exe = tmp_path / "cb"
    subprocess.run([gcc, "-std=c99", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)],
                   check=True)
    got = dict(tuple(map(int, line.split())) for line in
               subprocess.run([str(exe)], capture_output=True, text=True).stdout.split("\n") if line)
    assert got == {16: 32, 32: 32, 48: 64, 64: 64, 80: 128, 96: 128, 128: 128, 160: 128,
                   192: 128, 256: 128, 320: 128, 512: 128}


def test_tail_split_and_narrow_tile_rules(tmp_path):
    # int8conv_rules.h: i8c_pick_split (span model of the column parts) and
    # i8c_generic_bn (narrow N tiles for sub-wave layers whose BN tail
    # balancing cannot cut), compiled as C99 and evaluated on known cases.
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no gcc")
    src = tmp_path / "rules.c"
    src.write_text(
        '#include <stdio.h>\n#include "int8conv_rules.h"\n'
        'int main(void){\n'
        # (tiles, slots, bn) -> f
        ' printf("%d %d %d %d %d %d\\n", i8c_pick_split(25, 148, 128), i8c_pick_split(25, 148, 112),'
        ' i8c_pick_split(25, 148, 0), i8c_pick_split(296, 148, 256), i8c_pick_split(392, 74, 256),'
        ' i8c_pick_split(120, 148, 256));\n'
        # BN of GENERIC single CTAs on 148 SMs
        ' int8conv_shape c4 = {16, 14, 14, 48, 100, 3, 3, 1, 1, 1, 1, 1, 1};\n'
        ' int8conv_shape c2 = {32, 28, 28, 128, 128, 3, 3, 1, 1, 1, 1, 1, 1};\n'
        ' int8conv_shape s3 = {8, 14, 14, 128, 128, 3, 3, 1, 1, 1, 1, 1, 1};\n'
        ' int8conv_shape k300 = {1, 8, 8, 64, 300, 3, 3, 1, 1, 1, 1, 1, 1};\n'
        ' printf("%d %d %d %d %d\\n", i8c_generic_bn(&c4, 16, 148), i8c_generic_bn(&c2, 16, 148),'
        ' i8c_generic_bn(&s3, 16, 148), i8c_generic_bn(&c4, 16, 0), i8c_generic_bn(&k300, 16, 148));\n'
        ' printf("%d %d %d\\n", i8c_pick_bn(100, 16), i8c_pick_bn(100, 32), i8c_pick_bn(700, 16));\n'
        ' return 0;}\n')
    exe = tmp_path / "rules"
    subprocess.run([gcc, "-std=c99", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)],
                   check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True,
                           check=True).stdout.split("\n")
    # 25 tiles on 148 slots: quarters if BN allows (128), none for BN 112, the
    # model's own choice is quarters; full waves never split; 392 on 74 slots
    # leaves 22 in the last wave -> halves (span 5.7 tiles; quarters would
    # need two rounds of parts, 5.9); 120 tiles on 148 stay whole.
    assert list(map(int, lines[0].split())) == [4, 1, 4, 1, 2, 1]
    # 4c: 112 -> four 32-column tiles; cfg2 (196 tiles) and the 7-tile 14x14
    # layer (BN 128 splits into parts) keep their BN; no slots -> no change;
    # K = 300 on one row tile: BN 160 (two tiles) -> quarters of 40 -> 64.
    assert list(map(int, lines[1].split())) == [32, 128, 128, 112, 64]
    # K = 700: three equal tiles of ceil(700 / 3) = 234 -> 240 columns.
    assert list(map(int, lines[2].split())) == [112, 128, 240]


def im2col_encodable(s):
    """Restatement of i8c_im2col_ok (include/int8conv_rules.h): the TMA im2col
    tensor map's limits on pads, traversal strides, tap offsets and the
    bounding-box corners of a 4-D map."""
    def corner(extent, pad, stride, count):
        return -pad + (count - 1) * stride + 1 - extent
    return (s.valid and s.pad_h <= 127 and s.pad_w <= 127 and s.stride_h <= 8 and s.stride_w <= 8
            and (s.r - 1) * s.dilation_h <= 127 and (s.s - 1) * s.dilation_w <= 127
            and -128 <= corner(s.w, s.pad_w, s.stride_w, s.out_w) <= 127
            and -128 <= corner(s.h, s.pad_h, s.stride_h, s.out_h) <= 127)


# Shapes the reference's generic kernel computes (conv_shape.cuh:34-35 are its
# only conditions) that lie beyond the im2col map: patch embeds, strides past 8,
# a pad past 127, a tap span past 127.
BEYOND_IM2COL = {
    "patch16_s16": m.ConvShape(8, 224, 224, 16, 768, 16, 16, 0, 0, 16, 16, 1, 1),
    "patch32_s32": m.ConvShape(2, 448, 448, 16, 256, 32, 32, 0, 0, 32, 32, 1, 1),
    "stride9": m.ConvShape(2, 20, 20, 32, 16, 3, 3, 1, 1, 9, 9, 1, 1),
    "stride12": m.ConvShape(1, 25, 30, 16, 12, 2, 3, 0, 1, 12, 12, 1, 1),
    "pad130": m.ConvShape(1, 5, 5, 16, 8, 3, 3, 130, 130, 1, 1, 1, 1),
    "span140": m.ConvShape(1, 150, 145, 16, 8, 3, 2, 1, 1, 2, 2, 70, 140),
    # every parameter within its own limit, but the bounding box's upper
    # corner (1 - 135 = -134) is past the map's range
    "corner_only": m.ConvShape(1, 16, 135, 16, 8, 1, 2, 0, 0, 1, 8, 1, 127),
}


@pytest.mark.parametrize("name", sorted(BEYOND_IM2COL))
def test_generic_takes_shapes_beyond_the_im2col_map(name):
    s = BEYOND_IM2COL[name]
    assert s.valid and not im2col_encodable(s), name
    assert s.eligible("generic")
    for fam in ("strip", "halo", "splitk"):  # these stage through the im2col map
        assert not s.eligible(fam), (name, fam)
    assert s.select() == "generic"


def test_generic_eligible_is_shape_valid():
    # GENERIC computes every valid shape, as the reference's generic does.
    rng = np.random.RandomState(4)
    seen_beyond = 0
    for _ in range(3000):
        s = m.ConvShape(
            n=int(rng.randint(1, 5)), h=int(rng.randint(1, 300)), w=int(rng.randint(1, 300)),
            c=int(rng.choice([8, 16, 48, 64, 200, 256])), k=int(rng.randint(1, 900)),
            r=int(rng.randint(1, 40)), s=int(rng.randint(1, 40)),
            pad_h=int(rng.randint(0, 300)), pad_w=int(rng.randint(0, 300)),
            stride_h=int(rng.randint(1, 40)), stride_w=int(rng.randint(1, 40)),
            dilation_h=int(rng.randint(1, 20)), dilation_w=int(rng.randint(1, 20)))
        assert s.eligible("generic") == s.valid, s
        if s.valid:
            assert s.select() in ("generic", "splitk", "halo"), s
            if not im2col_encodable(s):
                seen_beyond += 1
                assert s.select() == "generic"
                assert not (s.eligible("strip") or s.eligible("halo") or s.eligible("splitk"))
    assert seen_beyond > 100
