"""sweep.py: the reference's flags and merge columns (scripts/sweep.py:10-66).

conv_lab is replaced by a stub script that prints one CSV row, so these tests
check the driver's host logic without a GPU.
"""
import csv
import stat

import pytest

from int8_kernel_lab_b200 import sweep

STUB = """#!/bin/sh
case_name=""
while [ $# -gt 0 ]; do
  if [ "$1" = "--case" ]; then case_name="$2"; fi
  shift
done
echo "case,generic_ms,strip_ms,halo_ms,splitk_ms,winner,selected"
if [ "$case_name" = "smoke" ]; then
  echo "smoke,0.02,0.03,-1,0.01,splitk,splitk"
else
  echo "$case_name,0.05,-1,0.07,-1,generic,generic"
fi
"""


@pytest.fixture
def stub(tmp_path):
    path = tmp_path / "conv_lab_stub"
    path.write_text(STUB)
    path.chmod(path.stat().st_mode | stat.S_IEXEC)
    return path


def read(path):
    with open(path, newline="") as stream:
        return list(csv.DictReader(stream))


def test_rows_follow_requested_cases(stub, tmp_path):
    out = tmp_path / "m.csv"
    assert sweep.main(["--cases", "smoke,cfg2_mid_3x3", "--output", str(out),
                       "--conv-lab", str(stub)]) == 0
    rows = read(out)
    assert [r["case"] for r in rows] == ["smoke", "cfg2_mid_3x3"]
    assert "cudnn_ms" not in rows[0]


def test_with_cudnn_keeps_merge_columns(stub, tmp_path):
    out = tmp_path / "m.csv"
    sweep.main(["--cases", "smoke,cfg2_mid_3x3", "--output", str(out), "--conv-lab", str(stub),
                "--with-cudnn"])
    rows = read(out)
    # The winner's time, for families the reference's mapping did not know.
    assert rows[0]["dispatch_ms"] == "0.01" and rows[1]["dispatch_ms"] == "0.05"
    assert all(r["comparison_contract"] == "cudnn_not_built" and r["cudnn_ms"] == ""
               for r in rows)


def test_unknown_case_and_arch_are_errors(stub, tmp_path):
    with pytest.raises(SystemExit, match="unknown cases"):
        sweep.main(["--cases", "smoke,nope", "--output", str(tmp_path / "m.csv"),
                    "--conv-lab", str(stub)])
    with pytest.raises(SystemExit, match="sm_100a"):
        sweep.main(["--arch", "sm_75", "--output", str(tmp_path / "m.csv"),
                    "--conv-lab", str(stub)])


def test_default_is_every_workload(stub, tmp_path):
    out = tmp_path / "m.csv"
    sweep.main(["--output", str(out), "--conv-lab", str(stub)])
    rows = read(out)
    assert len(rows) == 51 and rows[0]["case"] == "smoke" and rows[-1]["case"] == "cfg5c_1x7"


# A stub whose timings change with each call: calls are counted in a file
# next to it, so interleaving and averaging can be checked.
COUNTING_STUB = """#!/bin/sh
here=$(dirname "$0")
n=$(cat "$here/calls" 2>/dev/null || echo 0)
n=$((n + 1))
echo $n > "$here/calls"
echo "$n" >> "$here/order"
case_name=""
while [ $# -gt 0 ]; do
  if [ "$1" = "--case" ]; then case_name="$2"; fi
  shift
done
echo "$case_name" >> "$here/order"
echo "case,generic_ms,strip_ms,halo_ms,splitk_ms,winner,generic_correct,strip_correct,halo_correct,splitk_correct,tops,roofline_frac,graph_ms,selected"
if [ $((n % 2)) -eq 1 ]; then
  echo "$case_name,0.020,-1,0.030,0.018,splitk,1,1,1,1,10,0.5,0.006,splitk"
else
  echo "$case_name,0.016,-1,0.030,0.022,generic,1,1,1,0,12.5,0.625,0.004,splitk"
fi
"""


@pytest.fixture
def counting_stub(tmp_path):
    path = tmp_path / "stub_dir" / "conv_lab_stub"
    path.parent.mkdir()
    path.write_text(COUNTING_STUB)
    path.chmod(path.stat().st_mode | stat.S_IEXEC)
    return path


def test_repeat_interleaves_and_averages(counting_stub, tmp_path):
    out = tmp_path / "m.csv"
    assert sweep.main(["--cases", "smoke,cfg2_mid_3x3", "--output", str(out),
                       "--conv-lab", str(counting_stub), "--repeat", "2"]) == 0
    # Every case once, then every case again.
    order = (counting_stub.parent / "order").read_text().split()
    assert order[1::2] == ["smoke", "cfg2_mid_3x3", "smoke", "cfg2_mid_3x3"]
    rows = read(out)
    assert [r["case"] for r in rows] == ["smoke", "cfg2_mid_3x3"]
    smoke = rows[0]  # calls 1 and 3: both odd, identical rows
    assert smoke["repeats"] == "2" and smoke["winner"] == "splitk"
    assert float(smoke["splitk_ms"]) == pytest.approx(0.018)
    mid = rows[1]  # calls 2 and 4: both even
    assert mid["splitk_correct"] == "0" and mid["winner"] == "generic"


def test_repeat_means_and_correctness(tmp_path):
    # Two repetitions that disagree: means, all-or-nothing correctness, and a
    # winner, tops and roofline_frac that follow the means.
    a = {"case": "x", "generic_ms": "0.020", "strip_ms": "-1", "halo_ms": "0.030",
         "splitk_ms": "0.018", "winner": "splitk", "generic_correct": "1",
         "strip_correct": "1", "halo_correct": "1", "splitk_correct": "1",
         "tops": "10", "roofline_frac": "0.5", "graph_ms": "0.006"}
    b = dict(a, generic_ms="0.016", splitk_ms="0.022", winner="generic", tops="12.5",
             roofline_frac="0.625", graph_ms="0.004", halo_correct="0", halo_ms="-1")
    m = sweep.merge_repeats([a, b])
    assert float(m["generic_ms"]) == pytest.approx(0.018)
    assert float(m["splitk_ms"]) == pytest.approx(0.020)
    assert m["halo_ms"] == "-1" and m["halo_correct"] == "0" and m["strip_ms"] == "-1"
    assert m["winner"] == "generic" and m["repeats"] == "2"
    # The first row's winner (splitk, 0.018) ran at 10 TOPS; the merged winner
    # (generic, 0.018 mean) gives the same time, so the same TOPS.
    assert float(m["tops"]) == pytest.approx(10.0)
    assert float(m["roofline_frac"]) == pytest.approx(0.5)
    # graph_ms is each row's winner's graph time: only the repetition whose
    # winner is the merged winner (b, generic) counts.
    assert float(m["graph_ms"]) == pytest.approx(0.004)


def test_repeat_with_a_missing_row_is_not_correct():
    # Three repetitions ran, two returned a row: no family counts as correct.
    a = {"case": "x", "generic_ms": "0.020", "strip_ms": "-1", "halo_ms": "-1",
         "splitk_ms": "-1", "winner": "generic", "generic_correct": "1", "strip_correct": "1",
         "halo_correct": "1", "splitk_correct": "1", "tops": "10", "roofline_frac": "0.5",
         "graph_ms": "0.006"}
    m = sweep.merge_repeats([a, dict(a)], expected=3)
    assert m["generic_correct"] == "0" and m["repeats"] == "2"
    assert sweep.merge_repeats([a, dict(a)], expected=2)["generic_correct"] == "1"
    assert float(sweep.merge_repeats([a, dict(a)])["graph_ms"]) == pytest.approx(0.006)
