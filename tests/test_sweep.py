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
