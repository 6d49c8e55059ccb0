"""The conv_lab CLI: the reference's flags and CSV row (src/conv_lab.cu:112-145, :222-241)."""
import csv
import io
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LAB = ROOT / "int8_kernel_lab_b200" / "lib" / "conv_lab"

# conv_lab.cu:223-224, in order.
REFERENCE_COLUMNS = ["case", "n", "h", "w", "c", "k", "r", "s", "out_h", "out_w", "eligible_strip",
                     "generic_ms", "strip_ms", "winner", "generic_correct", "strip_correct"]
APPENDED = ["eligible_halo", "eligible_splitk", "halo_ms", "splitk_ms", "halo_correct",
            "splitk_correct", "gpus", "tops", "roofline_frac", "oracle_ms", "oracle_threads",
            "graph_ms", "selected", "epilogue", "l2"]


def run(*args):
    return subprocess.run([str(LAB), *args], capture_output=True, text=True, timeout=600)


@pytest.mark.parametrize("args", [
    ["--strategy", "fastest"], ["--iterations", "0"], ["--warmup", "-1"], ["--bogus"],
    ["--warmup"], ["--iterations", "x"], ["--pairing", "triple"], ["--values", "small"],
    ["--epilogue", "fp8"],
])
def test_bad_options_exit_nonzero(args):
    out = run(*args)
    assert out.returncode != 0
    assert "usage" in out.stderr or "invalid" in out.stderr


def test_unknown_case():
    out = run("--case", "no_such_case")
    assert out.returncode != 0 and "unknown case" in out.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("strategy", ["both", "all", "generic", "auto"])
def test_csv_row_keeps_reference_columns(strategy):
    out = run("--case", "smoke", "--strategy", strategy, "--csv", "--iterations", "5",
              "--warmup", "2")
    assert out.returncode == 0, out.stderr
    rows = list(csv.DictReader(io.StringIO(out.stdout)))
    assert len(rows) == 1
    header = out.stdout.splitlines()[0].split(",")
    assert header[:16] == REFERENCE_COLUMNS and header[16:] == APPENDED
    row = rows[0]
    assert row["case"] == "smoke" and row["out_h"] == "16" and row["out_w"] == "16"
    assert row["generic_correct"] == "1" and row["strip_correct"] == "1"
    assert row["winner"] in ("generic", "strip", "halo", "splitk")
    assert row["selected"] in ("generic", "strip", "halo", "splitk")


@pytest.mark.gpu
def test_human_line_and_reference_values():
    out = run("--case", "resnet_s3_3x3", "--values", "reference", "--iterations", "3",
              "--warmup", "1")
    assert out.returncode == 0, out.stderr
    assert out.stdout.startswith("resnet_s3_3x3: generic ") and "winner" in out.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("case, epilogue", [("cfg2_mid_3x3", "int8"), ("cfg2_mid_3x3", "int8x32"),
                                            ("cfg4c_tail_k100", "int8")])
def test_int8_epilogues_validate(case, epilogue):
    out = run("--case", case, "--strategy", "all", "--epilogue", epilogue, "--csv",
              "--iterations", "5", "--warmup", "2")
    assert out.returncode == 0, out.stderr
    row = next(csv.DictReader(io.StringIO(out.stdout)))
    assert row["epilogue"] == epilogue
    assert all(row[f + "_correct"] == "1" for f in ("generic", "strip", "halo", "splitk"))
