"""bench.py's clock sampler, against a fake nvidia-smi (no GPU needed).

The fake prints one sample every 20 ms in nvidia-smi's CSV form (timestamp
first, then the fields of ClockSampler.QUERY), so the tests check which
samples the sampler attributes to a timed region: those inside it, or for a
region shorter than the period, the nearest one on each side.
"""
import os
import stat
import sys
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402

FAKE = r"""#!/bin/bash
# Fake nvidia-smi: ignores its arguments, one sample every 20 ms.
while true; do
  echo "$(date +'%Y/%m/%d %H:%M:%S.%3N'), 0, 1500, 1965, 900.00, 0x4, Not Active, Not Active, Not Active, Active"
  sleep 0.02
done
"""


@pytest.fixture
def fake_smi(tmp_path, monkeypatch):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE)
    exe.chmod(exe.stat().st_mode | stat.S_IXUSR)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    return exe


def test_samples_inside_a_region(fake_smi):
    s = bench.ClockSampler("0")
    s.wait_ready()
    time.sleep(0.05)
    s.mark_start()
    time.sleep(0.2)
    s.mark_stop()
    clocks = s.stop()
    assert clocks["sm_mhz"] == 1500.0 and clocks["sm_max_mhz"] == 1965.0
    assert clocks["reasons"] == ["sw_power_cap"]
    assert clocks["samples_inside"] >= 3  # about 10 at a 20 ms period
    assert clocks["samples"] == clocks["samples_inside"]
    assert 195 <= clocks["region_ms"] < 1000
    assert not os.path.exists(s.path)


def test_region_shorter_than_the_period_takes_its_neighbours(fake_smi):
    s = bench.ClockSampler("0")
    s.wait_ready()
    time.sleep(0.05)
    s.mark_start()
    s.mark_stop()  # a region of microseconds: no sample can fall inside
    clocks = s.stop()
    assert clocks["samples_inside"] == 0
    assert clocks["samples"] == 2  # the last before and the first after
    assert clocks["sm_mhz"] == 1500.0


def test_no_nvidia_smi_gives_no_clocks(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))
    s = bench.ClockSampler("0")
    s.wait_ready()
    s.mark_start()
    s.mark_stop()
    assert s.stop() is None


def _run_bench(args, env_extra=None, timeout=600):
    import json
    import subprocess
    env = dict(os.environ, **(env_extra or {}))
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                         text=True, timeout=timeout, env=env, cwd=str(ROOT))
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    return out.returncode, [json.loads(l) for l in lines], out.stderr


def test_reference_arm_prints_one_line():
    # The reference's own CPU implementation (oracle/_ref when built from the
    # reference sources, else the oracle port) on a small workload.
    rc, lines, err = _run_bench(["--impl", "reference", "--workload", "cfg1_smoke",
                                 "--steps", "2", "--warmup", "1"])
    assert rc == 0, err
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference" and line["unit"] == "TOPS" and line["value"] > 0
    assert line["higher_is_better"] is True and line["steps"] == 2 and line["warmup"] == 1
    assert line["config"]["workload"] == "cfg1_smoke"
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "TOPS", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    rc, lines, err = _run_bench(["--impl", "reference", "--gpus", "2", "--steps", "1",
                                 "--warmup", "0"], {"RANK": "1", "WORLD_SIZE": "2"})
    assert rc == 0, err
    assert lines == []


SHAPE_ATTRS = ("n", "h", "w", "c", "k", "r", "s", "pad_h", "pad_w", "stride_h", "stride_w",
               "dilation_h", "dilation_w", "out_h", "out_w", "gemm_m", "gemm_k",
               "input_elements", "filter_elements", "output_elements", "ops")


def test_plain_shapes_and_inputs_match_the_package():
    # The reference arm computes shapes and inputs without this package; they
    # must be the GPU arm's, field for field and byte for byte.
    import numpy as np

    import int8_kernel_lab_b200 as m
    for name, s in m.load_workloads().items():
        p = bench.plain_workload(name)
        for a in SHAPE_ATTRS:
            assert getattr(p, a) == getattr(s, a), (name, a)
    for name in ("cfg4c_tail_k100", "g_like", "cfg1_smoke"):
        s = m.load_workloads().get(name) or m.ConvShape(2, 9, 7, 16, 24, 3, 3, 1, 1, 2, 2, 1, 1)
        p = bench.PlainShape(**{f: getattr(s, f) for f in bench.SHAPE_FIELDS})
        for got, want in zip(bench.plain_inputs(p), m.make_inputs(s)):
            assert got.dtype == want.dtype and np.array_equal(got, want), name


def test_both_arms_emit_the_same_config():
    import argparse

    import int8_kernel_lab_b200 as m
    args = argparse.Namespace(workload="cfg5a_stress_3x3")
    for world in (1, 8):
        ours = bench.workload_config(m.load_workloads()[args.workload], args, world)
        ref = bench.workload_config(bench.plain_workload(args.workload), args, world)
        assert ours == ref


def test_reference_arm_loads_nothing_of_the_package():
    import subprocess
    probe = (
        "import runpy, sys\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'cfg1_smoke',"
        " '--steps', '1', '--warmup', '0']\n"
        "try:\n"
        "    runpy.run_path('bench.py', run_name='__main__')\n"
        "except SystemExit as e:\n"
        "    assert not e.code, e.code\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('PKG', 'int8_kernel_lab_b200' in sys.modules, 'libint8conv' in maps)\n")
    out = subprocess.run([sys.executable, "-c", probe], capture_output=True, text=True,
                         cwd=str(ROOT), timeout=600)
    assert out.returncode == 0, out.stderr
    assert "PKG False False" in out.stdout
