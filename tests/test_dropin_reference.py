"""The drop-in, end to end: the reference's own program on this engine.

`make -C oracle dropin` compiles the reference's src/conv_lab.cu, unchanged,
with include/compat ahead of everything else on the include path.  Its
`#include "generic_implicit_gemm.cuh"` / `"spatial_strip.cuh"` and the case
header's `#include "conv_shape.cuh"` then resolve to this engine's header,
and the binary links libint8conv.so.  Running it exercises the reference's
call sites (src/conv_lab.cu:170-202), its own seeded inputs and its own
validation (reference_value, :39-86), and its CSV and exit-code contract
(:222-241).  The binaries are built where the reference sources exist and
travel with the tree (oracle/_ref/dropin_<case>).
"""
import csv
import io
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
BINARIES = sorted((ROOT / "oracle" / "_ref").glob("dropin_*"))

REFERENCE_STYLE_CALLER = r'''
#include "generic_implicit_gemm.cuh"
#include "spatial_strip.cuh"
#include "conv_shape.cuh"

using TestShape = ConvShape<32, 28, 28, 128, 128, 3, 3, 1, 1, 1, 1, 1, 1>;
static_assert(TestShape::output_elements == 32u * 28 * 28 * 128, "conv_shape formulas");

int main() {
  int status = 0;
  launch_generic_sm80<TestShape>(nullptr, nullptr, nullptr, nullptr);
  if constexpr (kSpatialStripEligible<TestShape>) {
    launch_spatial_strip<TestShape>(nullptr, nullptr, nullptr, nullptr);
  } else {
    status = 1;
  }
  return status;
}
'''


def test_compat_headers_resolve_the_reference_names(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no g++")
    src = tmp_path / "caller.cpp"
    src.write_text(REFERENCE_STYLE_CALLER)
    exe = tmp_path / "caller"
    lib_dir = ROOT / "int8_kernel_lab_b200" / "lib"
    subprocess.run([gxx, "-std=c++17", f"-I{ROOT / 'include' / 'compat'}",
                    f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", str(src), "-o", str(exe),
                    f"-L{lib_dir}", "-lint8conv", f"-Wl,-rpath,{lib_dir}"], check=True)
    assert subprocess.run([str(exe)]).returncode == 0


@pytest.mark.gpu
@pytest.mark.parametrize("binary", BINARIES, ids=[b.name for b in BINARIES])
def test_reference_harness_on_this_engine(binary):
    out = subprocess.run([str(binary), "--strategy", "both", "--csv", "--warmup", "2",
                          "--iterations", "5"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    row = next(csv.DictReader(io.StringIO(out.stdout)))
    assert row["case"] == binary.name[len("dropin_"):]
    assert row["generic_correct"] == "1" and row["strip_correct"] == "1"
    assert float(row["generic_ms"]) > 0
    if row["eligible_strip"] == "1":
        assert float(row["strip_ms"]) > 0
