"""The C++ drop-in header compiles against reference-style call sites and
links the C ABI; constexpr predicates evaluate at compile time."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent

SOURCE = r'''
#include "int8conv.hpp"
#include <cstdio>

// Reference-style compile-time shapes (workloads.csv rows).
using Smoke = ConvShape<1, 16, 16, 32, 32, 3, 3, 1, 1, 1, 1, 1, 1>;
using BigStrip = ConvShape<16, 256, 256, 256, 256, 3, 3, 1, 1, 1, 1, 1, 1>;
using Down = ConvShape<1, 56, 56, 256, 128, 3, 3, 1, 1, 2, 2, 1, 1>;
static_assert(Smoke::out_h == 16 && Smoke::gemm_k == 288, "conv_shape formulas");
static_assert(kSpatialStripEligible<BigStrip>, "reference strip shape stays eligible");
static_assert(kSpatialStripEligible<Smoke>, "B200 strip needs no out_w % 128");
static_assert(!kSpatialStripEligible<Down>, "stride_w 2 is not strip");
// Beyond the TMA im2col limits (stride 16, pad 130): still launch_generic
// shapes, as in the reference (gather staging).
using Patch16 = ConvShape<8, 224, 224, 16, 768, 16, 16, 0, 0, 16, 16, 1, 1>;
using Pad130 = ConvShape<1, 5, 5, 16, 8, 3, 3, 130, 130, 1, 1, 1, 1>;
static_assert(!kSpatialStripEligible<Patch16>, "stride 16 is not strip");

int main() {
  int status = 0;
  // Same call sites as src/conv_lab.cu:172-176 / :200-201 (null buffers: no GPU needed).
  if (launch_generic<Smoke>(nullptr, nullptr, nullptr, nullptr) != INT8CONV_BAD_POINTER) status = 1;
  if (launch_generic_sm80<Smoke>(nullptr, nullptr, nullptr, nullptr, 0) != INT8CONV_BAD_POINTER) status = 2;
  if (launch_generic<Patch16>(nullptr, nullptr, nullptr, nullptr) != INT8CONV_BAD_POINTER) status = 4;
  if (launch_generic_sm80<Pad130>(nullptr, nullptr, nullptr, nullptr) != INT8CONV_BAD_POINTER) status = 5;
  if constexpr (kSpatialStripEligible<BigStrip>) {
    if (launch_spatial_strip<BigStrip>(nullptr, nullptr, nullptr, nullptr) != INT8CONV_BAD_POINTER) status = 3;
  }
  std::printf("dropin %d\n", status);
  return status;
}
'''


def test_dropin_header_compiles_and_links(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no g++")
    src = tmp_path / "dropin.cpp"
    src.write_text(SOURCE)
    exe = tmp_path / "dropin"
    lib_dir = ROOT / "int8_kernel_lab_b200" / "lib"
    subprocess.run([gxx, "-std=c++17", "-O1", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include",
                    str(src), "-o", str(exe), f"-L{lib_dir}", "-lint8conv",
                    f"-Wl,-rpath,{lib_dir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "dropin 0" in out.stdout


def test_c_header_is_plain_c(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no gcc")
    src = tmp_path / "c_abi.c"
    src.write_text('#include "int8conv.h"\n#include "int8conv_rules.h"\n'
                   'int main(void){int8conv_shape s={1,8,8,16,4,3,3,1,1,1,1,1,1};'
                   'return i8c_generic_eligible(&s) && int8conv_abi_version()==INT8CONV_ABI_VERSION ? 0 : 1;}\n')
    exe = tmp_path / "c_abi"
    lib_dir = ROOT / "int8_kernel_lab_b200" / "lib"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(src), "-o",
                    str(exe), f"-L{lib_dir}", "-lint8conv", f"-Wl,-rpath,{lib_dir}"], check=True)
    assert subprocess.run([str(exe)]).returncode == 0
