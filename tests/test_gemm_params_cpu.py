"""The GEMM kernel's packed output switches (gemm_tc.cuh): the row scatter of
the fused tensor-parallel reduce-scatter (rows per owner, this rank's slot)
and the transposed-columns output (first V^T column, V^T row stride), each
packed into one int of the kernel's parameter block.  Compiled with nvcc as
host code and run without a GPU: every value in the documented ranges comes
back unchanged, including the range ends, and off stays distinguishable
from on."""
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(REPO, "vpipe-ltx-2.5_b200", "csrc")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

PROGRAM = r"""
#include <cstdio>
#include "gemm_tc.cuh"

int main()
{
  using namespace ltx;
  long bad = 0, checked = 0;
  const int rows_cases[] = {1, 2, 12, 1020, 2040, 4080, 32767, 65536, (1 << 28) - 1};
  for (int rows : rows_cases)
    for (int slot = 0; slot < 8; ++slot) {
      GemmParams p{};
      p.scatter = pack_scatter(rows, slot);
      ++checked;
      if (p.scatter <= 0 || scatter_rows(p) != rows || scatter_slot(p) != slot) ++bad;
    }
  const int col_cases[] = {0, 32, 256, 1024, 2048, 8192, 12288, 65504};
  const int ld_cases[] = {8, 128, 1056, 8160, 8192, 65536, (1 << 23) - 8};
  for (int col0 : col_cases)
    for (int ld : ld_cases) {
      GemmParams p{};
      p.vt_spec = pack_vt(col0, ld);
      ++checked;
      if (p.vt_spec == 0 || vt_col0(p) != col0 || vt_ld(p) != ld) ++bad;
    }
  GemmParams off{};
  std::printf("checked %ld bad %ld off %d %d\n", checked, bad, off.scatter, off.vt_spec);
  return bad == 0 ? 0 : 1;
}
"""


@pytest.mark.skipif(not os.path.exists(NVCC) or shutil.which("g++") is None,
                    reason="no nvcc / host compiler")
def test_packed_switches_round_trip(tmp_path):
    src = tmp_path / "params.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "params"
    subprocess.run([NVCC, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-I", CSRC, "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)],
                   check=True, timeout=300)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stdout
    assert out.stdout.strip() == "checked 128 bad 0 off 0 0", out.stdout
