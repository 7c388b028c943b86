"""The header-only C++ adapter (include/ltx25_cuda.hpp), the MetalOps /
QWeight stand-in a plugin maintainer compiles against, built and run as a
plain C++ program against the library without a GPU: it compiles cleanly
under -Wall -Wextra -Werror, links, reports the ABI version, refuses a
device that does not exist with a message, and turns a failing linear into
an exception instead of a silent no-op."""
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(REPO, "vpipe-ltx-2.5_b200", "lib")

PROGRAM = r"""
#include <cstdio>
#include <stdexcept>
#include <string>
#include <utility>
#include "ltx25_cuda.hpp"

int main()
{
  std::printf("abi %d\n", ltx_abi_version());
  ltx25::CudaOpsAdapter ops;
  std::string err;
  const bool ok = ops.init(9999, &err);           // no such device anywhere
  std::printf("init %d %s\n", ok ? 1 : 0, err.c_str());
  ltx25::CudaQWeight w, moved(std::move(w));
  std::printf("weight %d %d\n", w.valid() ? 1 : 0, moved.valid() ? 1 : 0);
  try {
    ops.linear(nullptr, nullptr, moved, nullptr, nullptr, 1, 64, 64);
    std::printf("linear returned\n");
  } catch (const std::runtime_error& e) {
    std::printf("linear threw %s\n", e.what());
  }
  std::printf("i8_takes %d\n", ops.i8_takes(8160, 4096, 16384) ? 1 : 0);
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_adapter_compiles_links_and_fails_loudly(tmp_path):
    lib = os.path.join(LIB_DIR, "libltx25_cuda.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    src = tmp_path / "adapter.cc"
    src.write_text(PROGRAM)
    exe = tmp_path / "adapter"
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror",
                    "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe),
                    "-L", LIB_DIR, "-lltx25_cuda", "-Wl,-rpath," + LIB_DIR],
                   check=True, timeout=300)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True,
                         timeout=120).stdout.splitlines()
    import ltx25_b200 as L
    assert out[0] == f"abi {L.load().ltx_abi_version()}"
    assert out[1].startswith("init 0 ltx_ctx_create(9999) failed"), out[1]
    assert out[2] == "weight 0 0"
    assert out[3] == "linear threw null context", out[3]
    assert out[4] == "i8_takes 0"
