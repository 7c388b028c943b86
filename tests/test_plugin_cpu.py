"""The plugin entry (vpipe-ltx-2.5_b200/plugin/ltx25-plugin-cuda.cc): the
reference's plugin symbol and registration shape (VPIPE_PLUGIN_DEFINE(&kInfo,
ltx25_register), kRequires = {kernel contract, accel bag},
src/ltx25-plugin.cc:50-136) against the in-repo vpipe stub headers, with
the metallib registration replaced by one CUDA kernel table.

A stand-in host (tests/plugin_host.cc) is compiled with -Wall -Wextra
-Werror, loads the plugin .so, checks the ABI integer, the info record and
the required features, registers it (twice: the second is refused), resolves
the table by name and drives the family's linear and block entries through
it.  Without a GPU those reach the C ABI and report its errors.
"""
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "vpipe-ltx-2.5_b200")
PLUGIN = os.path.join(PKG, "lib", "vpipe-ltx-2.5-b200.so")
CUDA = "/usr/local/cuda"


def build_host(tmp_path):
    if shutil.which("g++") is None:
        pytest.skip("no host C++ compiler")
    if not os.path.exists(PLUGIN):
        pytest.skip("plugin not built (python vpipe-ltx-2.5_b200/build.py)")
    exe = tmp_path / "plugin_host"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
                    "-I", os.path.join(REPO, "include"),
                    "-I", os.path.join(PKG, "plugin", "stub"),
                    "-I", os.path.join(CUDA, "include"),
                    os.path.join(REPO, "tests", "plugin_host.cc"), "-o", str(exe),
                    "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-ldl",
                    "-Wl,-rpath," + os.path.join(CUDA, "lib64")],
                   check=True, timeout=300)
    return str(exe)


def test_plugin_symbol_registration_and_table_without_gpu(tmp_path):
    exe = build_host(tmp_path)
    r = subprocess.run([exe, PLUGIN, "cpu"], capture_output=True, text=True, timeout=120)
    out = r.stdout.splitlines()
    assert r.returncode == 0, r.stdout + r.stderr
    assert out[0] == "abi 8 schema 1 name ltx-2.5"
    assert out[1] == "requires kernel-contract/1,accel-bag/1"
    assert out[2] == "tables 1 1"
    assert out[3] == "table ltx25-cuda-sm100a backend cuda/sm_100a version 1 abi 1 size_ok 1"
    assert out[4].startswith("ops_create -4 null 1 msg ltx_ctx_create(9999) failed"), out[4]
    assert out[5] == "linear_null -1"
    assert out[6] == "i8_takes 0"
    assert out[7] == "block_create_null -1"
    assert out[8] == "block_finalize_null -1"


def test_plugin_exports_only_the_plugin_entry():
    """The shim exports the three plugin symbols and nothing else of its own
    (the table is reached through registration, not by symbol)."""
    if not os.path.exists(PLUGIN) or shutil.which("nm") is None:
        pytest.skip("plugin not built or no nm")
    syms = subprocess.run(["nm", "-D", "--defined-only", PLUGIN], capture_output=True,
                          text=True, check=True).stdout.split()
    ours = sorted(s for s in syms if s.startswith(("vpipe_", "ltx")))
    assert ours == ["vpipe_plugin_abi", "vpipe_plugin_info", "vpipe_plugin_register"]
