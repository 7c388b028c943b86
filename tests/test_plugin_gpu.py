"""The plugin entry on a B200: the stand-in host (tests/plugin_host.cc)
loads lib/vpipe-ltx-2.5-b200.so, registers it, resolves the CUDA kernel
table by name and runs one w8g64 linear (192 x 512 -> 256) through the
table's ops_create / bind_qlinear / linear / wait_ok entries, against a
dequantise-then-dense f64 product computed on the host, at the reference
qlinear test's 3e-3 rel-L2 bar (tests/ltx25-qlinear-test.cc:188-197)."""
import subprocess

import pytest

from test_plugin_cpu import PLUGIN, build_host

pytestmark = pytest.mark.gpu


def test_linear_through_the_registered_table(tmp_path):
    exe = build_host(tmp_path)
    r = subprocess.run([exe, PLUGIN, "gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    last = r.stdout.splitlines()[-1].split()
    assert last[:4] == ["gpu", "linear", "wait_ok", "0"], r.stdout
    rel = float(last[5])
    assert rel < 3e-3, rel
