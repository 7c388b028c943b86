"""The C-ABI library: it is built, it loads, and it exports exactly what
include/ltx25_cuda.h declares (CPU only; no compute calls)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "ltx25_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"LTX_API\s+[\w\s\*]+?\b(ltx_\w+)\s*\(", src)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for must in ("ltx_ctx_create", "ltx_qweight_upload", "ltx_qlinear",
                 "ltx_qlinear_ex", "ltx_set_tiers", "ltx_i8_takes",
                 "ltx_ctx_check"):
        assert must in syms


def test_library_loads_and_exports_every_symbol():
    import ltx25_b200 as L
    lib = L.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.ltx_abi_version() == 1


def test_binding_covers_the_header():
    import ltx25_b200 as L
    assert sorted(L.SIGNATURES) == declared_symbols()


def test_null_arguments_rejected_without_a_device():
    import ltx25_b200 as L
    lib = L.load()
    assert lib.ltx_ctx_create(0, None) == -1                 # LTX_E_NULL
    assert lib.ltx_qlinear(None, None, None, None, None, 1, 64, 8, None) == -1
    assert lib.ltx_set_tiers(None, 1, 0, 0) == -1
    assert lib.ltx_i8_takes(None, 8160, 4096, 4096) == 0
    assert lib.ltx_stack_create(None, None) == -1
    assert lib.ltx_stack_add_block(None, None) == -1
    assert lib.ltx_stack_reserve(None, 1, 1, 1) == -1
    assert lib.ltx_stack_forward(None, None, None, 0, -1, None, None, None) == -1
    assert lib.ltx_stack_size(None) == 0
    assert lib.ltx_stack_last_error(None) == b"null stack"


def test_context_creation_fails_loudly_without_an_sm100_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the gpu tests")
    import ltx25_b200 as L
    with pytest.raises(L.LtxError):
        L.Context(0)


def test_rope_tables_match_reference_golden(golden):
    """The product's host RoPE builder against the reference's own tables
    (src/ltx25-rope.cc, frozen in tests/golden/rope.npz)."""
    import numpy as np
    import ltx25_b200 as L
    g = golden("rope.npz")
    s, e = L.video_spans(2, 3, 4)
    c, sn = L.rope_table(s, e, [20, 2048, 2048], 96, 4)
    np.testing.assert_allclose(c, g["video__cos"], atol=1.2e-7)
    np.testing.assert_allclose(sn, g["video__sin"], atol=1.2e-7)
    a_s, a_e = L.audio_seconds(7)
    c, sn = L.rope_table(a_s, a_e, [20], 64, 4)
    np.testing.assert_allclose(c, g["audio__cos"], atol=1.2e-7)
    np.testing.assert_array_equal(a_s[:9 if len(a_s) >= 9 else len(a_s)], g["atime"][:len(a_s)])
    c, sn = L.rope_table(g["cross__starts"], g["cross__ends"], [20], 32, 4)
    np.testing.assert_allclose(c, g["cross__cos"], atol=1.2e-7)
    # spans: the time axis equals the reference's video_time_seconds
    np.testing.assert_array_equal(np.unique(s[0]), g["vtime"][:2])


_ONE_THREAD_TABLE = """
import sys, numpy as np
sys.path.insert(0, sys.argv[1])
import ltx25_b200 as L
s, e = L.video_spans(16, 17, 30)
c, sn = L.rope_table(s, e, [20, 2048, 2048], 4096, 32)
np.save(sys.argv[2] + "/c.npy", c)
np.save(sys.argv[2] + "/s.npy", sn)
"""


def test_rope_table_threads_give_the_same_bits(tmp_path):
    """The video table at BASELINE config 4's geometry (8160 tokens, 32
    heads) built over the host's threads equals, bit for bit, the table
    built on one thread (LTX25_HOST_THREADS=1 in a child process)."""
    import os
    import subprocess
    import sys
    import numpy as np
    import ltx25_b200 as L
    s, e = L.video_spans(16, 17, 30)
    c, sn = L.rope_table(s, e, [20, 2048, 2048], 4096, 32)
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                       "vpipe-ltx-2.5_b200")
    env = dict(os.environ, LTX25_HOST_THREADS="1")
    subprocess.run([sys.executable, "-c", _ONE_THREAD_TABLE, pkg, str(tmp_path)], env=env,
                   check=True, timeout=300)
    assert np.array_equal(c.view(np.uint32), np.load(tmp_path / "c.npy").view(np.uint32))
    assert np.array_equal(sn.view(np.uint32), np.load(tmp_path / "s.npy").view(np.uint32))
