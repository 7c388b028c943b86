"""The CPU oracle against the reference's own outputs (CPU only).

The golden fixtures in tests/golden/ were produced by the reference's code
compiled from its sources (tests/golden/make_golden.py); when that build is
present here the restatement is also checked against it live.
"""
import numpy as np
import pytest

from oracle import block_np, lib, lora_np, ref, rope_np


def test_pack_matches_reference_golden(golden):
    """w8g64/w4 packs bit-exact vs tests/ltx25-qlinear-test.cc:94-141."""
    g = golden("pack.npz")
    names = sorted({k.split("__")[0] for k in g.files})
    assert len(names) >= 8
    for name in names:
        w = g[f"{name}__w"]
        bits, group = (int(v) for v in g[f"{name}__meta"])
        codes, scales, biases, deq = lib.pack_affine(w, bits, group)
        assert np.array_equal(codes, g[f"{name}__codes"]), name
        assert np.array_equal(scales, g[f"{name}__scales"]), name
        assert np.array_equal(biases, g[f"{name}__biases"]), name
        assert np.array_equal(deq, g[f"{name}__deq"]), name


def test_pack_edge_cases(golden):
    g = golden("pack.npz")
    codes, scales, _, _ = lib.pack_affine(g["edge__w"], 8, 64)
    # a constant group has scale 0 and every code 0 (qlinear-test.cc:129-131)
    assert np.all(codes[0] == 0) and np.all(scales[0] == 0)
    assert np.all(codes[1, :16] == 0)


def test_code_layout_low_bits_first():
    w = np.zeros((1, 64), np.float32)
    w[0, :] = np.arange(64, dtype=np.float32)      # codes ramp 0..255 scaled
    codes, scales, biases, _ = lib.pack_affine(w, 8, 64)
    b = codes.view(np.uint8).reshape(1, 64)        # little-endian bytes
    assert b[0, 0] == 0 and b[0, 63] == 255
    assert np.all(np.diff(b[0].astype(int)) > 0)


def test_dequant_bf16_within_one_ulp_of_reference_deq(golden):
    g = golden("pack.npz")
    for name in ("case0", "case1", "case6", "edge"):
        codes = g[f"{name}__codes"]
        K = g[f"{name}__w"].shape[1]
        d16 = lib.bf16_to_f32(lib.dequant_bf16(codes, g[f"{name}__scales"],
                                               g[f"{name}__biases"], K, 8, 64))
        want = lib.bf16_to_f32(lib.f32_to_bf16(g[f"{name}__deq"]))
        ulp = np.abs(want) * 2.0 ** -7 + 1e-30
        assert np.all(np.abs(d16 - want) <= ulp), name


def test_linear_matches_reference_golden(golden):
    g = golden("linear.npz")
    for i in range(3):
        b = g[f"lin{i}__b"] if f"lin{i}__b" in g.files else None
        y = lib.linear_f64(g[f"lin{i}__x"], g[f"lin{i}__w"], b, threads=2)
        assert np.array_equal(y, g[f"lin{i}__y"])


def test_rope_matches_reference_golden(golden):
    g = golden("rope.npz")
    c, s = rope_np.build_video_rope(2, 3, 4, [20, 2048, 2048], 96, 4)
    np.testing.assert_allclose(c, g["video__cos"], atol=1.2e-7)
    np.testing.assert_allclose(s, g["video__sin"], atol=1.2e-7)
    c, s = rope_np.build_audio_rope(7, 20, 64, 4)
    np.testing.assert_allclose(c, g["audio__cos"], atol=1.2e-7)
    c, s = rope_np.build_index_rope(6, 20, 64, 4)
    np.testing.assert_allclose(c, g["index__cos"], atol=1.2e-7)
    c, s = rope_np.build_cross_rope(g["cross__starts"], g["cross__ends"], 20, 32, 4)
    np.testing.assert_allclose(c, g["cross__cos"], atol=1.2e-7)
    np.testing.assert_array_equal(rope_np.video_time_seconds(3), g["vtime"])
    np.testing.assert_array_equal(rope_np.audio_time_seconds(9), g["atime"])


def _small_block(golden):
    g = golden("block_small.npz")
    cfg = dict(zip(("vdim", "vheads", "adim", "aheads", "vt", "at", "tt"),
                   (int(v) for v in g["cfg"])))
    t = {k[3:]: g[k] for k in g.files if k.startswith("w__")}
    ins = {}
    for s in ("video", "audio"):
        d = {}
        for k in g.files:
            if k.startswith(f"in_{s}__"):
                key = k[len(f"in_{s}__"):]
                if key.endswith("__cos") or key.endswith("__sin"):
                    continue
                d[key] = g[k]
        d["pe"] = (g[f"in_{s}__pe__cos"], g[f"in_{s}__pe__sin"])
        d["cross_pe"] = (g[f"in_{s}__cross_pe__cos"], g[f"in_{s}__cross_pe__sin"])
        ins[s] = d
    return g, cfg, t, ins


@pytest.mark.parametrize("mode", ["joint", "video", "audio"])
def test_block_np_matches_reference_golden(golden, mode):
    """block_np vs the reference block_forward, the bar of
    tests/ltx25-block-test.cc:205-227 (1e-5)."""
    g, cfg, t, ins = _small_block(golden)
    v = dict(ins["video"], present=(mode != "audio"))
    a = dict(ins["audio"], present=(mode != "video"))
    xv, xa = block_np.block_forward(t, v, a, cfg["vdim"], cfg["vheads"],
                                    cfg["adim"], cfg["aheads"])
    assert lib.rel_l2(xv, g[f"out_{mode}__video"]) < 1e-5
    assert lib.rel_l2(xa, g[f"out_{mode}__audio"]) < 1e-5


def test_block_np_structure_is_not_vacuous(golden):
    """Negative control: the pre-cross snapshot and the gate table matter."""
    g, cfg, t, ins = _small_block(golden)
    t2 = dict(t)
    t2["scale_shift_table_a2v_ca_video"] = t["scale_shift_table_a2v_ca_video"] * 3
    xv, _ = block_np.block_forward(t2, ins["video"], ins["audio"], cfg["vdim"],
                                   cfg["vheads"], cfg["adim"], cfg["aheads"])
    assert lib.rel_l2(xv, g["out_joint__video"]) > 1e-4


def test_quant_rows_i8_properties():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((7, 1024)).astype(np.float32)
    x[3, 10] = 40.0
    x[5, :] = 0.0
    xb = lib.f32_to_bf16(x)
    for group in (1024, 512, 64):
        q, s = lib.quant_rows_i8(xb, group)
        assert q.dtype == np.int8 and np.all(np.abs(q.astype(int)) <= 127)
        assert np.all(q[5] == 0) and np.all(s[5] == 0)
        xf = lib.bf16_to_f32(xb).reshape(7, -1, group)
        deq = q.astype(np.float32).reshape(7, -1, group) * s[:, :, None]
        assert np.all(np.abs(deq - xf) <= s[:, :, None] * 0.5 + 1e-7)
        # the absmax element of each nonzero group maps to +-127
        assert np.abs(q[3]).max() == 127


def test_i8_gemm_tracks_float_gemm():
    rng = np.random.default_rng(6)
    M, K, N = 32, 1024, 48
    x = lib.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    w = lib.f32_to_bf16((rng.standard_normal((N, K)) * 0.05).astype(np.float32))
    xq, sx = lib.quant_rows_i8(x, K)
    wq, sw = lib.quant_rows_i8(w, K)
    y = lib.i8_gemm(xq, sx, wq, sw, None, K, threads=2)
    ref_y = lib.linear_f64(lib.bf16_to_f32(x), lib.bf16_to_f32(w))
    r = lib.rel_l2(y, ref_y)
    assert 1e-5 < r < 3e-2


@pytest.mark.skipif(not ref.available(), reason="reference build absent")
def test_restatement_vs_live_reference():
    rng = np.random.default_rng(99)
    for (N, K, bits, group) in [(24, 192, 8, 64), (8, 64, 4, 32)]:
        w = (rng.standard_normal((N, K)) * 0.3).astype(np.float32)
        a = lib.pack_affine(w, bits, group)
        b = ref.pack(w, bits, group)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)


# ---- the trunk's adaLN chain and the adapters, pinned to the reference's own
# host helpers (src/ltx25-dit.cc:30-160, src/ltx25-lora.cc:27-67,
# tests/ltx25-lora-apply-test.cc:330-366, compiled into oracle/_ref)

def _need_ref():
    from oracle import ref
    if not ref.available():
        pytest.skip("oracle/_ref not built (no reference tree at build time)")
    return ref


@pytest.mark.parametrize("t", [0.0, 1.0, 500.0, 999.0])
def test_adaln_restatement_matches_the_reference_chain(t):
    ref = _need_ref()
    from oracle import adaln_np
    rng = np.random.default_rng(5)
    f = lambda *s, sc=1.0: lib.f32_to_bf16((rng.standard_normal(s) * sc).astype(np.float32))
    w = (f(96, 256, sc=0.1), f(96, sc=0.1), f(96, 96, sc=0.15), f(96, sc=0.1),
         f(4 * 96, 96, sc=0.15), f(4 * 96, sc=0.1))
    out, emb = ref.adaln_chain(t, *w)
    want, want_emb = adaln_np.chain(t, *w)
    assert lib.rel_l2(want, out) < 1e-6 and lib.rel_l2(want_emb, emb) < 1e-6
    # a chain without biases (the reference's gemv_host_ takes an empty b)
    out0, _ = ref.adaln_chain(t, w[0], None, w[2], None, w[4], None)
    want0, _ = adaln_np.chain(t, w[0], None, w[2], None, w[4], None)
    assert lib.rel_l2(want0, out0) < 1e-6


def test_lora_restatements_match_the_reference_helpers():
    ref = _need_ref()
    rng = np.random.default_rng(9)
    a_bits, b_bits = lora_np.make_pair(rng, 7, 96, 40)
    a, b = lib.bf16_to_f32(a_bits), lib.bf16_to_f32(b_bits)
    w = (rng.standard_normal((40, 96)) * 0.05).astype(np.float32)
    # W += B A: the test's fold, exactly (same f64 sum order per element)
    assert np.array_equal(lora_np.fold(w, a, b), ref.lora_fold(w, a, b))
    # the factor folded into A: one RNE rounding, bit for bit
    for factor in (1.0, 0.5, 0.37, 2.5):
        assert np.array_equal(lora_np.fold_scale(a_bits, factor), ref.lora_scale(a_bits, factor))
    # one row's delta against the reference's host adapter GEMV
    x = rng.standard_normal(96).astype(np.float32)
    y0 = rng.standard_normal(40).astype(np.float32)
    got = ref.lora_gemv(x, a_bits, b_bits, y0)
    want = y0.astype(np.float64) + lora_np.delta(x[None, :], a, b)[0]
    assert lib.rel_l2(got, want) < 1e-6
