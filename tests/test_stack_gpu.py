"""The block stack on the GPU (BASELINE config 5's single-GPU leg).

Mirrors the reference's ltx25-dit-stack-golden-test (tests/ltx25-dit-stack-
golden-test.cc:1-21, 166-170): the stack's hidden state is compared with the
CPU block_forward chained over the same weights at the taps {0, 1, 3, 7, 15,
31, 47}.  The full 48 blocks run at the model's real widths on a short clip
(the oracle at 8160 tokens would take hours per block); the token count does
not change any GEMM's K or N, only M.

Bars.  Against the f32-stream oracle the reference's own bar is 0.25 (a
48-deep bf16 chain "accumulates", only its shape is diagnostic; it measured
6.7e-3 -> 1.8e-2 on the real checkpoint, README.md:86); the taps must also
grow smoothly (no tap more than 2.5x the previous one, which a defect in one
block would break).  Against an oracle that stores the residual stream in
bf16 after every update, as the interface's bf16 x does on the device, the
chain must stay under 2e-2 at every tap: that isolates the kernels' own
error from the stream's storage.

Also pinned here: the stack's shared arena gives the same bits as private
per-block arenas, ranges compose, the progress hook stops between blocks,
and misuse is refused with the right codes.
"""
import numpy as np
import pytest

from oracle import block_np

from test_block_gpu import SMALL, bf16r, build, host, to_dev

pytestmark = pytest.mark.gpu

STACK_BAR = 2e-2          # small stack / bf16-stream oracle
REF_BAR = 2.5e-1          # tests/ltx25-dit-stack-golden-test.cc:166-170


def chain_oracle(weights, ins, cfg, x_round=None):
    v = {k: (np.array(x) if k == "x" else x) for k, x in ins["video"].items()}
    a = {k: (np.array(x) if k == "x" else x) for k, x in ins["audio"].items()}
    outs = []
    for ow in weights:
        v["x"], a["x"] = block_np.block_forward(ow, v, a, cfg["vdim"], cfg["vheads"],
                                                cfg["adim"], cfg["aheads"], x_round=x_round)
        outs.append((v["x"].copy(), a["x"].copy()))
    return outs


def small_stack(ctx, n):
    blocks, weights, ins = [], [], None
    for i in range(n):
        blk, ow, ins_i = build(ctx, SMALL, seed=100 + 7 * i, grid=(2, 3, 4))
        blocks.append(blk)
        weights.append(ow)
        ins = ins if ins is not None else ins_i     # one set of inputs for all
    return blocks, weights, ins


def test_stack_matches_chained_oracle(ctx):
    import torch
    import ltx25_b200 as L
    from oracle import lib
    blocks, weights, ins = small_stack(ctx, 4)
    st = L.Stack(ctx, blocks)
    st.reserve(SMALL["vt"], SMALL["at"], SMALL["tt"])
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    st.forward(dv, da)
    torch.cuda.synchronize()
    ctx.check()
    want = chain_oracle(weights, ins, SMALL)[-1]
    for name, got, w in (("video", host(dv["x"]), want[0]), ("audio", host(da["x"]), want[1])):
        r = lib.rel_l2(got, w)
        print(name, r)
        assert np.isfinite(got).all()
        assert r < STACK_BAR, f"{name}: {r:.3e}"
    st.close()


def test_shared_arena_is_bit_identical_to_private_arenas(ctx):
    import torch
    import ltx25_b200 as L
    blocks, _, ins = small_stack(ctx, 3)
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    for b in blocks:                         # private arenas (build() reserved)
        b.forward(dv, da)
    torch.cuda.synchronize()
    priv = dv["x"].clone(), da["x"].clone()
    st = L.Stack(ctx, blocks)
    st.reserve(SMALL["vt"], SMALL["at"], SMALL["tt"])
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    st.forward(dv, da)
    torch.cuda.synchronize()
    assert torch.equal(dv["x"], priv[0]) and torch.equal(da["x"], priv[1])
    st.close()


def test_ranges_compose_and_progress_stops(ctx):
    import torch
    import ltx25_b200 as L
    blocks, _, ins = small_stack(ctx, 4)
    st = L.Stack(ctx, blocks)
    st.reserve(SMALL["vt"], SMALL["at"], SMALL["tt"])
    assert len(st) == 4
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    st.forward(dv, da)
    full = dv["x"].clone(), da["x"].clone()
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    st.forward(dv, da, 0, 2)
    st.forward(dv, da, 2, 4)
    torch.cuda.synchronize()
    assert torch.equal(dv["x"], full[0]) and torch.equal(da["x"], full[1])

    seen = []
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    with pytest.raises(L.LtxError) as e:
        st.forward(dv, da, progress=lambda i, n: seen.append((i, n)) or i < 2)
    assert e.value.code == -9                      # LTX_E_ABORTED
    assert seen == [(0, 4), (1, 4), (2, 4)]
    dv2, da2 = to_dev(ins["video"]), to_dev(ins["audio"])
    st.forward(dv2, da2, 0, 2)
    torch.cuda.synchronize()
    assert torch.equal(dv["x"], dv2["x"]) and torch.equal(da["x"], da2["x"])
    st.close()


def test_stack_refuses_misuse(ctx):
    import ltx25_b200 as L
    blocks, _, ins = small_stack(ctx, 2)
    st = L.Stack(ctx, blocks)
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    with pytest.raises(L.LtxError) as e:
        st.forward(dv, da)
    assert e.value.code == -7                      # before reserve
    st.reserve(SMALL["vt"], SMALL["at"], SMALL["tt"])
    with pytest.raises(L.LtxError) as e:
        st.forward(dv, da, 1, 5)
    assert e.value.code == -2                      # range outside the stack
    big = dict(vdim=512, vheads=4, adim=128, aheads=2, vt=24, at=7, tt=5)
    other, _, _ = build(ctx, big, seed=3, grid=(2, 3, 4))
    with pytest.raises(L.LtxError) as e:
        st.add(other)
    assert e.value.code == -2                      # widths differ
    with pytest.raises(L.LtxError) as e:
        st.forward(to_dev(dict(ins["video"], x=np.zeros((SMALL["vt"] + 1, SMALL["vdim"]),
                                                         np.float32))), da)
    assert e.value.code == -7                      # geometry beyond the arena
    blocks[1].reserve(SMALL["vt"], SMALL["at"], SMALL["tt"])    # leaves the shared arena
    with pytest.raises(L.LtxError) as e:
        st.forward(dv, da)
    assert e.value.code == -7
    st.close()


TAPS = (0, 1, 3, 7, 15, 31, 47)


def test_stack_48_blocks_real_widths(ctx):
    """48 blocks at 4096/32 video and 2048/32 audio widths, 24 video tokens
    (2x3x4 grid), 8 audio, 16 text; hidden state checked at the reference's
    taps against the chained f32 oracle."""
    import torch
    import ltx25_b200 as L
    from ltx25_b200 import synth
    from oracle import lib
    cfg = dict(vdim=4096, vheads=32, adim=2048, aheads=32, vt=24, at=8, tt=16)
    ins = block_np.random_block_inputs(cfg, seed=5, video_grid=(2, 3, 4))
    for s in ("video", "audio"):
        for key in ("x", "context", "timesteps", "cross_scale_shift", "cross_gate",
                    "prompt_timestep"):
            ins[s][key] = bf16r(ins[s][key])
    fresh = lambda d: {k: (np.array(x) if k == "x" else x) for k, x in d.items()}
    v, a = fresh(ins["video"]), fresh(ins["audio"])
    vb, ab = fresh(ins["video"]), fresh(ins["audio"])
    st = L.Stack(ctx)
    taps, taps_b = {}, {}
    for i in range(48):
        blk, ow = synth.load_random_block(ctx, 4096, 32, 2048, 32, seed=9000 + i,
                                          effective=True)
        st.add(blk)
        v["x"], a["x"] = block_np.block_forward(ow, v, a, 4096, 32, 2048, 32)
        vb["x"], ab["x"] = block_np.block_forward(ow, vb, ab, 4096, 32, 2048, 32,
                                                  x_round=bf16r)
        if i in TAPS:
            taps[i] = (v["x"].copy(), a["x"].copy())
            taps_b[i] = (vb["x"].copy(), ab["x"].copy())
        del ow
    st.reserve(cfg["vt"], cfg["at"], cfg["tt"])
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    prev = 0
    errs, errs_b = {}, {}
    for t in TAPS:
        st.forward(dv, da, prev, t + 1)
        torch.cuda.synchronize()
        ctx.check()
        prev = t + 1
        gv, ga = host(dv["x"]), host(da["x"])
        assert np.isfinite(gv).all() and np.isfinite(ga).all()
        errs[t] = (lib.rel_l2(gv, taps[t][0]), lib.rel_l2(ga, taps[t][1]))
        errs_b[t] = (lib.rel_l2(gv, taps_b[t][0]), lib.rel_l2(ga, taps_b[t][1]))
    print("f32-stream oracle", {t: (f"{e[0]:.2e}", f"{e[1]:.2e}") for t, e in errs.items()})
    print("bf16-stream oracle", {t: (f"{e[0]:.2e}", f"{e[1]:.2e}") for t, e in errs_b.items()})
    last = None
    for t in TAPS:
        ev, ea = errs[t]
        assert ev < REF_BAR and ea < REF_BAR, (t, ev, ea)
        if last is not None:
            assert ev < 2.5 * last[0] and ea < 2.5 * last[1], ("jump", t, ev, ea, last)
        last = (ev, ea)
        bv, ba = errs_b[t]
        assert bv < STACK_BAR and ba < STACK_BAR, ("bf16-stream", t, bv, ba)
    st.close()
    for b in st.blocks:
        b.close()
