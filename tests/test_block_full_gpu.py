"""one joint AV block at 960x544x121 on the GPU vs the
CPU oracle.

Video 8160 tokens x 4096 (latent grid t=16, h=17, w=30, 3-axis RoPE in
seconds and pixels), audio 126 tokens x 2048 (1-D RoPE in seconds), text
256 tokens at each stream's width, cross tables on the time axis at the
audio width.  Random-init weights (matrices N(0, 1/sqrt(fan_in))), w8g64
packed; adaLN drivers drawn directly as N(0, 0.1) (one modulation level for
every token -- a single sigma).  The oracle (numpy restatement of
block_forward, f64 dot products) runs on the same dequantized weights.
"""
import numpy as np
import pytest

from oracle import block_np, lib

pytestmark = pytest.mark.gpu

CFG = dict(vdim=4096, vheads=32, adim=2048, aheads=32, vt=16 * 17 * 30, at=126, tt=256)


def test_block_full_size_matches_oracle(ctx):
    import time
    import torch
    from test_block_gpu import build, to_dev, host
    blk, ow, ins = build(ctx, CFG, seed=31, grid=(16, 17, 30))
    v, a = ins["video"], ins["audio"]
    dv, da = to_dev(v), to_dev(a)
    x0v, x0a = dv["x"].clone(), da["x"].clone()
    blk.forward(dv, da)
    torch.cuda.synchronize()
    gv, ga = host(dv["x"]), host(da["x"])
    # timing: restore the inputs each time (the block updates x in place)
    ts = []
    for _ in range(5):
        dv["x"].copy_(x0v)
        da["x"].copy_(x0a)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        blk.forward(dv, da)
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    print(f"\nblock forward at 960x544x121: {min(ts):.2f} ms (best of 5)")
    from test_block_gpu import bf16r, OUT_BAR, DELTA_BAR
    t0 = time.time()
    wv, wa = block_np.block_forward(ow, v, a, CFG["vdim"], CFG["vheads"],
                                    CFG["adim"], CFG["aheads"])
    bv, ba = block_np.block_forward(ow, v, a, CFG["vdim"], CFG["vheads"],
                                    CFG["adim"], CFG["aheads"], x_round=bf16r)
    print(f"oracle: {time.time() - t0:.1f} s")
    for name, got, want, wantb, x0 in (("video", gv, wv, bv, v["x"]),
                                       ("audio", ga, wa, ba, a["x"])):
        out_r = lib.rel_l2(got, want)
        delta_r = lib.rel_l2(got - x0, wantb - x0)
        print(f"{name}: output rel-L2 {out_r:.3e}, delta rel-L2 (bf16 stream) {delta_r:.3e}")
        assert out_r < OUT_BAR
        assert delta_r < DELTA_BAR
    blk.close()
