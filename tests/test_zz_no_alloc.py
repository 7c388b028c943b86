"""ltx_qlinear_i8_static: the int8 tier with its activation scratch in the
library's fixed device array, so that the call allocates nothing.

Checked against the existing entry point (ltx_qlinear with the int8 tier on)
on the same weights and inputs over two calls in a row of different shapes --
the second smaller, so the rows the first call left in the shared array must
not leak into it.  Both entry points run the same quantize kernel and the same
kind::i8 GEMM on the same operands, so the outputs must be equal bit for bit
(tighter than the int8 tests' 3e-3 rel-L2 bar).  The static calls run on a
second context whose own int8 scratch was never reserved, and neither that
context's scratch nor the device's free memory may change across them.
Collected last so that it also runs after every other test in the same
process.
"""
import numpy as np
import pytest

from oracle import lib

pytestmark = pytest.mark.gpu

TOL = 3e-3      # the int8 GEMM tests' rel-L2 bar


def _weight(ctx, N, K, seed):
    import ltx25_b200 as L
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    codes, scales, biases, _ = lib.pack_affine(w, 8, 64)
    return L.QWeight.upload(ctx, codes, scales, biases, N, K)


def _x(M, K, seed):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)


def test_static_scratch_matches_the_int8_tier_on_two_calls(ctx):
    import torch
    import ltx25_b200 as L
    cases = [(2048, 4096, 4096, 1), (1100, 4096, 2048, 2)]
    # the weights live on the shared test context, which makes their int8
    # copies; the static calls run on a fresh context of their own
    ws = [_weight(ctx, N, K, seed=10 + s) for (_, K, N, s) in cases]
    xs = [_x(M, K, seed=20 + s) for (M, K, _, s) in cases]
    bias = (torch.randn(4096, device="cuda") * 0.01).to(torch.bfloat16)
    bs = [bias[:N] for (_, _, N, _) in cases]
    ctx.set_tiers(i8_gemm=True)
    try:
        refs = []
        for (M, K, N, _), w, x, b in zip(cases, ws, xs, bs):
            assert ctx.i8_takes(M, K, N)
            refs.append(L.qlinear(ctx, w, x, bias=b).float())
        torch.cuda.synchronize()
    finally:
        ctx.set_tiers(i8_gemm=False)
    outs = [torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
            for (M, _, N, _) in cases]
    fresh = L.Context(0)
    try:
        # warm the entry point once (its first call on a device looks up the
        # array's address), then watch the allocations across the two calls
        L.qlinear_i8_static(fresh, ws[1], xs[1], bias=bs[1], out=outs[1])
        torch.cuda.synchronize()
        cap0 = fresh.scratch_bytes()
        free0 = torch.cuda.mem_get_info()[0]
        for w, x, b, o in zip(ws, xs, bs, outs):
            L.qlinear_i8_static(fresh, w, x, bias=b, out=o)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        fresh.check()
        assert fresh.scratch_bytes() == cap0 == 0, "the static path grew context scratch"
        assert free1 == free0, f"device free memory moved by {free0 - free1} bytes"
    finally:
        fresh.close()
    for (M, K, N, _), g, r in zip(cases, outs, refs):
        g = g.float()
        rel = float(((g - r).norm() / r.norm()).item())
        assert torch.isfinite(g).all()
        assert rel < TOL, ((M, K, N), rel)
        assert torch.equal(g, r), ((M, K, N), rel)
    for w in ws:
        w.free()


def test_static_scratch_refuses_what_it_cannot_hold(ctx):
    import torch
    import ltx25_b200 as L
    w = _weight(ctx, 256, 4096, seed=3)
    x = torch.zeros((8193, 4096), dtype=torch.bfloat16, device="cuda")   # 8193*4096 > 2^25
    with pytest.raises(L.LtxError) as e:
        L.qlinear_i8_static(ctx, w, x)
    assert e.value.code == -2
    fresh = _weight(ctx, 256, 4096, seed=4)      # no int8 copy made yet
    with pytest.raises(L.LtxError) as e:
        L.qlinear_i8_static(ctx, fresh, x[:16])
    assert e.value.code == -7
    w.free()
    fresh.free()
