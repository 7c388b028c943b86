"""ltx_qlinear_i8_static: the int8 tier with its activation scratch in the
library's fixed device array, so that the call allocates nothing.

Checked against the existing entry point (ltx_qlinear with the int8 tier on)
on the same weights and inputs, at the tolerance the int8 tests use, over two
calls in a row of different shapes -- the second smaller, so the rows the
first call left in the shared array must not leak into it.  Collected last so
that it also runs after every other test in the same process.
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
    got = [L.qlinear_i8_static(ctx, w, x, bias=b).float() for w, x, b in zip(ws, xs, bs)]
    torch.cuda.synchronize()
    ctx.check()
    for (M, K, N, _), g, r in zip(cases, got, refs):
        rel = float(((g - r).norm() / r.norm()).item())
        print((M, K, N), rel, bool(torch.equal(g, r)))
        assert torch.isfinite(g).all()
        assert rel < TOL, ((M, K, N), rel)
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
