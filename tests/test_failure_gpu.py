"""Failure detection without a GPU fault.

Every pipeline wait in the library's kernels is bounded: when it runs out,
the kernel records a code in the context's error word, drains and exits, and
the host learns it from ltx_ctx_check (LTX_E_KERNEL) while the context stays
usable.  ltx_ctx_selftest_timeout makes one such wait run out on purpose (a
barrier nothing arrives at, a 100 ms bound); nothing faults, traps or hangs.
"""
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives(ctx):
    import time
    import torch
    import ltx25_b200 as L
    ctx.check()                                   # clean to start with
    t0 = time.time()
    ctx.selftest_timeout(100)
    with pytest.raises(L.LtxError) as e:
        ctx.check()
    assert e.value.code == -6                     # LTX_E_KERNEL
    assert "bounded wait" in str(e.value)
    assert time.time() - t0 < 30                  # it gave up; it did not hang
    ctx.check()                                   # the word was cleared
    # and the context still computes
    w32 = torch.randn(256, 512, device="cuda") * 0.02
    c, s, b = L.pack_w8g64(ctx, w32)
    w = L.QWeight.upload(ctx, c, s, b, 256, 512, on_device=True)
    x = torch.randn(64, 512, device="cuda").to(torch.bfloat16)
    y = L.qlinear(ctx, w, x).float()
    ref = x.float() @ L.dequant(ctx, w).float().t()
    assert float(((y - ref).norm() / ref.norm()).item()) < 3e-3
    ctx.check()
    w.free()


def test_selftest_bound_is_limited(ctx):
    import ltx25_b200 as L
    for bad in (0, 5000):
        with pytest.raises(L.LtxError) as e:
            ctx.selftest_timeout(bad)
        assert e.value.code == -2
