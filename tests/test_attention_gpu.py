"""The tcgen05 flash attention (head_dim 128) against an fp32 PyTorch
reference of the same op on the GPU.

Covers the shapes the video stream runs (8160 self keys, 256 text keys),
ragged query and key tiles (not multiples of 128), one-token edges, the
per-head gate, and logits large enough that rows' running maxima grow
across key tiles (the in-TMEM rescale of O).  Bar: the warp-MMA kernel's
8e-3 rel-L2 (bf16 q/k/v/P/O).
"""
import pytest

pytestmark = pytest.mark.gpu

BAR = 8e-3


def reference(q, k, v, heads, gate=None):
    import torch
    tq, tk = q.shape[0], k.shape[0]
    D = q.shape[1] // heads
    qh = q.float().view(tq, heads, D).transpose(0, 1)
    kh = k.float().view(tk, heads, D).transpose(0, 1)
    vh = v.float().view(tk, heads, D).transpose(0, 1)
    p = torch.softmax(qh @ kh.transpose(1, 2) / D ** 0.5, dim=-1)
    o = (p @ vh).transpose(0, 1)                      # [tq][heads][D]
    if gate is not None:
        o = o * (2.0 * torch.sigmoid(gate.float()))[:, :, None]
    return o.reshape(tq, heads * D)


@pytest.mark.parametrize("tq,tk,heads,gated,qscale,D", [
    (128, 128, 1, False, 1.0, 128), (129, 300, 2, True, 1.0, 128), (1000, 777, 2, True, 1.0, 128),
    (1, 1, 1, False, 1.0, 128), (5, 1000, 3, True, 1.0, 128), (2048, 2048, 4, True, 1.0, 128),
    (8160, 256, 4, True, 1.0, 128), (1500, 1500, 2, False, 6.0, 128),
    (8160, 8160, 2, True, 1.0, 128), (300, 100, 2, True, 1.0, 128), (257, 129, 1, False, 1.0, 128),
    (200, 50, 2, True, 1.0, 128),
    # split over the keys (few query tiles): the video->audio shape and others
    (126, 8160, 32, True, 1.0, 64), (126, 2000, 4, False, 6.0, 64), (100, 4000, 2, True, 1.0, 128),
    (126, 8160, 4, True, 1.0, 64)])
def test_tc_attention_matches_fp32(ctx, tq, tk, heads, gated, qscale, D):
    import torch
    import ltx25_b200 as L
    g = torch.Generator(device="cuda")
    g.manual_seed(tq * 31 + tk)
    inner = heads * D
    q = (torch.randn((tq, inner), generator=g, device="cuda") * qscale).to(torch.bfloat16)
    kv = torch.randn((tk, 2 * inner), generator=g, device="cuda").to(torch.bfloat16)
    k, v = kv[:, :inner], kv[:, inner:]                # strided, as the GEMM writes them
    gate = torch.randn((tq, heads), generator=g, device="cuda").to(torch.bfloat16) if gated else None
    got = L.attention(ctx, q, k, v, heads, D, gate=gate).float()
    torch.cuda.synchronize()
    ctx.check()
    want = reference(q, k, v, heads, gate)
    rel = float(((got - want).norm() / want.norm()).item())
    print((tq, tk, heads, gated, qscale), rel)
    assert torch.isfinite(got).all()
    assert rel < BAR, rel


def test_tc_attention_writes_only_its_rows(ctx):
    """Rows past tq are computed in the last query tile but never stored."""
    import torch
    import ltx25_b200 as L
    heads, D, tq, tk = 2, 128, 130, 140
    q = torch.randn((tq, heads * D), device="cuda").to(torch.bfloat16)
    k = torch.randn((tk, heads * D), device="cuda").to(torch.bfloat16)
    v = torch.randn((tk, heads * D), device="cuda").to(torch.bfloat16)
    big = torch.full((tq + 64, heads * D), 7.0, device="cuda", dtype=torch.bfloat16)
    out = big[:tq]
    L.attention(ctx, q, k, v, heads, D, out=out)
    torch.cuda.synchronize()
    assert torch.all(big[tq:] == 7.0)
    want = reference(q, k, v, heads)
    assert float(((out.float() - want).norm() / want.norm()).item()) < BAR


@pytest.mark.parametrize("mode", ["tc", "mma"])
@pytest.mark.parametrize("tq,tk,heads,gated", [(126, 126, 32, True), (126, 256, 32, True),
                                               (8160, 126, 32, True), (100, 77, 3, False),
                                               (1, 5, 1, True)])
def test_attention_64_unsplit(tq, tk, heads, gated, mode):
    """The unsplit 64-wide attentions (the audio stream's, and the video
    queries over the audio keys) through each kernel LTX25_ATTN64 selects:
    tcgen05 and warp MMA (the default), on a context created with the switch
    set."""
    import os
    import torch
    import ltx25_b200 as L
    old = os.environ.get("LTX25_ATTN64")
    os.environ["LTX25_ATTN64"] = mode
    c = L.Context(0)
    try:
        g = torch.Generator(device="cuda")
        g.manual_seed(tq * 7 + tk)
        D, inner = 64, heads * 64
        q = torch.randn((tq, inner), generator=g, device="cuda").to(torch.bfloat16)
        kv = torch.randn((tk, 2 * inner), generator=g, device="cuda").to(torch.bfloat16)
        gate = torch.randn((tq, heads), generator=g, device="cuda").to(torch.bfloat16) if gated else None
        got = L.attention(c, q, kv[:, :inner], kv[:, inner:], heads, D, gate=gate).float()
        torch.cuda.synchronize()
        c.check()
        want = reference(q, kv[:, :inner], kv[:, inner:], heads, gate)
        rel = float(((got - want).norm() / want.norm()).item())
        assert torch.isfinite(got).all()
        assert rel < BAR, rel
    finally:
        c.close()
        if old is None:
            os.environ.pop("LTX25_ATTN64", None)
        else:
            os.environ["LTX25_ATTN64"] = old
