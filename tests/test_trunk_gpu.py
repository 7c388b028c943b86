"""The DiT trunk around the block loop on the GPU (src/ltx25-dit.cc): the
patchify projection with its token pack and keyframe embedding, and the
output head (LayerNorm, 2-row modulation, proj_out), at the model's widths,
against the numpy restatement of tests/ltx25-trunk-test.cc's formulas.

Bars: the reference's are 2e-2 (patchify) and 4e-2 (head) against its
goldens; against an oracle on the same dequantized weights these are bf16
outputs of one GEMM, held to 1e-2."""
import numpy as np
import pytest

from oracle import lib, lora_np, trunk_np

from test_block_gpu import bf16r, dev_bf16, host

pytestmark = pytest.mark.gpu

BAR = 1e-2


def _weight(ctx, rng, N, K, scale=0.05):
    import torch
    import ltx25_b200 as L
    w = torch.from_numpy((rng.standard_normal((N, K)) * scale).astype(np.float32)).cuda()
    c, s, b = L.pack_w8g64(ctx, w)
    q = L.QWeight.upload(ctx, c, s, b, N, K, on_device=True)
    return q, L.dequant(ctx, q).float().cpu().numpy()


def _bits(a):
    import torch
    return torch.from_numpy(np.asarray(a, np.uint16).view(np.int16)).cuda().view(torch.bfloat16)


@pytest.mark.parametrize("dim,grid,adapted", [(4096, (2, 3, 4), False), (4096, (2, 3, 4), True),
                                              (2048, (5, 1, 1), False)])
def test_patchify(ctx, dim, grid, adapted):
    import torch
    import ltx25_b200 as L
    rng = np.random.default_rng(dim + sum(grid))
    z = 128
    F, H, W = grid
    T = F * H * W
    q, wdeq = _weight(ctx, rng, dim, z)
    bias = bf16r(rng.standard_normal(dim) * 0.1)
    lat_cm = bf16r(rng.standard_normal((z, T)))          # [z][F][H][W] flattened
    prefix = bf16r(rng.standard_normal(dim) * 0.5)
    rows = H * W                                          # the first latent frame
    lo, a, b = None, None, None
    if adapted:
        a, b = lora_np.make_pair(rng, 16, z, dim)
        lo = L.Lora(ctx, _bits(a), _bits(b))
    got = L.patchify(ctx, q, dev_bf16(lat_cm), bias=dev_bf16(bias), lora=lo, channel_major=True,
                     prefix=dev_bf16(prefix), prefix_rows=rows)
    torch.cuda.synchronize()
    ctx.check()
    w_eff = wdeq if lo is None else lora_np.fold(wdeq, lib.bf16_to_f32(a), lib.bf16_to_f32(b))
    want = trunk_np.patchify(trunk_np.pack(lat_cm), w_eff, bias, prefix, rows)
    r = lib.rel_l2(host(got), want)
    print(dim, grid, adapted, r)
    assert r < BAR, r
    # token-major input gives the same result
    got2 = L.patchify(ctx, q, dev_bf16(trunk_np.pack(lat_cm)), bias=dev_bf16(bias), lora=lo,
                      prefix=dev_bf16(prefix), prefix_rows=rows)
    torch.cuda.synchronize()
    assert torch.equal(got, got2)
    # the keyframe rows moved, the others did not
    plain = L.patchify(ctx, q, dev_bf16(lat_cm), bias=dev_bf16(bias), lora=lo, channel_major=True)
    torch.cuda.synchronize()
    assert torch.equal(plain[rows:], got[rows:])
    assert not torch.equal(plain[:rows], got[:rows])


@pytest.mark.parametrize("T,dim,out_ch,adapted", [(6, 4096, 128, False), (300, 4096, 128, True),
                                                  (126, 2048, 128, False)])
def test_output_head(ctx, T, dim, out_ch, adapted):
    import torch
    import ltx25_b200 as L
    rng = np.random.default_rng(T + dim)
    q, wdeq = _weight(ctx, rng, out_ch, dim, scale=0.02)
    bias = bf16r(rng.standard_normal(out_ch) * 0.1)
    x = bf16r(rng.standard_normal((T, dim)) * 3.0 + 0.7)    # a mean LayerNorm must remove
    table = rng.standard_normal((2, dim)).astype(np.float32) * 0.2
    emb = rng.standard_normal(dim).astype(np.float32) * 0.2
    ss = (table + emb[None, :]).astype(np.float32)
    lo, a, b = None, None, None
    if adapted:
        a, b = lora_np.make_pair(rng, 8, dim, out_ch)
        lo = L.Lora(ctx, _bits(a), _bits(b))
    ssd = torch.from_numpy(ss).cuda()
    got = L.output_head(ctx, q, dev_bf16(x), ssd, bias=dev_bf16(bias), lora=lo)
    cm = L.output_head(ctx, q, dev_bf16(x), ssd, bias=dev_bf16(bias), lora=lo, channel_major=True)
    torch.cuda.synchronize()
    ctx.check()
    w_eff = wdeq if lo is None else lora_np.fold(wdeq, lib.bf16_to_f32(a), lib.bf16_to_f32(b))
    want = trunk_np.head(x, ss, w_eff, bias)
    r = lib.rel_l2(host(got), want)
    print(T, dim, out_ch, adapted, r)
    assert r < BAR, r
    assert torch.equal(cm, got.t().contiguous())
    # LayerNorm, not RMSNorm: an RMS-normalized head is far off
    rms = np.asarray(x, np.float64)
    rms = (rms / np.sqrt((rms ** 2).mean(axis=1, keepdims=True) + 1e-6)).astype(np.float32)
    wrong = trunk_np.linear(rms * (1 + ss[1]) + ss[0], w_eff, bias)
    assert lib.rel_l2(host(got), wrong) > 10 * r
