"""Low-rank adapters on the GPU (the reference's
tests/ltx25-lora-apply-test.cc): the standalone op against f64 on the host,
the adapted qlinear (delta in the GEMM's accumulator) against the oracle
under each epilogue, and the adapted block against the CPU block with the
pair folded into its base weight, site by site and all at once.

Bars: the op, 2e-2 (the reference's, two bf16 GEMMs); the block, the
reference's 4e-2 on the output, with controls that the fold is material and
that the adapter is applied (omitting it does not match)."""
import numpy as np
import pytest

from oracle import block_np, lib, lora_np

from test_block_gpu import bf16r, dev_bf16, host, to_dev

pytestmark = pytest.mark.gpu

OP_BAR = 2e-2
BLOCK_BAR = 4e-2


def _bits_to_dev(bits):
    import torch
    return torch.from_numpy(np.asarray(bits, np.uint16).view(np.int16)).cuda().view(
        torch.bfloat16)


@pytest.mark.parametrize("M,K,N,rank", [
    (12, 64, 64, 3), (8, 32, 64, 3), (12, 64, 32, 3), (12, 64, 4, 3), (12, 64, 256, 5),
    (6, 64, 64, 1), (128, 4096, 4096, 32), (128, 4096, 16384, 32), (64, 1024, 1024, 450)])
def test_lora_add_matches_f64(ctx, M, K, N, rank):
    """tests/ltx25-lora-apply-test.cc:389-480: y + (x A^T) B^T, f64 on the host."""
    import torch
    import ltx25_b200 as L
    rng = np.random.default_rng(M * 7 + K + N + rank)
    x = bf16r(rng.standard_normal((M, K)))
    a = lib.f32_to_bf16(rng.standard_normal((rank, K)) * 0.5)
    b = lib.f32_to_bf16(rng.standard_normal((N, rank)) * 0.5)
    y0 = bf16r(rng.standard_normal((M, N)))
    lo = L.Lora(ctx, _bits_to_dev(a), _bits_to_dev(b))
    xd, yd = dev_bf16(x), dev_bf16(y0)
    L.lora_add(ctx, lo, xd, yd)
    torch.cuda.synchronize()
    ctx.check()
    want = y0 + lora_np.delta(x, lib.bf16_to_f32(a), lib.bf16_to_f32(b))
    r = lib.rel_l2(host(yd), want)
    print((M, K, N, rank), r)
    assert r < OP_BAR, r
    lo.free()


def test_lora_scale_is_folded_into_a(ctx):
    """lora_scale * alpha/rank folded into A at upload (src/ltx25-lora.cc:
    56-68): the result follows the folded A, not A times the scale later."""
    import torch
    import ltx25_b200 as L
    rng = np.random.default_rng(3)
    M, K, N, rank, scale = 64, 512, 256, 16, 0.37
    x = bf16r(rng.standard_normal((M, K)))
    a = lib.f32_to_bf16(rng.standard_normal((rank, K)))
    b = lib.f32_to_bf16(rng.standard_normal((N, rank)))
    lo = L.Lora(ctx, _bits_to_dev(a), _bits_to_dev(b), scale=scale)
    yd = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda")
    L.lora_add(ctx, lo, dev_bf16(x), yd)
    torch.cuda.synchronize()
    want = lora_np.delta(x, lib.bf16_to_f32(lora_np.fold_scale(a, scale)), lib.bf16_to_f32(b))
    r = lib.rel_l2(host(yd), want)
    assert r < OP_BAR, r
    unscaled = lora_np.delta(x, lib.bf16_to_f32(a), lib.bf16_to_f32(b))
    assert lib.rel_l2(host(yd), unscaled) > 0.5
    lo.free()


def _quantized(ctx, rng, N, K):
    import torch
    import ltx25_b200 as L
    w = torch.from_numpy((rng.standard_normal((N, K)) * 0.02).astype(np.float32)).cuda()
    c, s, b = L.pack_w8g64(ctx, w)
    q = L.QWeight.upload(ctx, c, s, b, N, K, on_device=True)
    wdeq = L.dequant(ctx, q).float().cpu().numpy()
    return q, wdeq


@pytest.mark.parametrize("M", [126, 2048])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_qlinear_lora_matches_oracle(ctx, M, epi):
    """The delta in the linear's accumulator, before the epilogue: GELU and
    the gated residual see x W^T + b + (x A^T) B^T, as a folded weight would."""
    import torch
    import ltx25_b200 as L
    rng = np.random.default_rng(M + epi)
    K, N, rank = 1024, 512, 24
    q, wdeq = _quantized(ctx, rng, N, K)
    a, b = lora_np.make_pair(rng, rank, K, N)
    lo = L.Lora(ctx, _bits_to_dev(a), _bits_to_dev(b))
    x = bf16r(rng.standard_normal((M, K)))
    bias = bf16r(rng.standard_normal(N) * 0.1)
    gate = rng.standard_normal(N).astype(np.float32)
    y0 = bf16r(rng.standard_normal((M, N)))
    yd = dev_bf16(y0)
    L.qlinear_lora(ctx, q, lo, dev_bf16(x), bias=dev_bf16(bias), out=yd, epilogue=epi,
                   gate=torch.from_numpy(gate).cuda() if epi == 2 else None)
    torch.cuda.synchronize()
    ctx.check()
    acc = (x.astype(np.float64) @ wdeq.astype(np.float64).T + bias +
           lora_np.delta(x, lib.bf16_to_f32(a), lib.bf16_to_f32(b)))
    if epi == 0:
        want = acc
    elif epi == 1:
        want = block_np.gelu_tanh(acc.astype(np.float32))
    else:
        want = y0 + gate * acc
    r = lib.rel_l2(host(yd), want)
    print(M, epi, r)
    assert r < 1e-2, r
    # and the adapter is material: without it the result is far off
    plain = L.qlinear(ctx, q, dev_bf16(x), bias=dev_bf16(bias), out=dev_bf16(y0), epilogue=epi,
                      gate=torch.from_numpy(gate).cuda() if epi == 2 else None)
    torch.cuda.synchronize()
    assert lib.rel_l2(host(plain), want) > 10 * r
    lo.free()
    q.free()


@pytest.mark.parametrize("M,N,epi", [(2048, 1024, 2), (1900, 2048, 0)])
def test_dense_lora_tile_plans_agree(ctx, M, N, epi):
    """The adapter as a K extension of the expanded-weight GEMM: single CTAs,
    CTA pairs and pairs holding two weight blocks per CTA give the same bits
    (the same K order per output) and the oracle's result."""
    import torch
    import ltx25_b200 as L
    rng = np.random.default_rng(M + N)
    K, rank = 1024, 24
    q, wdeq = _quantized(ctx, rng, N, K)
    a, b = lora_np.make_pair(rng, rank, K, N)
    lo = L.Lora(ctx, _bits_to_dev(a), _bits_to_dev(b))
    x = bf16r(rng.standard_normal((M, K)))
    gate = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).cuda()
    y0 = bf16r(rng.standard_normal((M, N)))
    outs = {}
    ctx.set_route(L.ROUTE_DEQUANT_ONCE)
    try:
        for pair in (2, 1, 0):
            ctx.set_tile_plan(pair=pair, splits=1)
            yd = dev_bf16(y0)
            L.qlinear_lora(ctx, q, lo, dev_bf16(x), out=yd, epilogue=epi,
                           gate=gate if epi == 2 else None)
            torch.cuda.synchronize()
            outs[pair] = yd
    finally:
        ctx.set_tile_plan()
        ctx.set_route(L.ROUTE_AUTO)
    ctx.check()
    assert torch.equal(outs[2], outs[0])
    assert torch.equal(outs[1], outs[0])
    acc = x.astype(np.float64) @ wdeq.astype(np.float64).T + \
        lora_np.delta(x, lib.bf16_to_f32(a), lib.bf16_to_f32(b))
    want = acc if epi == 0 else y0 + gate.cpu().numpy() * acc
    assert lib.rel_l2(host(outs[2]), want) < 1e-2
    lo.free()
    q.free()


def test_qlinear_lora_without_adapter_is_qlinear(ctx):
    import torch
    import ltx25_b200 as L
    rng = np.random.default_rng(9)
    q, _ = _quantized(ctx, rng, 256, 512)
    x = dev_bf16(rng.standard_normal((300, 512)))
    a = L.qlinear_lora(ctx, q, None, x)
    b = L.qlinear(ctx, q, x)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    q.free()


# ---- the adapted block ------------------------------------------------------

CFG = dict(vdim=512, vheads=4, adim=256, aheads=4, vt=24, at=7, tt=5)

# (module, stream it writes): the reference's site list
# (tests/ltx25-lora-apply-test.cc:237-325)
SITES = [
    ("attn1.to_q", "video"), ("attn1.to_k", "video"), ("attn1.to_v", "video"),
    ("attn1.to_out.0", "video"), ("attn1.to_gate_logits", "video"),
    ("attn2.to_q", "video"), ("attn2.to_out.0", "video"),
    ("ff.net.0.proj", "video"), ("ff.net.2", "video"),
    ("audio_attn1.to_q", "audio"), ("audio_attn2.to_v", "audio"),
    ("audio_ff.net.0.proj", "audio"), ("audio_ff.net.2", "audio"),
    ("audio_to_video_attn.to_k", "video"), ("video_to_audio_attn.to_k", "audio"),
    ("audio_to_video_attn.to_v", "video"), ("audio_to_video_attn.to_out.0", "video"),
    ("video_to_audio_attn.to_out.0", "audio"),
]


def _block(ctx, t):
    import ltx25_b200 as L
    blk = L.Block(ctx, CFG["vdim"], CFG["vheads"], CFG["adim"], CFG["aheads"])
    deq = blk.load(t)
    ow = {}
    for k, v in deq.items():
        if L.is_quantized_name(k, np.ndim(t[k])):
            ow[k] = v
        elif k.endswith(".bias") or "to_gate_logits" in k:
            ow[k] = bf16r(v)
        else:
            ow[k] = v
    return blk, ow


def _inputs():
    ins = block_np.random_block_inputs(CFG, seed=41, video_grid=(2, 3, 4))
    for s in ("video", "audio"):
        for key in ("x", "context", "timesteps", "cross_scale_shift", "cross_gate",
                    "prompt_timestep"):
            ins[s][key] = bf16r(ins[s][key])
    return ins


def _gpu(blk, ins):
    import torch
    blk.reserve(CFG["vt"], CFG["at"], CFG["tt"])
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    blk.forward(dv, da)
    torch.cuda.synchronize()
    return {"video": host(dv["x"]), "audio": host(da["x"])}


def _cpu(ow, ins):
    v, a = block_np.block_forward(ow, ins["video"], ins["audio"], CFG["vdim"], CFG["vheads"],
                                  CFG["adim"], CFG["aheads"])
    return {"video": v, "audio": a}


def _both(d):
    return np.concatenate([d["video"].ravel(), d["audio"].ravel()])


@pytest.fixture(scope="module")
def base():
    return block_np.random_block_tensors(CFG["vdim"], CFG["vheads"], CFG["adim"],
                                         CFG["aheads"], seed=40)


def _adapt(ctx, blk, ow, module, rng, rank):
    """Attach a pair to `module` and fold it into the oracle's weights."""
    import ltx25_b200 as L
    wname = module + ".weight"
    n, k = ow[wname].shape
    a, b = lora_np.make_pair(rng, rank, k, n)
    lo = L.Lora(ctx, _bits_to_dev(a), _bits_to_dev(b))
    blk.set_lora(module, lo)
    ow[wname] = lora_np.fold(ow[wname], lib.bf16_to_f32(a), lib.bf16_to_f32(b))
    return lo


@pytest.mark.parametrize("module,stream", SITES)
def test_block_adapter_site(ctx, base, module, stream):
    """tests/ltx25-lora-apply-test.cc:699-765: runtime adapter == folded
    weight, the fold is material on the stream the site writes, and omitting
    the adapter does not match."""
    ins = _inputs()
    plain_blk, plain_ow = _block(ctx, base)
    plain_blk.finalize()
    plain_gpu = _gpu(plain_blk, ins)
    plain_cpu = _cpu(plain_ow, ins)
    plain_blk.close()
    blk, ow = _block(ctx, base)
    rng = np.random.default_rng(sum(module.encode()))
    lo = _adapt(ctx, blk, ow, module, rng, rank=5 if "ff" not in module else 40)
    blk.finalize()
    lo.free()                       # copied at finalize
    got = _gpu(blk, ins)
    want = _cpu(ow, ins)
    r = lib.rel_l2(_both(got), _both(want))
    moved = lib.rel_l2(want[stream], plain_cpu[stream])
    omitted = lib.rel_l2(plain_gpu[stream], want[stream])
    print(module, f"adapted {r:.3e} moved {moved:.3f} omitted {omitted:.3f}")
    assert r < BLOCK_BAR, r
    assert moved > 0.01, moved
    assert omitted > 5 * lib.rel_l2(got[stream], want[stream])
    blk.close()


def test_block_all_adapters_at_once(ctx, base):
    """Every site together: catches a pair applied twice or a scratch
    collision between sites sharing the arena (tests/ltx25-lora-apply-test.cc:
    767-795)."""
    ins = _inputs()
    blk, ow = _block(ctx, base)
    rng = np.random.default_rng(77)
    los = [_adapt(ctx, blk, ow, m, rng, rank=5) for m, _ in SITES]
    # the remaining modules too, so every site of every attention is adapted
    for extra in ("attn2.to_k", "attn2.to_v", "audio_attn1.to_k", "audio_attn1.to_v",
                  "audio_attn1.to_out.0", "audio_attn2.to_q", "audio_attn2.to_k",
                  "audio_to_video_attn.to_q", "video_to_audio_attn.to_q",
                  "video_to_audio_attn.to_v", "audio_attn1.to_gate_logits"):
        los.append(_adapt(ctx, blk, ow, extra, rng, rank=9))
    blk.finalize()
    got = _gpu(blk, ins)
    want = _cpu(ow, ins)
    r = lib.rel_l2(_both(got), _both(want))
    print("all sites", r)
    assert r < BLOCK_BAR, r
    blk.close()


def test_block_adapter_refusals(ctx, base):
    import ltx25_b200 as L
    blk, ow = _block(ctx, base)
    rng = np.random.default_rng(1)
    a, b = lora_np.make_pair(rng, 4, CFG["vdim"], CFG["vdim"])
    lo = L.Lora(ctx, _bits_to_dev(a), _bits_to_dev(b))
    with pytest.raises(L.LtxError) as e:
        blk.set_lora("attn1.to_qq", lo)           # a module this block does not apply
    assert e.value.code == -3
    # a pair whose widths disagree with the base linear: refused at finalize
    bad = L.Lora(ctx, *map(_bits_to_dev, lora_np.make_pair(rng, 4, CFG["vdim"], 64)))
    blk.set_lora("attn1.to_q", bad)
    with pytest.raises(L.LtxError) as e:
        blk.finalize()
    assert e.value.code == -2
    blk.close()
    blk, _ = _block(ctx, base)
    blk.finalize()
    with pytest.raises(L.LtxError) as e:
        blk.set_lora("attn1.to_q", lo)            # after finalize
    assert e.value.code == -7
    blk.close()
    lo.free()
    bad.free()
