"""Blocks and adapters bound from safetensors checkpoints (the reference's
loader, src/ltx25-dit-weights.cc): a block staged by ltx_block_load_st from
a file holding w8g64 packs (codes u32 + F16 or BF16 scales / biases, the reference's on-disk layout)
runs bit-identical to the same block staged tensor by tensor; a pack at
another group is refused; an adapter read with ltx_lora_load_st carries
the file's alpha / rank factor."""
import numpy as np
import pytest

from oracle import block_np, lib, lora_np

import st_file
from test_block_gpu import bf16r, host, to_dev

pytestmark = pytest.mark.gpu

CFG = dict(vdim=256, vheads=2, adim=128, aheads=2, vt=24, at=7, tt=5)
PREFIX = "model.diffusion_model.transformer_blocks.3."


def _checkpoint(tmp_path, t, f16_names=()):
    """Pack every quantized linear with the reference packer; scales and
    biases F16 for the names in f16_names (bf16 otherwise); float tensors
    F32, or BF16 for biases."""
    import ltx25_b200 as L
    tensors, bf16, packs = {}, [], {}
    for name, a in t.items():
        if L.is_quantized_name(name, np.ndim(a)):
            codes, sc, bz, _ = lib.pack_affine(a)
            base = PREFIX + name[:-len(".weight")]
            tensors[base + ".weight"] = codes
            if name in f16_names:
                sc = lib.bf16_to_f32(sc).astype(np.float16)
                bz = lib.bf16_to_f32(bz).astype(np.float16)
            else:
                bf16 += [base + ".scales", base + ".biases"]
            tensors[base + ".scales"] = sc
            tensors[base + ".biases"] = bz
            packs[name] = (codes, sc, bz)
        elif name.endswith(".bias"):
            tensors[PREFIX + name] = lib.f32_to_bf16(np.asarray(a, np.float32))
            bf16.append(PREFIX + name)
        else:
            tensors[PREFIX + name] = np.asarray(a, np.float32)
    tensors["model.diffusion_model.transformer_blocks.4.attn1.to_q.bias"] = \
        np.zeros(CFG["vdim"], np.float32)      # another block's tensor: not bound
    p = st_file.write(tmp_path / "block.safetensors", tensors, bf16=tuple(bf16))
    return p, packs


def _dev(a):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    if a.dtype == np.float16:
        return torch.from_numpy(a).cuda()
    return torch.from_numpy(a.astype(np.float32)).cuda()


def _forward(blk, ins):
    import torch
    blk.reserve(CFG["vt"], CFG["at"], CFG["tt"])
    dv, da = to_dev(ins["video"]), to_dev(ins["audio"])
    blk.forward(dv, da)
    torch.cuda.synchronize()
    return host(dv["x"]), host(da["x"])


def test_block_from_checkpoint_is_bit_identical(ctx, tmp_path):
    import ltx25_b200 as L
    t = block_np.random_block_tensors(CFG["vdim"], CFG["vheads"], CFG["adim"], CFG["aheads"],
                                      seed=31)
    f16 = ("attn1.to_q.weight", "audio_ff.net.2.weight")
    path, packs = _checkpoint(tmp_path, t, f16_names=f16)
    ins = block_np.random_block_inputs(CFG, seed=32, video_grid=(2, 3, 4))
    for s in ("video", "audio"):
        for key in ("x", "context", "timesteps", "cross_scale_shift", "cross_gate",
                    "prompt_timestep"):
            ins[s][key] = bf16r(ins[s][key])
    st = L.SafeTensors(path)
    a = L.Block(ctx, CFG["vdim"], CFG["vheads"], CFG["adim"], CFG["aheads"])
    a.load_st(st, PREFIX)
    a.finalize()
    got = _forward(a, ins)
    a.close()
    b = L.Block(ctx, CFG["vdim"], CFG["vheads"], CFG["adim"], CFG["aheads"])
    for name, arr in t.items():
        if name in packs:
            codes, sc, bz = packs[name]
            N, K = np.shape(arr)
            b.set_qlinear(name, _dev(codes), _dev(sc), _dev(bz), N, K,
                          sb_dtype=L.SB_F16 if name in f16 else L.SB_BF16)
        elif name.endswith(".bias"):
            b.set_tensor(name, _dev(bf16r(arr)))
        else:
            b.set_tensor(name, _dev(arr))
    b.finalize()
    want = _forward(b, ins)
    b.close()
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
    st.close()


def test_other_packs_are_refused(ctx, tmp_path):
    import ltx25_b200 as L
    rng = np.random.default_rng(2)
    codes, sc, bz, _ = lib.pack_affine(rng.standard_normal((64, 256)).astype(np.float32),
                                       bits=8, group=32)
    p = st_file.write(tmp_path / "g32.safetensors",
                      {PREFIX + "attn1.to_q.weight": codes, PREFIX + "attn1.to_q.scales": sc,
                       PREFIX + "attn1.to_q.biases": bz},
                      bf16=(PREFIX + "attn1.to_q.scales", PREFIX + "attn1.to_q.biases"))
    st = L.SafeTensors(p)
    blk = L.Block(ctx, CFG["vdim"], CFG["vheads"], CFG["adim"], CFG["aheads"])
    with pytest.raises(L.LtxError) as e:
        blk.load_st(st, PREFIX)
    assert e.value.code == -3
    blk.close()


def test_adapter_from_file_carries_alpha_over_rank(ctx, tmp_path):
    import torch
    import ltx25_b200 as L
    rng = np.random.default_rng(3)
    k, n, r = 256, 128, 12
    a, b = lora_np.make_pair(rng, r, k, n)
    mod = "diffusion_model.transformer_blocks.0.attn1.to_q"
    p = st_file.write(tmp_path / "lora.safetensors",
                      {mod + ".lora_A.weight": a, mod + ".lora_B.weight": b},
                      metadata={"lora_alpha": "6", "lora_rank": "12"},
                      bf16=(mod + ".lora_A.weight", mod + ".lora_B.weight"))
    st = L.SafeTensors(p)
    lo = L.lora_from_st(ctx, st, mod, k, n, lora_scale=0.8)
    assert lo.rank == r
    ref = L.Lora(ctx, _dev(a).view(torch.bfloat16), _dev(b).view(torch.bfloat16), scale=0.8 * 6 / 12)
    x = torch.from_numpy(rng.standard_normal((40, k)).astype(np.float32)).cuda().to(torch.bfloat16)
    y1 = torch.zeros((40, n), dtype=torch.bfloat16, device="cuda")
    y2 = torch.zeros_like(y1)
    L.lora_add(ctx, lo, x, y1)
    L.lora_add(ctx, ref, x, y2)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    with pytest.raises(L.LtxError) as e:
        L.lora_from_st(ctx, st, "diffusion_model.transformer_blocks.0.attn1.to_k", k, n)
    assert e.value.code == -7
    with pytest.raises(L.LtxError) as e:
        L.lora_from_st(ctx, st, mod, k, n + 2)
    assert e.value.code == -2
    st.close()
