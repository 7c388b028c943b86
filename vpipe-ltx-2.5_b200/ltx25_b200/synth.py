"""Seeded synthetic LTX-2.5 block weights and stream inputs, generated on
the device, under the reference's parameter names
(src/ltx25-block-ref.cc:424-523).  Used by bench.py and the stack runner
(there is no checkpoint here); matrices N(0, std) with std = 1/sqrt(fan_in)
by default (BASELINE's N(0, 0.02) for the 4096-wide linears is within 30% of
that), biases N(0, 0.02), norm gains 1 + N(0, 0.1), adaLN tables N(0, 0.1).
"""
import math


def tensor_specs(vdim, vheads, adim, aheads, ff_mult=4):
    """name -> (shape, kind); kind in {mat, bias, gain, table, gate, gate_b}."""
    specs = {}

    def attn(prefix, qdim, kvdim, inner, heads, odim):
        specs[f"{prefix}.to_q.weight"] = ((inner, qdim), "mat")
        specs[f"{prefix}.to_q.bias"] = ((inner,), "bias")
        specs[f"{prefix}.to_k.weight"] = ((inner, kvdim), "mat")
        specs[f"{prefix}.to_k.bias"] = ((inner,), "bias")
        specs[f"{prefix}.to_v.weight"] = ((inner, kvdim), "mat")
        specs[f"{prefix}.to_v.bias"] = ((inner,), "bias")
        specs[f"{prefix}.to_out.0.weight"] = ((odim, inner), "mat")
        specs[f"{prefix}.to_out.0.bias"] = ((odim,), "bias")
        specs[f"{prefix}.q_norm.weight"] = ((inner,), "gain")
        specs[f"{prefix}.k_norm.weight"] = ((inner,), "gain")
        specs[f"{prefix}.to_gate_logits.weight"] = ((heads, qdim), "gate")
        specs[f"{prefix}.to_gate_logits.bias"] = ((heads,), "gate_b")

    for pre, d, h in (("", vdim, vheads), ("audio_", adim, aheads)):
        attn(f"{pre}attn1", d, d, d, h, d)
        attn(f"{pre}attn2", d, d, d, h, d)
        specs[f"{pre}ff.net.0.proj.weight"] = ((ff_mult * d, d), "mat")
        specs[f"{pre}ff.net.2.weight"] = ((d, ff_mult * d), "mat")
        if pre == "audio_":
            specs[f"{pre}ff.net.0.proj.bias"] = ((ff_mult * d,), "bias")
            specs[f"{pre}ff.net.2.bias"] = ((d,), "bias")
        specs[f"{pre}scale_shift_table"] = ((9 * d,), "table")
        specs[f"{pre}prompt_scale_shift_table"] = ((2 * d,), "table")
    specs["scale_shift_table_a2v_ca_video"] = ((5 * vdim,), "table")
    specs["scale_shift_table_a2v_ca_audio"] = ((5 * adim,), "table")
    attn("audio_to_video_attn", vdim, adim, adim, aheads, vdim)
    attn("video_to_audio_attn", adim, vdim, adim, aheads, adim)
    return specs


def load_random_block(ctx, vdim, vheads, adim, aheads, seed, device="cuda",
                      effective=False):
    """A finalized ltx25_b200.Block with random weights made on the device.

    effective=True also returns the weights the device computes with, as
    host f32 numpy under the same names: the dequantized linears, the bf16
    biases and gate weights, the f32 gains and tables."""
    import torch
    from . import Block, QWeight, dequant, is_quantized_name, pack_w8g64
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    blk = Block(ctx, vdim, vheads, adim, aheads)
    eff = {}
    for name, (shape, kind) in tensor_specs(vdim, vheads, adim, aheads).items():
        t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
        if kind in ("mat", "gate"):
            t *= 1.0 / math.sqrt(shape[1])
        elif kind == "bias":
            t *= 0.02
        elif kind == "gain":
            t = 1.0 + 0.1 * t
        elif kind == "table":
            t *= 0.1
        elif kind == "gate_b":
            t *= 0.5
        if is_quantized_name(name, t.dim()):
            c, s, b = pack_w8g64(ctx, t)
            blk.set_qlinear(name, c, s, b, shape[0], shape[1])
            if effective:
                q = QWeight.upload(ctx, c, s, b, shape[0], shape[1], on_device=True)
                eff[name] = dequant(ctx, q).float().cpu().numpy()
                q.free()
            del c, s, b
        else:
            blk.set_tensor(name, t)
            if effective:
                bf16 = kind in ("bias", "gate", "gate_b")
                eff[name] = (t.to(torch.bfloat16).float() if bf16 else t).cpu().numpy()
        del t
    blk.finalize()
    return (blk, eff) if effective else blk


def video_grid(frames=16, height=17, width=30):
    return frames, height, width


def random_stream_inputs(dim, tokens, text_tokens, heads, gen, device="cuda",
                         pe=None, cross_pe=None):
    """Device inputs of one stream (bf16 activations and adaLN drivers)."""
    import torch

    def n(*shape, s=1.0):
        return (torch.randn(shape, generator=gen, device=device) * s).to(torch.bfloat16)

    return {
        "x": n(tokens, dim), "context": n(text_tokens, dim),
        "timesteps": n(9 * dim, s=0.1), "cross_scale_shift": n(4 * dim, s=0.1),
        "cross_gate": n(dim, s=0.1), "prompt_timestep": n(2 * dim, s=0.1),
        "pe": pe, "cross_pe": cross_pe, "present": True,
    }


def connector_tensors(dim, heads, layers, registers, seed=0, device="cuda", gated=True):
    """Random embeddings-connector weights under the reference's names, as
    device f32 tensors (fan-in scaled linears, small biases, unit-ish norm
    gains, N(0, 1) registers)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    n = lambda *s, sc=0.02: torch.randn(s, generator=g, device=device) * sc
    t = {}
    if registers > 0:
        t["learnable_registers"] = n(registers, dim, sc=1.0)
    for i in range(layers):
        p = f"transformer_1d_blocks.{i}."
        for m in ("to_q", "to_k", "to_v", "to_out.0"):
            t[p + f"attn1.{m}.weight"] = n(dim, dim, sc=dim ** -0.5)
            t[p + f"attn1.{m}.bias"] = n(dim)
        t[p + "attn1.q_norm.weight"] = 1.0 + n(dim, sc=0.1)
        t[p + "attn1.k_norm.weight"] = 1.0 + n(dim, sc=0.1)
        if gated:
            t[p + "attn1.to_gate_logits.weight"] = n(heads, dim, sc=dim ** -0.5)
            t[p + "attn1.to_gate_logits.bias"] = n(heads)
        t[p + "ff.net.0.proj.weight"] = n(4 * dim, dim, sc=dim ** -0.5)
        t[p + "ff.net.0.proj.bias"] = n(4 * dim)
        t[p + "ff.net.2.weight"] = n(dim, 4 * dim, sc=(4 * dim) ** -0.5)
        t[p + "ff.net.2.bias"] = n(dim)
    return t
