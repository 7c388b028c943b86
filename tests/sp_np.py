"""The sequence-parallel plan of the CUDA block, restated in numpy (test helper).

As host/ltx25-block-cuda.cc implements it for `world` ranks (every rank holds
the whole weights):
  * rank r owns video tokens [r T/W, (r+1) T/W): adaLN modulation, every video
    GEMM, the text and audio->video cross attentions and the feed-forward run
    on those rows only (their keys and values -- text, audio -- are
    replicated);
  * the video self-attention needs every token: q, k and v of the local rows
    (all heads, normed and rotated with the rows' GLOBAL RoPE positions) are
    exchanged so that rank r holds every token of heads [r H/W, (r+1) H/W),
    attends, and the outputs come back to their rows (the all-to-alls), the
    per-head gate applied on the way back;
  * video->audio: the audio queries are replicated, the video keys/values
    are exchanged to their heads' owners, each rank attends its heads and the
    outputs are gathered;
  * the 126-token audio stream is computed identically on every rank.
The exchanges are restated with gloo all-gathers (each rank then keeps the
slice an all-to-all would have delivered).  `block_forward_sp` must equal
block_np.block_forward on the gathered rows; tests/test_sp_cpu.py checks it.
"""
import numpy as np

from oracle import block_np, rope_np
from oracle.block_np import F32, F64

EPS = 1e-6


def _gather_rows(arr, world, allgather):
    """All ranks' row blocks in rank order (the receive side of the
    exchanges)."""
    return np.concatenate(allgather(arr), axis=0)


def _proj(t, prefix, name, x):
    return block_np.linear(x, t[f"{prefix}.{name}.weight"], t.get(f"{prefix}.{name}.bias"))


def _norm_rope(m, gain, pe, rows0, heads, hd):
    m = block_np.rms_norm_gain(m, gain)
    if pe is not None:
        cos, sin = pe
        n = m.shape[0]
        rope_np.apply_rope(cos[:, rows0:rows0 + n], sin[:, rows0:rows0 + n], m, heads, hd)
    return m


def _gate(t, prefix, x, heads):
    g = block_np.linear(x, t[f"{prefix}.to_gate_logits.weight"],
                        t.get(f"{prefix}.to_gate_logits.bias"))
    return (F32(2.0) / (F32(1.0) + np.exp(-g))).astype(F32)


def _self_attn_sp(t, prefix, x_loc, pe, row0, heads, hd, rank, world, allgather):
    q = _norm_rope(_proj(t, prefix, "to_q", x_loc), t[f"{prefix}.q_norm.weight"], pe, row0,
                   heads, hd)
    k = _norm_rope(_proj(t, prefix, "to_k", x_loc), t[f"{prefix}.k_norm.weight"], pe, row0,
                   heads, hd)
    v = _proj(t, prefix, "to_v", x_loc)
    hl = heads // world
    cols = slice(rank * hl * hd, (rank + 1) * hl * hd)
    # all-to-all: every token, this rank's heads
    qh = _gather_rows(q, world, allgather)[:, cols]
    kh = _gather_rows(k, world, allgather)[:, cols]
    vh = _gather_rows(v, world, allgather)[:, cols]
    oh = block_np.sdpa(qh, kh, vh, hl, hd)
    # all-to-all back: this rank's rows, every head
    allh = allgather(oh)                     # [rank][tokens][hl*hd]
    n = x_loc.shape[0]
    att = np.concatenate([a[row0:row0 + n] for a in allh], axis=1)
    g = _gate(t, prefix, x_loc, heads)
    att = (att.reshape(n, heads, hd) * g[:, :, None]).astype(F32).reshape(n, heads * hd)
    return block_np.linear(att, t[f"{prefix}.to_out.0.weight"], t.get(f"{prefix}.to_out.0.bias"))


def _v2a_sp(t, prefix, qa_in, a_pe, kv_loc, v_pe, row0, heads, hd, rank, world, allgather):
    q = _norm_rope(_proj(t, prefix, "to_q", qa_in), t[f"{prefix}.q_norm.weight"], a_pe, 0,
                   heads, hd)
    k = _norm_rope(_proj(t, prefix, "to_k", kv_loc), t[f"{prefix}.k_norm.weight"], v_pe, row0,
                   heads, hd)
    v = _proj(t, prefix, "to_v", kv_loc)
    hl = heads // world
    cols = slice(rank * hl * hd, (rank + 1) * hl * hd)
    kh = _gather_rows(k, world, allgather)[:, cols]
    vh = _gather_rows(v, world, allgather)[:, cols]
    oh = block_np.sdpa(q[:, cols], kh, vh, hl, hd)
    att = np.concatenate(allgather(oh), axis=1)      # gather the heads
    g = _gate(t, prefix, qa_in, heads)
    n = qa_in.shape[0]
    att = (att.reshape(n, heads, hd) * g[:, :, None]).astype(F32).reshape(n, heads * hd)
    return block_np.linear(att, t[f"{prefix}.to_out.0.weight"], t.get(f"{prefix}.to_out.0.bias"))


def block_forward_sp(t, video, audio, vdim, vheads, adim, aheads, rank, world, allgather):
    """block_np.block_forward (src/ltx25-block-ref.cc:308-389) with this
    rank's video rows; returns (this rank's video rows, audio x).
    `allgather(arr)` returns the list of every rank's `arr`."""
    tv = np.asarray(video["x"]).shape[0]
    tl = tv // world
    row0 = rank * tl
    v = dict(video)
    a = dict(audio)
    v["x"] = np.asarray(video["x"], F32)[row0:row0 + tl].copy()
    a["x"] = np.asarray(a["x"], F32).copy()
    vhd, ahd = vdim // vheads, adim // aheads

    # video first half: self-attention across ranks, text cross local
    table = t["scale_shift_table"]
    msa = block_np.ada_values(table, v["timesteps"], vdim, 0, 3)
    normed = block_np.ada_zero(v["x"], EPS, msa[1], msa[0])
    sa = _self_attn_sp(t, "attn1", normed, v.get("pe"), row0, vheads, vhd, rank, world,
                       allgather)
    v["x"] = (v["x"] + sa * msa[2]).astype(F32)
    xn = block_np.rms_norm(v["x"], EPS)
    ca = block_np.ada_values(table, v["timesteps"], vdim, 6, 9)
    qin = block_np.mod(xn, ca[1], ca[0])
    pst = np.asarray(t["prompt_scale_shift_table"], F32).ravel()
    shift, scale = pst[:vdim].copy(), pst[vdim:2 * vdim].copy()
    pts = np.asarray(v["prompt_timestep"], F32).ravel()
    shift = (shift + pts[:vdim]).astype(F32)
    scale = (scale + pts[vdim:2 * vdim]).astype(F32)
    kv = block_np.mod(v["context"], scale, shift)
    co = block_np.attention(block_np._attn_params(t, "attn2"), qin, kv, None, None, vheads, vhd)
    v["x"] = (v["x"] + co * ca[2]).astype(F32)

    # audio first half: replicated
    block_np.stream_first_half(t, "audio_", a, adim, aheads, EPS)

    # cross attentions on the pre-cross state
    vx_pre, ax_pre = v["x"].copy(), a["x"].copy()
    vtab = t["scale_shift_table_a2v_ca_video"]
    atab = t["scale_shift_table_a2v_ca_audio"]
    vsc, vsh, vg = block_np.av_ada(vtab, v.get("cross_scale_shift"), v.get("cross_gate"), vdim, 0)
    asc, ash, _ = block_np.av_ada(atab, a.get("cross_scale_shift"), a.get("cross_gate"), adim, 0)
    qv = block_np.ada_zero(vx_pre, EPS, vsc, vsh)
    kva = block_np.ada_zero(ax_pre, EPS, asc, ash)
    vcpe = v.get("cross_pe")
    vcpe_loc = (vcpe[0][:, row0:row0 + tl], vcpe[1][:, row0:row0 + tl])
    o = block_np.attention(block_np._attn_params(t, "audio_to_video_attn"), qv, kva, vcpe_loc,
                           a.get("cross_pe"), aheads, ahd)
    v["x"] = (v["x"] + o * vg).astype(F32)
    asc, ash, ag = block_np.av_ada(atab, a.get("cross_scale_shift"), a.get("cross_gate"), adim, 2)
    vsc, vsh, _ = block_np.av_ada(vtab, v.get("cross_scale_shift"), v.get("cross_gate"), vdim, 2)
    qa = block_np.ada_zero(ax_pre, EPS, asc, ash)
    kvv = block_np.ada_zero(vx_pre, EPS, vsc, vsh)
    o = _v2a_sp(t, "video_to_audio_attn", qa, a.get("cross_pe"), kvv, vcpe, row0, aheads, ahd,
                rank, world, allgather)
    a["x"] = (a["x"] + o * ag).astype(F32)

    block_np.stream_ff(t, "", v, vdim, EPS)
    block_np.stream_ff(t, "audio_", a, adim, EPS)
    return v["x"], a["x"]
