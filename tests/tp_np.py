"""The tensor-parallel plan of the CUDA block, restated in numpy (test helper).

Megatron-style sharding over `world` ranks, as host/ltx25-block-cuda.cc
implements it:
  * q/k/v projections, their biases, the q/k RMSNorm gains and the per-head
    gate logits keep this rank's heads [rank*H/W, (rank+1)*H/W);
  * the RMSNorm over the WHOLE inner width needs the per-token sum of
    squares of all heads: each rank sums its columns, the sums are reduced;
  * the output projection keeps its K columns of this rank's heads; the
    partial products are reduced, then the bias and the gated residual are
    applied once;
  * ff.net.0 keeps hidden columns [rank*F/W, ...) (GELU is per column),
    ff.net.2 the same K columns, reduced like the output projections;
  * everything else (adaLN rows, modulation, norms of x) is replicated;
  * a runtime adapter (y += (x A^T) B^T, lora_np) follows its linear: on a
    column-split site A is whole and B keeps this rank's output rows; on a
    row-split site (to_out.0, ff.net.2) A keeps this rank's K columns, B is
    whole, and the delta joins the partial product before the reduction.

`block_forward_tp` with world == 1 is block_np.block_forward; with world > 1
it must equal it up to summation order, which tests/test_tp_cpu.py checks
over gloo ranks.
"""
import numpy as np

from oracle import block_np, lora_np, rope_np
from oracle.block_np import F32, F64

EPS = 1e-6


def _lin(lora, module, inp, w, b, rows=slice(None), kcols=slice(None)):
    """One sharded linear plus its adapter's share: output rows `rows` of
    the full linear, reading only input columns `kcols` (a row-split site's
    partial product, no bias there)."""
    y = block_np.linear(inp, w, b)
    pair = None if lora is None else lora.get(module)
    if pair is None:
        return y
    a, bb = pair
    return (y.astype(F64) + lora_np.delta(inp, a[:, kcols], bb[rows])).astype(F32)


def _attn_tp(t, prefix, x, ctx, pe, k_pe, heads, head_dim, rank, world, allreduce,
             lora=None):
    hl = heads // world
    il = hl * head_dim
    c0 = rank * il
    inner = heads * head_dim
    cols = slice(c0, c0 + il)
    w = lambda n: t.get(f"{prefix}.{n}")

    def lin(inp, name):
        wt = w(f"{name}.weight")
        b = w(f"{name}.bias")
        return _lin(lora, f"{prefix}.{name}", inp, wt[cols], None if b is None else b[cols],
                    rows=cols)

    q = lin(x, "to_q")
    k = lin(ctx, "to_k")
    v = lin(ctx, "to_v")
    ss = np.concatenate([(q.astype(F64) ** 2).sum(axis=1), (k.astype(F64) ** 2).sum(axis=1)])
    allreduce(ss)
    sq, sk = ss[:q.shape[0]], ss[q.shape[0]:]

    def norm(m, s, gain):
        out = m.astype(F64) / np.sqrt(s / inner + EPS)[:, None]
        return (out * np.asarray(gain, F32)[cols].astype(F64)[None, :]).astype(F32)

    q = norm(q, sq, w("q_norm.weight"))
    k = norm(k, sk, w("k_norm.weight"))
    hs = slice(rank * hl, (rank + 1) * hl)
    if pe is not None:
        rope_np.apply_rope(pe[0][hs], pe[1][hs], q, hl, head_dim)
        kt = k_pe if k_pe is not None else pe
        rope_np.apply_rope(kt[0][hs], kt[1][hs], k, hl, head_dim)
    att = block_np.sdpa(q, k, v, hl, head_dim)
    gw = w("to_gate_logits.weight")
    if gw is not None:
        gb = w("to_gate_logits.bias")
        g = _lin(lora, f"{prefix}.to_gate_logits", x, gw[hs], None if gb is None else gb[hs],
                 rows=hs)
        gate = (F32(2.0) / (F32(1.0) + np.exp(-g))).astype(F32)
        att = (att.reshape(att.shape[0], hl, head_dim) * gate[:, :, None]).astype(F32) \
            .reshape(att.shape)
    part = _lin(lora, f"{prefix}.to_out.0", att, w("to_out.0.weight")[:, cols], None,
                kcols=cols).astype(F64)
    allreduce(part)
    b = w("to_out.0.bias")
    return (part + (0.0 if b is None else np.asarray(b, F32).astype(F64))).astype(F32)


def _ff_tp(t, pre, xin, rank, world, allreduce, lora=None):
    wi = t[f"{pre}ff.net.0.proj.weight"]
    fl = wi.shape[0] // world
    cols = slice(rank * fl, (rank + 1) * fl)
    bi = t.get(f"{pre}ff.net.0.proj.bias")
    h = block_np.gelu_tanh(_lin(lora, f"{pre}ff.net.0.proj", xin, wi[cols],
                                None if bi is None else bi[cols], rows=cols))
    part = _lin(lora, f"{pre}ff.net.2", h, t[f"{pre}ff.net.2.weight"][:, cols], None,
                kcols=cols).astype(F64)
    allreduce(part)
    bo = t.get(f"{pre}ff.net.2.bias")
    return (part + (0.0 if bo is None else np.asarray(bo, F32).astype(F64))).astype(F32)


def _first_half(t, pre, s, dim, heads, tp):
    hd = dim // heads
    table = t[f"{pre}scale_shift_table"]
    msa = block_np.ada_values(table, s["timesteps"], dim, 0, 3)
    normed = block_np.ada_zero(s["x"], EPS, msa[1], msa[0])
    sa = _attn_tp(t, f"{pre}attn1", normed, normed, s.get("pe"), None, heads, hd, *tp)
    s["x"] = (s["x"] + sa * msa[2]).astype(F32)
    xn = block_np.rms_norm(s["x"], EPS)
    ca = block_np.ada_values(table, s["timesteps"], dim, 6, 9)
    qin = block_np.mod(xn, ca[1], ca[0])
    pst = np.asarray(t[f"{pre}prompt_scale_shift_table"], F32).ravel()
    shift, scale = pst[:dim].copy(), pst[dim:2 * dim].copy()
    pts = s.get("prompt_timestep")
    if pts is not None and np.asarray(pts).size >= 2 * dim:
        pts = np.asarray(pts, F32).ravel()
        shift = (shift + pts[:dim]).astype(F32)
        scale = (scale + pts[dim:2 * dim]).astype(F32)
    kv = block_np.mod(s["context"], scale, shift)
    co = _attn_tp(t, f"{pre}attn2", qin, kv, None, None, heads, hd, *tp)
    s["x"] = (s["x"] + co * ca[2]).astype(F32)


def _ff(t, pre, s, dim, tp):
    mlp = block_np.ada_values(t[f"{pre}scale_shift_table"], s["timesteps"], dim, 3, 6)
    scaled = block_np.ada_zero(s["x"], EPS, mlp[1], mlp[0])
    s["x"] = (s["x"] + _ff_tp(t, pre, scaled, *tp) * mlp[2]).astype(F32)


def block_forward_tp(t, video, audio, vdim, vheads, adim, aheads, rank, world, allreduce,
                     lora=None):
    """block_np.block_forward (src/ltx25-block-ref.cc:308-389) on one rank's
    shard; `allreduce(arr)` sums a float64 numpy array in place over ranks.
    `lora`: module -> (A [rank][K], B [N][rank]) f32 values of the FULL
    adapters (each rank takes its share), or None."""
    tp = (rank, world, allreduce, lora)
    v = dict(video)
    a = dict(audio)
    v["x"] = np.asarray(v["x"], F32).copy()
    a["x"] = np.asarray(a["x"], F32).copy()
    _first_half(t, "", v, vdim, vheads, tp)
    _first_half(t, "audio_", a, adim, aheads, tp)
    vx_pre, ax_pre = v["x"].copy(), a["x"].copy()
    ahd = adim // aheads
    vtab = t["scale_shift_table_a2v_ca_video"]
    atab = t["scale_shift_table_a2v_ca_audio"]
    vsc, vsh, vg = block_np.av_ada(vtab, v.get("cross_scale_shift"), v.get("cross_gate"), vdim, 0)
    asc, ash, _ = block_np.av_ada(atab, a.get("cross_scale_shift"), a.get("cross_gate"), adim, 0)
    qv = block_np.ada_zero(vx_pre, EPS, vsc, vsh)
    kv = block_np.ada_zero(ax_pre, EPS, asc, ash)
    o = _attn_tp(t, "audio_to_video_attn", qv, kv, v.get("cross_pe"), a.get("cross_pe"),
                 aheads, ahd, *tp)
    v["x"] = (v["x"] + o * vg).astype(F32)
    asc, ash, ag = block_np.av_ada(atab, a.get("cross_scale_shift"), a.get("cross_gate"), adim, 2)
    vsc, vsh, _ = block_np.av_ada(vtab, v.get("cross_scale_shift"), v.get("cross_gate"), vdim, 2)
    qa = block_np.ada_zero(ax_pre, EPS, asc, ash)
    kvv = block_np.ada_zero(vx_pre, EPS, vsc, vsh)
    o = _attn_tp(t, "video_to_audio_attn", qa, kvv, a.get("cross_pe"), v.get("cross_pe"),
                 aheads, ahd, *tp)
    a["x"] = (a["x"] + o * ag).astype(F32)
    _ff(t, "", v, vdim, tp)
    _ff(t, "audio_", a, adim, tp)
    return v["x"], a["x"]


# ---- the row-sharded residual (tensor parallel with the video x kept by
# token rows between blocks, host/ltx25-block-cuda.cc `rows` paths) --------
#
# Rank r holds video rows [r*T/W, (r+1)*T/W) of x.  Each modulated input
# (ada_zero, row-local) is formed for those rows and all-gathered (for the
# cross attentions x's rows are gathered once and both modulations formed
# on all rows); the
# sharded projections then see all T rows exactly as above; each row-split
# product is reduce-scattered (here: summed over ranks, then the rank keeps
# its rows) and the gated residual touches only the rank's rows.  The audio
# stream stays whole on every rank.  At the end the video rows are gathered.

def _rows(arr, rank, world):
    n = arr.shape[0] // world
    return arr[rank * n:(rank + 1) * n]


def block_forward_tp_rows(t, video, audio, vdim, vheads, adim, aheads, rank, world,
                          allreduce, allgather):
    """The same block with the video residual sharded by rows.
    `allgather(local)` returns the rows of all ranks stacked in rank order."""
    tp = (rank, world, allreduce, None)
    v = dict(video)
    a = dict(audio)
    vx = _rows(np.asarray(v["x"], F32), rank, world).copy()     # this rank's rows
    a["x"] = np.asarray(a["x"], F32).copy()
    hd = vdim // vheads
    table = t["scale_shift_table"]
    # video first half
    msa = block_np.ada_values(table, v["timesteps"], vdim, 0, 3)
    normed = allgather(block_np.ada_zero(vx, EPS, msa[1], msa[0]))
    sa = _attn_tp(t, "attn1", normed, normed, v.get("pe"), None, vheads, hd, *tp)
    vx = (vx + _rows(sa, rank, world) * msa[2]).astype(F32)
    ca = block_np.ada_values(table, v["timesteps"], vdim, 6, 9)
    qin = allgather(block_np.mod(block_np.rms_norm(vx, EPS), ca[1], ca[0]))
    pst = np.asarray(t["prompt_scale_shift_table"], F32).ravel()
    shift, scale = pst[:vdim].copy(), pst[vdim:2 * vdim].copy()
    pts = v.get("prompt_timestep")
    if pts is not None and np.asarray(pts).size >= 2 * vdim:
        pts = np.asarray(pts, F32).ravel()
        shift = (shift + pts[:vdim]).astype(F32)
        scale = (scale + pts[vdim:2 * vdim]).astype(F32)
    kv = block_np.mod(v["context"], scale, shift)
    co = _attn_tp(t, "attn2", qin, kv, None, None, vheads, hd, *tp)
    vx = (vx + _rows(co, rank, world) * ca[2]).astype(F32)
    # audio first half, whole
    _first_half(t, "audio_", a, adim, aheads, tp)
    # cross attentions from the pre-cross state
    vx_pre, ax_pre = allgather(vx), a["x"].copy()     # x's rows gathered once
    ahd = adim // aheads
    vtab = t["scale_shift_table_a2v_ca_video"]
    atab = t["scale_shift_table_a2v_ca_audio"]
    vsc, vsh, vg = block_np.av_ada(vtab, v.get("cross_scale_shift"), v.get("cross_gate"), vdim, 0)
    asc, ash, _ = block_np.av_ada(atab, a.get("cross_scale_shift"), a.get("cross_gate"), adim, 0)
    qv = block_np.ada_zero(vx_pre, EPS, vsc, vsh)
    kva = block_np.ada_zero(ax_pre, EPS, asc, ash)
    o = _attn_tp(t, "audio_to_video_attn", qv, kva, v.get("cross_pe"), a.get("cross_pe"),
                 aheads, ahd, *tp)
    vx = (vx + _rows(o, rank, world) * vg).astype(F32)
    asc, ash, ag = block_np.av_ada(atab, a.get("cross_scale_shift"), a.get("cross_gate"), adim, 2)
    vsc, vsh, _ = block_np.av_ada(vtab, v.get("cross_scale_shift"), v.get("cross_gate"), vdim, 2)
    qa = block_np.ada_zero(ax_pre, EPS, asc, ash)
    kvv = block_np.ada_zero(vx_pre, EPS, vsc, vsh)
    o = _attn_tp(t, "video_to_audio_attn", qa, kvv, a.get("cross_pe"), v.get("cross_pe"),
                 aheads, ahd, *tp)
    a["x"] = (a["x"] + o * ag).astype(F32)
    # feed-forwards
    mlp = block_np.ada_values(table, v["timesteps"], vdim, 3, 6)
    scaled = allgather(block_np.ada_zero(vx, EPS, mlp[1], mlp[0]))
    vx = (vx + _rows(_ff_tp(t, "", scaled, *tp), rank, world) * mlp[2]).astype(F32)
    _ff(t, "audio_", a, adim, tp)
    return allgather(vx), a["x"]
