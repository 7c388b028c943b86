"""numpy restatement of the reference's CPU block (src/ltx25-block-ref.cc).

TEST INFRASTRUCTURE ONLY.  Same math as block_forward: f32 storage, f64 dot
products (linear_, sdpa_), f64 row statistics, f32 elementwise updates.
Pinned against the reference's compiled block_forward by
tests/test_oracle.py (tests/golden/block_small.npz, rel-L2 < 1e-5).

Weights are a name -> array map using the reference's own parameter names
(load_block_weights, src/ltx25-block-ref.cc:424-523).  A stream input is a
dict with keys x, context, timesteps, cross_scale_shift, cross_gate,
prompt_timestep, pe, cross_pe ((cos, sin) tables), present.
"""
import numpy as np

from . import rope_np

F32 = np.float32
F64 = np.float64
EPS = 1e-6


def linear(x, w, b=None):
    """src/ltx25-block-ref.cc:13-29."""
    y = np.asarray(x, F32).astype(F64) @ np.asarray(w, F32).astype(F64).T
    if b is not None and len(b) > 0:
        y += np.asarray(b, F32).astype(F64)
    return y.astype(F32)


def rms_norm_gain(m, gain, eps=1e-6):
    """src/ltx25-block-ref.cc:31-45: RMSNorm over the WHOLE row."""
    m64 = m.astype(F64)
    inv = 1.0 / np.sqrt((m64 * m64).sum(axis=1) / m.shape[1] + eps)
    out = m64 * inv[:, None]
    if gain is not None and len(gain) > 0:
        out = out * np.asarray(gain, F32).astype(F64)[None, :]
    return out.astype(F32)


def rms_norm(x, eps):
    """src/ltx25-block-ref.cc:149-157."""
    return rms_norm_gain(x, None, eps)


def sdpa(q, k, v, heads, head_dim):
    """src/ltx25-block-ref.cc:49-86: dense softmax attention, f64."""
    out = np.zeros((q.shape[0], heads * head_dim), F32)
    scale = 1.0 / np.sqrt(float(head_dim))
    for h in range(heads):
        sl = slice(h * head_dim, (h + 1) * head_dim)
        qh = q[:, sl].astype(F64)
        kh = k[:, sl].astype(F64)
        vh = v[:, sl].astype(F64)
        lg = (qh @ kh.T) * scale
        lg -= lg.max(axis=1, keepdims=True)
        p = np.exp(lg)
        out[:, sl] = ((p @ vh) / p.sum(axis=1, keepdims=True)).astype(F32)
    return out


def attention(w, x, ctx, pe, k_pe, heads, head_dim):
    """src/ltx25-block-ref.cc:90-130."""
    q = linear(x, w["to_q.weight"], w.get("to_q.bias"))
    k = linear(ctx, w["to_k.weight"], w.get("to_k.bias"))
    v = linear(ctx, w["to_v.weight"], w.get("to_v.bias"))
    q = rms_norm_gain(q, w.get("q_norm.weight"))
    k = rms_norm_gain(k, w.get("k_norm.weight"))
    if pe is not None:
        rope_np.apply_rope(pe[0], pe[1], q, heads, head_dim)
        kt = k_pe if k_pe is not None else pe
        rope_np.apply_rope(kt[0], kt[1], k, heads, head_dim)
    att = sdpa(q, k, v, heads, head_dim)
    if w.get("to_gate_logits.weight") is not None:
        g = linear(x, w["to_gate_logits.weight"], w.get("to_gate_logits.bias"))
        gate = (F32(2.0) / (F32(1.0) + np.exp(-g))).astype(F32)
        att = (att.reshape(att.shape[0], heads, head_dim) *
               gate[:, :, None]).astype(F32).reshape(att.shape)
    return linear(att, w["to_out.0.weight"], w.get("to_out.0.bias"))


def mod(x, scale, shift):
    """src/ltx25-block-ref.cc:134-145: x * (1 + scale) + shift, f32."""
    return (x * (F32(1.0) + np.asarray(scale, F32)) + np.asarray(shift, F32)).astype(F32)


def ada_zero(x, eps, scale, shift):
    """src/ltx25-block-ref.cc:159-165."""
    return mod(rms_norm(x, eps), scale, shift)


def ada_values(table, ts, dim, lo, hi):
    """src/ltx25-block-ref.cc:167-188: table[i] + timesteps[i], i in [lo, hi)."""
    table = np.asarray(table, F32).ravel()
    ts = np.zeros(0, F32) if ts is None else np.asarray(ts, F32).ravel()
    rows = []
    for i in range(lo, hi):
        a = np.zeros(dim, F32)
        b = np.zeros(dim, F32)
        seg = table[i * dim:(i + 1) * dim]
        a[:seg.size] = seg
        seg = ts[i * dim:(i + 1) * dim]
        b[:seg.size] = seg
        rows.append((a + b).astype(F32))
    return rows


def _attn_params(t, prefix):
    keys = ["to_q.weight", "to_q.bias", "to_k.weight", "to_k.bias",
            "to_v.weight", "to_v.bias", "to_out.0.weight", "to_out.0.bias",
            "q_norm.weight", "k_norm.weight", "to_gate_logits.weight",
            "to_gate_logits.bias"]
    return {k: t.get(f"{prefix}.{k}") for k in keys}


def _upd(x, sub, gate, x_round):
    y = (x + sub * gate).astype(F32)
    return x_round(y) if x_round is not None else y


def stream_first_half(t, pre, s, dim, heads, eps, x_round=None):
    """src/ltx25-block-ref.cc:196-262."""
    hd = dim // heads
    table = t[f"{pre}scale_shift_table"]
    msa = ada_values(table, s["timesteps"], dim, 0, 3)
    normed = ada_zero(s["x"], eps, msa[1], msa[0])
    sa = attention(_attn_params(t, f"{pre}attn1"), normed, normed, s.get("pe"),
                   None, heads, hd)
    s["x"] = _upd(s["x"], sa, msa[2], x_round)
    xn = rms_norm(s["x"], eps)
    ca = ada_values(table, s["timesteps"], dim, 6, 9)
    qin = mod(xn, ca[1], ca[0])
    pst = np.asarray(t[f"{pre}prompt_scale_shift_table"], F32).ravel()
    shift = pst[:dim].copy()
    scale = pst[dim:2 * dim].copy()
    pts = s.get("prompt_timestep")
    if pts is not None and np.asarray(pts).size >= 2 * dim:
        pts = np.asarray(pts, F32).ravel()
        shift = (shift + pts[:dim]).astype(F32)
        scale = (scale + pts[dim:2 * dim]).astype(F32)
    kv = mod(s["context"], scale, shift)
    co = attention(_attn_params(t, f"{pre}attn2"), qin, kv, None, None, heads, hd)
    s["x"] = _upd(s["x"], co, ca[2], x_round)


def gelu_tanh(h):
    """src/ltx25-block-ref.cc:266-272, in f64."""
    x = h.astype(F64)
    u = 0.7978845608028654 * (x + 0.044715 * x * x * x)
    return (0.5 * x * (1.0 + np.tanh(u))).astype(F32)


def stream_ff(t, pre, s, dim, eps, x_round=None):
    """src/ltx25-block-ref.cc:264-281."""
    table = t[f"{pre}scale_shift_table"]
    mlp = ada_values(table, s["timesteps"], dim, 3, 6)
    scaled = ada_zero(s["x"], eps, mlp[1], mlp[0])
    h = linear(scaled, t[f"{pre}ff.net.0.proj.weight"],
               t.get(f"{pre}ff.net.0.proj.bias"))
    h = gelu_tanh(h)
    o = linear(h, t[f"{pre}ff.net.2.weight"], t.get(f"{pre}ff.net.2.bias"))
    s["x"] = _upd(s["x"], o, mlp[2], x_round)


def av_ada(table, css, cg, dim, lo):
    """src/ltx25-block-ref.cc:283-303: (scale, shift, gate)."""
    ss = ada_values(table, css, dim, lo, lo + 2)
    table = np.asarray(table, F32).ravel()
    cg = np.zeros(dim, F32) if cg is None else np.asarray(cg, F32).ravel()
    gate = (table[4 * dim:5 * dim] + cg[:dim]).astype(F32)
    return ss[0], ss[1], gate


def block_forward(t, video, audio, vdim, vheads, adim, aheads, eps=EPS,
                  x_round=None):
    """src/ltx25-block-ref.cc:308-389.  Returns (video_x, audio_x); the
    input dicts are not modified.  `x_round`, when given, is applied to the
    residual stream after every update -- to model a device that stores x
    in bf16 (the reference's GPU block does); None is the reference's f32."""
    v = dict(video)
    a = dict(audio)
    v["x"] = np.asarray(v["x"], F32).copy()
    a["x"] = np.asarray(a["x"], F32).copy()
    rv = v.get("present", True) and v["x"].shape[0] > 0
    ra = a.get("present", True) and a["x"].shape[0] > 0
    if not rv and not ra:
        raise ValueError("neither stream is present")
    if rv:
        stream_first_half(t, "", v, vdim, vheads, eps, x_round)
    if ra:
        stream_first_half(t, "audio_", a, adim, aheads, eps, x_round)
    if rv and ra:
        vx_pre = v["x"].copy()
        ax_pre = a["x"].copy()
        ahd = adim // aheads
        vtab = t["scale_shift_table_a2v_ca_video"]
        atab = t["scale_shift_table_a2v_ca_audio"]
        vsc, vsh, vg = av_ada(vtab, v.get("cross_scale_shift"), v.get("cross_gate"), vdim, 0)
        asc, ash, _ = av_ada(atab, a.get("cross_scale_shift"), a.get("cross_gate"), adim, 0)
        qv = ada_zero(vx_pre, eps, vsc, vsh)
        kv = ada_zero(ax_pre, eps, asc, ash)
        o = attention(_attn_params(t, "audio_to_video_attn"), qv, kv,
                      v.get("cross_pe"), a.get("cross_pe"), aheads, ahd)
        v["x"] = _upd(v["x"], o, vg, x_round)
        asc, ash, ag = av_ada(atab, a.get("cross_scale_shift"), a.get("cross_gate"), adim, 2)
        vsc, vsh, _ = av_ada(vtab, v.get("cross_scale_shift"), v.get("cross_gate"), vdim, 2)
        qa = ada_zero(ax_pre, eps, asc, ash)
        kvv = ada_zero(vx_pre, eps, vsc, vsh)
        o = attention(_attn_params(t, "video_to_audio_attn"), qa, kvv,
                      a.get("cross_pe"), v.get("cross_pe"), aheads, ahd)
        a["x"] = _upd(a["x"], o, ag, x_round)
    if rv:
        stream_ff(t, "", v, vdim, eps, x_round)
    if ra:
        stream_ff(t, "audio_", a, adim, eps, x_round)
    return v["x"], a["x"]


# ---- seeded synthetic weights and inputs ---------------------------------

def random_block_tensors(vdim, vheads, adim, aheads, seed=0, ff_mult=4,
                         w_std=None, f32_draws=False):
    """Random-init weights under the reference's names.  Matrices are
    N(0, w_std) (default 1/sqrt(fan_in)); biases N(0, 0.02); norm gains
    1 + N(0, 0.1); adaLN tables N(0, 0.1); gate logits N(0, 1/sqrt(in)).
    The video feed-forward has no bias, the audio one does
    (src/ltx25-dit-weights.cc:482-486).  f32_draws draws the matrices in f32
    (other values, same distribution; for timing at the real widths)."""
    rng = np.random.default_rng(seed)

    def mat(o, i):
        s = w_std if w_std is not None else 1.0 / np.sqrt(i)
        if f32_draws:
            m = rng.standard_normal((o, i), dtype=F32)
            m *= F32(s)
            return m
        return (rng.standard_normal((o, i)) * s).astype(F32)

    def vec(n, s=0.02, mean=0.0):
        return (mean + rng.standard_normal(n) * s).astype(F32)

    t = {}

    def attn(prefix, qdim, kvdim, inner, heads, odim):
        t[f"{prefix}.to_q.weight"] = mat(inner, qdim)
        t[f"{prefix}.to_q.bias"] = vec(inner)
        t[f"{prefix}.to_k.weight"] = mat(inner, kvdim)
        t[f"{prefix}.to_k.bias"] = vec(inner)
        t[f"{prefix}.to_v.weight"] = mat(inner, kvdim)
        t[f"{prefix}.to_v.bias"] = vec(inner)
        t[f"{prefix}.to_out.0.weight"] = mat(odim, inner)
        t[f"{prefix}.to_out.0.bias"] = vec(odim)
        t[f"{prefix}.q_norm.weight"] = vec(inner, 0.1, 1.0)
        t[f"{prefix}.k_norm.weight"] = vec(inner, 0.1, 1.0)
        t[f"{prefix}.to_gate_logits.weight"] = (rng.standard_normal((heads, qdim)) / np.sqrt(qdim)).astype(F32)
        t[f"{prefix}.to_gate_logits.bias"] = vec(heads, 0.5)

    for pre, d, h in (("", vdim, vheads), ("audio_", adim, aheads)):
        attn(f"{pre}attn1", d, d, d, h, d)
        attn(f"{pre}attn2", d, d, d, h, d)
        t[f"{pre}ff.net.0.proj.weight"] = mat(ff_mult * d, d)
        t[f"{pre}ff.net.2.weight"] = mat(d, ff_mult * d)
        if pre == "audio_":
            t[f"{pre}ff.net.0.proj.bias"] = vec(ff_mult * d)
            t[f"{pre}ff.net.2.bias"] = vec(d)
        t[f"{pre}scale_shift_table"] = vec(9 * d, 0.1)
        t[f"{pre}prompt_scale_shift_table"] = vec(2 * d, 0.1)
    t["scale_shift_table_a2v_ca_video"] = vec(5 * vdim, 0.1)
    t["scale_shift_table_a2v_ca_audio"] = vec(5 * adim, 0.1)
    attn("audio_to_video_attn", vdim, adim, adim, aheads, vdim)
    attn("video_to_audio_attn", adim, vdim, adim, aheads, adim)
    return t


def random_block_inputs(cfg, seed=0, index_rope=False, video_grid=None):
    """Seeded stream inputs.  cfg: vdim, vheads, adim, aheads, vt, at, tt.
    index_rope: the reference goldens' arange tables
    (tests/ltx25-block-metal-test.cc:186-192); otherwise real geometry
    tables (video_grid = (frames, height, width), audio in seconds)."""
    rng = np.random.default_rng(seed)
    vd, vh, ad, ah = cfg["vdim"], cfg["vheads"], cfg["adim"], cfg["aheads"]
    vt, at, tt = cfg["vt"], cfg["at"], cfg["tt"]

    def n(*shape, s=1.0):
        return (rng.standard_normal(shape) * s).astype(F32)

    if index_rope:
        vpe = rope_np.build_index_rope(vt, 20, vd, vh)
        ape = rope_np.build_index_rope(at, 20, ad, ah)
        vcpe = rope_np.build_index_rope(vt, 20, ad, ah)
        acpe = ape
    else:
        f, hh, ww = video_grid
        assert f * hh * ww == vt
        vpe = rope_np.build_video_rope(f, hh, ww, [20, 2048, 2048], vd, vh)
        ape = rope_np.build_audio_rope(at, 20, ad, ah)
        vts = rope_np.video_time_seconds(f)
        vte = rope_np.video_time_seconds(f + 1)[1:]
        per = hh * ww
        vcpe = rope_np.build_cross_rope(np.repeat(vts, per), np.repeat(vte, per),
                                        20, ad, ah)
        a0 = rope_np.audio_time_seconds(at)
        a1 = rope_np.audio_time_seconds(at + 1)[1:]
        acpe = rope_np.build_cross_rope(a0, a1, 20, ad, ah)
    video = dict(x=n(vt, vd), context=n(tt, vd), timesteps=n(9 * vd, s=0.1),
                 cross_scale_shift=n(4 * vd, s=0.1), cross_gate=n(vd, s=0.1),
                 prompt_timestep=n(2 * vd, s=0.1), pe=vpe, cross_pe=vcpe,
                 present=True)
    audio = dict(x=n(at, ad), context=n(tt, ad), timesteps=n(9 * ad, s=0.1),
                 cross_scale_shift=n(4 * ad, s=0.1), cross_gate=n(ad, s=0.1),
                 prompt_timestep=n(2 * ad, s=0.1), pe=ape, cross_pe=acpe,
                 present=True)
    return {"video": video, "audio": audio}
