"""numpy restatement of the reference's RoPE (src/ltx25-rope.cc).

TEST INFRASTRUCTURE ONLY.  Tables are [heads][tokens][half] f32 (cos, sin).
Pinned against the reference's compiled builders by tests/test_oracle.py
through tests/golden/rope.npz (angles in f32 exactly as the reference forms
them; cos/sin of an f32 angle evaluated in f64 and rounded once, within
1 ulp of the reference's f32 cos/sin).
"""
import math

import numpy as np


def freq_ladder(theta, n_axes, inner_dim, f64_precision=True):
    """theta ** linspace(0, 1, n) * pi / 2, narrowed to f32
    (src/ltx25-rope.cc:46-70)."""
    n = inner_dim // (2 * n_axes)
    if n <= 0:
        return np.zeros(0, np.float32)
    i = np.arange(n, dtype=np.float64)
    if f64_precision:
        t = np.zeros(n) if n == 1 else i / (n - 1)
        return (np.power(theta, t) * math.pi / 2.0).astype(np.float32)
    step = np.float32(0.0) if n == 1 else np.float32(1.0) / np.float32(n - 1)
    t = i.astype(np.float32) * step
    v = np.power(np.float32(theta), t).astype(np.float32)
    v = (v * np.float32(math.pi)).astype(np.float32)
    return (v / np.float32(2.0)).astype(np.float32)


def build_rope(starts, ends, max_pos, inner_dim, heads, theta=10000.0,
               f64_precision=True):
    """src/ltx25-rope.cc:74-165."""
    n_axes = len(starts)
    if n_axes == 0 or len(ends) != n_axes or len(max_pos) != n_axes:
        raise ValueError("axis count mismatch")
    tokens = len(starts[0])
    head_dim = inner_dim // heads
    half = head_dim // 2
    ladder = freq_ladder(theta, n_axes, inner_dim, f64_precision)
    n_freq = ladder.size
    used = n_freq * n_axes
    pad = half * heads - used
    if pad < 0:
        raise ValueError("frequency table overruns head_dim/2 * heads")
    row_cos = np.ones((tokens, pad + used), np.float32)
    row_sin = np.zeros((tokens, pad + used), np.float32)
    for a in range(n_axes):
        s = np.asarray(starts[a], np.float64)
        e = np.asarray(ends[a], np.float64)
        mid = ((s + e) * 0.5).astype(np.float32)
        frac = (mid / np.float32(max_pos[a])).astype(np.float32)
        fr = (frac * np.float32(2.0) - np.float32(1.0)).astype(np.float32)
        ang = (ladder[None, :] * fr[:, None]).astype(np.float32)  # [T][F]
        cols = pad + np.arange(n_freq) * n_axes + a
        row_cos[:, cols] = np.cos(ang.astype(np.float64)).astype(np.float32)
        row_sin[:, cols] = np.sin(ang.astype(np.float64)).astype(np.float32)
    cos = row_cos[:, : half * heads].reshape(tokens, heads, half)
    sin = row_sin[:, : half * heads].reshape(tokens, heads, half)
    return (np.ascontiguousarray(cos.transpose(1, 0, 2)),
            np.ascontiguousarray(sin.transpose(1, 0, 2)))


def video_spans(frames, height, width, scale=(8, 32, 32), fps=24.0,
                causal_fix=True, pixel_frame_offset=0, single_pixel_frame=False):
    """src/ltx25-rope.cc:180-247: per-token (start, end) in seconds/pixels,
    (f, h, w) with w fastest."""
    st, sh, sw = scale
    tsec, tend = [], []
    for f in range(frames):
        t = float(f * st)
        e = float((f + 1) * st)
        if causal_fix:
            t = max(t + 1.0 - st, 0.0)
            e = max(e + 1.0 - st, 0.0)
        t += pixel_frame_offset
        e += pixel_frame_offset
        if single_pixel_frame:
            e = t + 1.0
        tsec.append(t / fps)
        tend.append(e / fps)
    f_idx, h_idx, w_idx = np.meshgrid(np.arange(frames), np.arange(height),
                                      np.arange(width), indexing="ij")
    f_idx, h_idx, w_idx = f_idx.ravel(), h_idx.ravel(), w_idx.ravel()
    starts = [np.asarray(tsec)[f_idx], h_idx * float(sh), w_idx * float(sw)]
    ends = [np.asarray(tend)[f_idx], (h_idx + 1) * float(sh),
            (w_idx + 1) * float(sw)]
    return starts, ends


def build_video_rope(frames, height, width, max_pos, inner_dim, heads,
                     scale=(8, 32, 32), fps=24.0, causal_fix=True):
    s, e = video_spans(frames, height, width, scale, fps, causal_fix)
    return build_rope(s, e, max_pos, inner_dim, heads)


def video_time_seconds(frames, scale_t=8, fps=24.0, causal_fix=True):
    """src/ltx25-rope.cc:249-260."""
    out = []
    for f in range(frames):
        t = float(f * scale_t)
        if causal_fix:
            t = t + 1.0 - scale_t
        out.append((0.0 if t < 0 else t) / fps)
    return np.asarray(out, np.float64)


def audio_time_seconds(tokens, downsample=4, hop=160, sample_rate=16000,
                       causal=True):
    """src/ltx25-rope.cc:262-276."""
    per = hop / sample_rate if sample_rate > 0 else 0.0
    out = []
    for t in range(tokens):
        mel = float(t * downsample)
        if causal:
            mel = mel + 1.0 - downsample
        out.append((0.0 if mel < 0 else mel) * per)
    return np.asarray(out, np.float64)


def build_audio_rope(tokens, max_pos, inner_dim, heads):
    """src/ltx25-rope.cc:282-296: 1-D, positions in seconds."""
    t0 = audio_time_seconds(tokens)
    t1 = audio_time_seconds(tokens + 1)[1:]
    return build_rope([t0], [t1], [max_pos], inner_dim, heads)


def build_index_rope(tokens, max_pos, inner_dim, heads):
    """src/ltx25-rope.cc:278-280 (raw indices; the goldens' arange grid)."""
    i = np.arange(tokens, dtype=np.float64)
    return build_rope([i], [i + 1.0], [max_pos], inner_dim, heads)


def build_cross_rope(starts, ends, max_pos, inner_dim, heads):
    """src/ltx25-rope.cc:298-323: the time-only a2v/v2a table."""
    return build_rope([np.asarray(starts)], [np.asarray(ends)], [max_pos],
                      inner_dim, heads)


def apply_rope(cos, sin, x, heads, head_dim):
    """Split-half rotation in place on x [tokens][heads*head_dim] f32
    (src/ltx25-rope.cc:325-352).  Returns x."""
    tokens = x.shape[0]
    half = head_dim // 2
    v = x.reshape(tokens, heads, head_dim)
    c = cos.transpose(1, 0, 2)
    s = sin.transpose(1, 0, 2)
    a = v[:, :, :half].copy()
    b = v[:, :, half:].copy()
    v[:, :, :half] = a * c - b * s
    v[:, :, half:] = b * c + a * s
    return x
