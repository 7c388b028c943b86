"""The DiT trunk's patchify and output head restated in numpy (TEST
INFRASTRUCTURE ONLY).

Follows Ltx25Dit's trunk (src/ltx25-dit.cc:1509-1540, 2000-2045) and the
formulas of its test (tests/ltx25-trunk-test.cc:146-240): the 1x1x1 patchify
packs the channel-major latent [z][F][H][W] to token-major [T][z] (w
fastest), projects it with bias, and adds the keyframe position embedding to
the first latent frame's tokens; the head is LayerNorm (no affine, eps
1e-6 -- not an RMSNorm), x * (1 + scale) + shift with shift = table[0] + emb
and scale = table[1] + emb, then proj_out.  The reference's goldens for these
(trunk_patch_*, trunk_head_*) are not in the tree, so parity is pinned to
those formulas, not to recorded outputs.
"""
import numpy as np

from .block_np import linear

F32 = np.float32
F64 = np.float64


def pack(latent_cm):
    """[z][T] -> [T][z] (tests/ltx25-trunk-test.cc:159-165)."""
    return np.ascontiguousarray(np.asarray(latent_cm, F32).T)


def patchify(latent_tm, w, b, prefix=None, prefix_rows=0):
    x = linear(latent_tm, w, b)
    if prefix is not None and prefix_rows > 0:
        x[:prefix_rows] = (x[:prefix_rows] + np.asarray(prefix, F32)).astype(F32)
    return x


def layer_norm(x, eps=1e-6):
    x64 = np.asarray(x, F32).astype(F64)
    mu = x64.mean(axis=1, keepdims=True)
    var = ((x64 - mu) ** 2).mean(axis=1, keepdims=True)
    return ((x64 - mu) / np.sqrt(var + eps)).astype(F32)


def head(x, shift_scale, w, b):
    """src/ltx25-dit.cc:2010-2031; shift_scale [2][dim], shift row first."""
    ss = np.asarray(shift_scale, F32)
    dim = ss.shape[1]
    m = (layer_norm(x) * (F32(1.0) + ss[1][None, :dim]) + ss[0][None, :dim]).astype(F32)
    return linear(m, w, b)
