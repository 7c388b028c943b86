"""The trunk's adaLN chain restated in numpy (TEST INFRASTRUCTURE ONLY).

Ltx25Dit::adaln_ (src/ltx25-dit.cc:51-160): the 256-channel timestep
sinusoid (max period 10000, downscale shift 0, flip_sin_to_cos so the row
is [cos | sin]), then emb.timestep_embedder.linear_1 -> SiLU -> linear_2
(= embedded_timestep) -> SiLU -> linear, host GEMVs over bf16 weights with
f64 sums stored f32.  No golden vectors exist in the tree (the reference's
trunk test reads goldens that are not shipped); these are its formulas.
"""
import numpy as np

from . import lib

F32 = np.float32
F64 = np.float64


def sinusoid(t, channels=256):
    half = channels // 2
    i = np.arange(half, dtype=F64)
    a = F64(t) * np.exp(-np.log(10000.0) * i / half)
    return np.concatenate([np.cos(a).astype(F32), np.sin(a).astype(F32)])


def gemv(x, w_bits, b_bits):
    """gemv_host_ (src/ltx25-dit.cc:51-67)."""
    w = lib.bf16_to_f32(w_bits).astype(F64)
    y = w @ np.asarray(x, F32).astype(F64)
    if b_bits is not None:
        y += lib.bf16_to_f32(b_bits).astype(F64)
    return y.astype(F32)


def silu(v):
    v = np.asarray(v, F32)
    return (v / (F32(1.0) + np.exp(-v))).astype(F32)


def chain(t, w1, b1, w2, b2, w3, b3):
    """(driver, embedded_timestep) for timestep t (src/ltx25-dit.cc:137-160)."""
    h1 = silu(gemv(sinusoid(t), w1, b1))
    h2 = gemv(h1, w2, b2)
    return gemv(silu(h2), w3, b3), h2
