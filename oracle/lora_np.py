"""Low-rank adapters restated in numpy (TEST INFRASTRUCTURE ONLY).

The reference applies one module's adapter at run time as
y += (x . A^T) . B^T (MetalOps::lora_add, src/ltx25-metal-ops.cc:986-1000),
between the linear and whatever consumes it (MetalBlock::lora_,
src/ltx25-block-metal.cc:404-420), with the scale folded into A at load:
a' = bf16(f32(a) * factor) (scaled_, src/ltx25-lora.cc:56-68).  Its tests
check the op against f64 on the host (tests/ltx25-lora-apply-test.cc:
418-440) and the adapted block against the CPU block with each pair folded
into its base weight, W += B . A (tests/ltx25-lora-apply-test.cc:357-370).
No golden vectors exist for this path in the reference; these are the
formulas its own tests compute.
"""
import numpy as np

from . import lib

F32 = np.float32
F64 = np.float64


def fold_scale(a_bits, scale):
    """bf16 bits of A with `scale` folded in, one RNE rounding
    (src/ltx25-lora.cc:62-66)."""
    a = lib.bf16_to_f32(np.asarray(a_bits, np.uint16))
    return lib.f32_to_bf16((a * F32(scale)).astype(F32))


def delta(x, a, b):
    """(x . A^T) . B^T in f64 (tests/ltx25-lora-apply-test.cc:420-440).
    x [M][K], a [rank][K], b [N][rank] as f32 values."""
    r = np.asarray(x, F32).astype(F64) @ np.asarray(a, F32).astype(F64).T
    return r @ np.asarray(b, F32).astype(F64).T


def fold(w, a, b):
    """W + B . A with f64 sums, stored f32 (tests/ltx25-lora-apply-test.cc:
    357-370).  w [N][K], a [rank][K], b [N][rank]."""
    ba = np.asarray(b, F32).astype(F64) @ np.asarray(a, F32).astype(F64)
    # each f64 sum is rounded to f32 first, then added in f32, as the
    # reference's `w.v[...] += (float)acc` does
    return (np.asarray(w, F32) + ba.astype(F32)).astype(F32)


def make_pair(rng, rank, k, n):
    """A pair whose delta is the order of the weight it rides on
    (tests/ltx25-lora-apply-test.cc:338-352): A ~ N(0, 9 / (rank k)),
    B ~ N(0, 1); returned as bf16 bits."""
    amp = 3.0 / np.sqrt(rank * k)
    a = (rng.standard_normal((rank, k)) * amp).astype(F32)
    b = rng.standard_normal((n, rank)).astype(F32)
    return lib.f32_to_bf16(a), lib.f32_to_bf16(b)
