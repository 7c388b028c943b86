"""Generate tests/golden/*.npz from the REFERENCE's own CPU code.

Runs only where the reference tree was present when `make -C oracle` built
oracle/_ref/libref_oracle.so (the reference's packer from
tests/ltx25-qlinear-test.cc:94-141, its dense linear_ from
src/ltx25-block-ref.cc:13-29, its RoPE builders from src/ltx25-rope.cc and
its block_forward from src/ltx25-block-ref.cc:308-389).  The fixtures are
committed so the CPU tests can pin the oracle restatement without the
reference tree.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import ref  # noqa: E402
from oracle import block_np  # noqa: E402


def pack_cases():
    """The reference test's six (N, K, bits, group) cases plus edge cases."""
    rng = np.random.default_rng(7)
    cases = {}
    shapes = [(128, 256, 8, 64), (128, 256, 8, 64), (128, 256, 4, 64),
              (128, 256, 4, 64), (128, 256, 4, 32), (64, 512, 8, 32),
              (16, 4096, 8, 64)]
    for i, (N, K, bits, group) in enumerate(shapes):
        w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
        cases[f"case{i}"] = (w, bits, group)
    # Edge cases: constant groups (scale 0 -> every code 0), an all-zero
    # row, one-sided groups, a wide dynamic range, exact ties.
    e = (rng.standard_normal((16, 128)) * 0.02).astype(np.float32)
    e[0, :] = 0.0
    e[1, :64] = 0.3
    e[2, :] = -1e-3
    e[3, :] = np.abs(e[3, :])
    e[4, :] *= 1e3
    e[5, ::2] = 1.0
    e[5, 1::2] = -1.0
    e[6, :] = np.linspace(-1, 1, 128, dtype=np.float32)
    cases["edge"] = (e, 8, 64)
    out = {}
    for name, (w, bits, group) in cases.items():
        c, s, b, d = ref.pack(w, bits, group)
        out[f"{name}__w"] = w
        out[f"{name}__meta"] = np.array([bits, group], np.int32)
        out[f"{name}__codes"] = c
        out[f"{name}__scales"] = s
        out[f"{name}__biases"] = b
        out[f"{name}__deq"] = d
    return out


def linear_cases():
    rng = np.random.default_rng(11)
    out = {}
    for i, (M, K, N, bias) in enumerate([(17, 300, 33, True), (8, 256, 64, False),
                                         (3, 1024, 16, True)]):
        x = rng.standard_normal((M, K)).astype(np.float32)
        w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
        b = (rng.standard_normal(N) * 0.1).astype(np.float32) if bias else None
        out[f"lin{i}__x"] = x
        out[f"lin{i}__w"] = w
        if b is not None:
            out[f"lin{i}__b"] = b
        out[f"lin{i}__y"] = ref.linear(x, w, b)
    return out


def rope_cases():
    out = {}
    c, s = ref.video_rope(2, 3, 4, [20, 2048, 2048], 96, 4)
    out["video__cos"], out["video__sin"] = c, s
    c, s = ref.audio_rope(7, 20, 64, 4)
    out["audio__cos"], out["audio__sin"] = c, s
    c, s = ref.index_rope(6, 20, 64, 4)
    out["index__cos"], out["index__sin"] = c, s
    vt = ref.video_time_seconds(3)
    at = ref.audio_time_seconds(9)
    out["vtime"], out["atime"] = vt, at
    starts = np.repeat(vt, 4)
    ends = np.repeat(ref.video_time_seconds(4)[1:], 4)
    c, s = ref.cross_rope(starts, ends, 20, 32, 4)
    out["cross__cos"], out["cross__sin"] = c, s
    out["cross__starts"], out["cross__ends"] = starts, ends
    return out


def block_cases():
    """The reference block on its SMALL geometry (video 64/4 heads, audio
    32/4, 6/4/3 tokens; tests/ltx25-block-test.cc:36-38) with seeded
    random weights, for three runs: joint, video-only, audio-only."""
    out = {}
    cfg = dict(vdim=64, vheads=4, adim=32, aheads=4, vt=6, at=4, tt=3)
    tensors = block_np.random_block_tensors(cfg["vdim"], cfg["vheads"],
                                            cfg["adim"], cfg["aheads"],
                                            seed=3)
    ins = block_np.random_block_inputs(cfg, seed=4, index_rope=True)
    for k, v in tensors.items():
        out[f"w__{k}"] = v
    for s in ("video", "audio"):
        for k, v in ins[s].items():
            if k in ("pe", "cross_pe"):
                out[f"in_{s}__{k}__cos"] = v[0]
                out[f"in_{s}__{k}__sin"] = v[1]
            elif v is not None and k != "present":
                out[f"in_{s}__{k}"] = v
    blk = ref.RefBlock(tensors, cfg["vdim"], cfg["vheads"], cfg["adim"],
                       cfg["aheads"])
    for mode in ("joint", "video", "audio"):
        v = dict(ins["video"], present=(mode != "audio"))
        a = dict(ins["audio"], present=(mode != "video"))
        xv, xa = blk.forward(v, a)
        out[f"out_{mode}__video"] = xv
        out[f"out_{mode}__audio"] = xa
    out["cfg"] = np.array([cfg[k] for k in ("vdim", "vheads", "adim", "aheads",
                                            "vt", "at", "tt")], np.int32)
    return out


def main():
    if not ref.available():
        raise SystemExit("oracle/_ref/libref_oracle.so missing: run "
                         "`make -C oracle` with the reference tree present")
    np.savez_compressed(os.path.join(HERE, "pack.npz"), **pack_cases())
    np.savez_compressed(os.path.join(HERE, "linear.npz"), **linear_cases())
    np.savez_compressed(os.path.join(HERE, "rope.npz"), **rope_cases())
    np.savez_compressed(os.path.join(HERE, "block_small.npz"), **block_cases())
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
