"""ctypes bindings for _ref/libref_oracle.so -- the reference's own CPU code
(src/ltx25-block-ref.cc, src/ltx25-rope.cc, and the packer of
tests/ltx25-qlinear-test.cc), compiled by oracle/Makefile.

TEST INFRASTRUCTURE ONLY.  `available()` is False when the library was not
built (no reference tree at build time); callers skip or fall back to the
committed golden fixtures.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_PATH = os.path.join(_HERE, "_ref", "libref_oracle.so")
_LIB = None

P = ctypes.c_void_p
I = ctypes.c_int
FP = ctypes.POINTER(ctypes.c_float)


class RefStream(ctypes.Structure):
    _fields_ = [
        ("x", P), ("tokens", I), ("dim", I), ("ctx", P), ("text_tokens", I),
        ("ts", P), ("ts_n", I), ("css", P), ("css_n", I), ("cg", P),
        ("cg_n", I), ("pts", P), ("pts_n", I), ("pe_cos", P), ("pe_sin", P),
        ("pe_heads", I), ("pe_half", I), ("cpe_cos", P), ("cpe_sin", P),
        ("cpe_heads", I), ("cpe_half", I), ("present", I),
    ]


def available():
    return os.path.exists(_PATH)


def load():
    global _LIB
    if _LIB is None:
        if not available():
            raise RuntimeError(f"{_PATH} missing: build with `make -C oracle` "
                               "where the reference tree is present")
        lib = ctypes.CDLL(_PATH)
        lib.ref_pack.argtypes = [P, I, I, I, I, P, P, P, P]
        lib.ref_pack.restype = I
        lib.ref_linear.argtypes = [P, P, P, P, I, I, I]
        lib.ref_linear.restype = None
        lib.ref_block_new.restype = P
        lib.ref_block_free.argtypes = [P]
        lib.ref_block_put.argtypes = [P, ctypes.c_char_p, P, I, I]
        lib.ref_block_load.argtypes = [P, I, I, I, I, ctypes.c_char_p, I]
        lib.ref_block_forward.argtypes = [P, ctypes.POINTER(RefStream),
                                          ctypes.POINTER(RefStream),
                                          ctypes.c_char_p, I]
        lib.ref_build_video_rope.argtypes = [I, I, I, P, I, I, I, I, I,
                                             ctypes.c_double, I, P, P]
        lib.ref_build_audio_rope.argtypes = [I, I, I, I, P, P]
        lib.ref_build_index_rope.argtypes = [I, I, I, I, P, P]
        lib.ref_build_cross_rope.argtypes = [P, P, I, I, I, I, P, P]
        lib.ref_video_time_seconds.argtypes = [I, I, ctypes.c_double, I, P]
        lib.ref_audio_time_seconds.argtypes = [I, P]
        lib.ref_adaln_chain.argtypes = [ctypes.c_double, P, P, P, P, P, P, I, I, P, P]
        lib.ref_adaln_chain.restype = I
        lib.ref_lora_gemv.argtypes = [P, P, P, I, I, I, P]
        lib.ref_lora_fold.argtypes = [P, P, P, I, I, I]
        lib.ref_lora_scale.argtypes = [P, P, ctypes.c_size_t, ctypes.c_double]
        _LIB = lib
    return _LIB


def _p(a):
    return None if a is None else a.ctypes.data_as(P)


def pack(w, bits=8, group=64):
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    codes = np.zeros((N, K * bits // 32), dtype=np.uint32)
    scales = np.zeros((N, K // group), dtype=np.uint16)
    biases = np.zeros((N, K // group), dtype=np.uint16)
    deq = np.zeros((N, K), dtype=np.float32)
    load().ref_pack(_p(w), N, K, bits, group, _p(codes), _p(scales),
                    _p(biases), _p(deq))
    return codes, scales, biases, deq


def linear(x, w, b=None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty((M, N), dtype=np.float32)
    load().ref_linear(_p(x), _p(w), _p(bb), _p(out), M, K, N)
    return out


def _tab(heads, tokens, half):
    return (np.zeros((heads, tokens, half), np.float32),
            np.zeros((heads, tokens, half), np.float32))


def video_rope(frames, height, width, max_pos, inner_dim, heads,
               scale=(8, 32, 32), fps=24.0, causal_fix=True):
    half = inner_dim // heads // 2
    c, s = _tab(heads, frames * height * width, half)
    mp = np.asarray(max_pos, dtype=np.int32)
    rc = load().ref_build_video_rope(frames, height, width, _p(mp), inner_dim,
                                     heads, scale[0], scale[1], scale[2], fps,
                                     int(causal_fix), _p(c), _p(s))
    if rc != 0:
        raise ValueError("ref video rope failed")
    return c, s


def audio_rope(tokens, max_pos, inner_dim, heads):
    half = inner_dim // heads // 2
    c, s = _tab(heads, tokens, half)
    load().ref_build_audio_rope(tokens, max_pos, inner_dim, heads, _p(c), _p(s))
    return c, s


def index_rope(tokens, max_pos, inner_dim, heads):
    half = inner_dim // heads // 2
    c, s = _tab(heads, tokens, half)
    load().ref_build_index_rope(tokens, max_pos, inner_dim, heads, _p(c), _p(s))
    return c, s


def cross_rope(starts, ends, max_pos, inner_dim, heads):
    starts = np.ascontiguousarray(starts, dtype=np.float64)
    ends = np.ascontiguousarray(ends, dtype=np.float64)
    half = inner_dim // heads // 2
    c, s = _tab(heads, starts.size, half)
    load().ref_build_cross_rope(_p(starts), _p(ends), starts.size, max_pos,
                                inner_dim, heads, _p(c), _p(s))
    return c, s


def video_time_seconds(frames, scale_t=8, fps=24.0, causal_fix=True):
    out = np.zeros(frames, np.float64)
    load().ref_video_time_seconds(frames, scale_t, fps, int(causal_fix), _p(out))
    return out


def audio_time_seconds(tokens):
    out = np.zeros(tokens, np.float64)
    load().ref_audio_time_seconds(tokens, _p(out))
    return out


def adaln_chain(t, w1, b1, w2, b2, w3, b3):
    """Ltx25Dit::adaln_ over the reference's own host helpers
    (src/ltx25-dit.cc:30-160): returns (driver, embedded_timestep) f32.
    Weights / biases are bf16 bits [out][in] / [out] (biases may be None)."""
    arrs = [None if a is None else np.ascontiguousarray(a, dtype=np.uint16)
            for a in (w1, b1, w2, b2, w3, b3)]
    dim, out_dim = arrs[0].shape[0], arrs[4].shape[0]
    out = np.zeros(out_dim, np.float32)
    emb = np.zeros(dim, np.float32)
    load().ref_adaln_chain(float(t), *[_p(a) for a in arrs], dim, out_dim, _p(out), _p(emb))
    return out, emb


def lora_gemv(x, a_bits, b_bits, y):
    """y + B (A x): the reference's host adapter GEMV (src/ltx25-dit.cc:77-103)."""
    a = np.ascontiguousarray(a_bits, np.uint16)
    b = np.ascontiguousarray(b_bits, np.uint16)
    xx = np.ascontiguousarray(x, np.float32)
    yy = np.ascontiguousarray(y, np.float32).copy()
    load().ref_lora_gemv(_p(xx), _p(a), _p(b), a.shape[0], a.shape[1], b.shape[0], _p(yy))
    return yy


def lora_fold(w, a, b):
    """W + B A by the reference adapter test's fold
    (tests/ltx25-lora-apply-test.cc:353-366); f32 values."""
    ww = np.ascontiguousarray(w, np.float32).copy()
    aa = np.ascontiguousarray(a, np.float32)
    bb = np.ascontiguousarray(b, np.float32)
    load().ref_lora_fold(_p(ww), _p(aa), _p(bb), aa.shape[0], aa.shape[1], bb.shape[0])
    return ww


def lora_scale(a_bits, factor):
    """bf16 bits of A with the factor folded in as scaled_ does it
    (src/ltx25-lora.cc:53-67)."""
    s = np.ascontiguousarray(a_bits, np.uint16)
    d = np.empty_like(s)
    load().ref_lora_scale(_p(s), _p(d), s.size, float(factor))
    return d


class RefBlock:
    """The reference's block_forward over a name -> tensor map."""

    def __init__(self, tensors, vdim, vheads, adim, aheads):
        lib = load()
        self._h = lib.ref_block_new()
        self._keep = []
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, dtype=np.float32)
            self._keep.append(a)
            rows, cols = (a.shape[0], a.shape[1]) if a.ndim == 2 else (a.size, 0)
            lib.ref_block_put(self._h, name.encode(), _p(a), rows, cols)
        err = ctypes.create_string_buffer(512)
        if lib.ref_block_load(self._h, vdim, vheads, adim, aheads, err, 512) != 0:
            raise ValueError(err.value.decode())

    def __del__(self):
        if getattr(self, "_h", None) and _LIB is not None:
            _LIB.ref_block_free(self._h)

    @staticmethod
    def _stream(d, keep):
        s = RefStream()
        x = np.ascontiguousarray(d["x"], dtype=np.float32).copy()
        keep.append(x)
        s.x = _p(x)
        s.tokens, s.dim = x.shape
        s.present = int(d.get("present", True))

        def arr(key):
            v = d.get(key)
            if v is None:
                return None, 0
            a = np.ascontiguousarray(v, dtype=np.float32)
            keep.append(a)
            return _p(a), a.size

        ctx, _ = arr("context")
        s.ctx = ctx
        s.text_tokens = 0 if d.get("context") is None else d["context"].shape[0]
        s.ts, s.ts_n = arr("timesteps")
        s.css, s.css_n = arr("cross_scale_shift")
        s.cg, s.cg_n = arr("cross_gate")
        s.pts, s.pts_n = arr("prompt_timestep")
        for pre, key in (("pe", "pe"), ("cpe", "cross_pe")):
            t = d.get(key)
            if t is not None:
                c = np.ascontiguousarray(t[0], np.float32)
                sn = np.ascontiguousarray(t[1], np.float32)
                keep += [c, sn]
                setattr(s, pre + "_cos", _p(c))
                setattr(s, pre + "_sin", _p(sn))
                setattr(s, pre + "_heads", c.shape[0])
                setattr(s, pre + "_half", c.shape[2])
        return s, x

    def forward(self, video, audio):
        keep = []
        sv, xv = self._stream(video, keep)
        sa, xa = self._stream(audio, keep)
        err = ctypes.create_string_buffer(512)
        rc = load().ref_block_forward(self._h, ctypes.byref(sv),
                                      ctypes.byref(sa), err, 512)
        if rc != 0:
            raise ValueError(err.value.decode())
        return xv, xa
