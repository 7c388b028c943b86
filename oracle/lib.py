"""ctypes bindings for liboracle.so (the C restatement in ltx_oracle.c).

TEST INFRASTRUCTURE ONLY.  Each wrapper names the reference lines the C
function restates.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def load():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} missing: run `make -C oracle`")
        lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        I = ctypes.c_int
        lib.ltxo_pack_affine.argtypes = [P, I, I, I, I, P, P, P, P]
        lib.ltxo_pack_affine.restype = I
        lib.ltxo_dequant_bf16.argtypes = [P, P, P, I, I, I, I, P]
        lib.ltxo_dequant_bf16.restype = I
        lib.ltxo_linear_f64.argtypes = [P, P, P, P, I, I, I, I]
        lib.ltxo_linear_f64.restype = None
        lib.ltxo_quant_rows_i8.argtypes = [P, I, I, I, P, P]
        lib.ltxo_quant_rows_i8.restype = I
        lib.ltxo_i8_gemm.argtypes = [P, P, P, P, P, P, I, I, I, I, I]
        lib.ltxo_i8_gemm.restype = None
        lib.ltxo_f32_to_bf16_n.argtypes = [P, P, ctypes.c_size_t]
        lib.ltxo_bf16_to_f32_n.argtypes = [P, P, ctypes.c_size_t]
        _LIB = lib
    return _LIB


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def f32_to_bf16(a):
    """RNE f32 -> bf16 bits (tests/ltx25-qlinear-test.cc:66-73)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    load().ltxo_f32_to_bf16_n(_p(a), _p(out), a.size)
    return out


def bf16_to_f32(h):
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    load().ltxo_bf16_to_f32_n(_p(h), _p(out), h.size)
    return out


def pack_affine(w, bits=8, group=64):
    """Group-affine pack (tests/ltx25-qlinear-test.cc:94-141).

    Returns (codes u32 [N][K*bits/32], scales bf16 bits [N][K/group],
    biases bf16 bits [N][K/group], deq f32 [N][K]).
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    codes = np.zeros((N, K * bits // 32), dtype=np.uint32)
    scales = np.zeros((N, K // group), dtype=np.uint16)
    biases = np.zeros((N, K // group), dtype=np.uint16)
    deq = np.zeros((N, K), dtype=np.float32)
    rc = load().ltxo_pack_affine(_p(w), N, K, bits, group, _p(codes),
                                 _p(scales), _p(biases), _p(deq))
    if rc != 0:
        raise ValueError(f"pack_affine: bad shape N={N} K={K} bits={bits} group={group}")
    return codes, scales, biases, deq


def dequant_bf16(codes, scales, biases, K, bits=8, group=64):
    """bf16 bits of s*q + z, one rounding -- the GPU kernels' contract."""
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    biases = np.ascontiguousarray(biases, dtype=np.uint16)
    N = codes.shape[0]
    out = np.empty((N, K), dtype=np.uint16)
    rc = load().ltxo_dequant_bf16(_p(codes), _p(scales), _p(biases), N, K,
                                  bits, group, _p(out))
    if rc != 0:
        raise ValueError("dequant_bf16: bad shape")
    return out


def linear_f64(x, w, b=None, threads=1):
    """out = x @ w.T + b with f64 accumulation (src/ltx25-block-ref.cc:13-29)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    bb = None if b is None else np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty((M, N), dtype=np.float32)
    load().ltxo_linear_f64(_p(x), _p(w), _p(bb), _p(out), M, K, N, threads)
    return out


def quant_rows_i8(x_bf16, group):
    """Symmetric int8 per (row, group); returns (q int8, scale f32)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, K = x.shape
    q = np.empty((rows, K), dtype=np.int8)
    s = np.empty((rows, K // group), dtype=np.float32)
    rc = load().ltxo_quant_rows_i8(_p(x), rows, K, group, _p(q), _p(s))
    if rc != 0:
        raise ValueError("quant_rows_i8: K % group != 0")
    return q, s


def i8_gemm(xq, sx, wq, sw, bias, group, threads=1):
    xq = np.ascontiguousarray(xq, dtype=np.int8)
    wq = np.ascontiguousarray(wq, dtype=np.int8)
    sx = np.ascontiguousarray(sx, dtype=np.float32)
    sw = np.ascontiguousarray(sw, dtype=np.float32)
    bb = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    M, K = xq.shape
    N = wq.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    load().ltxo_i8_gemm(_p(xq), _p(sx), _p(wq), _p(sw), _p(bb), _p(y), M, K,
                        N, group, threads)
    return y


def rel_l2(a, b):
    """||a-b|| / ||b||, as tests/ltx25-qlinear-test.cc:143-153 computes it."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    num = float(np.sum((a - b) ** 2))
    den = float(np.sum(b * b))
    return (num / den) ** 0.5 if den > 0 else num ** 0.5
