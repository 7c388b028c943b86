"""Python binding over the ltx25 C ABI (include/ltx25_cuda.h).

Used by the tests and bench.py to drive the CUDA library with torch-owned
device buffers.  Every call goes through libltx25_cuda.so; there is no CPU
path here -- a missing library raises LtxError at import of the first
context.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(_HERE)
LIB_PATH = os.path.join(PKG_DIR, "lib", "libltx25_cuda.so")

LTX_OK = 0
ERRORS = {
    -1: "LTX_E_NULL", -2: "LTX_E_SHAPE", -3: "LTX_E_UNSUPPORTED",
    -4: "LTX_E_CUDA", -5: "LTX_E_OOM", -6: "LTX_E_KERNEL", -7: "LTX_E_STATE",
    -8: "LTX_E_ALIGN",
}
SB_F16, SB_BF16, SB_F32 = 0, 1, 2
ROUTE_FUSED, ROUTE_DEQUANT_ONCE = 0, 1
EPI_STORE, EPI_GELU, EPI_GATED_RES = 0, 1, 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_LIB = None

# name -> (restype, argtypes); the single source of the binding's view of
# include/ltx25_cuda.h.
SIGNATURES = {
    "ltx_abi_version": (_I, []),
    "ltx_ctx_create": (_I, [_I, ctypes.POINTER(_P)]),
    "ltx_ctx_destroy": (None, [_P]),
    "ltx_ctx_last_error": (ctypes.c_char_p, [_P]),
    "ltx_ctx_reserve": (_I, [_P, _I, _I, _I]),
    "ltx_ctx_check": (_I, [_P, _P]),
    "ltx_ctx_set_trace": (_I, [_P, _P, _I]),
    "ltx_qweight_upload": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I,
                                ctypes.POINTER(_P)]),
    "ltx_dweight_upload": (_I, [_P, _P, _I, _I, _I, ctypes.POINTER(_P)]),
    "ltx_qweight_free": (None, [_P]),
    "ltx_qweight_info": (_I, [_P] + [ctypes.POINTER(_I)] * 5),
    "ltx_qlinear": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "ltx_qlinear_ex": (_I, [_P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _P,
                            _P]),
    "ltx_set_route": (_I, [_P, _I]),
    "ltx_set_tiers": (_I, [_P, _I, _I, _I]),
    "ltx_i8_takes": (_I, [_P, _I, _I, _I]),
    "ltx_dequant": (_I, [_P, _P, _P, _P]),
    "ltx_quant_rows_i8": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "ltx_pack_w8g64": (_I, [_P, _P, _I, _I, _P, _P, _P, _P]),
}


class LtxError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


def load():
    """The C library.  Raises when it is absent: there is no fallback."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise LtxError(-4, f"{LIB_PATH} not built; run "
                               "`python vpipe-ltx-2.5_b200/build.py`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def _ptr(t):
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


class Context:
    """ltx_ctx: one per device (MetalOps' counterpart)."""

    def __init__(self, device=0):
        self.lib = load()
        h = ctypes.c_void_p()
        rc = self.lib.ltx_ctx_create(device, ctypes.byref(h))
        if rc != LTX_OK:
            raise LtxError(rc, f"ltx_ctx_create(device={device}) failed")
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            self.lib.ltx_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def err(self):
        return self.lib.ltx_ctx_last_error(self.h).decode()

    def _ok(self, rc, what):
        if rc != LTX_OK:
            raise LtxError(rc, f"{what}: {self.err()}")

    def reserve(self, max_tokens, max_n, max_k):
        self._ok(self.lib.ltx_ctx_reserve(self.h, max_tokens, max_n, max_k),
                 "reserve")

    def check(self, stream=None):
        self._ok(self.lib.ltx_ctx_check(self.h, _stream(stream)), "check")

    def set_trace(self, buf=None, max_ctas=0):
        """Diagnostics: per-CTA phase stamps of every following GEMM into a
        device int64 tensor [max_ctas][16] (None turns it off)."""
        self._ok(self.lib.ltx_ctx_set_trace(self.h, _ptr(buf), max_ctas),
                 "set_trace")

    def set_route(self, route):
        self._ok(self.lib.ltx_set_route(self.h, route), "set_route")

    def set_tiers(self, i8_gemm=False, sage_attn=False, sage_dense_layers=0):
        self._ok(self.lib.ltx_set_tiers(self.h, int(i8_gemm), int(sage_attn),
                                        sage_dense_layers), "set_tiers")

    def i8_takes(self, M, K, N):
        return bool(self.lib.ltx_i8_takes(self.h, M, K, N))


class QWeight:
    """ltx_qweight: a w8g64 pack (or dense bf16 weight) resident in HBM."""

    def __init__(self, ctx, handle, N, K, quantized):
        self.ctx, self.h, self.N, self.K = ctx, handle, N, K
        self.quantized = quantized

    @classmethod
    def upload(cls, ctx, codes, scales, biases, N, K, sb_dtype=SB_BF16,
               bits=8, group=64, on_device=False):
        """codes/scales/biases: numpy arrays (host) or torch tensors (device
        when on_device)."""
        h = ctypes.c_void_p()
        if on_device:
            pc, ps, pb = _ptr(codes), _ptr(scales), _ptr(biases)
        else:
            import numpy as np
            codes = np.ascontiguousarray(codes)
            scales = np.ascontiguousarray(scales)
            biases = np.ascontiguousarray(biases)
            pc = codes.ctypes.data_as(_P)
            ps = scales.ctypes.data_as(_P)
            pb = biases.ctypes.data_as(_P)
        rc = ctx.lib.ltx_qweight_upload(ctx.h, pc, ps, pb, sb_dtype, N, K, bits,
                                        group, int(on_device), ctypes.byref(h))
        ctx._ok(rc, "qweight_upload")
        return cls(ctx, h, N, K, True)

    @classmethod
    def upload_dense(cls, ctx, w_bf16_bits, N, K):
        import numpy as np
        w = np.ascontiguousarray(w_bf16_bits, dtype=np.uint16)
        h = ctypes.c_void_p()
        rc = ctx.lib.ltx_dweight_upload(ctx.h, w.ctypes.data_as(_P), N, K, 0,
                                        ctypes.byref(h))
        ctx._ok(rc, "dweight_upload")
        return cls(ctx, h, N, K, False)

    def free(self):
        if self.h is not None and self.h.value:
            self.ctx.lib.ltx_qweight_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def qlinear(ctx, w, x, bias=None, out=None, epilogue=EPI_STORE, gate=None,
            stream=None, M=None):
    """y = x @ W.T (+ bias) on the GPU through ltx_qlinear_ex."""
    import torch
    if M is None:
        M = x.shape[0]
    if out is None:
        out = torch.empty((M, w.N), dtype=torch.bfloat16, device=x.device)
    rc = ctx.lib.ltx_qlinear_ex(ctx.h, w.h, _ptr(x), x.stride(0), _ptr(bias),
                                _ptr(out), out.stride(0), M, w.K, w.N, epilogue,
                                _ptr(gate), _stream(stream))
    ctx._ok(rc, "qlinear")
    return out


def dequant(ctx, w, stream=None):
    import torch
    out = torch.empty((w.N, w.K), dtype=torch.bfloat16,
                      device=f"cuda:{ctx.device}")
    ctx._ok(ctx.lib.ltx_dequant(ctx.h, w.h, _ptr(out), _stream(stream)),
            "dequant")
    return out


def quant_rows_i8(ctx, x, group, stream=None):
    import torch
    rows, K = x.shape
    q = torch.empty((rows, K), dtype=torch.int8, device=x.device)
    s = torch.empty((rows, K // group), dtype=torch.float32, device=x.device)
    ctx._ok(ctx.lib.ltx_quant_rows_i8(ctx.h, _ptr(x), rows, K, group, _ptr(q),
                                      _ptr(s), _stream(stream)), "quant_rows_i8")
    return q, s


def pack_w8g64(ctx, w, stream=None):
    """w8g64-pack a device f32 [N][K] weight on the GPU.  Returns device
    tensors (codes int32 [N][K/4] holding the u32 words, scales and
    zero-points as bf16-bit int16 [N][K/64])."""
    import torch
    N, K = w.shape
    codes = torch.empty((N, K // 4), dtype=torch.int32, device=w.device)
    scales = torch.empty((N, K // 64), dtype=torch.int16, device=w.device)
    biases = torch.empty((N, K // 64), dtype=torch.int16, device=w.device)
    ctx._ok(ctx.lib.ltx_pack_w8g64(ctx.h, _ptr(w.contiguous()), N, K, _ptr(codes),
                                   _ptr(scales), _ptr(biases), _stream(stream)),
            "pack_w8g64")
    return codes, scales, biases
