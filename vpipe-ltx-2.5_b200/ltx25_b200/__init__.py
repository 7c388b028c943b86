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
    -8: "LTX_E_ALIGN", -9: "LTX_E_ABORTED", -10: "LTX_E_HOST",
}
SB_F16, SB_BF16, SB_F32 = 0, 1, 2
TP_ID_BYTES = 128
ROUTE_FUSED, ROUTE_DEQUANT_ONCE, ROUTE_AUTO = 0, 1, 2
DEQUANT_MIN_M = 1536
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
    "ltx_ctx_scratch_bytes": (_I, [_P, ctypes.POINTER(ctypes.c_ulonglong)]),
    "ltx_ctx_check": (_I, [_P, _P]),
    "ltx_ctx_set_trace": (_I, [_P, _P, _I]),
    "ltx_ctx_selftest_timeout": (_I, [_P, _I, _P]),
    "ltx_qweight_upload": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I,
                                ctypes.POINTER(_P)]),
    "ltx_dweight_upload": (_I, [_P, _P, _I, _I, _I, ctypes.POINTER(_P)]),
    "ltx_qweight_free": (None, [_P]),
    "ltx_qweight_info": (_I, [_P] + [ctypes.POINTER(_I)] * 5),
    "ltx_qlinear": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "ltx_qlinear_ex": (_I, [_P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _P,
                            _P]),
    "ltx_qlinear_i8_static": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "ltx_lora_upload": (_I, [_P, _P, _P, _I, _I, _I, ctypes.c_float, _I, ctypes.POINTER(_P)]),
    "ltx_lora_free": (None, [_P]),
    "ltx_lora_info": (_I, [_P] + [ctypes.POINTER(_I)] * 3),
    "ltx_lora_add": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _I, _P]),
    "ltx_qlinear_lora": (_I, [_P, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "ltx_block_set_lora": (_I, [_P, ctypes.c_char_p, _P]),
    "ltx_patchify": (_I, [_P, _P, _P, _P, _P, _I, _P, _I, _P, _I, _I, _I, _P]),
    "ltx_st_open": (_I, [ctypes.c_char_p, ctypes.POINTER(_P), _P, _I]),
    "ltx_st_close": (None, [_P]),
    "ltx_st_count": (_I, [_P]),
    "ltx_st_name": (ctypes.c_char_p, [_P, _I]),
    "ltx_st_find": (_I, [_P, ctypes.c_char_p]),
    "ltx_st_info": (_I, [_P, _I, ctypes.POINTER(_I), ctypes.POINTER(_I),
                         ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(_P),
                         ctypes.POINTER(ctypes.c_uint64)]),
    "ltx_st_read_f32": (_I, [_P, _I, ctypes.c_uint64, ctypes.c_uint64, _P]),
    "ltx_st_metadata": (ctypes.c_char_p, [_P, ctypes.c_char_p]),
    "ltx_block_load_st": (_I, [_P, _P, ctypes.c_char_p]),
    "ltx_adaln_create": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, ctypes.POINTER(_P)]),
    "ltx_connector_create": (_I, [_P, _I, _I, _I, _I, _I, ctypes.c_double, _I, _I,
                                  ctypes.POINTER(_P)]),
    "ltx_connector_destroy": (None, [_P]),
    "ltx_connector_last_error": (ctypes.c_char_p, [_P]),
    "ltx_connector_set_qlinear": (_I, [_P, ctypes.c_char_p, _P, _P, _P, _I, _I, _I, _I]),
    "ltx_connector_set_tensor": (_I, [_P, ctypes.c_char_p, _P, _I, _I, _I]),
    "ltx_connector_load_st": (_I, [_P, _P, ctypes.c_char_p]),
    "ltx_connector_finalize": (_I, [_P]),
    "ltx_connector_reserve": (_I, [_P, _I]),
    "ltx_connector_forward": (_I, [_P, _P, _P, _I, _I, _P]),
    "ltx_adaln_load_st": (_I, [_P, ctypes.c_char_p, ctypes.POINTER(_P), _P, _I]),
    "ltx_adaln_free": (None, [_P]),
    "ltx_adaln_dims": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "ltx_adaln_run": (_I, [_P, ctypes.c_double, _P, _P, _I]),
    "ltx_adaln_run_many": (_I, [_P, _P, _P, _P, _I, _I]),
    "ltx_lora_load_st": (_I, [_P, _P, ctypes.c_char_p, _I, _I, ctypes.c_float,
                              ctypes.POINTER(_P)]),
    "ltx_output_head": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "ltx_launch_count": (ctypes.c_ulonglong, []),
    "ltx_tp_unique_id": (_I, [_P, _I]),
    "ltx_ctx_set_tp": (_I, [_P, _I, _I, _P]),
    "ltx_ctx_set_sp": (_I, [_P, _I, _I, _P]),
    "ltx_tp_allreduce": (_I, [_P, _P, ctypes.c_size_t, _I, _P]),
    "ltx_set_route": (_I, [_P, _I]),
    "ltx_set_tile_plan": (_I, [_P, _I, _I, _I]),
    "ltx_set_tiers": (_I, [_P, _I, _I, _I]),
    "ltx_i8_takes": (_I, [_P, _I, _I, _I]),
    "ltx_sage_takes": (_I, [_P, _I]),
    "ltx_block_set_layer": (_I, [_P, _I]),
    "ltx_dequant": (_I, [_P, _P, _P, _P]),
    "ltx_quant_rows_i8": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "ltx_pack_w8g64": (_I, [_P, _P, _I, _I, _P, _P, _P, _P]),
    "ltx_ada_zero": (_I, [_P, _P, _P, _I, _I, _P, _P, _I, _P]),
    "ltx_qk_norm_rope": (_I, [_P, _P, _I, _P, _I, _I, _I, _P, _P, _P, _P]),
    "ltx_attention": (_I, [_P, _P, _I, _P, _I, _P, _I, _P, _I, _P, _I, _I, _I,
                           _I, _I, _P]),
    "ltx_block_create": (_I, [_P, _I, _I, _I, _I, ctypes.POINTER(_P)]),
    "ltx_block_destroy": (None, [_P]),
    "ltx_block_last_error": (ctypes.c_char_p, [_P]),
    "ltx_block_set_qlinear": (_I, [_P, ctypes.c_char_p, _P, _P, _P, _I, _I, _I,
                                   _I]),
    "ltx_block_set_tensor": (_I, [_P, ctypes.c_char_p, _P, _I, _I, _I]),
    "ltx_block_finalize": (_I, [_P]),
    "ltx_block_reserve": (_I, [_P, _I, _I, _I]),
    "ltx_block_forward": (_I, [_P, _P, _P, _P]),
    "ltx_stack_create": (_I, [_P, ctypes.POINTER(_P)]),
    "ltx_stack_destroy": (None, [_P]),
    "ltx_stack_last_error": (ctypes.c_char_p, [_P]),
    "ltx_stack_add_block": (_I, [_P, _P]),
    "ltx_stack_size": (_I, [_P]),
    "ltx_stack_reserve": (_I, [_P, _I, _I, _I]),
    "ltx_stack_forward": (_I, [_P, _P, _P, _I, _I, _P, _P, _P]),
    "ltx_rope_table": (_I, [_P, _P, _I, _I, _P, _I, _I, ctypes.c_double, _I,
                            _P, _P]),
    "ltx_rope_video_spans": (_I, [_I, _I, _I, _I, _I, _I, ctypes.c_double, _I,
                                  _P, _P]),
    "ltx_rope_audio_seconds": (_I, [_I, _P, _P]),
}


class StreamIO(ctypes.Structure):
    """ltx_stream_io (include/ltx25_cuda.h)."""
    _fields_ = [
        ("x", _P), ("context", _P), ("timesteps", _P),
        ("cross_scale_shift", _P), ("cross_gate", _P),
        ("prompt_timestep", _P), ("pe_cos", _P), ("pe_sin", _P),
        ("cross_pe_cos", _P), ("cross_pe_sin", _P), ("tokens", _I),
        ("text_tokens", _I), ("present", _I),
    ]


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

    def scratch_bytes(self):
        """ltx_ctx_scratch_bytes: device scratch the context holds now."""
        n = ctypes.c_ulonglong(0)
        self._ok(self.lib.ltx_ctx_scratch_bytes(self.h, ctypes.byref(n)), "scratch_bytes")
        return int(n.value)

    def check(self, stream=None):
        self._ok(self.lib.ltx_ctx_check(self.h, _stream(stream)), "check")

    def set_trace(self, buf=None, max_ctas=0):
        """Diagnostics: per-CTA phase stamps of every following GEMM into a
        device int64 tensor [max_ctas][16] (None turns it off)."""
        self._ok(self.lib.ltx_ctx_set_trace(self.h, _ptr(buf), max_ctas),
                 "set_trace")

    def set_route(self, route):
        self._ok(self.lib.ltx_set_route(self.h, route), "set_route")

    def set_tile_plan(self, pair=-1, tn=-1, splits=-1):
        """ltx_set_tile_plan: force CTA pairs / token tile / K split (-1 = the
        planner's choice)."""
        self._ok(self.lib.ltx_set_tile_plan(self.h, pair, tn, splits), "set_tile_plan")

    def set_tiers(self, i8_gemm=False, sage_attn=False, sage_dense_layers=0):
        self._ok(self.lib.ltx_set_tiers(self.h, int(i8_gemm), int(sage_attn),
                                        sage_dense_layers), "set_tiers")

    def selftest_timeout(self, bound_ms=100, stream=None):
        """Launch the bounded-wait self-test (ltx_ctx_selftest_timeout)."""
        self._ok(self.lib.ltx_ctx_selftest_timeout(self.h, bound_ms, _stream(stream)),
                 "selftest_timeout")

    def set_tp(self, rank, world, uid=None):
        """Join a tensor-parallel group (uid: the bytes of tp_unique_id() made
        on rank 0; ignored when world == 1)."""
        buf = None
        if world > 1:
            buf = ctypes.create_string_buffer(bytes(uid), TP_ID_BYTES)
        self._ok(self.lib.ltx_ctx_set_tp(self.h, rank, world, buf), "set_tp")
        self.tp = (rank, world)

    def set_sp(self, rank, world, uid=None):
        """Join a sequence-parallel group (see ltx_ctx_set_sp)."""
        buf = None
        if world > 1:
            buf = ctypes.create_string_buffer(bytes(uid), TP_ID_BYTES)
        self._ok(self.lib.ltx_ctx_set_sp(self.h, rank, world, buf), "set_sp")
        self.sp = (rank, world)

    def allreduce(self, t, stream=None):
        """In-place sum of a contiguous f32 or bf16 device tensor over the group."""
        import torch
        dtype = {torch.float32: 0, torch.bfloat16: 1}[t.dtype]
        self._ok(self.lib.ltx_tp_allreduce(self.h, _ptr(t), t.numel(), dtype,
                                           _stream(stream)), "tp_allreduce")

    def sage_takes(self, head_dim):
        return bool(self.lib.ltx_sage_takes(self.h, head_dim))

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


class Lora:
    """ltx_lora: one module's low-rank adapter pair (a [rank][k], b [n][rank],
    bf16), `scale` folded into a at upload."""

    def __init__(self, ctx, a, b, scale=1.0):
        """a, b: torch bf16 tensors on the device (or numpy uint16 bf16 bits on
        the host)."""
        import numpy as np
        self.ctx = ctx
        rank, k = a.shape
        n = b.shape[0]
        if b.shape[1] != rank:
            raise ValueError("lora: a is [rank][k], b must be [n][rank]")
        h = ctypes.c_void_p()
        if isinstance(a, np.ndarray):
            a = np.ascontiguousarray(a, dtype=np.uint16)
            b = np.ascontiguousarray(b, dtype=np.uint16)
            pa, pb, dev = a.ctypes.data_as(_P), b.ctypes.data_as(_P), 0
        else:
            a, b = a.contiguous(), b.contiguous()
            pa, pb, dev = _ptr(a), _ptr(b), 1
        ctx._ok(ctx.lib.ltx_lora_upload(ctx.h, pa, pb, rank, k, n, float(scale), dev,
                                        ctypes.byref(h)), "lora_upload")
        self.h, self.rank, self.k, self.n = h, rank, k, n

    def free(self):
        if self.h is not None and self.h.value:
            self.ctx.lib.ltx_lora_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


ST_DTYPES = {0: "F32", 1: "F16", 2: "BF16", 3: "U32", 4: "I32", 5: "U8", 6: "I8", 7: "F64",
             8: "I64", 9: "U16", 10: "I16", 11: "BOOL"}


class SafeTensors:
    """ltx_st: a safetensors checkpoint mapped by the library (no GPU)."""

    def __init__(self, path):
        self.lib = load()
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(512)
        rc = self.lib.ltx_st_open(str(path).encode(), ctypes.byref(h), buf, 512)
        if rc != LTX_OK:
            raise LtxError(rc, f"st_open: {buf.value.decode()}")
        self.h = h

    def __len__(self):
        return self.lib.ltx_st_count(self.h)

    def names(self):
        return [self.lib.ltx_st_name(self.h, i).decode() for i in range(len(self))]

    def find(self, name):
        return self.lib.ltx_st_find(self.h, name.encode())

    def info(self, i):
        dt, nd = ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 8)()
        data, nbytes = ctypes.c_void_p(), ctypes.c_uint64()
        rc = self.lib.ltx_st_info(self.h, i, ctypes.byref(dt), ctypes.byref(nd), shape,
                                  ctypes.byref(data), ctypes.byref(nbytes))
        if rc != LTX_OK:
            raise LtxError(rc, "st_info")
        return ST_DTYPES[dt.value], [shape[d] for d in range(nd.value)], data.value, nbytes.value

    def raw(self, name):
        """The tensor's bytes (a copy) as a numpy uint8 array."""
        import numpy as np
        _, _, ptr, nbytes = self.info(self.find(name))
        return np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(ptr)).copy() \
            if nbytes else np.zeros(0, np.uint8)

    def read_f32(self, name):
        import numpy as np
        i = self.find(name)
        _, shape, _, _ = self.info(i)
        n = int(np.prod(shape)) if shape else 1
        out = np.empty(n, np.float32)
        rc = self.lib.ltx_st_read_f32(self.h, i, 0, n, out.ctypes.data_as(_P))
        if rc != LTX_OK:
            raise LtxError(rc, f"st_read_f32({name})")
        return out.reshape(shape)

    def metadata(self, key):
        v = self.lib.ltx_st_metadata(self.h, key.encode())
        return None if v is None else v.decode()

    def close(self):
        if self.h is not None and self.h.value:
            self.lib.ltx_st_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Connector:
    """ltx_connector: the embeddings connector on the GPU."""

    def __init__(self, ctx, heads, head_dim, layers, registers, norm_output=True, theta=10000.0,
                 max_pos=4096, rope_f64=True):
        self.ctx = ctx
        h = ctypes.c_void_p()
        ctx._ok(ctx.lib.ltx_connector_create(ctx.h, heads, head_dim, layers, registers,
                                             int(norm_output), float(theta), max_pos,
                                             int(rope_f64), ctypes.byref(h)), "connector_create")
        self.h, self.dim = h, heads * head_dim
        self._keep = []

    def err(self):
        return self.ctx.lib.ltx_connector_last_error(self.h).decode()

    def _ok(self, rc, what):
        if rc != LTX_OK:
            raise LtxError(rc, f"{what}: {self.err()}")

    def load(self, tensors, device="cuda", want_deq=True):
        """Stage a name -> f32 array (numpy or torch) map: the 2-D linears
        w8g64-packed on the device, the rest as f32.  Returns the weights
        as the GPU uses them (numpy; empty when want_deq is False)."""
        import numpy as np
        import torch
        deq = {}
        for name, arr in tensors.items():
            if isinstance(arr, torch.Tensor):
                t = arr.to(device=device, dtype=torch.float32)
            else:
                t = torch.as_tensor(np.ascontiguousarray(arr, dtype=np.float32)).to(device)
            if t.dim() == 2 and name.endswith(".weight") and "to_gate_logits" not in name:
                N, K = t.shape
                c, s, b = pack_w8g64(self.ctx, t)
                self._ok(self.ctx.lib.ltx_connector_set_qlinear(
                    self.h, name.encode(), _ptr(c), _ptr(s), _ptr(b), SB_BF16, N, K, 1),
                    f"set_qlinear({name})")
                if want_deq:
                    q = QWeight.upload(self.ctx, c, s, b, N, K, on_device=True)
                    deq[name] = dequant(self.ctx, q).float().cpu().numpy()
                    q.free()
            else:
                t = t.contiguous()
                self._keep.append(t)
                rows, cols = (t.shape[0], t.shape[1]) if t.dim() == 2 else (t.numel(), 0)
                self._ok(self.ctx.lib.ltx_connector_set_tensor(
                    self.h, name.encode(), _ptr(t), rows, cols, 1), f"set_tensor({name})")
                if want_deq:
                    deq[name] = t.float().cpu().numpy()
        torch.cuda.synchronize()
        return deq

    def load_st(self, st, root):
        self._ok(self.ctx.lib.ltx_connector_load_st(self.h, st.h, root.encode()), "load_st")

    def finalize(self):
        self._ok(self.ctx.lib.ltx_connector_finalize(self.h), "connector_finalize")
        self._keep = []

    def reserve(self, tokens):
        self._ok(self.ctx.lib.ltx_connector_reserve(self.h, tokens), "connector_reserve")

    def forward(self, x, n_valid, out=None, stream=None):
        import torch
        if out is None:
            out = torch.empty_like(x)
        self._ok(self.ctx.lib.ltx_connector_forward(self.h, _ptr(x), _ptr(out), x.shape[0],
                                                    n_valid, _stream(stream)),
                 "connector_forward")
        return out

    def close(self):
        if self.h is not None and self.h.value:
            self.ctx.lib.ltx_connector_destroy(self.h)
            self.h = None


def adaln_run_many(chains, timesteps, threads=0):
    """ltx_adaln_run_many: a denoise step's chains at once on one set of host
    threads.  Returns [(driver, embedded_timestep)] as f32 numpy, in order;
    the same bits as calling each chain alone."""
    import numpy as np
    if len(chains) != len(timesteps):
        raise ValueError("one timestep per chain")
    n = len(chains)
    if n == 0:
        return []
    outs = [np.empty(c.out_dim, np.float32) for c in chains]
    embs = [np.empty(c.dim, np.float32) for c in chains]
    hs = (_P * n)(*[c.h.value for c in chains])
    ts = (ctypes.c_double * n)(*[float(t) for t in timesteps])
    po = (_P * n)(*[o.ctypes.data for o in outs])
    pe = (_P * n)(*[e.ctypes.data for e in embs])
    rc = chains[0].lib.ltx_adaln_run_many(hs, ts, po, pe, n, threads)
    if rc != LTX_OK:
        raise LtxError(rc, "adaln_run_many")
    return list(zip(outs, embs))


class AdaLN:
    """ltx_adaln: one trunk adaLN chain on the host (no GPU)."""

    def __init__(self, w1=None, b1=None, w2=None, b2=None, w3=None, b3=None, st=None,
                 prefix=None):
        """bf16-bit numpy arrays [dim][256], [dim], [dim][dim], [dim],
        [out][dim], [out] -- or a SafeTensors and the chain's prefix."""
        import numpy as np
        self.lib = load()
        h = ctypes.c_void_p()
        if st is not None:
            buf = ctypes.create_string_buffer(512)
            rc = self.lib.ltx_adaln_load_st(st.h, prefix.encode(), ctypes.byref(h), buf, 512)
            if rc != LTX_OK:
                raise LtxError(rc, f"adaln_load_st: {buf.value.decode()}")
        else:
            arrs = [None if a is None else np.ascontiguousarray(a, np.uint16)
                    for a in (w1, b1, w2, b2, w3, b3)]
            self._keep = arrs
            ptrs = [None if a is None else a.ctypes.data_as(_P) for a in arrs]
            rc = self.lib.ltx_adaln_create(*ptrs, arrs[0].shape[0], arrs[4].shape[0],
                                           ctypes.byref(h))
            if rc != LTX_OK:
                raise LtxError(rc, "adaln_create")
        self.h = h
        d, od = ctypes.c_int(), ctypes.c_int()
        self.lib.ltx_adaln_dims(h, ctypes.byref(d), ctypes.byref(od))
        self.dim, self.out_dim = d.value, od.value

    def __call__(self, timestep, threads=0):
        """(driver [out_dim], embedded_timestep [dim]) as f32 numpy."""
        import numpy as np
        out = np.empty(self.out_dim, np.float32)
        emb = np.empty(self.dim, np.float32)
        rc = self.lib.ltx_adaln_run(self.h, float(timestep), out.ctypes.data_as(_P),
                                    emb.ctypes.data_as(_P), threads)
        if rc != LTX_OK:
            raise LtxError(rc, "adaln_run")
        return out, emb

    def close(self):
        if self.h is not None and self.h.value:
            self.lib.ltx_adaln_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def lora_from_st(ctx, st, module, k, n, lora_scale=1.0):
    """ltx_lora_load_st: one module's pair from an adapter file."""
    h = ctypes.c_void_p()
    ctx._ok(ctx.lib.ltx_lora_load_st(ctx.h, st.h, module.encode(), k, n, float(lora_scale),
                                     ctypes.byref(h)), f"lora_load_st({module})")
    lo = Lora.__new__(Lora)
    lo.ctx, lo.h = ctx, h
    r = ctypes.c_int()
    ctx.lib.ltx_lora_info(h, ctypes.byref(r), None, None)
    lo.rank, lo.k, lo.n = r.value, k, n
    return lo


def lora_add(ctx, lora, x, y, stream=None):
    """ltx_lora_add: y += (x @ A.T) @ B.T in place (MetalOps::lora_add)."""
    M = x.shape[0]
    ctx._ok(ctx.lib.ltx_lora_add(ctx.h, lora.h, _ptr(x), x.stride(0), _ptr(y), y.stride(0),
                                 M, lora.k, lora.n, _stream(stream)), "lora_add")
    return y


def qlinear_lora(ctx, w, lora, x, bias=None, out=None, epilogue=EPI_STORE, gate=None,
                 stream=None):
    """ltx_qlinear_lora: y = epilogue(x @ W.T + bias + (x @ A.T) @ B.T)."""
    import torch
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, w.N), dtype=torch.bfloat16, device=x.device)
    ctx._ok(ctx.lib.ltx_qlinear_lora(ctx.h, w.h, lora.h if lora is not None else None, _ptr(x),
                                     x.stride(0), _ptr(bias), _ptr(out), out.stride(0), M, w.K,
                                     w.N, epilogue, _ptr(gate), _stream(stream)),
            "qlinear_lora")
    return out


def patchify(ctx, w, latent, bias=None, lora=None, channel_major=False, prefix=None,
             prefix_rows=0, out=None, stream=None):
    """ltx_patchify: latent [T][z] (or [z][T] with channel_major) -> x [T][dim]."""
    import torch
    T = latent.shape[1] if channel_major else latent.shape[0]
    z, dim = w.K, w.N
    if out is None:
        out = torch.empty((T, dim), dtype=torch.bfloat16, device=latent.device)
    ctx._ok(ctx.lib.ltx_patchify(ctx.h, w.h, _ptr(bias), lora.h if lora is not None else None,
                                 _ptr(latent), int(channel_major), _ptr(prefix), prefix_rows,
                                 _ptr(out), T, z, dim, _stream(stream)), "patchify")
    return out


def output_head(ctx, w, x, shift_scale, bias=None, lora=None, channel_major=False, out=None,
                stream=None):
    """ltx_output_head: LayerNorm, modulate by shift_scale f32 [2][dim], proj_out."""
    import torch
    T, dim = x.shape
    oc = w.N
    if out is None:
        shape = (oc, T) if channel_major else (T, oc)
        out = torch.empty(shape, dtype=torch.bfloat16, device=x.device)
    ctx._ok(ctx.lib.ltx_output_head(ctx.h, _ptr(x), _ptr(shift_scale), w.h, _ptr(bias),
                                    lora.h if lora is not None else None, _ptr(out),
                                    int(channel_major), T, dim, oc, _stream(stream)),
            "output_head")
    return out


def qlinear_i8_static(ctx, w, x, bias=None, out=None, stream=None):
    """ltx_qlinear_i8_static: the int8 tier on the library's fixed scratch
    array (no device allocation in the call).  x: contiguous [M][K] bf16."""
    import torch
    M = x.shape[0]
    if out is None:
        out = torch.empty((M, w.N), dtype=torch.bfloat16, device=x.device)
    ctx._ok(ctx.lib.ltx_qlinear_i8_static(ctx.h, w.h, _ptr(x), _ptr(bias), _ptr(out),
                                          M, w.K, w.N, _stream(stream)),
            "qlinear_i8_static")
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


def ada_zero(ctx, x, scale=None, shift=None, normalize=True, out=None,
             stream=None):
    import torch
    rows, dim = x.shape
    if out is None:
        out = torch.empty_like(x)
    ctx._ok(ctx.lib.ltx_ada_zero(ctx.h, _ptr(x), _ptr(out), rows, dim,
                                 _ptr(scale), _ptr(shift), int(normalize),
                                 _stream(stream)), "ada_zero")
    return out


def qk_norm_rope(ctx, x, heads, head_dim, gain=None, cos=None, sin=None,
                 rows=None, stream=None):
    import torch
    rows = x.shape[0] if rows is None else rows
    out = torch.empty((rows, heads * head_dim), dtype=torch.bfloat16,
                      device=x.device)
    ctx._ok(ctx.lib.ltx_qk_norm_rope(ctx.h, _ptr(x), x.stride(0), _ptr(out),
                                     rows, heads, head_dim, _ptr(gain),
                                     _ptr(cos), _ptr(sin), _stream(stream)),
            "qk_norm_rope")
    return out


def attention(ctx, q, k, v, heads, head_dim, gate=None, tq=None, tk=None,
              stream=None, out=None):
    import torch
    tq = q.shape[0] if tq is None else tq
    tk = k.shape[0] if tk is None else tk
    o = out if out is not None else torch.empty((tq, heads * head_dim), dtype=torch.bfloat16,
                                                device=q.device)
    ctx._ok(ctx.lib.ltx_attention(
        ctx.h, _ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v),
        v.stride(0), _ptr(o), o.stride(0), _ptr(gate),
        0 if gate is None else gate.stride(0), tq, tk, heads, head_dim,
        _stream(stream)), "attention")
    return o


def is_quantized_name(name, ndim):
    """The w8g64 recipe's choice for a block tensor: every 2-D linear in the
    blocks except the gate logits and the adaLN tables
    (src/ltx25-quant-family.cc:50-71)."""
    return ndim == 2 and "to_gate_logits" not in name and "scale_shift" not in name


class Block:
    """ltx_block: one joint audio-video DiT block on the GPU."""

    def __init__(self, ctx, vdim, vheads, adim, aheads):
        self.ctx = ctx
        h = ctypes.c_void_p()
        ctx._ok(ctx.lib.ltx_block_create(ctx.h, vdim, vheads, adim, aheads,
                                         ctypes.byref(h)), "block_create")
        self.h = h
        self._keep = []

    def err(self):
        return self.ctx.lib.ltx_block_last_error(self.h).decode()

    def _ok(self, rc, what):
        if rc != LTX_OK:
            raise LtxError(rc, f"{what}: {self.err()}")

    def set_qlinear(self, name, codes, scales, biases, N, K, on_device=True,
                    sb_dtype=SB_BF16):
        self._ok(self.ctx.lib.ltx_block_set_qlinear(
            self.h, name.encode(), _ptr(codes), _ptr(scales), _ptr(biases),
            sb_dtype, N, K, int(on_device)), f"set_qlinear({name})")

    def set_tensor(self, name, t):
        """t: device f32 torch tensor (1-D or 2-D)."""
        t = t.contiguous()
        self._keep.append(t)
        rows, cols = (t.shape[0], t.shape[1]) if t.dim() == 2 else (t.numel(), 0)
        self._ok(self.ctx.lib.ltx_block_set_tensor(
            self.h, name.encode(), _ptr(t), rows, cols, 1),
            f"set_tensor({name})")

    def load(self, tensors, device="cuda"):
        """Stage a name -> f32 array map: 2-D linears are w8g64-packed on the
        device (bit-identical to the reference packer), the rest as is.
        Returns the dequantized f32 weights the GPU will use, as numpy (for
        an oracle run on the same weights)."""
        import numpy as np
        import torch
        deq = {}
        for name, arr in tensors.items():
            t = torch.as_tensor(np.ascontiguousarray(arr, dtype=np.float32)).to(device)
            if is_quantized_name(name, t.dim()):
                N, K = t.shape
                c, s, b = pack_w8g64(self.ctx, t)
                self.set_qlinear(name, c, s, b, N, K)
                q = QWeight.upload(self.ctx, c, s, b, N, K, on_device=True)
                deq[name] = dequant(self.ctx, q).float().cpu().numpy()
                q.free()
            else:
                self.set_tensor(name, t)
                deq[name] = np.asarray(arr, dtype=np.float32)
        torch.cuda.synchronize()
        return deq

    def load_st(self, st, prefix):
        """ltx_block_load_st: stage every tensor under `prefix` of a checkpoint."""
        self._ok(self.ctx.lib.ltx_block_load_st(self.h, st.h, prefix.encode()), "load_st")

    def set_lora(self, module, lora):
        """ltx_block_set_lora: attach `lora` (a Lora) to the module named as
        the reference names it ("attn1.to_q", "ff.net.2", ...)."""
        self._keep.append(lora)
        self._ok(self.ctx.lib.ltx_block_set_lora(self.h, module.encode(), lora.h),
                 f"set_lora({module})")

    def finalize(self):
        # Staged device tensors are read here; they may be dropped after.
        self._ok(self.ctx.lib.ltx_block_finalize(self.h), "block_finalize")
        self._keep = []

    def reserve(self, max_video, max_audio, max_text):
        self._ok(self.ctx.lib.ltx_block_reserve(self.h, max_video, max_audio,
                                                max_text), "block_reserve")

    def set_layer(self, layer):
        self._ok(self.ctx.lib.ltx_block_set_layer(self.h, layer), "block_set_layer")

    @staticmethod
    def make_io(s):
        """s: dict of device tensors (x, context, timesteps, cross_scale_shift,
        cross_gate, prompt_timestep, pe=(cos, sin), cross_pe=(cos, sin),
        present)."""
        io = StreamIO()
        if s is None:
            io.present = 0
            return io
        io.x = _ptr(s["x"])
        io.context = _ptr(s.get("context"))
        io.timesteps = _ptr(s.get("timesteps"))
        io.cross_scale_shift = _ptr(s.get("cross_scale_shift"))
        io.cross_gate = _ptr(s.get("cross_gate"))
        io.prompt_timestep = _ptr(s.get("prompt_timestep"))
        pe = s.get("pe")
        if pe is not None:
            io.pe_cos, io.pe_sin = _ptr(pe[0]), _ptr(pe[1])
        cpe = s.get("cross_pe")
        if cpe is not None:
            io.cross_pe_cos, io.cross_pe_sin = _ptr(cpe[0]), _ptr(cpe[1])
        io.tokens = s["x"].shape[0]
        io.text_tokens = 0 if s.get("context") is None else s["context"].shape[0]
        io.present = int(s.get("present", True))
        return io

    def forward(self, video, audio, stream=None):
        v = self.make_io(video)
        a = self.make_io(audio)
        self._ok(self.ctx.lib.ltx_block_forward(self.h, ctypes.byref(v),
                                                ctypes.byref(a),
                                                _stream(stream)),
                 "block_forward")

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            self.ctx.lib.ltx_block_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def launch_count():
    """Kernels the library has launched in this process so far."""
    return int(load().ltx_launch_count())


def tp_unique_id():
    """A fresh tensor-parallel rendezvous id (bytes), made on rank 0."""
    buf = ctypes.create_string_buffer(TP_ID_BYTES)
    rc = load().ltx_tp_unique_id(buf, TP_ID_BYTES)
    if rc != LTX_OK:
        raise LtxError(rc, "tp_unique_id: NCCL unavailable")
    return buf.raw


PROGRESS_FN = ctypes.CFUNCTYPE(_I, _I, _I, _P)


class Stack:
    """ltx_stack: blocks run in order over one shared scratch arena.  Holds
    Python references to its blocks so they outlive it."""

    def __init__(self, ctx, blocks=()):
        self.ctx = ctx
        h = ctypes.c_void_p()
        ctx._ok(ctx.lib.ltx_stack_create(ctx.h, ctypes.byref(h)), "stack_create")
        self.h = h
        self.blocks = []
        for b in blocks:
            self.add(b)

    def err(self):
        return self.ctx.lib.ltx_stack_last_error(self.h).decode()

    def _ok(self, rc, what):
        if rc != LTX_OK:
            raise LtxError(rc, f"{what}: {self.err()}")

    def add(self, block):
        self._ok(self.ctx.lib.ltx_stack_add_block(self.h, block.h), "stack_add_block")
        self.blocks.append(block)

    def __len__(self):
        return self.ctx.lib.ltx_stack_size(self.h)

    def reserve(self, max_video, max_audio, max_text):
        self._ok(self.ctx.lib.ltx_stack_reserve(self.h, max_video, max_audio,
                                                max_text), "stack_reserve")

    def forward(self, video, audio, begin=0, end=-1, progress=None, stream=None):
        """progress(block, blocks) -> bool; False stops (LTX_E_ABORTED)."""
        v = Block.make_io(video)
        a = Block.make_io(audio)
        cb = None
        if progress is not None:
            cb = PROGRESS_FN(lambda i, n, _u: 1 if progress(i, n) else 0)
        self._ok(self.ctx.lib.ltx_stack_forward(
            self.h, ctypes.byref(v), ctypes.byref(a), begin, end,
            ctypes.cast(cb, _P) if cb is not None else None, None,
            _stream(stream)), "stack_forward")

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            self.ctx.lib.ltx_stack_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- RoPE tables (host) --------------------------------------------------

def _np_ptr(a):
    return a.ctypes.data_as(_P)


def rope_table(starts, ends, max_pos, inner_dim, heads, theta=10000.0,
               f64_precision=True):
    """cos, sin [heads][tokens][half] f32 numpy (ltx_rope_table)."""
    import numpy as np
    starts = np.ascontiguousarray(np.atleast_2d(starts), dtype=np.float64)
    ends = np.ascontiguousarray(np.atleast_2d(ends), dtype=np.float64)
    n_axes, tokens = starts.shape
    mp = np.ascontiguousarray(np.atleast_1d(max_pos), dtype=np.int32)
    half = inner_dim // heads // 2
    cos = np.empty((heads, tokens, half), np.float32)
    sin = np.empty((heads, tokens, half), np.float32)
    rc = load().ltx_rope_table(_np_ptr(starts), _np_ptr(ends), n_axes, tokens,
                               _np_ptr(mp), inner_dim, heads, theta,
                               int(f64_precision), _np_ptr(cos), _np_ptr(sin))
    if rc != LTX_OK:
        raise LtxError(rc, "rope_table")
    return cos, sin


def video_spans(frames, height, width, scale=(8, 32, 32), fps=24.0,
                causal_fix=True):
    import numpy as np
    T = frames * height * width
    s = np.empty((3, T), np.float64)
    e = np.empty((3, T), np.float64)
    rc = load().ltx_rope_video_spans(frames, height, width, scale[0], scale[1],
                                     scale[2], fps, int(causal_fix),
                                     _np_ptr(s), _np_ptr(e))
    if rc != LTX_OK:
        raise LtxError(rc, "video_spans")
    return s, e


def audio_seconds(tokens):
    import numpy as np
    s = np.empty(tokens, np.float64)
    e = np.empty(tokens, np.float64)
    rc = load().ltx_rope_audio_seconds(tokens, _np_ptr(s), _np_ptr(e))
    if rc != LTX_OK:
        raise LtxError(rc, "audio_seconds")
    return s, e


def geometry_tables(frames, height, width, audio_tokens, vdim, vheads, adim,
                    aheads, max_pos_v=(20, 2048, 2048), max_pos_a=20):
    """The four tables one generation needs: video self (3 axes), audio self
    (seconds), and the two time-only cross tables at the audio width."""
    s, e = video_spans(frames, height, width)
    v_self = rope_table(s, e, list(max_pos_v), vdim, vheads)
    v_cross = rope_table(s[0:1], e[0:1], [max_pos_a], adim, aheads)
    a_s, a_e = audio_seconds(audio_tokens)
    a_self = rope_table(a_s, a_e, [max_pos_a], adim, aheads)
    return v_self, a_self, v_cross, a_self


from .watch import RankWatch  # noqa: E402  (host-only: the stack's progress hook over ranks)
