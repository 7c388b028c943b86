// capi.cc -- the extern "C" boundary declared in include/ltx25_cuda.h, over
// the C++ host mirror (CudaOps and friends).
#include <cstring>
#include <new>
#include <string>

#include "../../include/ltx25_cuda.h"
#include "../csrc/kernels.h"
#include "ltx25-cuda-ops.h"

struct ltx_ctx {
  ltx25::CudaOps ops;
  std::string err;
};

struct ltx_qweight {
  ltx25::QWeight w;
};

namespace {

int fail(ltx_ctx* c, int code, const std::string& m)
{
  if (c != nullptr) c->err = m;
  return code;
}

cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Map a message from the host mirror to an error code.
int code_for(const std::string& m)
{
  if (m.find("cudaMalloc") != std::string::npos) return LTX_E_OOM;
  if (m.find("aligned") != std::string::npos) return LTX_E_ALIGN;
  if (m.find("shape") != std::string::npos || m.find("need") != std::string::npos)
    return LTX_E_SHAPE;
  if (m.find("not run by this build") != std::string::npos) return LTX_E_UNSUPPORTED;
  if (m.find("null") != std::string::npos) return LTX_E_NULL;
  return LTX_E_CUDA;
}

}  // namespace

extern "C" {

int ltx_abi_version(void) { return LTX25_ABI_VERSION; }

int ltx_ctx_create(int device, ltx_ctx** out)
{
  if (out == nullptr) return LTX_E_NULL;
  *out = nullptr;
  ltx_ctx* c = new (std::nothrow) ltx_ctx();
  if (c == nullptr) return LTX_E_OOM;
  std::string e;
  if (!c->ops.init(device, &e)) {
    delete c;
    return LTX_E_CUDA;
  }
  *out = c;
  return LTX_OK;
}

void ltx_ctx_destroy(ltx_ctx* ctx) { delete ctx; }

const char* ltx_ctx_last_error(const ltx_ctx* ctx)
{
  return ctx == nullptr ? "null context" : ctx->err.c_str();
}

int ltx_ctx_reserve(ltx_ctx* ctx, int max_tokens, int max_n, int max_k)
{
  if (ctx == nullptr) return LTX_E_NULL;
  std::string e;
  if (!ctx->ops.reserve(max_tokens, max_n, max_k, &e)) return fail(ctx, code_for(e), e);
  return LTX_OK;
}

int ltx_ctx_check(ltx_ctx* ctx, void* stream)
{
  if (ctx == nullptr) return LTX_E_NULL;
  std::string e;
  const int h = ctx->ops.check(S(stream), &e);
  if (h < 0) return fail(ctx, LTX_E_CUDA, e);
  if (h > 0) return fail(ctx, LTX_E_KERNEL, e);
  return LTX_OK;
}

int ltx_ctx_set_trace(ltx_ctx* ctx, void* buf, int max_ctas)
{
  if (ctx == nullptr) return LTX_E_NULL;
  ctx->ops.set_trace(static_cast<unsigned long long*>(buf),
                     buf == nullptr ? 0 : max_ctas);
  return LTX_OK;
}

int ltx_qweight_upload(ltx_ctx* ctx, const uint32_t* codes, const void* scales,
                       const void* biases, int sb_dtype, int N, int K, int bits,
                       int group, int on_device, ltx_qweight** out)
{
  if (ctx == nullptr || out == nullptr) return LTX_E_NULL;
  *out = nullptr;
  ltx_qweight* q = new (std::nothrow) ltx_qweight();
  if (q == nullptr) return fail(ctx, LTX_E_OOM, "host allocation failed");
  std::string e;
  if (!ltx25::upload_qweight(ctx->ops, codes, scales, biases, sb_dtype, N, K,
                             bits, group, on_device != 0, &q->w, &e)) {
    delete q;
    return fail(ctx, code_for(e), e);
  }
  *out = q;
  return LTX_OK;
}

int ltx_dweight_upload(ltx_ctx* ctx, const uint16_t* w_bf16, int N, int K,
                       int on_device, ltx_qweight** out)
{
  if (ctx == nullptr || out == nullptr) return LTX_E_NULL;
  *out = nullptr;
  ltx_qweight* q = new (std::nothrow) ltx_qweight();
  if (q == nullptr) return fail(ctx, LTX_E_OOM, "host allocation failed");
  std::string e;
  if (!ltx25::upload_dweight(ctx->ops, w_bf16, N, K, on_device != 0, &q->w, &e)) {
    delete q;
    return fail(ctx, code_for(e), e);
  }
  *out = q;
  return LTX_OK;
}

void ltx_qweight_free(ltx_qweight* w)
{
  if (w == nullptr) return;
  ltx25::free_qweight(&w->w);
  delete w;
}

int ltx_qweight_info(const ltx_qweight* w, int* N, int* K, int* bits,
                     int* group, int* quantized)
{
  if (w == nullptr) return LTX_E_NULL;
  if (N) *N = w->w.N;
  if (K) *K = w->w.K;
  if (bits) *bits = w->w.quantized ? w->w.bits : 16;
  if (group) *group = w->w.quantized ? w->w.group : 0;
  if (quantized) *quantized = w->w.quantized ? 1 : 0;
  return LTX_OK;
}

int ltx_qlinear_ex(ltx_ctx* ctx, const ltx_qweight* w, const void* x, int ldx,
                   const void* bias, void* y, int ldy, int M, int K, int N,
                   int epilogue, const void* gate, void* stream)
{
  if (ctx == nullptr) return LTX_E_NULL;
  if (w == nullptr || x == nullptr || y == nullptr)
    return fail(ctx, LTX_E_NULL, "qlinear: null weight, x or y");
  if (epilogue < LTX_EPI_STORE || epilogue > LTX_EPI_GATED_RES)
    return fail(ctx, LTX_E_SHAPE, "qlinear: unknown epilogue");
  std::string e;
  if (!ctx->ops.linear(S(stream), static_cast<const __nv_bfloat16*>(x), ldx, w->w,
                       static_cast<const __nv_bfloat16*>(bias),
                       static_cast<__nv_bfloat16*>(y), ldy, M, K, N, epilogue,
                       static_cast<const __nv_bfloat16*>(gate), &e))
    return fail(ctx, code_for(e), e);
  return LTX_OK;
}

int ltx_qlinear(ltx_ctx* ctx, const ltx_qweight* w, const void* x,
                const void* bias, void* y, int M, int K, int N, void* stream)
{
  return ltx_qlinear_ex(ctx, w, x, K, bias, y, N, M, K, N, LTX_EPI_STORE,
                        nullptr, stream);
}

int ltx_set_route(ltx_ctx* ctx, int route)
{
  if (ctx == nullptr) return LTX_E_NULL;
  if (route != LTX_ROUTE_FUSED && route != LTX_ROUTE_DEQUANT_ONCE)
    return fail(ctx, LTX_E_SHAPE, "unknown route");
  ctx->ops.set_route(route == LTX_ROUTE_FUSED ? ltx25::Route::Fused
                                              : ltx25::Route::DequantOnce);
  return LTX_OK;
}

int ltx_set_tiers(ltx_ctx* ctx, int i8_gemm, int sage_attn,
                  int sage_dense_layers)
{
  if (ctx == nullptr) return LTX_E_NULL;
  ctx->ops.set_i8_gemm(i8_gemm != 0);
  ctx->ops.set_sage(sage_attn != 0, sage_dense_layers < 0 ? 0 : sage_dense_layers);
  return LTX_OK;
}

int ltx_i8_takes(const ltx_ctx* ctx, int M, int K, int N)
{
  if (ctx == nullptr) return 0;
  return ctx->ops.i8_takes(M, K, N) ? 1 : 0;
}

int ltx_dequant(ltx_ctx* ctx, const ltx_qweight* w, void* out, void* stream)
{
  if (ctx == nullptr) return LTX_E_NULL;
  if (w == nullptr || out == nullptr) return fail(ctx, LTX_E_NULL, "dequant: null");
  if (!w->w.quantized) return fail(ctx, LTX_E_SHAPE, "dequant: weight is dense");
  if (ltx::launch_dequant_w8(w->w.codes, w->w.sz, w->w.N, w->w.K,
                             static_cast<__nv_bfloat16*>(out), S(stream)) != 0)
    return fail(ctx, LTX_E_CUDA, "dequant launch failed");
  return LTX_OK;
}

int ltx_quant_rows_i8(ltx_ctx* ctx, const void* x, int rows, int K, int group,
                      void* q, void* scale, void* stream)
{
  if (ctx == nullptr) return LTX_E_NULL;
  if (x == nullptr || q == nullptr || scale == nullptr)
    return fail(ctx, LTX_E_NULL, "quant_rows_i8: null");
  if (rows <= 0 || K <= 0 || group <= 0 || K % group != 0 || group % 8 != 0)
    return fail(ctx, LTX_E_SHAPE, "quant_rows_i8: need K % group == 0, group % 8 == 0");
  if (ltx::launch_quant_rows_i8(static_cast<const __nv_bfloat16*>(x), rows, K, K,
                                group, static_cast<int8_t*>(q),
                                static_cast<float*>(scale), S(stream)) != 0)
    return fail(ctx, LTX_E_CUDA, "quant_rows_i8 launch failed");
  return LTX_OK;
}

int ltx_pack_w8g64(ltx_ctx* ctx, const float* w, int N, int K, uint32_t* codes,
                   uint16_t* scales, uint16_t* biases, void* stream)
{
  if (ctx == nullptr) return LTX_E_NULL;
  if (w == nullptr || codes == nullptr || scales == nullptr || biases == nullptr)
    return fail(ctx, LTX_E_NULL, "pack_w8g64: null");
  if (N <= 0 || K <= 0 || K % 64 != 0)
    return fail(ctx, LTX_E_SHAPE, "pack_w8g64: need K % 64 == 0");
  if (ltx::launch_pack_w8g64(w, N, K, codes, scales, biases, S(stream)) != 0)
    return fail(ctx, LTX_E_CUDA, "pack_w8g64 launch failed");
  return LTX_OK;
}

}  // extern "C"
