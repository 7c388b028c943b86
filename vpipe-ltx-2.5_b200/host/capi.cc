// capi.cc -- the extern "C" boundary declared in include/ltx25_cuda.h, over
// the C++ host mirror (CudaOps and friends).
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "../../include/ltx25_cuda.h"
#include "../csrc/kernels.h"
#include "../csrc/block_ops.h"
#include "ltx25-block-cuda.h"
#include "ltx25-cuda-ops.h"
#include "ltx25-adaln.h"
#include "ltx25-connector-cuda.h"
#include "ltx25-safetensors.h"

struct ltx_ctx {
  ltx25::CudaOps ops;
  std::string err;
};

struct ltx_qweight {
  ltx25::QWeight w;
};

struct ltx_lora {
  ltx25::LoraPair p;
};

struct ltx_st {
  ltx25::SafeTensors f;
};

struct ltx_adaln {
  ltx25::AdaLNChain c;
};

namespace {

int fail(ltx_ctx* c, int code, const std::string& m)
{
  if (c != nullptr) c->err = m;
  return code;
}

cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Every call on a context, or on an object made from one, runs on the
// context's device whatever device the calling thread has selected (one
// thread may drive several contexts); the thread's own selection is put
// back on return.  ltx_ctx_create alone leaves its device selected.
class OnDevice {
public:
  explicit OnDevice(int dev)
  {
    int cur = -1;
    if (dev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != dev &&
        cudaSetDevice(dev) == cudaSuccess)
      _prev = cur;
  }
  ~OnDevice()
  {
    if (_prev >= 0) cudaSetDevice(_prev);
  }
  OnDevice(const OnDevice&) = delete;
  OnDevice& operator=(const OnDevice&) = delete;

private:
  int _prev = -1;
};

int dev_of(const ltx_ctx* c) { return c == nullptr ? -1 : c->ops.device(); }

// No C++ exception leaves the C ABI: a host allocation that fails becomes
// LTX_E_OOM, any other exception from the library's host code LTX_E_HOST.
template <class Body>
int guarded(const Body& body) noexcept
{
  try {
    return body();
  } catch (const std::bad_alloc&) {
    return LTX_E_OOM;
  } catch (...) {
    return LTX_E_HOST;
  }
}

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
  return guarded([&]() -> int {
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
  });
}

void ltx_ctx_destroy(ltx_ctx* ctx) { delete ctx; }

const char* ltx_ctx_last_error(const ltx_ctx* ctx)
{
  return ctx == nullptr ? "null context" : ctx->err.c_str();
}

int ltx_ctx_reserve(ltx_ctx* ctx, int max_tokens, int max_n, int max_k)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    std::string e;
    if (!ctx->ops.reserve(max_tokens, max_n, max_k, &e)) return fail(ctx, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_ctx_scratch_bytes(const ltx_ctx* ctx, unsigned long long* bytes)
{
  return guarded([&]() -> int {
    if (ctx == nullptr || bytes == nullptr) return LTX_E_NULL;
    *bytes = (unsigned long long)ctx->ops.scratch_bytes();
    return LTX_OK;
  });
}

int ltx_ctx_check(ltx_ctx* ctx, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    std::string e;
    const int h = ctx->ops.check(S(stream), &e);
    if (h < 0) return fail(ctx, LTX_E_CUDA, e);
    if (h > 0) return fail(ctx, LTX_E_KERNEL, e);
    return LTX_OK;
  });
}

int ltx_ctx_selftest_timeout(ltx_ctx* ctx, int bound_ms, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    const int rc = ltx::launch_watchdog_probe(ctx->ops.err_word(), bound_ms, S(stream));
    if (rc == -2) return fail(ctx, LTX_E_SHAPE, "selftest: bound_ms outside 1..2000");
    if (rc != 0) return fail(ctx, LTX_E_CUDA, "selftest launch failed");
    return LTX_OK;
  });
}

int ltx_ctx_set_trace(ltx_ctx* ctx, void* buf, int max_ctas)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    ctx->ops.set_trace(static_cast<unsigned long long*>(buf),
                       buf == nullptr ? 0 : max_ctas);
    return LTX_OK;
  });
}

int ltx_qweight_upload(ltx_ctx* ctx, const uint32_t* codes, const void* scales,
                       const void* biases, int sb_dtype, int N, int K, int bits,
                       int group, int on_device, ltx_qweight** out)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
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
  });
}

int ltx_dweight_upload(ltx_ctx* ctx, const uint16_t* w_bf16, int N, int K,
                       int on_device, ltx_qweight** out)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
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
  });
}

void ltx_qweight_free(ltx_qweight* w)
{
  OnDevice on_(w == nullptr ? -1 : w->w.device);
  if (w == nullptr) return;
  ltx25::free_qweight(&w->w);
  delete w;
}

int ltx_qweight_info(const ltx_qweight* w, int* N, int* K, int* bits,
                     int* group, int* quantized)
{
  return guarded([&]() -> int {
    if (w == nullptr) return LTX_E_NULL;
    if (N) *N = w->w.N;
    if (K) *K = w->w.K;
    if (bits) *bits = w->w.quantized ? w->w.bits : 16;
    if (group) *group = w->w.quantized ? w->w.group : 0;
    if (quantized) *quantized = w->w.quantized ? 1 : 0;
    return LTX_OK;
  });
}

int ltx_qlinear_ex(ltx_ctx* ctx, const ltx_qweight* w, const void* x, int ldx,
                   const void* bias, void* y, int ldy, int M, int K, int N,
                   int epilogue, const void* gate, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (w == nullptr || x == nullptr || y == nullptr)
      return fail(ctx, LTX_E_NULL, "qlinear: null weight, x or y");
    if (epilogue < LTX_EPI_STORE || epilogue > LTX_EPI_GATED_RES)
      return fail(ctx, LTX_E_SHAPE, "qlinear: unknown epilogue");
    std::string e;
    if (!ctx->ops.linear(S(stream), static_cast<const __nv_bfloat16*>(x), ldx, w->w,
                         static_cast<const __nv_bfloat16*>(bias),
                         static_cast<__nv_bfloat16*>(y), ldy, M, K, N, epilogue,
                         static_cast<const float*>(gate), &e))
      return fail(ctx, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_lora_upload(ltx_ctx* ctx, const uint16_t* a, const uint16_t* b, int rank, int k,
                    int n, float scale, int on_device, ltx_lora** out)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr || out == nullptr) return LTX_E_NULL;
    *out = nullptr;
    ltx_lora* l = new (std::nothrow) ltx_lora();
    if (l == nullptr) return fail(ctx, LTX_E_OOM, "host allocation failed");
    std::string e;
    if (!ltx25::upload_lora(ctx->ops, a, b, rank, k, n, scale, on_device != 0, &l->p, &e)) {
      delete l;
      return fail(ctx, code_for(e), e);
    }
    *out = l;
    return LTX_OK;
  });
}

void ltx_lora_free(ltx_lora* l)
{
  OnDevice on_(l == nullptr ? -1 : l->p.device);
  if (l == nullptr) return;
  ltx25::free_lora(&l->p);
  delete l;
}

int ltx_lora_info(const ltx_lora* l, int* rank, int* k, int* n)
{
  return guarded([&]() -> int {
    if (l == nullptr) return LTX_E_NULL;
    if (rank) *rank = l->p.rank;
    if (k) *k = l->p.k;
    if (n) *n = l->p.n;
    return LTX_OK;
  });
}

int ltx_lora_add(ltx_ctx* ctx, const ltx_lora* l, const void* x, int ldx, void* y, int ldy,
                 int M, int K, int N, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (l == nullptr || x == nullptr || y == nullptr)
      return fail(ctx, LTX_E_NULL, "lora_add: null adapter, x or y");
    if (K != l->p.k || N != l->p.n)
      return fail(ctx, LTX_E_SHAPE,
                  "lora_add shape: K " + std::to_string(K) + ", N " + std::to_string(N) +
                      " against the pair's k " + std::to_string(l->p.k) + ", n " +
                      std::to_string(l->p.n));
    if (M <= 0) return LTX_OK;
    std::string e;
    ltx25::LoraExt ext;
    ext.a = l->p.a;
    ext.b = l->p.b;
    ext.r = l->p.r8;
    ext.rbuf = ctx->ops.lora_rbuf((size_t)M * l->p.r8, &e);
    if (ext.rbuf == nullptr) return fail(ctx, code_for(e), e);
    if (!ctx->ops.lora_add(S(stream), static_cast<const __nv_bfloat16*>(x), ldx, ext,
                           static_cast<__nv_bfloat16*>(y), ldy, M, K, N, &e))
      return fail(ctx, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_qlinear_lora(ltx_ctx* ctx, const ltx_qweight* w, const ltx_lora* l, const void* x,
                     int ldx, const void* bias, void* y, int ldy, int M, int K, int N,
                     int epilogue, const void* gate, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (l == nullptr)
      return ltx_qlinear_ex(ctx, w, x, ldx, bias, y, ldy, M, K, N, epilogue, gate, stream);
    if (w == nullptr || x == nullptr || y == nullptr)
      return fail(ctx, LTX_E_NULL, "qlinear_lora: null weight, x or y");
    if (epilogue < LTX_EPI_STORE || epilogue > LTX_EPI_GATED_RES)
      return fail(ctx, LTX_E_SHAPE, "qlinear_lora: unknown epilogue");
    if (K != l->p.k || N != l->p.n)
      return fail(ctx, LTX_E_SHAPE,
                  "qlinear_lora shape: K " + std::to_string(K) + ", N " + std::to_string(N) +
                      " against the pair's k " + std::to_string(l->p.k) + ", n " +
                      std::to_string(l->p.n));
    if (M <= 0) return fail(ctx, LTX_E_SHAPE, "qlinear_lora shape: M <= 0");
    std::string e;
    ltx25::LoraExt ext;
    ext.a = l->p.a;
    ext.b = l->p.b;
    ext.r = l->p.r8;
    ext.rbuf = ctx->ops.lora_rbuf((size_t)M * l->p.r8, &e);
    if (ext.rbuf == nullptr) return fail(ctx, code_for(e), e);
    if (!ctx->ops.linear(S(stream), static_cast<const __nv_bfloat16*>(x), ldx, w->w,
                         static_cast<const __nv_bfloat16*>(bias),
                         static_cast<__nv_bfloat16*>(y), ldy, M, K, N, epilogue,
                         static_cast<const float*>(gate), &e, &ext))
      return fail(ctx, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_patchify(ltx_ctx* ctx, const ltx_qweight* w, const void* bias, const ltx_lora* l,
                 const void* latent, int channel_major, const void* prefix, int prefix_rows,
                 void* x, int T, int z, int dim, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (w == nullptr) return fail(ctx, LTX_E_NULL, "patchify: null weight");
    if (w->w.K != z || w->w.N != dim)
      return fail(ctx, LTX_E_SHAPE, "patchify shape: the weight is [" + std::to_string(w->w.N) +
                                        "][" + std::to_string(w->w.K) + "]");
    std::string e;
    if (!ctx->ops.patchify(S(stream), w->w, static_cast<const __nv_bfloat16*>(bias),
                           l != nullptr ? &l->p : nullptr,
                           static_cast<const __nv_bfloat16*>(latent), channel_major != 0,
                           static_cast<const __nv_bfloat16*>(prefix), prefix_rows,
                           static_cast<__nv_bfloat16*>(x), T, z, dim, &e))
      return fail(ctx, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_output_head(ltx_ctx* ctx, const void* x, const float* shift_scale, const ltx_qweight* w,
                    const void* bias, const ltx_lora* l, void* out, int channel_major, int T,
                    int dim, int out_ch, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (w == nullptr) return fail(ctx, LTX_E_NULL, "output head: null weight");
    if (w->w.K != dim || w->w.N != out_ch)
      return fail(ctx, LTX_E_SHAPE, "output head shape: proj_out is [" + std::to_string(w->w.N) +
                                        "][" + std::to_string(w->w.K) + "]");
    std::string e;
    if (!ctx->ops.output_head(S(stream), static_cast<const __nv_bfloat16*>(x), shift_scale, w->w,
                              static_cast<const __nv_bfloat16*>(bias),
                              l != nullptr ? &l->p : nullptr, static_cast<__nv_bfloat16*>(out),
                              channel_major != 0, T, dim, out_ch, &e))
      return fail(ctx, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_qlinear(ltx_ctx* ctx, const ltx_qweight* w, const void* x,
                const void* bias, void* y, int M, int K, int N, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    return ltx_qlinear_ex(ctx, w, x, K, bias, y, N, M, K, N, LTX_EPI_STORE,
                          nullptr, stream);
  });
}

int ltx_qlinear_i8_static(ltx_ctx* ctx, const ltx_qweight* w, const void* x,
                          const void* bias, void* y, int M, int K, int N,
                          void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (w == nullptr || x == nullptr || y == nullptr)
      return fail(ctx, LTX_E_NULL, "qlinear_i8_static: null weight, x or y");
    if (M <= 0 || K <= 0 || (size_t)M * (size_t)K > (size_t)LTX_I8_STATIC_MAX_CODES ||
        M > LTX_I8_STATIC_MAX_ROWS)
      return fail(ctx, LTX_E_SHAPE,
                  "qlinear_i8_static: M*K = " + std::to_string((long long)M * K) +
                      " codes, M = " + std::to_string(M) + "; the fixed scratch holds " +
                      std::to_string(LTX_I8_STATIC_MAX_CODES) + " codes and " +
                      std::to_string(LTX_I8_STATIC_MAX_ROWS) + " rows");
    if (!w->w.quantized)
      return fail(ctx, LTX_E_UNSUPPORTED, "qlinear_i8_static: weight is dense");
    int8_t* xq = nullptr;
    float* sx = nullptr;
    std::string e;
    if (!ltx::i8_static_scratch(ctx->ops.device(), &xq, &sx, &e))
      return fail(ctx, LTX_E_CUDA, e);
    if (!ctx->ops.linear_i8_scratch(S(stream), static_cast<const __nv_bfloat16*>(x), w->w,
                                    static_cast<const __nv_bfloat16*>(bias),
                                    static_cast<__nv_bfloat16*>(y), M, K, N, xq, sx, &e)) {
      int code = code_for(e);
      if (e.find("int8 tier state") != std::string::npos) code = LTX_E_STATE;
      return fail(ctx, code, e);
    }
    return LTX_OK;
  });
}

unsigned long long ltx_launch_count(void) { return ltx::launch_count(); }

int ltx_tp_unique_id(void* id, int bytes)
{
  return guarded([&]() -> int {
    if (id == nullptr) return LTX_E_NULL;
    if (bytes < LTX_TP_ID_BYTES) return LTX_E_SHAPE;
    std::string e;
    return ltx25::Comm::unique_id(id, &e) ? LTX_OK : LTX_E_CUDA;
  });
}

int ltx_ctx_set_tp(ltx_ctx* ctx, int rank, int world, const void* id)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (world < 1 || rank < 0 || rank >= world)
      return fail(ctx, LTX_E_SHAPE, "set_tp: rank outside [0, world)");
    if (ctx->ops.comm() != nullptr) return fail(ctx, LTX_E_STATE, "set_tp: already set");
    if (world == 1) return LTX_OK;
    if (id == nullptr) return fail(ctx, LTX_E_NULL, "set_tp: null id");
    auto c = std::make_unique<ltx25::Comm>();
    std::string e;
    if (!c->init(ctx->ops.device(), rank, world, id, &e)) return fail(ctx, LTX_E_CUDA, e);
    // A second communicator lets the audio stream's all-reduces run on the
    // side stream beside the video stream's; without it, one stream.
    auto side = std::make_unique<ltx25::Comm>();
    if (!c->split(side.get(), &e)) side.reset();
    ctx->ops.set_comm(std::move(c), false, std::move(side));
    return LTX_OK;
  });
}

int ltx_ctx_set_sp(ltx_ctx* ctx, int rank, int world, const void* id)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (world < 1 || rank < 0 || rank >= world)
      return fail(ctx, LTX_E_SHAPE, "set_sp: rank outside [0, world)");
    if (ctx->ops.comm() != nullptr) return fail(ctx, LTX_E_STATE, "set_sp: already set");
    if (world == 1) return LTX_OK;
    if (id == nullptr) return fail(ctx, LTX_E_NULL, "set_sp: null id");
    auto c = std::make_unique<ltx25::Comm>();
    std::string e;
    if (!c->init(ctx->ops.device(), rank, world, id, &e)) return fail(ctx, LTX_E_CUDA, e);
    ctx->ops.set_comm(std::move(c), /*sequence*/ true);
    return LTX_OK;
  });
}

int ltx_tp_allreduce(ltx_ctx* ctx, void* buf, size_t count, int dtype, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (buf == nullptr && count > 0) return fail(ctx, LTX_E_NULL, "tp_allreduce: null buffer");
    if (dtype != 0 && dtype != 1) return fail(ctx, LTX_E_SHAPE, "tp_allreduce: dtype 0 or 1");
    if (ctx->ops.comm() == nullptr) return LTX_OK;   // one rank: the sum is itself
    std::string e;
    if (!ctx->ops.comm()->allreduce_sum(buf, count, dtype, S(stream), &e))
      return fail(ctx, LTX_E_CUDA, e);
    return LTX_OK;
  });
}

int ltx_set_route(ltx_ctx* ctx, int route)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (route != LTX_ROUTE_FUSED && route != LTX_ROUTE_DEQUANT_ONCE && route != LTX_ROUTE_AUTO)
      return fail(ctx, LTX_E_SHAPE, "unknown route");
    ctx->ops.set_route(route == LTX_ROUTE_FUSED ? ltx25::Route::Fused
                       : route == LTX_ROUTE_DEQUANT_ONCE ? ltx25::Route::DequantOnce
                                                         : ltx25::Route::Auto);
    return LTX_OK;
  });
}

int ltx_set_tile_plan(ltx_ctx* ctx, int force_pair, int force_tn, int force_splits)
{
  return guarded([&]() -> int {
    if (ctx == nullptr) return LTX_E_NULL;
    if (force_pair < -1 || force_pair > 2 || !(force_tn == -1 || force_tn == 128 || force_tn == 256) ||
        force_splits < -1 || force_splits == 0 || force_splits > 8)
      return fail(ctx, LTX_E_SHAPE, "set_tile_plan: pair -1/0/1/2, tn -1/128/256, splits -1 or 1..8");
    ltx25::PlanKnobs k;
    k.pair = force_pair;
    k.tn = force_tn;
    k.splits = force_splits;
    ctx->ops.set_plan_knobs(k);
    return LTX_OK;
  });
}

int ltx_set_tiers(ltx_ctx* ctx, int i8_gemm, int sage_attn,
                  int sage_dense_layers)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    ctx->ops.set_i8_gemm(i8_gemm != 0);
    ctx->ops.set_sage(sage_attn != 0, sage_dense_layers < 0 ? 0 : sage_dense_layers);
    return LTX_OK;
  });
}

int ltx_i8_takes(const ltx_ctx* ctx, int M, int K, int N)
{
  return guarded([&]() -> int {
    if (ctx == nullptr) return 0;
    return ctx->ops.i8_takes(M, K, N) ? 1 : 0;
  });
}

int ltx_sage_takes(const ltx_ctx* ctx, int head_dim)
{
  return guarded([&]() -> int {
    if (ctx == nullptr) return 0;
    return ctx->ops.sage_takes(head_dim) ? 1 : 0;
  });
}

int ltx_dequant(ltx_ctx* ctx, const ltx_qweight* w, void* out, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (w == nullptr || out == nullptr) return fail(ctx, LTX_E_NULL, "dequant: null");
    if (!w->w.quantized) return fail(ctx, LTX_E_SHAPE, "dequant: weight is dense");
    if (ltx::launch_dequant_w8(w->w.codes, w->w.sz, w->w.N, w->w.K,
                               static_cast<__nv_bfloat16*>(out), S(stream)) != 0)
      return fail(ctx, LTX_E_CUDA, "dequant launch failed");
    return LTX_OK;
  });
}

int ltx_quant_rows_i8(ltx_ctx* ctx, const void* x, int rows, int K, int group,
                      void* q, void* scale, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
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
  });
}

int ltx_pack_w8g64(ltx_ctx* ctx, const float* w, int N, int K, uint32_t* codes,
                   uint16_t* scales, uint16_t* biases, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (w == nullptr || codes == nullptr || scales == nullptr || biases == nullptr)
      return fail(ctx, LTX_E_NULL, "pack_w8g64: null");
    if (N <= 0 || K <= 0 || K % 64 != 0)
      return fail(ctx, LTX_E_SHAPE, "pack_w8g64: need K % 64 == 0");
    if (ltx::launch_pack_w8g64(w, N, K, codes, scales, biases, S(stream)) != 0)
      return fail(ctx, LTX_E_CUDA, "pack_w8g64 launch failed");
    return LTX_OK;
  });
}

int ltx_ada_zero(ltx_ctx* ctx, const void* x, void* out, int rows, int dim,
                 const float* scale, const float* shift, int normalize,
                 void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (x == nullptr || out == nullptr) return fail(ctx, LTX_E_NULL, "ada_zero: null");
    const int rc = ltx::launch_ada_zero(static_cast<const __nv_bfloat16*>(x), dim,
                                        static_cast<__nv_bfloat16*>(out), dim, rows,
                                        dim, scale, shift, 1e-6f, normalize != 0,
                                        S(stream));
    if (rc == -2) return fail(ctx, LTX_E_SHAPE, "ada_zero: dim % 8 != 0 or > 8192");
    if (rc != 0) return fail(ctx, LTX_E_CUDA, "ada_zero launch failed");
    return LTX_OK;
  });
}

int ltx_qk_norm_rope(ltx_ctx* ctx, const void* in, int ld_in, void* out,
                     int rows, int heads, int head_dim, const float* gain,
                     const float* cos_tab, const float* sin_tab, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (in == nullptr || out == nullptr) return fail(ctx, LTX_E_NULL, "qk_norm_rope: null");
    if ((cos_tab == nullptr) != (sin_tab == nullptr))
      return fail(ctx, LTX_E_NULL, "qk_norm_rope: cos and sin go together");
    const int rc = ltx::launch_qk_norm_rope(
        static_cast<const __nv_bfloat16*>(in), ld_in, static_cast<__nv_bfloat16*>(out),
        heads * head_dim, rows, heads, head_dim, gain, cos_tab, sin_tab, 1e-6f, S(stream));
    if (rc == -2) return fail(ctx, LTX_E_SHAPE, "qk_norm_rope: bad head geometry");
    if (rc != 0) return fail(ctx, LTX_E_CUDA, "qk_norm_rope launch failed");
    return LTX_OK;
  });
}

int ltx_attention(ltx_ctx* ctx, const void* q, int ldq, const void* k, int ldk,
                  const void* v, int ldv, void* o, int ldo,
                  const void* gate_logits, int ldg, int tq, int tk, int heads,
                  int head_dim, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr) return LTX_E_NULL;
    if (q == nullptr || k == nullptr || v == nullptr || o == nullptr)
      return fail(ctx, LTX_E_NULL, "attention: null");
    std::string e;
    if (!ctx->ops.attention(S(stream), static_cast<const __nv_bfloat16*>(q), ldq,
                            static_cast<const __nv_bfloat16*>(k), ldk,
                            static_cast<const __nv_bfloat16*>(v), ldv,
                            static_cast<__nv_bfloat16*>(o), ldo,
                            static_cast<const __nv_bfloat16*>(gate_logits), ldg, tq, tk,
                            heads, head_dim, &e, /*layer*/ 1 << 30))
      return fail(ctx, code_for(e), e);
    return LTX_OK;
  });
}

}  // extern "C"

struct ltx_block {
  ltx_ctx* ctx = nullptr;
  ltx25::CudaBlock* blk = nullptr;
  std::string err;
};

namespace {

int bfail(ltx_block* b, int code, const std::string& m)
{
  if (b != nullptr) b->err = m;
  return code;
}

ltx25::StreamIO to_io(const ltx_stream_io* s)
{
  ltx25::StreamIO io;
  if (s == nullptr) {
    io.present = false;
    return io;
  }
  io.x = static_cast<__nv_bfloat16*>(s->x);
  io.context = static_cast<const __nv_bfloat16*>(s->context);
  io.timesteps = static_cast<const __nv_bfloat16*>(s->timesteps);
  io.cross_scale_shift = static_cast<const __nv_bfloat16*>(s->cross_scale_shift);
  io.cross_gate = static_cast<const __nv_bfloat16*>(s->cross_gate);
  io.prompt_timestep = static_cast<const __nv_bfloat16*>(s->prompt_timestep);
  io.pe_cos = s->pe_cos;
  io.pe_sin = s->pe_sin;
  io.cpe_cos = s->cross_pe_cos;
  io.cpe_sin = s->cross_pe_sin;
  io.tokens = s->tokens;
  io.text_tokens = s->text_tokens;
  io.present = s->present != 0;
  return io;
}

}  // namespace

extern "C" {

int ltx_block_create(ltx_ctx* ctx, int video_dim, int video_heads,
                     int audio_dim, int audio_heads, ltx_block** out)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr || out == nullptr) return LTX_E_NULL;
    *out = nullptr;
    if (video_dim <= 0 || video_heads <= 0 || audio_dim <= 0 || audio_heads <= 0 ||
        video_dim % video_heads != 0 || audio_dim % audio_heads != 0)
      return fail(ctx, LTX_E_SHAPE, "block: widths must be positive multiples of the heads");
    ltx_block* b = new (std::nothrow) ltx_block();
    if (b == nullptr) return fail(ctx, LTX_E_OOM, "host allocation failed");
    b->ctx = ctx;
    b->blk = new (std::nothrow) ltx25::CudaBlock(&ctx->ops, video_dim, video_heads,
                                                 audio_dim, audio_heads);
    if (b->blk == nullptr) {
      delete b;
      return fail(ctx, LTX_E_OOM, "host allocation failed");
    }
    *out = b;
    return LTX_OK;
  });
}

void ltx_block_destroy(ltx_block* b)
{
  OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
  if (b == nullptr) return;
  delete b->blk;
  delete b;
}

const char* ltx_block_last_error(const ltx_block* b)
{
  return b == nullptr ? "null block" : b->err.c_str();
}

int ltx_block_set_qlinear(ltx_block* b, const char* name, const uint32_t* codes,
                          const void* scales, const void* biases, int sb_dtype,
                          int N, int K, int on_device)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
    if (b == nullptr) return LTX_E_NULL;
    if (name == nullptr) return bfail(b, LTX_E_NULL, "set_qlinear: null name");
    std::string e;
    if (!b->blk->set_qlinear(name, codes, scales, biases, sb_dtype, N, K,
                             on_device != 0, &e))
      return bfail(b, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_block_set_tensor(ltx_block* b, const char* name, const float* data,
                         int rows, int cols, int on_device)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
    if (b == nullptr) return LTX_E_NULL;
    if (name == nullptr || data == nullptr) return bfail(b, LTX_E_NULL, "set_tensor: null");
    std::string e;
    if (!b->blk->set_tensor(name, data, rows, cols, on_device != 0, &e))
      return bfail(b, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_block_set_lora(ltx_block* b, const char* module, const ltx_lora* l)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
    if (b == nullptr) return LTX_E_NULL;
    if (module == nullptr || l == nullptr)
      return bfail(b, LTX_E_NULL, "set_lora: null module name or adapter");
    std::string e;
    if (!b->blk->set_lora(module, l->p, &e)) {
      const int code = e.find("finalized") != std::string::npos ? LTX_E_STATE : code_for(e);
      return bfail(b, code, e);
    }
    return LTX_OK;
  });
}

int ltx_block_finalize(ltx_block* b)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
    if (b == nullptr) return LTX_E_NULL;
    std::string e;
    if (!b->blk->finalize(&e)) {
      const int code = e.find("missing") != std::string::npos ? LTX_E_STATE : code_for(e);
      return bfail(b, code, e);
    }
    return LTX_OK;
  });
}

int ltx_block_reserve(ltx_block* b, int max_video_tokens, int max_audio_tokens,
                      int max_text_tokens)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
    if (b == nullptr) return LTX_E_NULL;
    std::string e;
    if (!b->blk->reserve(max_video_tokens, max_audio_tokens, max_text_tokens, &e))
      return bfail(b, b->blk->finalized() ? code_for(e) : LTX_E_STATE, e);
    return LTX_OK;
  });
}

int ltx_block_set_layer(ltx_block* b, int layer)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
    if (b == nullptr) return LTX_E_NULL;
    if (layer < 0) return bfail(b, LTX_E_SHAPE, "set_layer: negative layer");
    b->blk->set_layer(layer);
    return LTX_OK;
  });
}

int ltx_block_forward(ltx_block* b, const ltx_stream_io* video,
                      const ltx_stream_io* audio, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
    if (b == nullptr) return LTX_E_NULL;
    ltx25::StreamIO v = to_io(video), a = to_io(audio);
    std::string e;
    if (!b->blk->forward(S(stream), v, a, &e)) {
      int code = code_for(e);
      if (e.find("before finalize") != std::string::npos || e.find("arena") != std::string::npos)
        code = LTX_E_STATE;
      if (e.find("neither stream") != std::string::npos || e.find("missing") != std::string::npos)
        code = LTX_E_NULL;
      return bfail(b, code, e);
    }
    return LTX_OK;
  });
}

}  // extern "C"

struct ltx_stack {
  ltx_ctx* ctx = nullptr;
  std::vector<ltx_block*> blocks;
  std::shared_ptr<ltx25::BlockArena> arena;
  bool reserved = false;
  std::string err;
};

namespace {

int sfail(ltx_stack* s, int code, const std::string& m)
{
  if (s != nullptr) s->err = m;
  return code;
}

}  // namespace

extern "C" {

int ltx_stack_create(ltx_ctx* ctx, ltx_stack** out)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr || out == nullptr) return LTX_E_NULL;
    *out = nullptr;
    ltx_stack* s = new (std::nothrow) ltx_stack();
    if (s == nullptr) return fail(ctx, LTX_E_OOM, "host allocation failed");
    s->ctx = ctx;
    *out = s;
    return LTX_OK;
  });
}

void ltx_stack_destroy(ltx_stack* s)
{
  OnDevice on_(dev_of(s == nullptr ? nullptr : s->ctx));
  delete s;
}

const char* ltx_stack_last_error(const ltx_stack* s)
{
  return s == nullptr ? "null stack" : s->err.c_str();
}

int ltx_stack_add_block(ltx_stack* s, ltx_block* b)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(s == nullptr ? nullptr : s->ctx));
    if (s == nullptr) return LTX_E_NULL;
    if (b == nullptr) return sfail(s, LTX_E_NULL, "add_block: null block");
    if (b->ctx != s->ctx) return sfail(s, LTX_E_STATE, "add_block: block of another context");
    if (!b->blk->finalized()) return sfail(s, LTX_E_STATE, "add_block: block not finalized");
    if (!s->blocks.empty() && !s->blocks[0]->blk->same_widths(*b->blk))
      return sfail(s, LTX_E_SHAPE, "add_block: widths differ from block 0");
    b->blk->set_layer((int)s->blocks.size());
    s->blocks.push_back(b);
    s->reserved = false;
    return LTX_OK;
  });
}

int ltx_stack_size(const ltx_stack* s) { return s == nullptr ? 0 : (int)s->blocks.size(); }

int ltx_stack_reserve(ltx_stack* s, int max_video_tokens, int max_audio_tokens,
                      int max_text_tokens)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(s == nullptr ? nullptr : s->ctx));
    if (s == nullptr) return LTX_E_NULL;
    if (s->blocks.empty()) return sfail(s, LTX_E_STATE, "reserve: empty stack");
    if (!s->arena) s->arena = std::make_shared<ltx25::BlockArena>();
    std::string e;
    for (ltx_block* b : s->blocks)
      if (!b->blk->reserve(max_video_tokens, max_audio_tokens, max_text_tokens, &e,
                           s->arena))
        return sfail(s, code_for(e), e);
    s->reserved = true;
    return LTX_OK;
  });
}

int ltx_stack_forward(ltx_stack* s, const ltx_stream_io* video,
                      const ltx_stream_io* audio, int begin, int end,
                      ltx_progress_fn progress, void* user, void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(s == nullptr ? nullptr : s->ctx));
    if (s == nullptr) return LTX_E_NULL;
    const int n = (int)s->blocks.size();
    if (end < 0) end = n;
    if (begin < 0 || begin > end || end > n)
      return sfail(s, LTX_E_SHAPE, "forward: block range outside the stack");
    if (!s->reserved) return sfail(s, LTX_E_STATE, "forward before reserve");
    ltx25::StreamIO whole = to_io(video), a = to_io(audio);
    // Sequence parallel, and tensor parallel with the residual sharded by
    // rows: each rank runs its token shard of x through every block and the
    // shards are gathered once, after the last.
    ltx25::StreamIO v = whole;
    const bool sp = s->blocks[0]->blk->shards_video(whole.present ? whole.tokens : 0);
    if (sp) {
      std::string e;
      if (!s->blocks[0]->blk->shard_io(whole, &v, &e)) return sfail(s, LTX_E_SHAPE, e);
    }
    for (int i = begin; i < end; ++i) {
      if (progress != nullptr && progress(i, n, user) == 0)
        // (sequence parallel: x's shards stay where each rank left them, and
        // every rank must take the same decision -- the next collective
        // would otherwise wait for ranks that stopped)
        return sfail(s, LTX_E_ABORTED, "aborted at block " + std::to_string(i));
      ltx25::CudaBlock* blk = s->blocks[(size_t)i]->blk;
      if (blk->arena() != s->arena)
        return sfail(s, LTX_E_STATE, "block " + std::to_string(i) +
                                         " was reserved outside the stack");
      std::string e;
      if (!(sp ? blk->forward_shard(S(stream), v, a, &e) : blk->forward(S(stream), v, a, &e))) {
        int code = code_for(e);
        if (e.find("arena") != std::string::npos) code = LTX_E_STATE;
        if (e.find("neither stream") != std::string::npos || e.find("missing") != std::string::npos)
          code = LTX_E_NULL;
        return sfail(s, code, "block " + std::to_string(i) + ": " + e);
      }
    }
    if (sp && end > begin) {
      std::string e;
      if (!s->blocks[0]->blk->gather_video(S(stream), whole, &e)) return sfail(s, LTX_E_CUDA, e);
    }
    return LTX_OK;
  });
}


// ---- checkpoints ----------------------------------------------------------

int ltx_st_open(const char* path, ltx_st** out, char* err, int err_len)
{
  return guarded([&]() -> int {
    if (out == nullptr || path == nullptr) return LTX_E_NULL;
    *out = nullptr;
    ltx_st* f = new (std::nothrow) ltx_st();
    if (f == nullptr) return LTX_E_OOM;
    std::string e;
    if (!f->f.open(path, &e)) {
      delete f;
      if (err != nullptr && err_len > 0) {
        std::strncpy(err, e.c_str(), (size_t)err_len - 1);
        err[err_len - 1] = '\0';
      }
      return e.find("cannot") != std::string::npos ? LTX_E_STATE : LTX_E_SHAPE;
    }
    *out = f;
    return LTX_OK;
  });
}

void ltx_st_close(ltx_st* f) { delete f; }

int ltx_st_count(const ltx_st* f) { return f == nullptr ? 0 : f->f.count(); }

const char* ltx_st_name(const ltx_st* f, int i)
{
  if (f == nullptr || i < 0 || i >= f->f.count()) return nullptr;
  return f->f.at(i).name.c_str();
}

int ltx_st_find(const ltx_st* f, const char* name)
{
  return guarded([&]() -> int {
    if (f == nullptr || name == nullptr) return -1;
    return f->f.find(name);
  });
}

int ltx_st_info(const ltx_st* f, int i, int* dtype, int* ndim, int64_t* shape,
                const void** data, uint64_t* bytes)
{
  return guarded([&]() -> int {
    if (f == nullptr) return LTX_E_NULL;
    if (i < 0 || i >= f->f.count()) return LTX_E_SHAPE;
    const ltx25::StTensor& t = f->f.at(i);
    if (dtype) *dtype = t.dtype;
    if (ndim) *ndim = (int)t.shape.size();
    if (shape)
      for (size_t d = 0; d < t.shape.size() && d < 8; ++d) shape[d] = t.shape[d];
    if (data) *data = t.data;
    if (bytes) *bytes = t.bytes;
    return LTX_OK;
  });
}

int ltx_st_read_f32(const ltx_st* f, int i, uint64_t off, uint64_t n, float* out)
{
  return guarded([&]() -> int {
    if (f == nullptr || out == nullptr) return LTX_E_NULL;
    if (i < 0 || i >= f->f.count()) return LTX_E_SHAPE;
    if (!ltx25::SafeTensors::to_f32(f->f.at(i), (size_t)off, (size_t)n, out)) return LTX_E_SHAPE;
    return LTX_OK;
  });
}

const char* ltx_st_metadata(const ltx_st* f, const char* key)
{
  if (f == nullptr || key == nullptr) return nullptr;
  const std::string* v = f->f.metadata(key);
  return v == nullptr ? nullptr : v->c_str();
}

}  // extern "C"

namespace {

// Stage every tensor under `pre`: the "X.weight" u32 codes / "X.scales" /
// "X.biases" triplets through `qfn` (need_q_, src/ltx25-dit-weights.cc:
// 352-403; this build runs w8g64: 8-bit codes, K = 4 x the u32 columns, in
// groups of 64; any other pack that closes is refused, not mis-read), every
// other float tensor as f32 through `tfn`.  Returns an LTX_* code.
template <class Q, class T>
int load_prefix(const ltx25::SafeTensors& st, const std::string& pre, Q qfn, T tfn,
                std::string* msg)
{
  int bound = 0;
  std::vector<bool> used((size_t)st.count(), false);
  for (int i = 0; i < st.count(); ++i) {
    const ltx25::StTensor& sc = st.at(i);
    const std::string& n = sc.name;
    if (n.compare(0, pre.size(), pre) != 0 || n.size() < 7 ||
        n.compare(n.size() - 7, 7, ".scales") != 0)
      continue;
    const std::string base = n.substr(0, n.size() - 7);
    const int wi = st.find(base + ".weight"), bi = st.find(base + ".biases");
    if (wi < 0 || bi < 0) {
      *msg = "load: '" + base + "' has scales but no weight or biases";
      return LTX_E_STATE;
    }
    const ltx25::StTensor& cw = st.at(wi);
    const ltx25::StTensor& bz = st.at(bi);
    if (cw.dtype != ltx25::ST_U32 || cw.shape.size() != 2 || sc.shape.size() != 2 ||
        bz.shape != sc.shape || bz.dtype != sc.dtype || cw.shape[0] != sc.shape[0]) {
      *msg = "load: '" + base + "' is not a u32 codes / scales / biases triplet of matching rows";
      return LTX_E_SHAPE;
    }
    const int64_t N = cw.shape[0], K = cw.shape[1] * 4, G = sc.shape[1];
    if (G <= 0 || K % G != 0 || K / G != 64) {
      *msg = "load: '" + base + "' closes at K " + std::to_string(K) + " with " +
             std::to_string(G) + " groups; this build runs the w8g64 pack only "
             "(not run by this build)";
      return LTX_E_UNSUPPORTED;
    }
    int sbd = -1;
    if (sc.dtype == ltx25::ST_F16) sbd = LTX_SB_F16;
    else if (sc.dtype == ltx25::ST_BF16) sbd = LTX_SB_BF16;
    else if (sc.dtype == ltx25::ST_F32) sbd = LTX_SB_F32;
    if (sbd < 0) {
      *msg = "load: '" + base + "' scales dtype";
      return LTX_E_UNSUPPORTED;
    }
    std::string e;
    if (!qfn(base.substr(pre.size()) + ".weight", reinterpret_cast<const uint32_t*>(cw.data),
             sc.data, bz.data, sbd, (int)N, (int)K, &e)) {
      *msg = e;
      return code_for(e);
    }
    used[(size_t)i] = used[(size_t)wi] = used[(size_t)bi] = true;
    ++bound;
  }
  std::vector<float> buf;
  for (int i = 0; i < st.count(); ++i) {
    const ltx25::StTensor& t = st.at(i);
    if (used[(size_t)i] || t.name.compare(0, pre.size(), pre) != 0) continue;
    if (t.dtype != ltx25::ST_F32 && t.dtype != ltx25::ST_F16 && t.dtype != ltx25::ST_BF16) {
      *msg = "load: '" + t.name + "' is not a float tensor";
      return LTX_E_UNSUPPORTED;
    }
    size_t n = 1;
    for (int64_t d : t.shape) n *= (size_t)d;
    if (n == 0) continue;
    buf.resize(n);
    if (!ltx25::SafeTensors::to_f32(t, 0, n, buf.data())) {
      *msg = "load: '" + t.name + "' could not be read";
      return LTX_E_SHAPE;
    }
    const int rows = t.shape.empty() ? 1 : (int)t.shape[0];
    const int cols = t.shape.size() <= 1 ? 0 : (int)(n / (size_t)rows);
    std::string e;
    if (!tfn(t.name.substr(pre.size()), buf.data(), rows, cols, &e)) {
      *msg = e;
      return code_for(e);
    }
    ++bound;
  }
  if (bound == 0) {
    *msg = "load: no tensor under '" + pre + "'";
    return LTX_E_STATE;
  }
  return LTX_OK;
}

}  // namespace

extern "C" {

int ltx_block_load_st(ltx_block* b, const ltx_st* f, const char* prefix)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(b == nullptr ? nullptr : b->ctx));
    if (b == nullptr) return LTX_E_NULL;
    if (f == nullptr || prefix == nullptr)
      return bfail(b, LTX_E_NULL, "load: null checkpoint or prefix");
    std::string msg;
    const int rc = load_prefix(
        f->f, prefix,
        [&](const std::string& n, const uint32_t* c, const void* sc, const void* bz, int sbd, int N,
            int K, std::string* e) { return b->blk->set_qlinear(n, c, sc, bz, sbd, N, K, false, e); },
        [&](const std::string& n, const float* d, int rows, int cols, std::string* e) {
          return b->blk->set_tensor(n, d, rows, cols, false, e);
        },
        &msg);
    return rc == LTX_OK ? LTX_OK : bfail(b, rc, msg);
  });
}

int ltx_lora_load_st(ltx_ctx* ctx, const ltx_st* f, const char* module, int k, int n,
                     float lora_scale, ltx_lora** out)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr || out == nullptr) return LTX_E_NULL;
    *out = nullptr;
    if (f == nullptr || module == nullptr)
      return fail(ctx, LTX_E_NULL, "lora load: null checkpoint or module");
    const ltx25::SafeTensors& st = f->f;
    const std::string m(module);
    const int ai = st.find(m + ".lora_A.weight"), bi = st.find(m + ".lora_B.weight");
    if (ai < 0 && bi < 0) return fail(ctx, LTX_E_STATE, "lora load: '" + m + "' is not adapted");
    if (ai < 0 || bi < 0)
      return fail(ctx, LTX_E_SHAPE, "lora load: '" + m + "' has only one of lora_A / lora_B");
    const ltx25::StTensor& a = st.at(ai);
    const ltx25::StTensor& b = st.at(bi);
    // rank from each tensor's size against the base widths, cross-checked
    // (bind_pair_, src/ltx25-lora.cc:96-117)
    const size_t ea = a.bytes / std::max<size_t>(1, ltx25::SafeTensors::elem_size(a.dtype));
    const size_t eb = b.bytes / std::max<size_t>(1, ltx25::SafeTensors::elem_size(b.dtype));
    if (k <= 0 || n <= 0 || ea % (size_t)k != 0 || eb % (size_t)n != 0)
      return fail(ctx, LTX_E_SHAPE, "lora load: '" + m + "' does not divide by its base widths");
    const size_t ra = ea / (size_t)k, rb = eb / (size_t)n;
    if (ra == 0 || ra != rb)
      return fail(ctx, LTX_E_SHAPE, "lora load: '" + m + "' rank disagrees between lora_A (" +
                                        std::to_string(ra) + ") and lora_B (" + std::to_string(rb) +
                                        ")");
    // lora_scale times alpha / rank when the file's metadata names both
    // (LoraAdapter::load, src/ltx25-lora.cc:265-287)
    double factor = lora_scale;
    auto num = [&](const char* key, double* v) {
      const std::string* s = st.metadata(key);
      if (s == nullptr || s->empty()) return false;
      char* end = nullptr;
      *v = std::strtod(s->c_str(), &end);
      return end != s->c_str() && std::isfinite(*v);
    };
    double alpha = 0.0, rank = 0.0;
    if (num("lora_alpha", &alpha) && num("lora_rank", &rank) && rank > 0.0 && alpha > 0.0)
      factor *= alpha / rank;
    std::vector<uint16_t> ab(ea), bb(eb);
    if (!ltx25::SafeTensors::to_bf16(a, 0, ea, ab.data()) ||
        !ltx25::SafeTensors::to_bf16(b, 0, eb, bb.data()))
      return fail(ctx, LTX_E_UNSUPPORTED, "lora load: '" + m + "' is not a float pair");
    return ltx_lora_upload(ctx, ab.data(), bb.data(), (int)ra, k, n, (float)factor, 0, out);
  });
}


// ---- the embeddings connector -------------------------------------------------

}  // extern "C"

struct ltx_connector {
  ltx_ctx* ctx = nullptr;
  ltx25::CudaConnector* c = nullptr;
  std::string err;
};

namespace {

int cfail(ltx_connector* c, int code, const std::string& m)
{
  if (c != nullptr) c->err = m;
  return code;
}

}  // namespace

extern "C" {

int ltx_connector_create(ltx_ctx* ctx, int heads, int head_dim, int layers, int registers,
                         int norm_output, double theta, int max_pos, int rope_f64,
                         ltx_connector** out)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(ctx));
    if (ctx == nullptr || out == nullptr) return LTX_E_NULL;
    *out = nullptr;
    if (heads <= 0 || head_dim <= 0 || layers <= 0 || registers < 0 || max_pos <= 0)
      return fail(ctx, LTX_E_SHAPE, "connector shape");
    ltx_connector* c = new (std::nothrow) ltx_connector();
    if (c == nullptr) return LTX_E_OOM;
    c->ctx = ctx;
    c->c = new (std::nothrow) ltx25::CudaConnector(&ctx->ops, heads, head_dim, layers, registers,
                                                   norm_output != 0, theta, max_pos,
                                                   rope_f64 != 0);
    if (c->c == nullptr) {
      delete c;
      return LTX_E_OOM;
    }
    *out = c;
    return LTX_OK;
  });
}

void ltx_connector_destroy(ltx_connector* c)
{
  OnDevice on_(dev_of(c == nullptr ? nullptr : c->ctx));
  if (c == nullptr) return;
  delete c->c;
  delete c;
}

const char* ltx_connector_last_error(const ltx_connector* c)
{
  return c == nullptr ? "null connector" : c->err.c_str();
}

int ltx_connector_set_qlinear(ltx_connector* c, const char* name, const uint32_t* codes,
                              const void* scales, const void* biases, int sb_dtype, int N, int K,
                              int on_device)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(c == nullptr ? nullptr : c->ctx));
    if (c == nullptr) return LTX_E_NULL;
    if (name == nullptr) return cfail(c, LTX_E_NULL, "set_qlinear: null name");
    std::string e;
    if (!c->c->set_qlinear(name, codes, scales, biases, sb_dtype, N, K, on_device != 0, &e))
      return cfail(c, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_connector_set_tensor(ltx_connector* c, const char* name, const float* data, int rows,
                             int cols, int on_device)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(c == nullptr ? nullptr : c->ctx));
    if (c == nullptr) return LTX_E_NULL;
    if (name == nullptr) return cfail(c, LTX_E_NULL, "set_tensor: null name");
    std::string e;
    if (!c->c->set_tensor(name, data, rows, cols, on_device != 0, &e))
      return cfail(c, code_for(e), e);
    return LTX_OK;
  });
}

int ltx_connector_load_st(ltx_connector* c, const ltx_st* f, const char* root)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(c == nullptr ? nullptr : c->ctx));
    if (c == nullptr) return LTX_E_NULL;
    if (f == nullptr || root == nullptr)
      return cfail(c, LTX_E_NULL, "load: null checkpoint or root");
    std::string msg;
    const int rc = load_prefix(
        f->f, root,
        [&](const std::string& n, const uint32_t* q, const void* sc, const void* bz, int sbd, int N,
            int K, std::string* e) { return c->c->set_qlinear(n, q, sc, bz, sbd, N, K, false, e); },
        [&](const std::string& n, const float* d, int rows, int cols, std::string* e) {
          return c->c->set_tensor(n, d, rows, cols, false, e);
        },
        &msg);
    return rc == LTX_OK ? LTX_OK : cfail(c, rc, msg);
  });
}

int ltx_connector_finalize(ltx_connector* c)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(c == nullptr ? nullptr : c->ctx));
    if (c == nullptr) return LTX_E_NULL;
    std::string e;
    if (!c->c->finalize(&e))
      return cfail(c, e.find("missing") != std::string::npos ? LTX_E_STATE : code_for(e), e);
    return LTX_OK;
  });
}

int ltx_connector_reserve(ltx_connector* c, int tokens)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(c == nullptr ? nullptr : c->ctx));
    if (c == nullptr) return LTX_E_NULL;
    std::string e;
    if (!c->c->reserve(tokens, &e))
      return cfail(c, e.find("before") != std::string::npos ? LTX_E_STATE : code_for(e), e);
    return LTX_OK;
  });
}

int ltx_connector_forward(ltx_connector* c, const void* in, void* out, int tokens, int n_valid,
                          void* stream)
{
  return guarded([&]() -> int {
    OnDevice on_(dev_of(c == nullptr ? nullptr : c->ctx));
    if (c == nullptr) return LTX_E_NULL;
    std::string e;
    if (!c->c->forward(S(stream), static_cast<const __nv_bfloat16*>(in),
                       static_cast<__nv_bfloat16*>(out), tokens, n_valid, &e))
      return cfail(c, e.find("before") != std::string::npos ? LTX_E_STATE : code_for(e), e);
    return LTX_OK;
  });
}

// ---- the trunk's adaLN chains (host) ---------------------------------------

int ltx_adaln_create(const uint16_t* w1, const uint16_t* b1, const uint16_t* w2,
                     const uint16_t* b2, const uint16_t* w3, const uint16_t* b3, int dim,
                     int out_dim, ltx_adaln** out)
{
  return guarded([&]() -> int {
    if (out == nullptr || w1 == nullptr || w2 == nullptr || w3 == nullptr) return LTX_E_NULL;
    *out = nullptr;
    if (dim <= 0 || out_dim <= 0) return LTX_E_SHAPE;
    ltx_adaln* a = new (std::nothrow) ltx_adaln();
    if (a == nullptr) return LTX_E_OOM;
    ltx25::AdaLNChain& c = a->c;
    c.dim = dim;
    c.out_dim = out_dim;
    const size_t d = (size_t)dim, od = (size_t)out_dim;
    c.w1.assign(w1, w1 + d * 256);
    c.w2.assign(w2, w2 + d * d);
    c.w3.assign(w3, w3 + od * d);
    if (b1 != nullptr) c.b1.assign(b1, b1 + d);
    if (b2 != nullptr) c.b2.assign(b2, b2 + d);
    if (b3 != nullptr) c.b3.assign(b3, b3 + od);
    *out = a;
    return LTX_OK;
  });
}

int ltx_adaln_load_st(const ltx_st* f, const char* prefix, ltx_adaln** out, char* err,
                      int err_len)
{
  return guarded([&]() -> int {
    if (out == nullptr || f == nullptr || prefix == nullptr) return LTX_E_NULL;
    *out = nullptr;
    const std::string pre(prefix);
    const ltx25::SafeTensors& st = f->f;
    auto say = [&](const std::string& m, int code) {
      if (err != nullptr && err_len > 0) {
        std::strncpy(err, m.c_str(), (size_t)err_len - 1);
        err[err_len - 1] = '\0';
      }
      return code;
    };
    // bind_adaln_'s names (src/ltx25-lora.cc:145-158): the timestep
    // embedder's two linears, then the root projection
    const std::string n1 = pre + "emb.timestep_embedder.linear_1", n2 =
                           pre + "emb.timestep_embedder.linear_2", n3 = pre + "linear";
    const int i1 = st.find(n1 + ".weight"), i2 = st.find(n2 + ".weight"),
              i3 = st.find(n3 + ".weight");
    if (i1 < 0 || i2 < 0 || i3 < 0)
      return say("adaln: missing '" + (i1 < 0 ? n1 : i2 < 0 ? n2 : n3) + ".weight'", LTX_E_STATE);
    const ltx25::StTensor &t1 = st.at(i1), &t2 = st.at(i2), &t3 = st.at(i3);
    if (t1.shape.size() != 2 || t1.shape[1] != 256 || t2.shape.size() != 2 ||
        t2.shape[0] != t1.shape[0] || t2.shape[1] != t1.shape[0] || t3.shape.size() != 2 ||
        t3.shape[1] != t1.shape[0])
      return say("adaln: shapes are not [dim][256], [dim][dim], [out][dim]", LTX_E_SHAPE);
    ltx_adaln* a = new (std::nothrow) ltx_adaln();
    if (a == nullptr) return LTX_E_OOM;
    ltx25::AdaLNChain& c = a->c;
    c.dim = (int)t1.shape[0];
    c.out_dim = (int)t3.shape[0];
    auto rd = [&](const ltx25::StTensor& t, std::vector<uint16_t>* v) {
      size_t n = 1;
      for (int64_t d : t.shape) n *= (size_t)d;
      v->resize(n);
      return ltx25::SafeTensors::to_bf16(t, 0, n, v->data());
    };
    auto bias = [&](const std::string& n, size_t want, std::vector<uint16_t>* v) {
      const int i = st.find(n + ".bias");
      if (i < 0) return true;   // a linear without bias
      return rd(st.at(i), v) && v->size() == want;
    };
    if (!rd(t1, &c.w1) || !rd(t2, &c.w2) || !rd(t3, &c.w3) ||
        !bias(n1, (size_t)c.dim, &c.b1) || !bias(n2, (size_t)c.dim, &c.b2) ||
        !bias(n3, (size_t)c.out_dim, &c.b3)) {
      delete a;
      return say("adaln: a tensor is not float or a bias has the wrong width", LTX_E_SHAPE);
    }
    *out = a;
    return LTX_OK;
  });
}

void ltx_adaln_free(ltx_adaln* a) { delete a; }

int ltx_adaln_dims(const ltx_adaln* a, int* dim, int* out_dim)
{
  return guarded([&]() -> int {
    if (a == nullptr) return LTX_E_NULL;
    if (dim) *dim = a->c.dim;
    if (out_dim) *out_dim = a->c.out_dim;
    return LTX_OK;
  });
}

int ltx_adaln_run(const ltx_adaln* a, double timestep, float* out, float* embedded, int threads)
{
  return guarded([&]() -> int {
    if (a == nullptr || out == nullptr) return LTX_E_NULL;
    ltx25::adaln_run(a->c, timestep, out, embedded, threads);
    return LTX_OK;
  });
}

int ltx_adaln_run_many(const ltx_adaln* const* chains, const double* timesteps,
                       float* const* outs, float* const* embedded, int count, int threads)
{
  return guarded([&]() -> int {
    if (count < 0) return LTX_E_SHAPE;
    if (count == 0) return LTX_OK;
    if (chains == nullptr || timesteps == nullptr || outs == nullptr) return LTX_E_NULL;
    std::vector<const ltx25::AdaLNChain*> cs((size_t)count);
    for (int i = 0; i < count; ++i) {
      if (chains[i] == nullptr || outs[i] == nullptr) return LTX_E_NULL;
      cs[(size_t)i] = &chains[i]->c;
    }
    ltx25::adaln_run_many(cs.data(), timesteps, outs, embedded, count, threads);
    return LTX_OK;
  });
}

}  // extern "C"
