// ltx25-plugin-cuda.cc -- the B200 build's plugin entry: the same plugin
// symbol and registration shape as the reference's src/ltx25-plugin.cc:50-136
// (VPIPE_PLUGIN_DEFINE(&kInfo, ltx25_register), kRequires = {kernel
// contract, accel bag}), with the kernel registration swapped: where the
// reference hands the host three metallibs for MetalOps / MetalBlock, this
// hands it one table of entry points (include/ltx25_plugin.h) that routes
// the family's linear, weight binding, block and acceleration tiers through
// the C++ adapter of include/ltx25_cuda.hpp onto the sm_100a library.
//
// The reference's other registrations -- the video family's denoise loop,
// the conditioner / model-config / upscale stages, the VAE and quantize
// families, the catalog -- are that plugin's own code, outside this path;
// a B200 build of the plugin keeps them and links this file in place of
// the metallib registration.
//
// Built against the in-repo stub headers under plugin/stub (the vpipe SDK
// is not in this tree) into lib/vpipe-ltx-2.5-b200.so.
#include "plugin/plugin-abi.h"
#include "plugin/plugin-context.h"

#include <cstdio>
#include <cstring>
#include <exception>
#include <new>
#include <string>

#include "ltx25_cuda.hpp"
#include "ltx25_plugin.h"

// Opaque handles of the table: the adapters themselves.
struct ltx25_ops {
  ltx25::CudaOpsAdapter ops;
};
struct ltx25_block {
  ltx25::CudaBlockAdapter blk;
};

namespace {

// What this plugin cannot run without beyond the ABI integer, as in the
// reference (src/ltx25-plugin.cc:51-57): the host dispatches its kernels by
// name through the kernel contract, and the tiers arrive in the accel bag.
const char* const kRequires[] = {
    VPIPE_FEATURE_KERNEL_CONTRACT,
    VPIPE_FEATURE_ACCEL_BAG,
    nullptr,
};

const VpipePluginInfo kInfo = {
    VPIPE_PLUGIN_INFO_SCHEMA,
    "ltx-2.5",
    "0.2.0+b200",
    "ltx25-b200",
    "Apache-2.0 (plugin); the LTX-2.5 weights are under the LTX-2.x Community License",
    "LTX-2.5 joint audio-video DiT for generate-video: w8g64 qlinear and the AV block "
    "on B200 (sm_100a)",
    kRequires,
};

void put(char* err, int len, const std::string& msg)
{
  if (err == nullptr || len <= 0) return;
  const size_t n = std::min(msg.size(), (size_t)len - 1);
  std::memcpy(err, msg.data(), n);
  err[n] = '\0';
}

// Runs `body`; a C++ exception becomes LTX_E_HOST with its message.
template <typename Body>
int guard(char* err, int len, const Body& body) noexcept
{
  try {
    return body();
  } catch (const std::bad_alloc&) {
    put(err, len, "host allocation failed");
    return LTX_E_OOM;
  } catch (const std::exception& e) {
    put(err, len, e.what());
    return LTX_E_HOST;
  } catch (...) {
    put(err, len, "unknown host exception");
    return LTX_E_HOST;
  }
}

int ops_create(int device, ltx25_ops** out, char* err, int len)
{
  if (out == nullptr) return LTX_E_NULL;
  *out = nullptr;
  return guard(err, len, [&]() -> int {
    auto* o = new ltx25_ops();
    std::string e;
    if (!o->ops.init(device, &e)) {
      delete o;
      put(err, len, e);
      return LTX_E_CUDA;
    }
    *out = o;
    return LTX_OK;
  });
}

void ops_destroy(ltx25_ops* o) { delete o; }

ltx_ctx* ops_ctx(const ltx25_ops* o) { return o != nullptr ? o->ops.ctx() : nullptr; }

int bind_qlinear(ltx25_ops* o, const uint32_t* codes, const void* scales, const void* biases,
                 int sb_dtype, int N, int K, ltx_qweight** out, char* err, int len)
{
  if (o == nullptr || out == nullptr) return LTX_E_NULL;
  *out = nullptr;
  return guard(err, len, [&]() -> int {
    ltx25::CudaQWeight w;
    std::string e;
    if (!o->ops.bind_qlinear(codes, scales, biases, sb_dtype, N, K, &w, &e)) {
      put(err, len, e);
      return LTX_E_SHAPE;
    }
    // the model layer owns the handle from here and frees it with
    // qweight_free
    *out = w.release();
    return LTX_OK;
  });
}

void qweight_free(ltx_qweight* w) { ltx_qweight_free(w); }

int linear(ltx25_ops* o, void* stream, const void* x, const ltx_qweight* w, const void* bias,
           void* y, int M, int K, int N, char* err, int len)
{
  if (o == nullptr || w == nullptr) return LTX_E_NULL;
  return guard(err, len, [&]() -> int {
    o->ops.linear(stream, x, w, bias, y, M, K, N);
    return LTX_OK;
  });
}

int set_tiers(ltx25_ops* o, int i8_gemm, int sage_attn, int sage_dense_layers, char* err,
              int len)
{
  if (o == nullptr) return LTX_E_NULL;
  return guard(err, len, [&]() -> int {
    o->ops.set_tiers(i8_gemm != 0, sage_attn != 0, sage_dense_layers);
    return LTX_OK;
  });
}

int i8_takes(const ltx25_ops* o, int M, int K, int N)
{
  return o != nullptr && o->ops.i8_takes(M, K, N) ? 1 : 0;
}

int wait_ok(ltx25_ops* o, void* stream, char* err, int len)
{
  if (o == nullptr) return LTX_E_NULL;
  return guard(err, len, [&]() -> int {
    std::string e;
    if (o->ops.wait_ok(stream, &e)) return LTX_OK;
    put(err, len, e);
    return LTX_E_KERNEL;
  });
}

int block_create(ltx25_ops* o, int vdim, int vheads, int adim, int aheads, ltx25_block** out,
                 char* err, int len)
{
  if (o == nullptr || out == nullptr) return LTX_E_NULL;
  *out = nullptr;
  return guard(err, len, [&]() -> int {
    auto* b = new ltx25_block();
    std::string e;
    if (!b->blk.create(o->ops, vdim, vheads, adim, aheads, &e)) {
      delete b;
      put(err, len, e);
      return LTX_E_SHAPE;
    }
    *out = b;
    return LTX_OK;
  });
}

// The block calls: the adapter's bool + message, as MetalBlock's.
template <typename Call>
int block_call(ltx25_block* b, char* err, int len, const Call& call)
{
  if (b == nullptr) return LTX_E_NULL;
  return guard(err, len, [&]() -> int {
    std::string e;
    if (call(b->blk, &e)) return LTX_OK;
    put(err, len, e);
    return LTX_E_SHAPE;
  });
}

int block_set_qlinear(ltx25_block* b, const char* name, const uint32_t* codes,
                      const void* scales, const void* biases, int sb_dtype, int N, int K,
                      char* err, int len)
{
  return block_call(b, err, len, [&](ltx25::CudaBlockAdapter& a, std::string* e) {
    return a.set_qlinear(name, codes, scales, biases, sb_dtype, N, K, e);
  });
}

int block_set_tensor(ltx25_block* b, const char* name, const float* data, int rows, int cols,
                     char* err, int len)
{
  return block_call(b, err, len, [&](ltx25::CudaBlockAdapter& a, std::string* e) {
    return a.set_tensor(name, data, rows, cols, e);
  });
}

int block_finalize(ltx25_block* b, char* err, int len)
{
  return block_call(b, err, len,
                    [&](ltx25::CudaBlockAdapter& a, std::string* e) { return a.finalize(e); });
}

int block_reserve(ltx25_block* b, int vt, int at, int tt, char* err, int len)
{
  return block_call(b, err, len, [&](ltx25::CudaBlockAdapter& a, std::string* e) {
    return a.reserve(vt, at, tt, e);
  });
}

int block_set_layer(ltx25_block* b, int layer, char* err, int len)
{
  return block_call(b, err, len, [&](ltx25::CudaBlockAdapter& a, std::string* e) {
    return a.set_layer(layer, e);
  });
}

int block_forward(ltx25_block* b, void* stream, const ltx_stream_io* video,
                  const ltx_stream_io* audio, char* err, int len)
{
  return block_call(b, err, len, [&](ltx25::CudaBlockAdapter& a, std::string* e) {
    return a.forward(stream, video, audio, e);
  });
}

void block_destroy(ltx25_block* b) { delete b; }

const ltx25_cuda_kernels kTable = {
    LTX25_CUDA_KERNELS_VERSION,
    LTX25_ABI_VERSION,
    ops_create,
    ops_destroy,
    ops_ctx,
    bind_qlinear,
    qweight_free,
    linear,
    set_tiers,
    i8_takes,
    wait_ok,
    block_create,
    block_set_qlinear,
    block_set_tensor,
    block_finalize,
    block_reserve,
    block_set_layer,
    block_forward,
    block_destroy,
};

void ltx25_register(vpipe::VpipePluginContext* ctx)
{
  if (ctx == nullptr) return;
  // The kernels, before anything can dispatch them (the reference's
  // register_metal_library calls, src/ltx25-plugin.cc:117-133): one table,
  // refused by the host if the name is taken.  A library built for another
  // C ABI than this header's is not registered at all.
  if (ltx_abi_version() != LTX25_ABI_VERSION) return;
  const vpipe::KernelTable t = {LTX25_CUDA_KERNELS_NAME, "cuda/sm_100a", &kTable,
                                sizeof(kTable)};
  ctx->register_kernel_table(t);
}

}  // namespace

VPIPE_PLUGIN_DEFINE(&kInfo, ltx25_register)
