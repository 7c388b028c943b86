// ltx25_cuda.hpp -- header-only C++ adapter over the C ABI in ltx25_cuda.h:
// the stand-in a plugin maintainer swaps in for MetalOps and QWeight on the
// quantized-linear path, keeping the plugin's call sites as they are.
//
//   MetalOps::init(mc, err)                  -> CudaOpsAdapter::init(device, err)
//   bind_qlinear(ws, mc, name, K, ...)       -> CudaOpsAdapter::bind_qlinear(...)
//     (src/ltx25-dit-weights.h:170-175; the checkpoint's u32 codes and F16
//      scales / biases as they sit)
//   MetalOps::linear(enc, x, w, bias, y, M, K, N)  (src/ltx25-metal-ops.h:100-105)
//                                            -> CudaOpsAdapter::linear(stream, ...)
//   set_i8_gemm / set_sage / i8_takes        -> set_tiers / i8_takes
//   wait_ok() after a command buffer         -> wait_ok(stream, err)
//   MetalBlock::create/upload/reserve/forward (src/ltx25-block-metal.h:245-325)
//                                            -> CudaBlockAdapter
//
// MetalOps::linear returns nothing and reports shape errors at bind time; the
// adapter's linear() throws std::runtime_error with the library's message on
// any failure, so a caller that ignored the reference's silent path cannot
// miss one here.  Objects are move-only owners of their C handles.
#pragma once

#include <stdexcept>
#include <string>
#include <utility>

#include "ltx25_cuda.h"

namespace ltx25 {

// One uploaded linear (the reference's QWeight).
class CudaQWeight {
public:
  CudaQWeight() = default;
  ~CudaQWeight() { ltx_qweight_free(h_); }
  CudaQWeight(CudaQWeight&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
  CudaQWeight& operator=(CudaQWeight&& o) noexcept
  {
    if (this != &o) {
      ltx_qweight_free(h_);
      h_ = std::exchange(o.h_, nullptr);
    }
    return *this;
  }
  CudaQWeight(const CudaQWeight&) = delete;
  CudaQWeight& operator=(const CudaQWeight&) = delete;

  ltx_qweight* handle() const { return h_; }
  bool valid() const { return h_ != nullptr; }
  // Gives up ownership: the caller frees the handle with ltx_qweight_free.
  ltx_qweight* release() { return std::exchange(h_, nullptr); }

private:
  friend class CudaOpsAdapter;
  ltx_qweight* h_ = nullptr;
};

class CudaOpsAdapter {
public:
  CudaOpsAdapter() = default;
  ~CudaOpsAdapter() { ltx_ctx_destroy(ctx_); }
  CudaOpsAdapter(const CudaOpsAdapter&) = delete;
  CudaOpsAdapter& operator=(const CudaOpsAdapter&) = delete;

  // Selects the device and checks it is sm_100 (MetalOps::init checks the
  // Metal device and its kernels the same way: a hard failure, not a
  // fallback).
  bool init(int device, std::string* err)
  {
    const int rc = ltx_ctx_create(device, &ctx_);
    if (rc != LTX_OK) {
      if (err != nullptr)
        *err = "ltx_ctx_create(" + std::to_string(device) + ") failed with " +
               std::to_string(rc) + ": no usable sm_100a device";
      return false;
    }
    return true;
  }

  // bind_qlinear for a w8g64 pack: u32 codes [N][K/4], scales and biases
  // [N][K/64] in `sb_dtype` (LTX_SB_F16 as a checkpoint stores them).
  bool bind_qlinear(const uint32_t* codes, const void* scales, const void* biases,
                    int sb_dtype, int N, int K, CudaQWeight* out, std::string* err)
  {
    ltx_qweight* h = nullptr;
    const int rc = ltx_qweight_upload(ctx_, codes, scales, biases, sb_dtype, N, K,
                                      /*bits*/ 8, /*group*/ 64, /*on_device*/ 0, &h);
    if (rc != LTX_OK) {
      if (err != nullptr) *err = ltx_ctx_last_error(ctx_);
      return false;
    }
    *out = CudaQWeight();
    out->h_ = h;
    return true;
  }

  // MetalOps::linear: y[M][N] = x[M][K] . W^T (+ bias); the encoder becomes a
  // CUDA stream, the buffers are device pointers the caller owns.
  void linear(void* stream, const void* x, const CudaQWeight& w, const void* bias, void* y,
              int M, int K, int N) const
  {
    linear(stream, x, w.handle(), bias, y, M, K, N);
  }
  // The same on a handle the caller keeps owning.
  void linear(void* stream, const void* x, const ltx_qweight* w, const void* bias, void* y,
              int M, int K, int N) const
  {
    const int rc = ltx_qlinear(ctx_, w, x, bias, y, M, K, N, stream);
    if (rc != LTX_OK) throw std::runtime_error(ltx_ctx_last_error(ctx_));
  }

  // The accel bag's keys: i8_gemm, sage_attn, sage_dense_layers.
  void set_tiers(bool i8_gemm, bool sage_attn, int sage_dense_layers)
  {
    if (ltx_set_tiers(ctx_, i8_gemm ? 1 : 0, sage_attn ? 1 : 0, sage_dense_layers) != LTX_OK)
      throw std::runtime_error(ltx_ctx_last_error(ctx_));
  }
  bool i8_takes(int M, int K, int N) const { return ltx_i8_takes(ctx_, M, K, N) != 0; }

  // wait_ok(): surfaces a kernel that gave up on a bounded wait, or any
  // other asynchronous failure on `stream`.
  bool wait_ok(void* stream, std::string* err) const
  {
    if (ltx_ctx_check(ctx_, stream) == LTX_OK) return true;
    if (err != nullptr) *err = ltx_ctx_last_error(ctx_);
    return false;
  }

  ltx_ctx* ctx() const { return ctx_; }

private:
  ltx_ctx* ctx_ = nullptr;
};

// One joint audio-video block (the reference's MetalBlock): tensors staged
// under the reference's parameter names, finalize, reserve once per
// geometry, then forward with x updated in place.  bool + err string like
// MetalBlock's own calls.
class CudaBlockAdapter {
public:
  CudaBlockAdapter() = default;
  ~CudaBlockAdapter() { ltx_block_destroy(b_); }
  CudaBlockAdapter(const CudaBlockAdapter&) = delete;
  CudaBlockAdapter& operator=(const CudaBlockAdapter&) = delete;

  bool create(const CudaOpsAdapter& ops, int video_dim, int video_heads, int audio_dim,
              int audio_heads, std::string* err)
  {
    const int rc = ltx_block_create(ops.ctx(), video_dim, video_heads, audio_dim,
                                    audio_heads, &b_);
    if (rc != LTX_OK && err != nullptr)
      *err = ops.ctx() != nullptr ? ltx_ctx_last_error(ops.ctx()) : "no context";
    return rc == LTX_OK;
  }
  bool set_qlinear(const char* name, const uint32_t* codes, const void* scales,
                   const void* biases, int sb_dtype, int N, int K, std::string* err)
  {
    return ok_(ltx_block_set_qlinear(b_, name, codes, scales, biases, sb_dtype, N, K, 0), err);
  }
  bool set_tensor(const char* name, const float* data, int rows, int cols, std::string* err)
  {
    return ok_(ltx_block_set_tensor(b_, name, data, rows, cols, 0), err);
  }
  bool finalize(std::string* err) { return ok_(ltx_block_finalize(b_), err); }
  bool reserve(int video_tokens, int audio_tokens, int text_tokens, std::string* err)
  {
    return ok_(ltx_block_reserve(b_, video_tokens, audio_tokens, text_tokens), err);
  }
  bool set_layer(int layer, std::string* err) { return ok_(ltx_block_set_layer(b_, layer), err); }
  bool forward(void* stream, const ltx_stream_io* video, const ltx_stream_io* audio,
               std::string* err)
  {
    return ok_(ltx_block_forward(b_, video, audio, stream), err);
  }
  ltx_block* handle() const { return b_; }

private:
  bool ok_(int rc, std::string* err) const
  {
    if (rc == LTX_OK) return true;
    if (err != nullptr) *err = b_ != nullptr ? ltx_block_last_error(b_) : "no block";
    return false;
  }
  ltx_block* b_ = nullptr;
};

}  // namespace ltx25
