/* ltx25_plugin.h -- the kernel table the B200 plugin shim registers with the
 * vpipe host, and the model layer resolves by name.
 *
 * The reference plugin registers its kernels as three metallibs "under the
 * names the model layer resolves with load_library()" (src/ltx25-plugin.cc:
 * 117-133) and its model layer drives them through MetalOps / MetalBlock
 * (src/ltx25-metal-ops.h:80-151, src/ltx25-block-metal.h:245-325).  On B200
 * the shim (vpipe-ltx-2.5_b200/plugin/ltx25-plugin-cuda.cc, built into
 * lib/vpipe-ltx-2.5-b200.so) registers this one table under
 * LTX25_CUDA_KERNELS_NAME instead; every entry goes through the C++ adapter
 * of ltx25_cuda.hpp over the C ABI of ltx25_cuda.h.
 *
 * Every entry returns LTX_OK or an LTX_E_* code and, where it takes one,
 * writes a message into err[err_len]; nothing throws across the table.  */
#ifndef LTX25_PLUGIN_H
#define LTX25_PLUGIN_H

#include "ltx25_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LTX25_CUDA_KERNELS_NAME "ltx25-cuda-sm100a"
#define LTX25_CUDA_KERNELS_VERSION 1

/* One MetalOps stand-in (a CudaOpsAdapter) and one MetalBlock stand-in (a
 * CudaBlockAdapter). */
typedef struct ltx25_ops ltx25_ops;
typedef struct ltx25_block ltx25_block;

typedef struct ltx25_cuda_kernels {
  int version;        /* LTX25_CUDA_KERNELS_VERSION */
  int abi;            /* LTX25_ABI_VERSION the table was built against */
  /* MetalOps::init: a context on `device`; refuses a device that is not sm_100 */
  int (*ops_create)(int device, ltx25_ops** out, char* err, int err_len);
  void (*ops_destroy)(ltx25_ops* ops);
  ltx_ctx* (*ops_ctx)(const ltx25_ops* ops);
  /* bind_qlinear (src/ltx25-dit-weights.h:170-175): a w8g64 pack as the
   * checkpoint stores it (u32 codes, F16/BF16/F32 scales and biases) */
  int (*bind_qlinear)(ltx25_ops* ops, const uint32_t* codes, const void* scales,
                      const void* biases, int sb_dtype, int N, int K, ltx_qweight** out,
                      char* err, int err_len);
  void (*qweight_free)(ltx_qweight* w);
  /* MetalOps::linear (src/ltx25-metal-ops.h:100-105): y = x . W^T (+ bias),
   * device buffers the caller owns, enqueued on `stream` */
  int (*linear)(ltx25_ops* ops, void* stream, const void* x, const ltx_qweight* w,
                const void* bias, void* y, int M, int K, int N, char* err, int err_len);
  /* the accel bag's tiers (src/ltx25-generator.cc:297-375) */
  int (*set_tiers)(ltx25_ops* ops, int i8_gemm, int sage_attn, int sage_dense_layers,
                   char* err, int err_len);
  int (*i8_takes)(const ltx25_ops* ops, int M, int K, int N);
  /* a command buffer's wait_ok(): asynchronous failures on `stream` */
  int (*wait_ok)(ltx25_ops* ops, void* stream, char* err, int err_len);
  /* MetalBlock (src/ltx25-block-metal.h:245-325), one CudaBlockAdapter */
  int (*block_create)(ltx25_ops* ops, int video_dim, int video_heads, int audio_dim,
                      int audio_heads, ltx25_block** out, char* err, int err_len);
  int (*block_set_qlinear)(ltx25_block* b, const char* name, const uint32_t* codes,
                           const void* scales, const void* biases, int sb_dtype, int N,
                           int K, char* err, int err_len);
  int (*block_set_tensor)(ltx25_block* b, const char* name, const float* data, int rows,
                          int cols, char* err, int err_len);
  int (*block_finalize)(ltx25_block* b, char* err, int err_len);
  int (*block_reserve)(ltx25_block* b, int video_tokens, int audio_tokens, int text_tokens,
                       char* err, int err_len);
  int (*block_set_layer)(ltx25_block* b, int layer, char* err, int err_len);
  int (*block_forward)(ltx25_block* b, void* stream, const ltx_stream_io* video,
                       const ltx_stream_io* audio, char* err, int err_len);
  void (*block_destroy)(ltx25_block* b);
} ltx25_cuda_kernels;

#ifdef __cplusplus
}
#endif

#endif /* LTX25_PLUGIN_H */
