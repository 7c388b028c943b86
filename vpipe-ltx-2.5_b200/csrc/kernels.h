// kernels.h -- host-side launchers for the ltx25 CUDA kernels.  Internal to
// the library: the public surface is include/ltx25_cuda.h.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>

#include "gemm_tc.cuh"

namespace ltx {

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType,
                                    cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle,
                                    CUtensorMapL2promotion,
                                    CUtensorMapFloatOOBfill);

struct GemmLaunch {
  int mode = MODE_W8G64;   // GemmMode
  int tn = 256;            // token tile: 128 or 256
  bool pair = false;       // cta_group::2 pairs (MODE_W8G64 / MODE_BF16, tn 256)
  int wb = 1;              // weight blocks per CTA: 2 for dense pairs only
                           // (512 weight rows per tile, n_tiles = N / 512)
  int epi = EPI_STORE;     // EpiMode
  int num_sms = 148;
  const void* x = nullptr; // bf16 [M][ldx] (int8 for MODE_I8)
  int ldx = 0;             // elements
  const void* w = nullptr; // u8 codes [N][K] / bf16 [N][K] / int8 [N][K]
  const uint32_t* sz = nullptr;  // MODE_W8G64: [K/64][N] (scale | zp << 16)
  // K extension (MODE_BF16): ext_w bf16 [N][ext_k] and ext_x bf16
  // [M][ld_ext], contracted over ext_k after the main K (ext_k % 8 == 0).
  const void* ext_w = nullptr;
  const void* ext_x = nullptr;
  int ext_k = 0;
  int ld_ext = 0;
  GemmParams p{};
};

// 0 on success; negative on a launch/encode failure.
int gemm_launch(const GemmLaunch& L, cudaStream_t stream);
int gemm_smem_bytes(int mode, int tn);

// scales/biases [N][G] (dtype: 0 f16, 1 bf16, 2 f32) -> sz [G][N] u32 with
// the bf16 scale in the low half and the bf16 zero-point in the high half.
int launch_pack_sz(const void* scales, const void* biases, int dtype, int N,
                   int G, uint32_t* sz, cudaStream_t stream);
// The reference w8g64 quantizer on the device: w f32 [N][K] -> codes u32
// [N][K/4], scales / zero-points bf16 [N][K/64].
int launch_pack_w8g64(const float* w, int N, int K, uint32_t* codes,
                      uint16_t* scales, uint16_t* biases, cudaStream_t stream);
// codes u8 [N][K] + sz -> bf16 [N][K] (s*q + z, one rounding).
int launch_dequant_w8(const uint8_t* codes, const uint32_t* sz, int N, int K,
                      __nv_bfloat16* out, cudaStream_t stream);
// Symmetric int8 per (row, group): q = rint(x / (absmax/127)).
int launch_quant_rows_i8(const __nv_bfloat16* x, int rows, int K, int ldx,
                         int group, int8_t* q, float* scale,
                         cudaStream_t stream);

// Device address of the fixed int8-tier scratch array on `device`
// (i8_static.cu): LTX_I8_STATIC_MAX_CODES codes, then LTX_I8_STATIC_MAX_ROWS
// f32 scales.
bool i8_static_scratch(int device, int8_t** codes, float** scales, std::string* err);

// A one-thread kernel that waits `bound_ms` (1..2000) on an mbarrier nothing
// arrives at and records the timeout in `err` (watchdog.cu).
int launch_watchdog_probe(int* err, int bound_ms, cudaStream_t s);

}  // namespace ltx
