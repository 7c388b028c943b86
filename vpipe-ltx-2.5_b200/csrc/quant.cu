// quant.cu -- byte/integer kernels around the w8g64 pack and the int8 tier:
// the one-time scale/zero-point relayout, the dequant-once expansion, and
// symmetric int8 row quantization.  All HBM-bound.
#include <cuda_fp16.h>

#include "block_ops.h"
#include "kernels.h"

namespace ltx {

namespace {

__device__ __forceinline__ uint16_t to_bf16_bits(float f)
{
  const __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<const uint16_t*>(&b);
}

// One-time relayout at upload (src/ltx25-dit-weights.cc:230-277 converts
// F16 scales/biases to bf16 with RNE; the per-group pair is then stored
// K-group-major so one 512-byte TMA box serves a 128-row weight tile).
__global__ void pack_sz_kernel(const void* __restrict__ scales,
                               const void* __restrict__ biases, int dtype,
                               int N, int G, uint32_t* __restrict__ sz)
{
  pdl_wait();
  pdl_trigger();
  const long long total = (long long)N * G;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
       i < total; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / G), g = (int)(i % G);
    uint16_t s, z;
    if (dtype == 0) {
      s = to_bf16_bits(__half2float(reinterpret_cast<const __half*>(scales)[i]));
      z = to_bf16_bits(__half2float(reinterpret_cast<const __half*>(biases)[i]));
    } else if (dtype == 1) {
      s = reinterpret_cast<const uint16_t*>(scales)[i];
      z = reinterpret_cast<const uint16_t*>(biases)[i];
    } else {
      s = to_bf16_bits(reinterpret_cast<const float*>(scales)[i]);
      z = to_bf16_bits(reinterpret_cast<const float*>(biases)[i]);
    }
    sz[(size_t)g * N + n] = (uint32_t)s | ((uint32_t)z << 16);
  }
}

// Dequant-once: 16 codes per thread, one fma.rn.bf16x2 per pair -- the same
// arithmetic the fused GEMM uses, so both arms see identical weights.
__global__ void dequant_w8_kernel(const uint8_t* __restrict__ codes,
                                  const uint32_t* __restrict__ sz, int N,
                                  int K, __nv_bfloat16* __restrict__ out)
{
  pdl_wait();
  pdl_trigger();
  const long long chunks = (long long)N * (K / 16);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
       i < chunks; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / (K / 16));
    const int k = (int)(i % (K / 16)) * 16;
    const uint4 c = *reinterpret_cast<const uint4*>(codes + (size_t)n * K + k);
    const uint32_t p = sz[(size_t)(k / 64) * N + n];
    const uint32_t s2 = __byte_perm(p, 0, 0x1010);
    const uint32_t z2 = __byte_perm(p, 0, 0x3232);
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
    uint32_t o[8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float f0 = __uint_as_float(__byte_perm(w[u], 0x4B000000u, 0x7650 | (2 * h))) - 8388608.0f;
        const float f1 = __uint_as_float(__byte_perm(w[u], 0x4B000000u, 0x7650 | (2 * h + 1))) - 8388608.0f;
        const uint32_t q2 = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
        uint32_t r;
        asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(q2), "r"(s2), "r"(z2));
        o[u * 2 + h] = r;
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)n * K + k);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// One CTA per (row, group).  absmax -> scale = absmax / 127 (IEEE divide),
// q = rint(x / scale) clamped to [-127, 127]: the exact arithmetic of the
// CPU restatement, so the codes match bit for bit.
__global__ void quant_rows_i8_kernel(const __nv_bfloat16* __restrict__ x,
                                     int K, int ldx, int group,
                                     int8_t* __restrict__ q,
                                     float* __restrict__ scale)
{
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.y;
  const int g = blockIdx.x;
  const __nv_bfloat16* xs = x + (size_t)row * ldx + (size_t)g * group;
  float amax = 0.0f;
  for (int k = threadIdx.x * 8; k < group; k += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xs + k);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1)
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float a = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1)
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (threadIdx.x == 0) red[0] = a;
  }
  __syncthreads();
  amax = red[0];
  const float sc = __fdiv_rn(amax, 127.0f);
  const int gcols = K / group;
  if (threadIdx.x == 0) scale[(size_t)row * gcols + g] = sc;
  int8_t* qs = q + (size_t)row * K + (size_t)g * group;
  for (int k = threadIdx.x * 8; k < group; k += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xs + k);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
    uint32_t packed[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      int a = 0, b = 0;
      if (amax != 0.0f) {
        a = (int)fminf(fmaxf(rintf(__fdiv_rn(f.x, sc)), -127.0f), 127.0f);
        b = (int)fminf(fmaxf(rintf(__fdiv_rn(f.y, sc)), -127.0f), 127.0f);
      }
      const uint32_t pair = ((uint32_t)(a & 0xff)) | ((uint32_t)(b & 0xff) << 8);
      packed[i >> 1] |= pair << (16 * (i & 1));
    }
    *reinterpret_cast<uint2*>(qs + k) = make_uint2(packed[0], packed[1]);
  }
}

// The w8g64 quantizer, one warp per (row, 64-group).  The arithmetic of the
// reference's packer (tests/ltx25-qlinear-test.cc:94-141) -- min/max, scale
// = (hi - lo) / 255 and both rounded to bf16, q = lround((w - lo) / scale)
// clamped to [0, 255], 0 when the scale is 0 -- done in IEEE single
// operations, so the pack is bit-identical.
__global__ void pack_w8g64_kernel(const float* __restrict__ w, int N, int K,
                                  uint32_t* __restrict__ codes,
                                  uint16_t* __restrict__ scales,
                                  uint16_t* __restrict__ biases)
{
  pdl_wait();
  pdl_trigger();
  const int G = K / 64;
  const long long warp_id =
      (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= (long long)N * G) return;
  const int n = (int)(warp_id / G), g = (int)(warp_id % G);
  const float2 v =
      *reinterpret_cast<const float2*>(w + (size_t)n * K + g * 64 + lane * 2);
  float lo = fminf(v.x, v.y), hi = fmaxf(v.x, v.y);
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  const float sc = __fdiv_rn(__fsub_rn(hi, lo), 255.0f);
  const uint16_t sc_b = to_bf16_bits(sc), lo_b = to_bf16_bits(lo);
  const float scr = __uint_as_float((uint32_t)sc_b << 16);
  const float lor = __uint_as_float((uint32_t)lo_b << 16);
  int q0 = 0, q1 = 0;
  if (scr > 0.0f) {
    q0 = (int)lroundf(__fdiv_rn(__fsub_rn(v.x, lor), scr));
    q1 = (int)lroundf(__fdiv_rn(__fsub_rn(v.y, lor), scr));
    q0 = min(max(q0, 0), 255);
    q1 = min(max(q1, 0), 255);
  }
  const uint32_t half = (uint32_t)q0 | ((uint32_t)q1 << 8);
  const uint32_t other = __shfl_down_sync(0xffffffffu, half, 1);
  if ((lane & 1) == 0)
    codes[(size_t)n * (K / 4) + g * 16 + lane / 2] = half | (other << 16);
  if (lane == 0) {
    scales[(size_t)n * G + g] = sc_b;
    biases[(size_t)n * G + g] = lo_b;
  }
}

int grid_for(long long work, int threads)
{
  long long g = (work + threads - 1) / threads;
  if (g > 148LL * 16) g = 148LL * 16;
  if (g < 1) g = 1;
  return (int)g;
}

}  // namespace

int launch_pack_sz(const void* scales, const void* biases, int dtype, int N,
                   int G, uint32_t* sz, cudaStream_t stream)
{
  launch_k(pack_sz_kernel, dim3(grid_for((long long)N * G, 256)), dim3(256), 0, stream, 1, scales, biases, dtype, N, G, sz);
  return launched();
}

int launch_pack_w8g64(const float* w, int N, int K, uint32_t* codes,
                      uint16_t* scales, uint16_t* biases, cudaStream_t stream)
{
  if (K % 64 != 0 || N <= 0) return -1;
  const long long threads = (long long)N * (K / 64) * 32;
  const int block = 256;
  const long long grid = (threads + block - 1) / block;
  launch_k(pack_w8g64_kernel, dim3((unsigned)grid), dim3(block), 0, stream, 1, w, N, K, codes, scales, biases);
  return launched();
}

int launch_dequant_w8(const uint8_t* codes, const uint32_t* sz, int N, int K,
                      __nv_bfloat16* out, cudaStream_t stream)
{
  launch_k(dequant_w8_kernel, dim3(grid_for((long long)N * (K / 16), 256)), dim3(256), 0, stream, 1, codes, sz, N, K, out);
  return launched();
}

int launch_quant_rows_i8(const __nv_bfloat16* x, int rows, int K, int ldx,
                         int group, int8_t* q, float* scale,
                         cudaStream_t stream)
{
  if (group % 8 != 0 || K % group != 0) return -1;
  int threads = group / 8;
  if (threads > 256) threads = 256;
  threads = (threads + 31) / 32 * 32;
  dim3 grid(K / group, rows);
  launch_k(quant_rows_i8_kernel, dim3(grid), dim3(threads), 0, stream, 1, x, K, ldx, group, q, scale);
  return launched();
}

}  // namespace ltx
