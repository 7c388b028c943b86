// block_ops.cu -- the bandwidth-bound row ops of the LTX-2.5 AV block.
//
// Each replaces a plugin Metal kernel of the reference (src/ltx25-kernels
// .metal) and follows the CPU reference's math (src/ltx25-block-ref.cc):
//
//   vec_add          adaLN rows: table[i] + timesteps[i]   (ada_values, av_ada_)
//   ada_zero         rms_norm(x) * (1 + scale) + shift     (ltx_ada_zero)
//                    with scale = shift = 0 it is ltx_rms_norm_out
//   modulate         x * (1 + scale) + shift               (adaln_modulate)
//   qk_norm_rope     RMSNorm over the WHOLE inner width with a gain, then the
//                    split-half rotation per head          (ltx_rms_norm_gain
//                                                           + ltx_rope_half_perhead)
//
// bf16 storage, f32 arithmetic, one CTA per row, 16-byte vector accesses.
#include "block_ops.h"

#include <atomic>
#include <cstdlib>

namespace ltx {

namespace {
std::atomic<unsigned long long> g_launches{0};
}  // namespace

int launched()
{
  if (cudaGetLastError() != cudaSuccess) return -1;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return 0;
}

unsigned long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red)
{
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8])
{
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8])
{
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = v;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi)
{
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void vec_add_kernel(const float* __restrict__ a,
                               const __nv_bfloat16* __restrict__ b,
                               float* __restrict__ out, int n)
{
  pdl_wait();
  pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += gridDim.x * blockDim.x) {
    out[i] = a[i] + (b != nullptr ? __bfloat162float(b[i]) : 0.0f);
  }
}

// out = (rms_norm(x) if norm) * (1 + scale) + shift.  scale/shift may be
// null (0).  dim % 8 == 0; a thread owns 8-element chunks of ROWS rows, so
// ROWS rows of loads are in flight together.  The rows stay in registers as
// raw bf16 (4 registers a chunk, widened when used) and the f32 scale/shift
// chunks are read only after the reduction, so the kernel fits three CTAs
// on an SM (12 rows in flight) where a float-resident form fits two.  Per
// row the arithmetic and the reduction order are those of a one-row CTA.
template <bool NORM, int ROWS, int CH>
__global__ void __launch_bounds__(kRowThreads, 3)
    row_mod_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                   __nv_bfloat16* __restrict__ out, int ldo, int rows, int dim,
                   const float* __restrict__ scale,
                   const float* __restrict__ shift, float eps)
{
  pdl_wait();
  pdl_trigger();
  __shared__ float red[ROWS][33];
  const int r0 = blockIdx.x * ROWS;
  uint4 v[ROWS][CH];
  float ss[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    ss[r] = 0.0f;
    const bool live = r0 + r < rows;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int k = (c * kRowThreads + threadIdx.x) * 8;
      v[r][c] = make_uint4(0u, 0u, 0u, 0u);
      if (live && k < dim)
        v[r][c] = *reinterpret_cast<const uint4*>(x + (size_t)(r0 + r) * ldx + k);
    }
  }
  if (NORM) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[r][c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 t = __bfloat1622float2(h[i]);
          ss[r] = fmaf(t.x, t.x, ss[r]);
          ss[r] = fmaf(t.y, t.y, ss[r]);
        }
      }
    }
  }
  float inv[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) inv[r] = 1.0f;
  if (NORM) {
    // block_sum for ROWS values at once (same tree per row)
    const int w = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      float t = ss[r];
      for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if ((threadIdx.x & 31) == 0) red[r][w] = t;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[r][threadIdx.x] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[r][32] = t;
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < ROWS; ++r) inv[r] = rsqrtf(red[r][32] / (float)dim + eps);
  }
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int k = (c * kRowThreads + threadIdx.x) * 8;
    if (k >= dim) continue;
    float sc[8], sh[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) sc[i] = sh[i] = 0.0f;
    if (scale != nullptr) {
      const float4 a = *reinterpret_cast<const float4*>(scale + k);
      const float4 b = *reinterpret_cast<const float4*>(scale + k + 4);
      sc[0] = a.x; sc[1] = a.y; sc[2] = a.z; sc[3] = a.w;
      sc[4] = b.x; sc[5] = b.y; sc[6] = b.z; sc[7] = b.w;
    }
    if (shift != nullptr) {
      const float4 a = *reinterpret_cast<const float4*>(shift + k);
      const float4 b = *reinterpret_cast<const float4*>(shift + k + 4);
      sh[0] = a.x; sh[1] = a.y; sh[2] = a.z; sh[3] = a.w;
      sh[4] = b.x; sh[5] = b.y; sh[6] = b.z; sh[7] = b.w;
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      if (r0 + r >= rows) break;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[r][c]);
      float o[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 t = __bfloat1622float2(h[i]);
        o[2 * i] = fmaf(t.x * inv[r], 1.0f + sc[2 * i], sh[2 * i]);
        o[2 * i + 1] = fmaf(t.y * inv[r], 1.0f + sc[2 * i + 1], sh[2 * i + 1]);
      }
      store8(out + (size_t)(r0 + r) * ldo + k, o);
    }
  }
}

// q/k normalization over the whole inner width, gain, then RoPE (optional).
// in: row stride ldi (the fused-QKV output), out: compact [rows][inner].
// cos/sin: [heads][tokens][half] f32.
__global__ void __launch_bounds__(kRowThreads)
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ in, int ldi,
                        __nv_bfloat16* __restrict__ out, int ldo, int heads,
                        int head_dim, const float* __restrict__ gain,
                        const float* __restrict__ cosb,
                        const float* __restrict__ sinb, int tokens, float eps,
                        const float* __restrict__ sumsq, int norm_width,
                        int head0, int tbl_tokens, int tok0)
{
  pdl_wait();
  pdl_trigger();
  extern __shared__ float srow[];   // the normalized row, f32 [inner]
  __shared__ float red[33];
  const int inner = heads * head_dim;
  const int t = blockIdx.x;
  const __nv_bfloat16* xr = in + (size_t)t * ldi;
  float ss = 0.0f;
  for (int k = threadIdx.x * 8; k < inner; k += kRowThreads * 8) {
    float v[8];
    load8(xr + k, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ss = fmaf(v[i], v[i], ss);
      srow[k + i] = v[i];
    }
  }
  // A tensor-parallel rank holds only its heads' columns: the row's sum of
  // squares over the whole width then comes in already reduced.
  float total;
  if (sumsq != nullptr) {
    __syncthreads();   // publish srow
    total = sumsq[t];
  } else {
    total = block_sum(ss, red);   // (its barriers also publish srow)
  }
  const float inv = rsqrtf(total / (float)norm_width + eps);
  const int half = head_dim / 2;
  __nv_bfloat16* orow = out + (size_t)t * ldo;
  // Four consecutive rotation pairs (j .. j+3 of one head) per step: float4
  // gain / cos / sin reads, 8-byte stores.  half % 4 == 0 (32 or 64).
  const int quads = heads * half / 4;
  for (int idx = threadIdx.x; idx < quads; idx += kRowThreads) {
    const int h = (idx * 4) / half, j = (idx * 4) % half;
    const int ia = h * head_dim + j, ib = ia + half;
    float a[4], b[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      a[e] = srow[ia + e] * inv;
      b[e] = srow[ib + e] * inv;
    }
    if (gain != nullptr) {
      const float4 ga = *reinterpret_cast<const float4*>(gain + ia);
      const float4 gb = *reinterpret_cast<const float4*>(gain + ib);
      a[0] *= ga.x; a[1] *= ga.y; a[2] *= ga.z; a[3] *= ga.w;
      b[0] *= gb.x; b[1] *= gb.y; b[2] *= gb.z; b[3] *= gb.w;
    }
    if (cosb != nullptr) {
      const size_t o = ((size_t)(head0 + h) * tbl_tokens + tok0 + t) * half + j;
      const float4 c4 = *reinterpret_cast<const float4*>(cosb + o);
      const float4 s4 = *reinterpret_cast<const float4*>(sinb + o);
      const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float ra = a[e] * cc[e] - b[e] * sn[e];
        const float rb = b[e] * cc[e] + a[e] * sn[e];
        a[e] = ra;
        b[e] = rb;
      }
    }
    uint2 wa, wb;
    wa.x = pack2(a[0], a[1]);
    wa.y = pack2(a[2], a[3]);
    wb.x = pack2(b[0], b[1]);
    wb.y = pack2(b[2], b[3]);
    *reinterpret_cast<uint2*>(orow + ia) = wa;
    *reinterpret_cast<uint2*>(orow + ib) = wb;
  }
}

// The same op with each row held in registers: TR = quads / Q threads per
// row, Q rotation quads (four pairs j..j+3 of one head, both halves) per
// thread, 256 / TR rows per CTA.  One pass over the row: load, sum of
// squares (warp shuffles, then the row's warps through shared memory),
// normalize, gain, rotate, store -- no f32 copy of the row in shared
// memory, and narrow rows (a tensor-parallel rank's heads) share a CTA.
// Same arithmetic per element as qk_norm_rope_kernel; the sum of squares
// is added in another order.
template <int Q>
__global__ void __launch_bounds__(kRowThreads)
    qk_norm_rope_reg_kernel(const __nv_bfloat16* __restrict__ in, int ldi,
                            __nv_bfloat16* __restrict__ out, int ldo, int heads,
                            int head_dim, const float* __restrict__ gain,
                            const float* __restrict__ cosb,
                            const float* __restrict__ sinb, int tokens, float eps,
                            const float* __restrict__ sumsq, int norm_width,
                            int head0, int tbl_tokens, int tok0, int tr)
{
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kRowThreads / 32];
  const int half = head_dim / 2;
  const int rl = threadIdx.x / tr, li = threadIdx.x % tr;
  const int t = blockIdx.x * (kRowThreads / tr) + rl;
  const bool live = t < tokens;
  const __nv_bfloat16* xr = in + (size_t)(live ? t : 0) * ldi;
  float a[Q][4], b[Q][4];
  int ia_[Q];
  float ss = 0.0f;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const int idx = li + q * tr;
    const int h = (idx * 4) / half, j = (idx * 4) % half;
    const int ia = h * head_dim + j;
    ia_[q] = ia;
    uint2 ua = make_uint2(0u, 0u), ub = make_uint2(0u, 0u);
    if (live) {
      ua = *reinterpret_cast<const uint2*>(xr + ia);
      ub = *reinterpret_cast<const uint2*>(xr + ia + half);
    }
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&ua);
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&ub);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float2 fa = __bfloat1622float2(ha[e]), fb = __bfloat1622float2(hb[e]);
      a[q][2 * e] = fa.x;
      a[q][2 * e + 1] = fa.y;
      b[q][2 * e] = fb.x;
      b[q][2 * e + 1] = fb.y;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) ss = fmaf(a[q][e], a[q][e], fmaf(b[q][e], b[q][e], ss));
  }
  float total;
  if (sumsq != nullptr) {
    total = live ? sumsq[t] : 0.0f;
  } else {
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = ss;
    __syncthreads();
    const int w0 = (rl * tr) >> 5, nw = tr >> 5;
    total = 0.0f;
    for (int i = 0; i < nw; ++i) total += red[w0 + i];
  }
  if (!live) return;
  const float inv = rsqrtf(total / (float)norm_width + eps);
  __nv_bfloat16* orow = out + (size_t)t * ldo;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    const int ia = ia_[q], ib = ia + half;
    const int h = ia / head_dim, j = ia % head_dim;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      a[q][e] *= inv;
      b[q][e] *= inv;
    }
    if (gain != nullptr) {
      const float4 ga = *reinterpret_cast<const float4*>(gain + ia);
      const float4 gb = *reinterpret_cast<const float4*>(gain + ib);
      a[q][0] *= ga.x; a[q][1] *= ga.y; a[q][2] *= ga.z; a[q][3] *= ga.w;
      b[q][0] *= gb.x; b[q][1] *= gb.y; b[q][2] *= gb.z; b[q][3] *= gb.w;
    }
    if (cosb != nullptr) {
      const size_t o = ((size_t)(head0 + h) * tbl_tokens + tok0 + t) * half + j;
      const float4 c4 = *reinterpret_cast<const float4*>(cosb + o);
      const float4 s4 = *reinterpret_cast<const float4*>(sinb + o);
      const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float ra = a[q][e] * cc[e] - b[q][e] * sn[e];
        const float rb = b[q][e] * cc[e] + a[q][e] * sn[e];
        a[q][e] = ra;
        b[q][e] = rb;
      }
    }
    uint2 wa, wb;
    wa.x = pack2(a[q][0], a[q][1]);
    wa.y = pack2(a[q][2], a[q][3]);
    wb.x = pack2(b[q][0], b[q][1]);
    wb.y = pack2(b[q][2], b[q][3]);
    *reinterpret_cast<uint2*>(orow + ia) = wa;
    *reinterpret_cast<uint2*>(orow + ib) = wb;
  }
}

// One warp per row, eight rows per CTA: out[t] = the sum of squares of row
// t's `cols` values (f32), for the tensor-parallel q/k norms.
__global__ void __launch_bounds__(kRowThreads)
    row_sumsq_warp_kernel(const __nv_bfloat16* __restrict__ in, int ldi, int rows, int cols,
                          float* __restrict__ out)
{
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * (kRowThreads / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= rows) return;
  const __nv_bfloat16* xr = in + (size_t)t * ldi;
  float ss = 0.0f;
  for (int k = lane * 8; k < cols; k += 32 * 8) {
    float v[8];
    load8(xr + k, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) out[t] = ss;
}

// out[t] = sum of squares of row t's `cols` values (f32).
__global__ void __launch_bounds__(kRowThreads)
    row_sumsq_kernel(const __nv_bfloat16* __restrict__ in, int ldi, int cols,
                     float* __restrict__ out)
{
  pdl_wait();
  pdl_trigger();
  __shared__ float red[33];
  const __nv_bfloat16* xr = in + (size_t)blockIdx.x * ldi;
  float ss = 0.0f;
  for (int k = threadIdx.x * 8; k < cols; k += kRowThreads * 8) {
    float v[8];
    load8(xr + k, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
  }
  const float tot = block_sum(ss, red);
  if (threadIdx.x == 0) out[blockIdx.x] = tot;
}

// x = x + gate * (part + bias): the gated residual of a row-split output
// projection once its partial sums are reduced (the GEMM epilogue's
// EPI_GATED_RES arithmetic: a = acc + bias; x = fma(gate, a, x)).
__global__ void gated_residual_kernel(__nv_bfloat16* __restrict__ x, int ldx,
                                      const __nv_bfloat16* __restrict__ part,
                                      const __nv_bfloat16* __restrict__ bias,
                                      const float* __restrict__ gate, int rows,
                                      int dim, int nslot, size_t slot_stride)
{
  pdl_wait();
  pdl_trigger();
  const int chunks = dim / 8;
  const size_t total = (size_t)rows * chunks;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / chunks);
    const int k = (int)(i % chunks) * 8;
    float xv[8], pv[8];
    load8(x + (size_t)r * ldx + k, xv);
    load8(part + (size_t)r * dim + k, pv);
    // further partials (one per source rank), summed in slot order
    for (int sl = 1; sl < nslot; ++sl) {
      float qv[8];
      load8(part + sl * slot_stride + (size_t)r * dim + k, qv);
#pragma unroll
      for (int j = 0; j < 8; ++j) pv[j] += qv[j];
    }
    float bv[8];
    if (bias != nullptr) {
      load8(bias + k, bv);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) bv[j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) xv[j] = fmaf(gate[k + j], pv[j] + bv[j], xv[j]);
    store8(x + (size_t)r * ldx + k, xv);
  }
}

// dst[p][t][c] = src[t][p * cpr + c]: a token-major [rows][ranks * cpr]
// matrix regrouped into one contiguous [rows][cpr] block per rank (the send
// side of an all-to-all).  8 columns per thread.
__global__ void a2a_pack_kernel(const __nv_bfloat16* __restrict__ src, int ld, int rows,
                                int ranks, int cpr, __nv_bfloat16* __restrict__ dst)
{
  pdl_wait();
  pdl_trigger();
  const int c8 = cpr / 8;
  const size_t total = (size_t)ranks * rows * c8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % c8) * 8;
    const size_t pt = i / c8;
    const int t = (int)(pt % rows), p = (int)(pt / rows);
    *reinterpret_cast<uint4*>(dst + ((size_t)p * rows + t) * cpr + c) =
        *reinterpret_cast<const uint4*>(src + (size_t)t * ld + (size_t)p * cpr + c);
  }
}

// dst[t][p * cpr + c] = src[p][t][c] (* 2 sigmoid(gate[t][p * cpr / D + c / D])
// when gate is given): the receive side of an all-to-all back to token-major
// rows, applying the attention's per-head gate on the way.
__global__ void a2a_unpack_kernel(const __nv_bfloat16* __restrict__ src, int rows, int ranks,
                                  int cpr, __nv_bfloat16* __restrict__ dst, int ldd,
                                  const __nv_bfloat16* __restrict__ gate, int ldg, int head_dim)
{
  pdl_wait();
  pdl_trigger();
  const int c8 = cpr / 8;
  const size_t total = (size_t)ranks * rows * c8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % c8) * 8;
    const size_t pt = i / c8;
    const int t = (int)(pt % rows), p = (int)(pt / rows);
    uint4 w = *reinterpret_cast<const uint4*>(src + ((size_t)p * rows + t) * cpr + c);
    if (gate != nullptr) {
      const int col = p * cpr + c;
      const float g = __bfloat162float(gate[(size_t)t * ldg + col / head_dim]);
      const float f = 2.0f / (1.0f + __expf(-g));
      float v[8];
      load8(reinterpret_cast<const __nv_bfloat16*>(&w), v);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] *= f;
      store8(reinterpret_cast<__nv_bfloat16*>(&w), v);
    }
    *reinterpret_cast<uint4*>(dst + (size_t)t * ldd + (size_t)p * cpr + c) = w;
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ a,
                                   __nv_bfloat16* __restrict__ out, size_t n)
{
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(a[i]);
}

// The DiT output head's normalization (src/ltx25-dit.cc:2010-2031):
// out = LayerNorm(x) * (1 + scale) + shift, LayerNorm without affine
// (population variance, eps), f32 statistics in two block reductions.  One
// CTA per row; a thread holds CH chunks of 8 elements (dim <= 256 * 8 * CH).
template <int CH>
__global__ void __launch_bounds__(kRowThreads)
    layer_norm_mod_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                          __nv_bfloat16* __restrict__ out, int ldo, int dim,
                          const float* __restrict__ shift, const float* __restrict__ scale,
                          float eps)
{
  pdl_wait();
  pdl_trigger();
  __shared__ float red[33];
  const int row = blockIdx.x;
  float v[CH][8];
  float sum = 0.0f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int k = (c * kRowThreads + threadIdx.x) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[c][i] = 0.0f;
    if (k < dim) {
      load8(x + (size_t)row * ldx + k, v[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) sum += v[c][i];
    }
  }
  auto block_sum = [&](float t) {
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x < 32) {
      float u = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
      for (int o = 16; o > 0; o >>= 1) u += __shfl_xor_sync(0xffffffffu, u, o);
      if (threadIdx.x == 0) red[32] = u;
    }
    __syncthreads();
    const float r = red[32];
    __syncthreads();
    return r;
  };
  const float mean = block_sum(sum) / (float)dim;
  float sq = 0.0f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int k = (c * kRowThreads + threadIdx.x) * 8;
    if (k < dim) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[c][i] - mean;
        sq = fmaf(d, d, sq);
      }
    }
  }
  const float inv = rsqrtf(block_sum(sq) / (float)dim + eps);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int k = (c * kRowThreads + threadIdx.x) * 8;
    if (k >= dim) continue;
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o[i] = fmaf((v[c][i] - mean) * inv, 1.0f + scale[k + i], shift[k + i]);
    store8(out + (size_t)row * ldo + k, o);
  }
}

// x[r][c] += vec[c] for r < rows (the keyframe position embedding added to
// the first frame's tokens, src/ltx25-kernels.metal:349-358)
__global__ void add_row_prefix_kernel(__nv_bfloat16* __restrict__ x, int ldx,
                                      const __nv_bfloat16* __restrict__ vec, int rows, int cols)
{
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / cols, c = i - r * cols;
    __nv_bfloat16* p = x + r * ldx + c;
    *p = __float2bfloat16_rn(__bfloat162float(*p) + __bfloat162float(vec[c]));
  }
}

// dst[c][r] = src[r][c] through a 32 x 33 shared tile (coalesced both sides)
__global__ void transpose_bf16_kernel(const __nv_bfloat16* __restrict__ src, int lds,
                                      __nv_bfloat16* __restrict__ dst, int ldd, int rows,
                                      int cols)
{
  pdl_wait();
  pdl_trigger();
  __shared__ __nv_bfloat16 t[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[i][threadIdx.x] = src[(size_t)r * lds + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[(size_t)c * ldd + r] = t[threadIdx.x][i];
  }
}

// x[t][d] = regs[t % R][d] for t >= n_valid: the learnable registers tiled
// over the padded positions (src/ltx25-kernels.metal:382-396)
__global__ void fill_registers_kernel(__nv_bfloat16* __restrict__ x, int ldx,
                                      const __nv_bfloat16* __restrict__ regs, int dim, int R,
                                      int n_valid, int T)
{
  pdl_wait();
  pdl_trigger();
  const size_t n = (size_t)(T - n_valid) * dim;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const int t = n_valid + (int)(i / dim), d = (int)(i % dim);
    x[(size_t)t * ldx + d] = regs[(size_t)(t % R) * dim + d];
  }
}

__global__ void fill_f32_kernel(float* __restrict__ out, float v, size_t n)
{
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = v;
}

// out = bf16(f32(in) * scale), one rounding (the adapter's scale fold,
// src/ltx25-lora.cc:56-68)
__global__ void scale_bf16_kernel(const __nv_bfloat16* __restrict__ in,
                                  __nv_bfloat16* __restrict__ out, float scale, size_t n)
{
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(__bfloat162float(in[i]) * scale);
}

}  // namespace

int launch_layer_norm_mod(const __nv_bfloat16* x, int ldx, __nv_bfloat16* out, int ldo,
                          int rows, int dim, const float* shift, const float* scale, float eps,
                          cudaStream_t s)
{
  if (rows <= 0) return 0;
  if (dim % 8 != 0 || dim > kRowThreads * 8 * 4 || shift == nullptr || scale == nullptr ||
      ldx % 8 != 0 || ldo % 8 != 0)
    return -2;
  if (dim <= kRowThreads * 8 * 2)
    launch_k(layer_norm_mod_kernel<2>, dim3(rows), dim3(kRowThreads), 0, s, 1, x, ldx, out, ldo,
             dim, shift, scale, eps);
  else
    launch_k(layer_norm_mod_kernel<4>, dim3(rows), dim3(kRowThreads), 0, s, 1, x, ldx, out, ldo,
             dim, shift, scale, eps);
  return launched();
}

int launch_add_row_prefix(__nv_bfloat16* x, int ldx, const __nv_bfloat16* vec, int rows,
                          int cols, cudaStream_t s)
{
  if (rows <= 0 || cols <= 0) return 0;
  size_t grid = ((size_t)rows * cols + 255) / 256;
  if (grid > 4096) grid = 4096;
  launch_k(add_row_prefix_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, x, ldx, vec, rows,
           cols);
  return launched();
}

int launch_transpose_bf16(const __nv_bfloat16* src, int lds, __nv_bfloat16* dst, int ldd,
                          int rows, int cols, cudaStream_t s)
{
  if (rows <= 0 || cols <= 0) return 0;
  launch_k(transpose_bf16_kernel, dim3((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32)),
           dim3(32, 8), 0, s, 1, src, lds, dst, ldd, rows, cols);
  return launched();
}

int launch_fill_registers(__nv_bfloat16* x, int ldx, const __nv_bfloat16* regs, int dim, int R,
                          int n_valid, int T, cudaStream_t s)
{
  if (R <= 0 || n_valid >= T) return 0;
  if (n_valid < 0) return -2;
  size_t grid = ((size_t)(T - n_valid) * dim + 255) / 256;
  if (grid > 4096) grid = 4096;
  launch_k(fill_registers_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, x, ldx, regs, dim, R,
           n_valid, T);
  return launched();
}

int launch_fill_f32(float* out, float v, size_t n, cudaStream_t s)
{
  if (n == 0) return 0;
  size_t grid = (n + 255) / 256;
  if (grid > 4096) grid = 4096;
  launch_k(fill_f32_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, out, v, n);
  return launched();
}

int launch_scale_bf16(const __nv_bfloat16* in, __nv_bfloat16* out, float scale, size_t n,
                      cudaStream_t s)
{
  if (n == 0) return 0;
  size_t grid = (n + 255) / 256;
  if (grid > 4096) grid = 4096;
  launch_k(scale_bf16_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, in, out, scale, n);
  return launched();
}

int launch_f32_to_bf16(const float* a, __nv_bfloat16* out, size_t n,
                       cudaStream_t s)
{
  if (n == 0) return 0;
  size_t grid = (n + 255) / 256;
  if (grid > 4096) grid = 4096;
  launch_k(f32_to_bf16_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, a, out, n);
  return launched();
}

int launch_vec_add(const float* a, const __nv_bfloat16* b, float* out, int n,
                   cudaStream_t s)
{
  if (n <= 0) return 0;
  const int threads = 256;
  int grid = (n + threads - 1) / threads;
  if (grid > 1024) grid = 1024;
  launch_k(vec_add_kernel, dim3(grid), dim3(threads), 0, s, 1, a, b, out, n);
  return launched();
}

int launch_ada_zero(const __nv_bfloat16* x, int ldx, __nv_bfloat16* out,
                    int ldo, int rows, int dim, const float* scale,
                    const float* shift, float eps, bool norm, cudaStream_t s)
{
  if (rows <= 0) return 0;
  if (dim % 8 != 0 || dim > kRowThreads * 8 * 4) return -2;
  if (((reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(shift)) & 15u) != 0)
    return -2;
  if (dim <= kRowThreads * 8 * 2) {
    constexpr int R = 4;
    const unsigned grid = (unsigned)((rows + R - 1) / R);
    if (norm)
      launch_k(row_mod_kernel<true, R, 2>, dim3(grid), dim3(kRowThreads), 0, s, 1, x, ldx, out, ldo, rows, dim, scale, shift, eps);
    else
      launch_k(row_mod_kernel<false, R, 2>, dim3(grid), dim3(kRowThreads), 0, s, 1, x, ldx, out, ldo, rows, dim, scale, shift, eps);
  } else {
    if (norm)
      launch_k(row_mod_kernel<true, 1, 4>, dim3(rows), dim3(kRowThreads), 0, s, 1, x, ldx, out, ldo, rows, dim, scale, shift, eps);
    else
      launch_k(row_mod_kernel<false, 1, 4>, dim3(rows), dim3(kRowThreads), 0, s, 1, x, ldx, out, ldo, rows, dim, scale, shift, eps);
  }
  return launched();
}

int launch_qk_norm_rope(const __nv_bfloat16* in, int ldi, __nv_bfloat16* out,
                        int ldo, int rows, int heads, int head_dim,
                        const float* gain, const float* cosb,
                        const float* sinb, float eps, cudaStream_t s,
                        const float* sumsq, int norm_width, int head0, int tbl_tokens,
                        int tok0)
{
  if (rows <= 0) return 0;
  const int inner = heads * head_dim;
  if (inner % 8 != 0 || head_dim % 8 != 0 || ldo % 4 != 0 ||
      ((reinterpret_cast<uintptr_t>(gain) | reinterpret_cast<uintptr_t>(cosb) |
        reinterpret_cast<uintptr_t>(sinb)) & 15u) != 0)
    return -2;
  // The register form when a row's rotation quads split into whole warps
  // that tile a CTA: Q = 4 quads a thread (2 for narrow rows).
  const int half = head_dim / 2;
  const int quads = heads * half / 4;
  static const bool smem_form = [] {
    const char* e = std::getenv("LTX25_QK_SMEM");   // A/B: the shared-memory form
    return e != nullptr && e[0] == '1';
  }();
  if (!smem_form && half % 4 == 0 && ldi % 4 == 0 && ldo % 4 == 0 &&
      (reinterpret_cast<uintptr_t>(in) & 7u) == 0 && (reinterpret_cast<uintptr_t>(out) & 7u) == 0) {
    for (const int Q : {4, 2}) {
      const int tr = quads / Q;
      if (quads % Q != 0 || tr % 32 != 0 || tr > kRowThreads || kRowThreads % tr != 0) continue;
      const int rpb = kRowThreads / tr;
      const dim3 grid((unsigned)((rows + rpb - 1) / rpb));
      const int nw = norm_width > 0 ? norm_width : inner;
      const int tt = tbl_tokens > 0 ? tbl_tokens : rows;
      if (Q == 4)
        launch_k(qk_norm_rope_reg_kernel<4>, grid, dim3(kRowThreads), 0, s, 1, in, ldi, out, ldo, heads, head_dim, gain, cosb, sinb, rows, eps, sumsq, nw, head0, tt, tok0, tr);
      else
        launch_k(qk_norm_rope_reg_kernel<2>, grid, dim3(kRowThreads), 0, s, 1, in, ldi, out, ldo, heads, head_dim, gain, cosb, sinb, rows, eps, sumsq, nw, head0, tt, tok0, tr);
      return launched();
    }
  }
  const size_t smem = (size_t)inner * sizeof(float);
  if (smem > 48 * 1024) {
    static std::atomic<unsigned long long> attr{0};
    if (!smem_limit_once(qk_norm_rope_kernel, 96 * 1024, attr)) return -1;
  }
  launch_k(qk_norm_rope_kernel, dim3(rows), dim3(kRowThreads), smem, s, 1, in, ldi, out, ldo, heads, head_dim, gain, cosb, sinb, rows, eps, sumsq, norm_width > 0 ? norm_width : inner, head0, tbl_tokens > 0 ? tbl_tokens : rows, tok0);
  return launched();
}

int launch_a2a_pack(const __nv_bfloat16* src, int ld, int rows, int ranks, int cpr,
                    __nv_bfloat16* dst, cudaStream_t s)
{
  if (rows <= 0) return 0;
  if (cpr % 8 != 0 || ld % 8 != 0) return -2;
  const size_t total = (size_t)ranks * rows * (cpr / 8);
  size_t grid = (total + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  launch_k(a2a_pack_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, src, ld, rows, ranks, cpr, dst);
  return launched();
}

int launch_a2a_unpack(const __nv_bfloat16* src, int rows, int ranks, int cpr,
                      __nv_bfloat16* dst, int ldd, const __nv_bfloat16* gate, int ldg,
                      int head_dim, cudaStream_t s)
{
  if (rows <= 0) return 0;
  if (cpr % 8 != 0 || ldd % 8 != 0 || (gate != nullptr && head_dim % 8 != 0)) return -2;
  const size_t total = (size_t)ranks * rows * (cpr / 8);
  size_t grid = (total + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  launch_k(a2a_unpack_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, src, rows, ranks, cpr, dst, ldd, gate, ldg, head_dim);
  return launched();
}

int launch_row_sumsq(const __nv_bfloat16* in, int ldi, int rows, int cols,
                     float* out, cudaStream_t s)
{
  if (rows <= 0) return 0;
  if (cols % 8 != 0 || ldi % 8 != 0) return -2;
  if (cols <= 2048) {
    const int rpb = kRowThreads / 32;
    launch_k(row_sumsq_warp_kernel, dim3((unsigned)((rows + rpb - 1) / rpb)), dim3(kRowThreads), 0, s, 1, in, ldi, rows, cols, out);
    return launched();
  }
  launch_k(row_sumsq_kernel, dim3(rows), dim3(kRowThreads), 0, s, 1, in, ldi, cols, out);
  return launched();
}

int launch_gated_residual(__nv_bfloat16* x, int ldx, const __nv_bfloat16* part,
                          const __nv_bfloat16* bias, const float* gate, int rows,
                          int dim, cudaStream_t s, int nslot, size_t slot_stride)
{
  if (rows <= 0) return 0;
  if (dim % 8 != 0 || ldx % 8 != 0 || nslot < 1 || slot_stride % 8 != 0) return -2;
  const size_t total = (size_t)rows * (dim / 8);
  size_t grid = (total + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  launch_k(gated_residual_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, x, ldx, part, bias, gate, rows, dim, nslot, slot_stride);
  return launched();
}

}  // namespace ltx
