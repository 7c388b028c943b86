// attention.cu -- non-causal softmax attention for the LTX-2.5 block.
//
// Replaces the reference's steel flash attention + ltx_gate_heads
// (src/ltx25-metal-ops.cc:1117-1289, src/ltx25-kernels.metal:85-103) and
// follows the CPU math of sdpa_ + the per-head gate (src/ltx25-block-ref.cc:
// 49-127):  o[t][h] = softmax(q k^T / sqrt(D)) v  *  2 sigmoid(g[t][h]).
//
// q, k, v are TOKEN-major [tokens][row stride] with head h at columns
// [h*D, (h+1)*D) -- the GEMM outputs read in place, no head transposes.
// Query and key lengths differ (text / audio<->video cross attention).
//
// Online-softmax flash attention on warp-level bf16 MMA (m16n8k16): a CTA of
// four warps owns 64 query rows of one head and streams 64-key K/V tiles
// through a double-buffered, XOR-swizzled shared-memory ring (cp.async).
#include "block_ops.h"

namespace ltx {

namespace {

constexpr int kBM = 64;    // query rows per CTA (16 per warp)
constexpr int kBN = 64;    // keys per tile

__device__ __forceinline__ uint32_t saddr(const void* p)
{
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async copy; zero-fills when `valid` is false.
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid)
{
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst),
               "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ void cp_commit()
{
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_wait()
{
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1,
                                        uint32_t& r2, uint32_t& r3)
{
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t& r0,
                                          uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3)
{
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(a));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0,
                                         uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1)
{
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
      "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi)
{
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `c` of row `r` in a [rows][D] bf16 tile with
// the chunk index XOR-swizzled by the row (conflict-free ldmatrix).
template <int D>
__device__ __forceinline__ int swz(int r, int c)
{
  return r * (D * 2) + ((c ^ (r & 7)) << 4);
}

template <int D>
__global__ void __launch_bounds__(128)
    flash_attn_kernel(const __nv_bfloat16* __restrict__ q, int ldq,
                      const __nv_bfloat16* __restrict__ k, int ldk,
                      const __nv_bfloat16* __restrict__ v, int ldv,
                      __nv_bfloat16* __restrict__ o, int ldo,
                      const __nv_bfloat16* __restrict__ gate, int ldg, int tq,
                      int tk, float scale_log2)
{
  pdl_wait();
  pdl_trigger();
  constexpr int kChunks = D / 8;               // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sq = smem;                          // [64][D]
  uint8_t* sk = sq + kBM * D * 2;              // 2 x [64][D]
  uint8_t* sv = sk + 2 * kBN * D * 2;          // 2 x [64][D]

  const int h = blockIdx.y;
  const int q0 = blockIdx.x * kBM;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tq4 = lane & 3;
  const __nv_bfloat16* qh = q + (size_t)h * D;
  const __nv_bfloat16* kh = k + (size_t)h * D;
  const __nv_bfloat16* vh = v + (size_t)h * D;

  auto load_tile = [&](uint8_t* dst, const __nv_bfloat16* src, int ld, int r0,
                       int rmax) {
    for (int i = tid; i < kBN * kChunks; i += 128) {
      const int r = i / kChunks, c = i % kChunks;
      const int gr = r0 + r;
      const bool ok = gr < rmax;
      cp16(saddr(dst + swz<D>(r, c)),
           src + (size_t)(ok ? gr : 0) * ld + c * 8, ok);
    }
  };

  load_tile(sq, qh, ldq, q0, tq);
  load_tile(sk, kh, ldk, 0, tk);
  load_tile(sv, vh, ldv, 0, tk);
  cp_commit();

  const int ntiles = (tk + kBN - 1) / kBN;
  float m0 = -INFINITY, m1 = -INFINITY;    // rows gid, gid + 8
  float l0 = 0.0f, l1 = 0.0f;
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
  uint32_t qf[D / 16][4];

  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1;
    if (it + 1 < ntiles) {
      load_tile(sk + (buf ^ 1) * kBN * D * 2, kh, ldk, (it + 1) * kBN, tk);
      load_tile(sv + (buf ^ 1) * kBN * D * 2, vh, ldv, (it + 1) * kBN, tk);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (it == 0) {
      // Q fragments for this warp's 16 rows, loaded once.
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(saddr(sq + swz<D>(r, c)), qf[kk][0], qf[kk][1], qf[kk][2],
                qf[kk][3]);
      }
    }
    const uint8_t* skb = sk + buf * kBN * D * 2;
    const uint8_t* svb = sv + buf * kBN * D * 2;

    // S = Q K^T for 16 rows x 64 keys: 8 n-tiles of 8 keys.
    float s[kBN / 8][4];
#pragma unroll
    for (int j = 0; j < kBN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int jp = 0; jp < kBN / 16; ++jp) {
        const int r = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(saddr(skb + swz<D>(r, c)), b0, b1, b2, b3);
        mma16816(s[2 * jp], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma16816(s[2 * jp + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // Mask keys past the end, scale into the exp2 domain, online softmax.
    const int kbase = it * kBN;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < kBN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kbase + j * 8 + tq4 * 2 + (e & 1);
        s[j][e] = key < tk ? s[j][e] * scale_log2 : -INFINITY;
      }
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float corr0 = exp2f(m0 - mx0), corr1 = exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.0f, rs1 = 0.0f;
    uint32_t pf[kBN / 16][4];
#pragma unroll
    for (int j = 0; j < kBN / 8; ++j) {
      const float p0 = exp2f(s[j][0] - m0), p1 = exp2f(s[j][1] - m0);
      const float p2 = exp2f(s[j][2] - m1), p3 = exp2f(s[j][3] - m1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      pf[j / 2][(j & 1) * 2 + 0] = pack_bf16(p0, p1);
      pf[j / 2][(j & 1) * 2 + 1] = pack_bf16(p2, p3);
    }
    l0 = l0 * corr0 + rs0;
    l1 = l1 * corr1 + rs1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      acc[i][0] *= corr0;
      acc[i][1] *= corr0;
      acc[i][2] *= corr1;
      acc[i][3] *= corr1;
    }
    // O += P V: k = 64 keys (4 steps of 16), n = D (D/8 tiles).
#pragma unroll
    for (int kk = 0; kk < kBN / 16; ++kk) {
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(saddr(svb + swz<D>(r, c)), b0, b1, b2, b3);
        mma16816(acc[2 * dp], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b0, b1);
        mma16816(acc[2 * dp + 1], pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3], b2, b3);
      }
    }
    __syncthreads();   // the next iteration's loads overwrite this buffer
  }

  // Row sums across the quad, normalize, gate, store.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const int r0 = q0 + warp * 16 + gid, r1 = r0 + 8;
  float f0 = 1.0f / l0, f1 = 1.0f / l1;
  if (gate != nullptr) {
    if (r0 < tq) f0 *= 2.0f / (1.0f + __expf(-__bfloat162float(gate[(size_t)r0 * ldg + h])));
    if (r1 < tq) f1 *= 2.0f / (1.0f + __expf(-__bfloat162float(gate[(size_t)r1 * ldg + h])));
  }
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int col = h * D + i * 8 + tq4 * 2;
    if (r0 < tq)
      *reinterpret_cast<uint32_t*>(o + (size_t)r0 * ldo + col) =
          pack_bf16(acc[i][0] * f0, acc[i][1] * f0);
    if (r1 < tq)
      *reinterpret_cast<uint32_t*>(o + (size_t)r1 * ldo + col) =
          pack_bf16(acc[i][2] * f1, acc[i][3] * f1);
  }
}

}  // namespace

int launch_attention(const __nv_bfloat16* q, int ldq, const __nv_bfloat16* k,
                     int ldk, const __nv_bfloat16* v, int ldv,
                     __nv_bfloat16* o, int ldo, const __nv_bfloat16* gate,
                     int ldg, int tq, int tk, int heads, int head_dim,
                     cudaStream_t s)
{
  if (tq <= 0 || tk <= 0 || heads <= 0) return 0;
  if ((ldq | ldk | ldv) % 8 != 0 || ldo % 2 != 0) return -2;
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  const dim3 grid((tq + kBM - 1) / kBM, heads);
  if (head_dim == 128) {
    const int smem = (kBM + 4 * kBN) * 128 * 2;
    static std::atomic<unsigned long long> attr{0};
    if (!smem_limit_once(flash_attn_kernel<128>, smem, attr)) return -1;
    launch_k(flash_attn_kernel<128>, dim3(grid), dim3(128), smem, s, 1, q, ldq, k, ldk, v, ldv, o, ldo, gate, ldg, tq, tk, scale_log2);
  } else if (head_dim == 64) {
    const int smem = (kBM + 4 * kBN) * 64 * 2;
    launch_k(flash_attn_kernel<64>, dim3(grid), dim3(128), smem, s, 1, q, ldq, k, ldk, v, ldv, o, ldo, gate, ldg, tq, tk, scale_log2);
  } else {
    return -2;
  }
  return launched();
}

}  // namespace ltx
