// gemm_tc.cu -- kernel body and launcher for the tcgen05 GEMM described in
// gemm_tc.cuh.
#include <cstdio>

#include "gemm_tc.cuh"
#include "kernels.h"

namespace ltx {

namespace {

constexpr int kGroupM = 8;  // raster: 8 token tiles share each weight sweep

__device__ __forceinline__ void decode_tile(const GemmParams& p, int t,
                                            int& m_tile, int& n_tile,
                                            int& kb0, int& kb1)
{
  const int split = t % p.splits;
  const int mn = t / p.splits;
  const int group = kGroupM * p.n_tiles;
  const int g = mn / group;
  const int first_m = g * kGroupM;
  const int gm = min(p.m_tiles - first_m, kGroupM);
  const int r = mn - g * group;
  m_tile = first_m + r % gm;
  n_tile = r / gm;
  kb0 = (int)((long long)split * p.kblocks / p.splits);
  kb1 = (int)((long long)(split + 1) * p.kblocks / p.splits);
}

// Two u8 codes -> bf16x2 of s*q + z, rounded once (fma.rn.bf16x2).  The
// codes become exact f32 integers through the 2^23 magic, whose upper half
// is then exactly the bf16 of the code (an integer below 2^8 has no bits in
// the low half of its f32).
__device__ __forceinline__ uint32_t deq_pair(uint32_t word, int sel0, int sel1,
                                             uint32_t s2, uint32_t z2)
{
  const float f0 = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650 | sel0)) - 8388608.0f;
  const float f1 = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650 | sel1)) - 8388608.0f;
  const uint32_t q2 = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
  uint32_t out;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(q2), "r"(s2), "r"(z2));
  return out;
}

__device__ __forceinline__ float gelu_tanh(float x)
{
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), the "gelu-approximate"
  // the model is trained with (src/ltx25-block-ref.cc:266-272).  The tanh is
  // the hardware approximation (max rel. error ~2^-11), below the bf16
  // rounding of the output.
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * x * (1.0f + t);
}

template <int EPI>
__device__ __forceinline__ uint32_t epi_pair(float a, float b, int n,
                                             const GemmParams& p,
                                             const __nv_bfloat16* yrow)
{
  if (p.bias != nullptr) {
    const __nv_bfloat162 bb =
        *reinterpret_cast<const __nv_bfloat162*>(p.bias + n);
    a += __bfloat162float(bb.x);
    b += __bfloat162float(bb.y);
  }
  if constexpr (EPI == EPI_GELU) {
    a = gelu_tanh(a);
    b = gelu_tanh(b);
  } else if constexpr (EPI == EPI_GATED_RES) {
    const __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(p.gate + n);
    const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(yrow + n);
    a = fmaf(__bfloat162float(g.x), a, __bfloat162float(h.x));
    b = fmaf(__bfloat162float(g.y), b, __bfloat162float(h.y));
  }
  const __nv_bfloat162 o = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&o);
}

}  // namespace

template <int MODE, int TN, int EPI>
__global__ void __launch_bounds__(320, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_sz, GemmParams p)
{
  using C = GemmCfg<MODE, TN>;
  constexpr int S = C::kStages;
  constexpr int A = C::kASlots > 0 ? C::kASlots : 1;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_x = base;
  uint8_t* s_w = s_x + S * C::kXStage;
  uint32_t* s_sz = reinterpret_cast<uint32_t*>(s_w + S * C::kWStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      reinterpret_cast<uint8_t*>(s_sz) + S * C::kSZStage);
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;
  uint64_t* aempty = afull + A;
  uint64_t* accfull = aempty + A;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], MODE == MODE_W8G64 ? 5 : 1);
    }
    for (int i = 0; i < A; ++i) {
      mbar_init(&afull[i], 4);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], 4);
    }
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    if constexpr (MODE == MODE_W8G64) tma_prefetch_desc(&tm_sz);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_par = 0;   // per-stage: armed once / parity
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        int mt, nt, kb0, kb1;
        decode_tile(p, t, mt, nt, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, s_abort, p.err,
                         KERR_WAIT_PRODUCER))
            goto producer_done;
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          armed |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          const int kx = kb * C::kKPerStage;
          tma_load_2d(&tm_x, &full[stage], s_x + stage * C::kXStage, kx,
                      mt * TN);
          tma_load_2d(&tm_w, &full[stage], s_w + stage * C::kWStage, kx,
                      nt * C::kBM);
          if constexpr (MODE == MODE_W8G64) {
            tma_load_2d(&tm_sz, &full[stage], s_sz + stage * C::kBM,
                        nt * C::kBM, kb);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:
      // Let every load this CTA issued land before the CTA can exit.
      for (int s = 0; s < S; ++s) {
        if (armed & (1u << s)) {
          volatile int no_abort = 0;
          mbar_wait(&full[s], (armed_par >> s) & 1u, &no_abort, p.err,
                    KERR_DRAIN);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc =
          MODE == MODE_I8 ? idesc_s8(C::kBM, TN) : idesc_bf16(C::kBM, TN);
      int stage = 0, aslot = 0, acc = 0;
      uint32_t phase = 0, aphase = 0, accphase = 0;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        int mt, nt, kb0, kb1;
        decode_tile(p, t, mt, nt, kb0, kb1);
        if (!mbar_wait(&accempty[acc], accphase ^ 1, s_abort, p.err,
                       KERR_WAIT_MMA))
          goto mma_done;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * TN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, s_abort, p.err, KERR_WAIT_MMA))
            goto mma_done;
          if constexpr (MODE == MODE_W8G64) {
            if (!mbar_wait(&afull[aslot], aphase, s_abort, p.err,
                           KERR_WAIT_MMA))
              goto mma_done;
          }
          tc_fence_after();
          const uint64_t bdesc =
              sdesc_k128_sw128(smem_u32(s_x + stage * C::kXStage));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t accum = (kb > kb0 || kk > 0) ? 1u : 0u;
            if constexpr (MODE == MODE_W8G64) {
              umma_f16_ts(d, tmem + (uint32_t)(C::kACol0 + aslot * 32 + kk * 8),
                          bdesc + (uint64_t)(2 * kk), idesc, accum);
            } else {
              const uint64_t adesc =
                  sdesc_k128_sw128(smem_u32(s_w + stage * C::kWStage));
              if constexpr (MODE == MODE_I8) {
                umma_i8_ss(d, adesc + (uint64_t)(2 * kk),
                           bdesc + (uint64_t)(2 * kk), idesc, accum);
              } else {
                umma_f16_ss(d, adesc + (uint64_t)(2 * kk),
                            bdesc + (uint64_t)(2 * kk), idesc, accum);
              }
            }
          }
          umma_commit(&empty[stage]);
          if constexpr (MODE == MODE_W8G64) {
            umma_commit(&aempty[aslot]);
            if (++aslot == C::kASlots) {
              aslot = 0;
              aphase ^= 1;
            }
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&accfull[acc]);
        if (++acc == C::kNAcc) {
          acc = 0;
          accphase ^= 1;
        }
      }
    mma_done:
      // Every MMA issued above has completed once `drain` flips.
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.err, KERR_DRAIN);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ dequant
    if constexpr (MODE == MODE_W8G64) {
      const int q = warp & 3;                 // TMEM lane quarter
      const int r = q * 32 + (int)lane;       // weight row within the tile
      const int sw = (r >> 1) & 3;            // TMA SWIZZLE_64B chunk xor
      const uint32_t lane_base = (uint32_t)(q * 32) << 16;
      int stage = 0, aslot = 0;
      uint32_t phase = 0, aphase = 0;
      for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
        int mt, nt, kb0, kb1;
        decode_tile(p, t, mt, nt, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, s_abort, p.err,
                         KERR_WAIT_DEQUANT))
            goto deq_done;
          const uint8_t* rowp = s_w + stage * C::kWStage + r * 64;
          uint4 c[4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
            c[j] = *reinterpret_cast<const uint4*>(rowp + 16 * (j ^ sw));
          const uint32_t sz = s_sz[stage * C::kBM + r];
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[stage]);
          const uint32_t s2 = __byte_perm(sz, 0, 0x1010);
          const uint32_t z2 = __byte_perm(sz, 0, 0x3232);
          uint32_t out[32];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t w4[4] = {c[j].x, c[j].y, c[j].z, c[j].w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              out[j * 8 + u * 2 + 0] = deq_pair(w4[u], 0, 1, s2, z2);
              out[j * 8 + u * 2 + 1] = deq_pair(w4[u], 2, 3, s2, z2);
            }
          }
          if (!mbar_wait(&aempty[aslot], aphase ^ 1, s_abort, p.err,
                         KERR_WAIT_DEQUANT))
            goto deq_done;
          tc_fence_after();
          tmem_st32(tmem + lane_base + (uint32_t)(C::kACol0 + aslot * 32), out);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[aslot]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
          if (++aslot == C::kASlots) {
            aslot = 0;
            aphase ^= 1;
          }
        }
      }
    deq_done:;
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int acc = 0;
    uint32_t accphase = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int mt, nt, kb0, kb1;
      decode_tile(p, t, mt, nt, kb0, kb1);
      if (!mbar_wait(&accfull[acc], accphase, s_abort, p.err,
                     KERR_WAIT_EPILOGUE))
        goto epi_done;
      tc_fence_after();
      // Pair layout: lanes (2i, 2i+1) own features (n, n+1); the even lane
      // writes even tokens, the odd lane odd tokens.
      const int n_pair = nt * C::kBM + q * 32 + (int)(lane & ~1u);
      const int odd = (int)(lane & 1u);
      float csx = 1.0f;
      if constexpr (MODE == MODE_I8) {
        const int nn = nt * C::kBM + q * 32 + (int)lane;
        csx = nn < p.N ? p.sw[nn] : 0.0f;
      }
#pragma unroll 1
      for (int c = 0; c < TN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + (uint32_t)(acc * TN + c * 32), v);
        tmem_wait_ld();
        if (c == TN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[acc]);
        }
        float f[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if constexpr (MODE == MODE_I8) {
            f[i] = (float)(int)v[i] * csx;
          } else {
            f[i] = __uint_as_float(v[i]);
          }
        }
        const int j0 = mt * TN + c * 32;
        if (p.splits > 1) {
          // K-split partial: park it in this CTA's shared memory as
          // red[token][feature] f32 (the pipeline buffers are idle now);
          // the cluster reduces it after the role loops.
          float* red = reinterpret_cast<float*>(s_x);
          const int nl = q * 32 + (int)lane;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float val = f[i];
            if constexpr (MODE == MODE_I8) {
              const int j = j0 + i;
              val *= j < p.M ? p.sx[j] : 0.0f;
            }
            red[(c * 32 + i) * C::kBM + nl] = val;
          }
          continue;
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          // even lane keeps token 2k, odd lane keeps token 2k+1
          const float send = odd ? f[2 * k] : f[2 * k + 1];
          const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
          float a = odd ? recv : f[2 * k];           // feature n_pair
          float b = odd ? f[2 * k + 1] : recv;       // feature n_pair + 1
          const int j = j0 + 2 * k + odd;
          if constexpr (MODE == MODE_I8) {
            const float s = j < p.M ? p.sx[j] : 0.0f;
            a *= s;
            b *= s;
          }
          if (j < p.M && n_pair < p.N) {
            __nv_bfloat16* yrow = p.y + (size_t)j * p.ldy;
            const uint32_t o = epi_pair<EPI>(a, b, n_pair, p, yrow);
            *reinterpret_cast<uint32_t*>(yrow + n_pair) = o;
          }
        }
      }
      if (++acc == C::kNAcc) {
        acc = 0;
        accphase ^= 1;
      }
    }
  epi_done:;
  }

  tc_fence_before();
  __syncthreads();

  if (p.splits > 1) {
    // One cluster per output tile, one CTA per K split (cluster rank ==
    // split).  Each CTA reduces a band of token rows across the cluster's
    // partials through DSMEM, in rank order, and stores the bf16 result.
    cluster_sync_all();
    int mt, nt, kb0, kb1;
    decode_tile(p, blockIdx.x, mt, nt, kb0, kb1);
    const int rank = (int)cluster_ctarank();
    const int per = (TN + p.splits - 1) / p.splits;
    const int r0 = rank * per;
    const int r1 = min(TN, r0 + per);
    const uint32_t red = smem_u32(s_x);
    for (int idx = threadIdx.x; idx < (r1 - r0) * (C::kBM / 4); idx += blockDim.x) {
      const int jl = r0 + idx / (C::kBM / 4);
      const int c4 = (idx % (C::kBM / 4)) * 4;
      const int j = mt * TN + jl;
      const int n = nt * C::kBM + c4;
      if (j >= p.M || n >= p.N) continue;
      const uint32_t off = (uint32_t)((jl * C::kBM + c4) * 4);
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp = 0; sp < p.splits; ++sp) {
        const float4 v = ld_dsmem_f4(mapa_shared(red + off, (uint32_t)sp));
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      __nv_bfloat16* yrow = p.y + (size_t)j * p.ldy;
      const uint32_t o0 = epi_pair<EPI>(s.x, s.y, n, p, yrow);
      const uint32_t o1 = epi_pair<EPI>(s.z, s.w, n + 2, p, yrow);
      *reinterpret_cast<uint32_t*>(yrow + n) = o0;
      *reinterpret_cast<uint32_t*>(yrow + n + 2) = o1;
    }
    // Peers may still be reading this CTA's partial: leave together.
    cluster_sync_all();
  }

  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- host

namespace {

PFN_encodeTiled g_encode = nullptr;

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* gaddr,
               uint64_t inner, uint64_t outer, uint64_t row_bytes,
               uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swz)
{
  if (g_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                cudaEnableDefault, &q) != cudaSuccess ||
        fn == nullptr) {
      return false;
    }
    g_encode = reinterpret_cast<PFN_encodeTiled>(fn);
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(map, dt, 2, const_cast<void*>(gaddr), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MODE, int TN, int EPI>
int launch_t(const GemmLaunch& L, cudaStream_t stream)
{
  using C = GemmCfg<MODE, TN>;
  CUtensorMap tx, tw, tsz;
  memset(&tsz, 0, sizeof(tsz));
  const GemmParams& p = L.p;
  if (MODE == MODE_I8) {
    if (!encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.x, p.K, p.M, L.ldx,
                   128, TN, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
    if (!encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.w, p.K, p.N, p.K,
                   128, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
  } else {
    if (!encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, L.x, p.K, p.M,
                   (uint64_t)L.ldx * 2, 64, TN, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
    if (MODE == MODE_W8G64) {
      if (!encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.w, p.K, p.N, p.K,
                     64, 128, CU_TENSOR_MAP_SWIZZLE_64B))
        return -1;
      if (!encode_2d(&tsz, CU_TENSOR_MAP_DATA_TYPE_UINT32, L.sz, p.N,
                     p.K / 64, (uint64_t)p.N * 4, 128, 1,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
        return -1;
    } else {
      if (!encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, L.w, p.K, p.N,
                     (uint64_t)p.K * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
        return -1;
    }
  }
  auto kern = gemm_tc_kernel<MODE, TN, EPI>;
  static bool attr_done = false;
  if (!attr_done) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmemBytes) != cudaSuccess)
      return -2;
    attr_done = true;
  }
  if (p.splits > 1) {
    // One cluster of `splits` CTAs per output tile, one unit per CTA.
    if (p.num_tiles > L.num_sms || p.splits > 8) return -5;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p.num_tiles, 1, 1);
    cfg.blockDim = dim3(C::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, tx, tw, tsz, p) != cudaSuccess) return -3;
    return 0;
  }
  const int grid = p.num_tiles < L.num_sms ? p.num_tiles : L.num_sms;
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(tx, tw, tsz, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <int MODE, int TN>
int launch_epi(const GemmLaunch& L, cudaStream_t stream)
{
  switch (L.epi) {
    case EPI_STORE: return launch_t<MODE, TN, EPI_STORE>(L, stream);
    case EPI_GELU: return launch_t<MODE, TN, EPI_GELU>(L, stream);
    case EPI_GATED_RES: return launch_t<MODE, TN, EPI_GATED_RES>(L, stream);
  }
  return -4;
}

template <int MODE>
int launch_tn(const GemmLaunch& L, cudaStream_t stream)
{
  switch (L.tn) {
    case 128: return launch_epi<MODE, 128>(L, stream);
    case 192: return launch_epi<MODE, 192>(L, stream);
    case 256: return launch_epi<MODE, 256>(L, stream);
  }
  return -4;
}

}  // namespace

int gemm_smem_bytes(int mode, int tn)
{
  switch (mode * 1000 + tn) {
    case MODE_W8G64 * 1000 + 128: return GemmCfg<MODE_W8G64, 128>::kSmemBytes;
    case MODE_W8G64 * 1000 + 192: return GemmCfg<MODE_W8G64, 192>::kSmemBytes;
    case MODE_W8G64 * 1000 + 256: return GemmCfg<MODE_W8G64, 256>::kSmemBytes;
    case MODE_BF16 * 1000 + 128: return GemmCfg<MODE_BF16, 128>::kSmemBytes;
    case MODE_BF16 * 1000 + 192: return GemmCfg<MODE_BF16, 192>::kSmemBytes;
    case MODE_BF16 * 1000 + 256: return GemmCfg<MODE_BF16, 256>::kSmemBytes;
    case MODE_I8 * 1000 + 128: return GemmCfg<MODE_I8, 128>::kSmemBytes;
    case MODE_I8 * 1000 + 192: return GemmCfg<MODE_I8, 192>::kSmemBytes;
    case MODE_I8 * 1000 + 256: return GemmCfg<MODE_I8, 256>::kSmemBytes;
  }
  return -1;
}

int gemm_launch(const GemmLaunch& L, cudaStream_t stream)
{
  switch (L.mode) {
    case MODE_W8G64: return launch_tn<MODE_W8G64>(L, stream);
    case MODE_BF16: return launch_tn<MODE_BF16>(L, stream);
    case MODE_I8: return launch_tn<MODE_I8>(L, stream);
  }
  return -4;
}

}  // namespace ltx
