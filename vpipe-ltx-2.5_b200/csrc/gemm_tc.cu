// gemm_tc.cu -- kernel body and launcher for the tcgen05 GEMM described in
// gemm_tc.cuh.
#include <cstdio>
#include <cstdlib>
#include <type_traits>

#include "gemm_tc.cuh"
#include "block_ops.h"
#include "kernels.h"

namespace ltx {

namespace {

constexpr int kGroupM = 8;  // default raster: 8 token tiles share each weight sweep

__device__ __forceinline__ void decode_tile(const GemmParams& p, int t,
                                            int& m_tile, int& n_tile,
                                            int& kb0, int& kb1)
{
  const int split = t % p.splits;
  const int mn = t / p.splits;
  const int group_m = p.group_m > 0 ? p.group_m : kGroupM;
  const int group = group_m * p.n_tiles;
  const int g = mn / group;
  const int first_m = g * group_m;
  const int gm = min(p.m_tiles - first_m, group_m);
  const int r = mn - g * group;
  m_tile = first_m + r % gm;
  n_tile = r / gm;
  kb0 = (int)((long long)split * p.kblocks / p.splits);
  kb1 = (int)((long long)(split + 1) * p.kblocks / p.splits);
}

// Unit u of the persistent loop: its tile, and the weight blocks it takes
// (blocks [blk0, blk0 + nblk) of the tile's WB).
template <int WB>
__device__ __forceinline__ void decode_unit(const GemmParams& p, int u, int& m_tile,
                                            int& n_tile, int& kb0, int& kb1,
                                            int& blk0, int& nblk)
{
  int t = u;
  blk0 = 0;
  nblk = WB;
  if (WB > 1 && u >= p.full_units) {
    const int h = u - p.full_units;
    t = p.full_units + (h >> 1);
    blk0 = h & 1;
    nblk = 1;
  }
  decode_tile(p, t, m_tile, n_tile, kb0, kb1);
}

// The i-th k-block a tile visits.  With one token tile (M <= TN: every CTA
// of the grid reads the same activation rows), each weight tile starts its
// K range at its own offset, so the CTAs that share a K range do not all
// request the same activation lines from L2 at the same moment; otherwise
// in order.  The producer and the MMA issuer walk the same sequence.
__device__ __forceinline__ int kb_at(const GemmParams& p, int i, int n_tile, int kb0, int kb1)
{
  const int nkb = kb1 - kb0;
  if (p.krot == 0 || p.m_tiles != 1 || nkb <= 1) return kb0 + i;
  int j = i + n_tile % nkb;
  if (j >= nkb) j -= nkb;
  return kb0 + j;
}

// Row j of the output: y's row, or under a row scatter (store epilogue
// only: the host refuses it with the others) its owner's slot.
template <int EPI>
__device__ __forceinline__ __nv_bfloat16* out_row(const GemmParams& p, int j)
{
  if (EPI == EPI_STORE && p.scatter > 0) {
    const int rows = scatter_rows(p);
    const int o = j / rows;
    return p.ys[o] + ((size_t)scatter_slot(p) * rows + (j - o * rows)) * p.ldy;
  }
  return p.y + (size_t)j * p.ldy;
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

// One output pair (features n, n+1 of one token): bias, then GELU or the
// gated residual (x = x + gate * (acc + bias), `res` the two bf16 of x).
// bias / gate are this thread's pair, loaded once per tile.
template <int EPI>
__device__ __forceinline__ uint32_t epi_pair(float a, float b, bool has_bias,
                                             float2 bias, float2 g, uint32_t res)
{
  if (has_bias) {
    a += bias.x;
    b += bias.y;
  }
  if constexpr (EPI == EPI_GELU) {
    a = gelu_tanh(a);
    b = gelu_tanh(b);
  } else if constexpr (EPI == EPI_GATED_RES) {
    const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&res);
    a = fmaf(g.x, a, __bfloat162float(h.x));
    b = fmaf(g.y, b, __bfloat162float(h.y));
  }
  const __nv_bfloat162 o = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&o);
}

}  // namespace

template <int MODE, int TN, int EPI, bool PAIR, int WB>
__global__ void __launch_bounds__(GemmCfg<MODE, TN, PAIR, WB>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_sz,
                   const __grid_constant__ CUtensorMap tm_ew,
                   const __grid_constant__ CUtensorMap tm_ex, GemmParams p)
{
  using C = GemmCfg<MODE, TN, PAIR, WB>;
  constexpr int S = C::kStages;
  constexpr int A = C::kASlots > 0 ? C::kASlots : 1;
  constexpr int kDeqWarps = 8;
  constexpr int kCta = PAIR ? 2 : 1;
  // weight rows per tile; weight block g of a tile starts kBlk rows after
  // block g - 1, and CTA `rank` holds rows [rank * kBM, +kBM) of each block
  constexpr int kBlk = kCta * C::kBM;
  constexpr int kWT = WB * kBlk;
  static_assert(!PAIR || MODE == MODE_W8G64 || MODE == MODE_BF16,
                "pairs run the w8g64 and bf16 paths");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_x = base;
  uint8_t* s_w = s_x + S * C::kXStage;
  uint32_t* s_sz = reinterpret_cast<uint32_t*>(s_w + S * C::kWStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      reinterpret_cast<uint8_t*>(s_sz) + S * C::kSZStage);
  uint64_t* full = bars;            // X (+ codes, scales when !PAIR)
  uint64_t* cfull = full + S;       // PAIR: this CTA's codes + scales
  uint64_t* empty = cfull + S;
  uint64_t* afull = empty + S;
  uint64_t* aempty = afull + A;
  uint64_t* accfull = aempty + A;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const int rank = PAIR ? (int)cluster_ctarank() : 0;
  const bool leader = rank == 0;
  const int unit0 = PAIR ? (int)blockIdx.x / 2 : (int)blockIdx.x;
  const int unit_step = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
  unsigned long long* tr = (p.trace != nullptr && (int)blockIdx.x < p.trace_ctas)
                               ? p.trace + (size_t)blockIdx.x * kTraceSlots
                               : nullptr;
  if (tr != nullptr && threadIdx.x == 0) tr[TR_ENTRY] = clock64();

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&cfull[i], 1);
      mbar_init(&empty[i], MODE == MODE_W8G64 ? 5 : 1);
    }
    for (int i = 0; i < A; ++i) {
      mbar_init(&afull[i], PAIR ? 8 : 4);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], kCta * C::kEpiWarps);
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
    if constexpr (PAIR) {
      tmem_alloc_pair(s_tmem, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(s_tmem, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();   // peer barriers live before use
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // prologue done (barriers, TMEM): wait for the previous kernel, let the
  // next one start its own prologue
  pdl_wait();
  pdl_trigger();
  if (tr != nullptr && threadIdx.x == 0) tr[TR_SETUP] = clock64();

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_par = 0;   // per-stage: armed once / parity
      unsigned long long w_empty = 0;
      bool first = true;
      for (int u = unit0; u < p.num_units; u += unit_step) {
        int mt, nt, kb0, kb1, blk0, nblk;
        decode_unit<WB>(p, u, mt, nt, kb0, kb1, blk0, nblk);
        const int wrow0 = nt * kWT + blk0 * kBlk + rank * C::kBM;
        const int xrow0 = mt * TN + rank * C::kXRows;
        for (int i = 0; i < kb1 - kb0; ++i) {
          const int kb = kb_at(p, i, nt, kb0, kb1);
          const unsigned long long c0 = tr ? clock64() : 0ull;
          if (!mbar_wait(&empty[stage], phase ^ 1, s_abort, p.err,
                         KERR_WAIT_PRODUCER))
            goto producer_done;
          if (tr) w_empty += clock64() - c0;
          armed |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          // K blocks past kblocks_main contract the extension (r.B^T)
          const bool ext = MODE == MODE_BF16 && p.kblocks_main > 0 && kb >= p.kblocks_main;
          const CUtensorMap* mx = ext ? &tm_ex : &tm_x;
          const CUtensorMap* mw = ext ? &tm_ew : &tm_w;
          const int kx = (ext ? kb - p.kblocks_main : kb) * C::kKPerStage;
          if constexpr (PAIR && MODE == MODE_BF16) {
            // Both CTAs' halves of both operands complete on the leader's
            // barrier, which the leader arms for all four.
            if (leader)
              mbar_arrive_expect_tx(&full[stage], 2 * (C::kXStage + nblk * (C::kBM * 128)));
            const uint32_t lf = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_2d_pair(mx, lf, s_x + stage * C::kXStage, kx, xrow0);
            for (int g = 0; g < nblk; ++g)
              tma_load_2d_pair(mw, lf, s_w + stage * C::kWStage + g * (C::kBM * 128), kx,
                               wrow0 + g * kBlk);
          } else if constexpr (PAIR) {
            // Both halves of the activation tile complete on the leader's
            // barrier (it arms them); the codes on this CTA's own.
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::kXStage);
            mbar_arrive_expect_tx(&cfull[stage], C::kWStage + C::kSZStage);
            tma_load_2d_pair(&tm_x, mapa_shared(smem_u32(&full[stage]), 0),
                             s_x + stage * C::kXStage, kx, xrow0);
            tma_load_2d(&tm_w, &cfull[stage], s_w + stage * C::kWStage, kx, wrow0);
            tma_load_2d(&tm_sz, &cfull[stage], s_sz + stage * C::kBM, wrow0, kb);
          } else {
            mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
            tma_load_2d(mx, &full[stage], s_x + stage * C::kXStage, kx, xrow0);
            tma_load_2d(mw, &full[stage], s_w + stage * C::kWStage, kx, wrow0);
            if constexpr (MODE == MODE_W8G64) {
              tma_load_2d(&tm_sz, &full[stage], s_sz + stage * C::kBM, wrow0, kb);
            }
          }
          if (tr && first) {
            tr[TR_FIRST_TMA] = clock64();
            first = false;
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:
      if (tr) {
        tr[TR_LAST_TMA] = clock64();
        tr[TR_PROD_WAIT_EMPTY] = w_empty;
      }
      // Let every load this CTA tracks land before the CTA can exit (in a
      // pair, the activation halves are tracked by the leader's MMA).
      // (A dense pair's loads all complete on the leader's barriers: the
      // leader drains them, and the final cluster barrier holds the peer.)
      const bool drains = !(PAIR && MODE == MODE_BF16) || leader;
      for (int s = 0; s < S && drains; ++s) {
        if (armed & (1u << s)) {
          volatile int no_abort = 0;
          mbar_wait((PAIR && MODE == MODE_W8G64) ? &cfull[s] : &full[s],
                    (armed_par >> s) & 1u, &no_abort, p.err, KERR_DRAIN);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = MODE == MODE_I8
                                     ? idesc_s8(C::kBM, TN)
                                     : idesc_bf16(PAIR ? 2 * C::kBM : C::kBM, TN);
      int stage = 0, aslot = 0, acc = 0;
      uint32_t phase = 0, aphase = 0, accphase = 0;
      unsigned long long w_full = 0, w_a = 0, w_acc = 0, n_tiles = 0;
      bool first = true;
      for (int u = unit0; u < p.num_units; u += unit_step) {
        int mt, nt, kb0, kb1, blk0, nblk;
        decode_unit<WB>(p, u, mt, nt, kb0, kb1, blk0, nblk);
        ++n_tiles;
        unsigned long long c0 = tr ? clock64() : 0ull;
        if (!mbar_wait(&accempty[acc * WB], accphase ^ 1, s_abort, p.err,
                       KERR_WAIT_MMA))
          goto mma_done;
        if (tr) w_acc += clock64() - c0;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * WB * TN);
        for (int i = 0; i < kb1 - kb0; ++i) {
          if (tr) c0 = clock64();
          if (!mbar_wait(&full[stage], phase, s_abort, p.err, KERR_WAIT_MMA))
            goto mma_done;
          if (tr) {
            const unsigned long long c1 = clock64();
            w_full += c1 - c0;
            c0 = c1;
          }
          if constexpr (MODE == MODE_W8G64) {
            if (!mbar_wait(&afull[aslot], aphase, s_abort, p.err,
                           KERR_WAIT_MMA))
              goto mma_done;
          }
          if (tr) {
            w_a += clock64() - c0;
            if (first) {
              tr[TR_FIRST_MMA] = clock64();
              first = false;
            }
          }
          tc_fence_after();
          const uint64_t bdesc =
              sdesc_k128_sw128(smem_u32(s_x + stage * C::kXStage));
          if constexpr (PAIR && MODE == MODE_BF16) {
#pragma unroll
            for (int g = 0; g < WB; ++g) {
              if (g > 0 && i == 0) {
                // A later accumulator of the set is claimed only here, so
                // the first block's MMAs overlap the epilogue's drain of it.
                // (A half unit leaves it unwritten but still completes its
                // phase, so the barrier phases stay one per unit.)
                if (!mbar_wait(&accempty[acc * WB + g], accphase ^ 1, s_abort, p.err,
                               KERR_WAIT_MMA))
                  goto mma_done;
                tc_fence_after();
              }
              if (g >= nblk) continue;
              const uint64_t adesc = sdesc_k128_sw128(
                  smem_u32(s_w + stage * C::kWStage + g * (C::kBM * 128)));
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                umma_f16_ss_pair(d + (uint32_t)(g * TN), adesc + (uint64_t)(2 * kk),
                                 bdesc + (uint64_t)(2 * kk), idesc,
                                 (i > 0 || kk > 0) ? 1u : 0u);
              }
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t accum = (i > 0 || kk > 0) ? 1u : 0u;
              if constexpr (PAIR) {
                umma_f16_ts_pair(d, tmem + (uint32_t)(C::kACol0 + aslot * 32 + kk * 8),
                                 bdesc + (uint64_t)(2 * kk), idesc, accum);
              } else if constexpr (MODE == MODE_W8G64) {
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
          }
          if constexpr (PAIR) {
            umma_commit_pair(smem_u32(&empty[stage]));
            umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
            if constexpr (MODE == MODE_W8G64) {
              umma_commit_pair(smem_u32(&aempty[aslot]));
              umma_commit_pair(mapa_shared(smem_u32(&aempty[aslot]), 1));
            }
          } else {
            umma_commit(&empty[stage]);
            if constexpr (MODE == MODE_W8G64) umma_commit(&aempty[aslot]);
          }
          if constexpr (MODE == MODE_W8G64) {
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
#pragma unroll
        for (int g = 0; g < WB; ++g) {
          if constexpr (PAIR) {
            umma_commit_pair(smem_u32(&accfull[acc * WB + g]));
            umma_commit_pair(mapa_shared(smem_u32(&accfull[acc * WB + g]), 1));
          } else {
            umma_commit(&accfull[acc * WB + g]);
          }
        }
        if (++acc == C::kNAcc) {
          acc = 0;
          accphase ^= 1;
        }
      }
    mma_done:
      if (tr) {
        tr[TR_LAST_COMMIT] = clock64();
        tr[TR_MMA_WAIT_FULL] = w_full;
        tr[TR_MMA_WAIT_A] = w_a;
        tr[TR_MMA_WAIT_ACC] = w_acc;
        tr[TR_TILES] = n_tiles;
      }
      // Every MMA issued above has completed once `drain` flips.
      if constexpr (PAIR) {
        umma_commit_pair(smem_u32(drain));
      } else {
        umma_commit(drain);
      }
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.err, KERR_DRAIN);
    }
  } else if (warp < C::kEpiWarp0) {
    // ------------------------------------------------------------ dequant
    // Two groups of four warps (one warp per TMEM lane quarter each) take
    // alternate k-blocks: codes from shared memory -> bf16 -> TMEM A slot.
    if constexpr (MODE == MODE_W8G64) {
      const int q = warp & 3;                 // TMEM lane quarter
      const int grp = (warp - 2) >> 2;        // 0: even blocks, 1: odd
      const int r = q * 32 + (int)lane;       // weight row within the tile
      const int sw = (r >> 1) & 3;            // TMA SWIZZLE_64B chunk xor
      const uint32_t lane_base = (uint32_t)(q * 32) << 16;
      uint64_t* cbar = PAIR ? cfull : full;
      int seq = 0;                            // CTA-wide k-block sequence
      const bool tw = tr != nullptr && warp == 2 && lane == 0;
      unsigned long long d_full = 0, d_load = 0, d_math = 0, d_st = 0,
                         d_ae = 0, d_blocks = 0;
      for (int u = unit0; u < p.num_units; u += unit_step) {
        int mt, nt, kb0, kb1;
        decode_tile(p, u, mt, nt, kb0, kb1);   // one weight block: units are tiles
        for (int kb = kb0; kb < kb1; ++kb, ++seq) {
          if ((seq & 1) != grp) continue;
          const int stage = seq % S;
          const uint32_t phase = (uint32_t)(seq / S) & 1u;
          const int aslot = seq % C::kASlots;
          const uint32_t aphase = (uint32_t)(seq / C::kASlots) & 1u;
          unsigned long long c0 = tw ? clock64() : 0ull;
          if (!mbar_wait(&cbar[stage], phase, s_abort, p.err,
                         KERR_WAIT_DEQUANT))
            goto deq_done;
          if (tr && warp == 2 && lane == 0 && seq == 0) tr[TR_FIRST_FULL_DEQ] = clock64();
          if (tw) {
            const unsigned long long c1 = clock64();
            d_full += c1 - c0;
            c0 = c1;
          }
          const uint8_t* rowp = s_w + stage * C::kWStage + r * 64;
          uint4 c[4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
            c[j] = *reinterpret_cast<const uint4*>(rowp + 16 * (j ^ sw));
          const uint32_t sz = s_sz[stage * C::kBM + r];
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[stage]);
          if (tw) {
            const unsigned long long c1 = clock64();
            d_load += c1 - c0;
            c0 = c1;
          }
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
          if (tw) {
            const unsigned long long c1 = clock64();
            d_math += c1 - c0;
            c0 = c1;
          }
          if (!mbar_wait(&aempty[aslot], aphase ^ 1, s_abort, p.err,
                         KERR_WAIT_DEQUANT))
            goto deq_done;
          if (tw) {
            const unsigned long long c1 = clock64();
            d_ae += c1 - c0;
            c0 = c1;
          }
          tc_fence_after();
          tmem_st32(tmem + lane_base + (uint32_t)(C::kACol0 + aslot * 32), out);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) {
              mbar_arrive_cluster(mapa_shared(smem_u32(&afull[aslot]), 0));
            } else {
              mbar_arrive(&afull[aslot]);
            }
          }
          if (tw) {
            d_st += clock64() - c0;
            ++d_blocks;
          }
        }
      }
    deq_done:
      if (tw) {
        tr[TR_DEQ_WAIT_FULL] = d_full;
        tr[TR_DEQ_LOAD] = d_load;
        tr[TR_DEQ_MATH] = d_math;
        tr[TR_DEQ_WAIT_ST] = d_st;
        tr[TR_DEQ_WAIT_AEMPTY] = d_ae;
        tr[TR_DEQ_BLOCKS] = d_blocks;
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    // Groups of four warps (one per lane quarter) drain alternate 32-column
    // chunks, so the accumulator is held for a fraction of a tile.
    constexpr int kEG = C::kEpiWarps / 4;
    const int q = warp & 3;
    const int egrp = (warp - C::kEpiWarp0) >> 2;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int acc = 0;
    uint32_t accphase = 0;
    const bool te = tr != nullptr && warp == C::kEpiWarp0 && lane == 0;
    unsigned long long e_wait = 0, e_work = 0;
    for (int u = unit0; u < p.num_units; u += unit_step) {
      int mt, nt, kb0, kb1, blk0, nblk;
      decode_unit<WB>(p, u, mt, nt, kb0, kb1, blk0, nblk);
      unsigned long long ce = te ? clock64() : 0ull;
#pragma unroll 1
      for (int g = 0; g < WB; ++g) {
        const int slot = acc * WB + g;   // accumulator g of the set
        // Pair layout: lanes (2i, 2i+1) own features (n, n+1); the even lane
        // writes even tokens, the odd lane odd tokens.
        const int nrow = nt * kWT + (blk0 + g) * kBlk + rank * C::kBM + q * 32;
        const int n_pair = nrow + (int)(lane & ~1u);
        const int odd = (int)(lane & 1u);
        float csx = 1.0f;
        if constexpr (MODE == MODE_I8) {
          const int nn = nrow + (int)lane;
          csx = nn < p.N ? p.sw[nn] : 0.0f;
        }
        float2 ebias = make_float2(0.0f, 0.0f), egate = make_float2(0.0f, 0.0f);
        if (n_pair < p.N) {
          if (p.bias != nullptr) {
            const __nv_bfloat162 bb = *reinterpret_cast<const __nv_bfloat162*>(p.bias + n_pair);
            ebias = make_float2(__bfloat162float(bb.x), __bfloat162float(bb.y));
          }
          if constexpr (EPI == EPI_GATED_RES) egate = *reinterpret_cast<const float2*>(p.gate + n_pair);
        }
        // The gated residual of a token chunk's 16 sites, all loaded before
        // any store (one memory latency per chunk, not one per token).
        auto load_res = [&](int c, uint32_t (&res)[16]) {
          if constexpr (EPI == EPI_GATED_RES) {
            if (!PAIR && p.splits > 1) return;   // the cluster reduction adds it
            const int j0 = mt * TN + c * 32;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int j = j0 + 2 * k + odd;
              res[k] = (j < p.M && n_pair < p.N)
                           ? *reinterpret_cast<const uint32_t*>(out_row<EPI>(p, j) + n_pair)
                           : 0u;
            }
          }
        };
        // On two-block pairs (no second accumulator set to hide the drain
        // behind) the first chunk's residual is fetched while the
        // accumulator fills, so nothing but the TMEM loads stands between
        // the accumulator becoming full and its release (elsewhere the
        // registers it holds over the wait would spill).
        constexpr bool kPrefetch = EPI == EPI_GATED_RES && PAIR && WB == 2;
        uint32_t res0[16];
        if constexpr (kPrefetch) load_res(egrp, res0);
        if (!mbar_wait(&accfull[slot], accphase, s_abort, p.err,
                       KERR_WAIT_EPILOGUE))
          goto epi_done;
        if (te) {
          const unsigned long long c1 = clock64();
          e_wait += c1 - ce;
          ce = c1;
        }
        if (te && u == unit0 && g == 0) tr[TR_FIRST_ACC] = clock64();
        tc_fence_after();
        if (g >= nblk) {
          // a half unit's unused accumulator: hand it straight back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) {
              mbar_arrive_cluster(mapa_shared(smem_u32(&accempty[slot]), 0));
            } else {
              mbar_arrive(&accempty[slot]);
            }
          }
          continue;
        }
        // One 32-column chunk of the accumulator, from registers to y.
        // `pre`: std::true_type when rpre already holds the chunk's residual.
        auto emit = [&](const uint32_t (&v)[32], int c, const uint32_t (&rpre)[16], auto pre) {
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
          if (!PAIR && p.splits > 1) {
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
            return;
          }
          uint32_t res[16];
          if constexpr (EPI == EPI_GATED_RES) {
            if constexpr (decltype(pre)::value) {
#pragma unroll
              for (int k = 0; k < 16; ++k) res[k] = rpre[k];
            } else {
              load_res(c, res);
            }
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
              const float sj = j < p.M ? p.sx[j] : 0.0f;
              a *= sj;
              b *= sj;
            }
            if (j < p.M && n_pair < p.N) {
              const uint32_t o = epi_pair<EPI>(a, b, p.bias != nullptr, ebias, egate,
                                               EPI == EPI_GATED_RES ? res[k] : 0u);
              *reinterpret_cast<uint32_t*>(out_row<EPI>(p, j) + n_pair) = o;
            }
          }
        };
        // V^T: this lane's feature over a chunk's 32 tokens, 64 contiguous
        // bytes (the warp's 32 features all lie at or past vt_col0, a
        // multiple of 32).
        auto emit_vt = [&](const uint32_t (&v)[32], int c) {
          const int n = nrow + (int)lane;
          const int j0 = mt * TN + c * 32;
          if (n >= p.N) return;
          const float bn = p.bias != nullptr ? __bfloat162float(p.bias[n]) : 0.0f;
          __nv_bfloat16* dst = p.vt + (size_t)(n - vt_col0(p)) * vt_ld(p) + j0;
          if (j0 + 32 <= p.M) {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(
                    __uint_as_float(v[8 * q4 + 2 * e]) + bn, __uint_as_float(v[8 * q4 + 2 * e + 1]) + bn);
                w[e] = *reinterpret_cast<const uint32_t*>(&h2);
              }
              *reinterpret_cast<uint4*>(dst + 8 * q4) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (j0 + i < p.M) dst[i] = __float2bfloat16_rn(__uint_as_float(v[i]) + bn);
          }
        };
        constexpr bool kVt = EPI == EPI_STORE && MODE != MODE_I8;
        const bool vt_warp = kVt && p.vt_spec != 0 && nrow >= vt_col0(p);
        auto release = [&]() {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) {
              mbar_arrive_cluster(mapa_shared(smem_u32(&accempty[slot]), 0));
            } else {
              mbar_arrive(&accempty[slot]);
            }
          }
        };
        constexpr int kChunks = TN / 32;
        constexpr int kPer = kChunks / kEG;   // chunks this warp drains per accumulator
        static_assert(kChunks % kEG == 0, "chunks split evenly over the groups");
        // Pull every chunk out of TMEM first and hand the accumulator back
        // before the first store, so the MMA waits for the loads only --
        // where the held chunks fit the register budget without spilling
        // (not beside a gated residual's loads or the int8 rescale).
        constexpr bool kHold = kPer <= 2 && MODE == MODE_BF16 && EPI != EPI_GATED_RES;
        if (kHold && vt_warp) {
          // V^T warps stream their chunks (light stores, no exchange)
#pragma unroll 1
          for (int h = 0; h < kPer; ++h) {
            const int c = egrp + h * kEG;
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + (uint32_t)(slot * TN + c * 32), v);
            tmem_wait_ld();
            if (h == kPer - 1) release();
            emit_vt(v, c);
          }
        } else if constexpr (kHold) {
          uint32_t v[kPer][32];
#pragma unroll
          for (int h = 0; h < kPer; ++h)
            tmem_ld32(tmem + lane_base + (uint32_t)(slot * TN + (egrp + h * kEG) * 32), v[h]);
          tmem_wait_ld();
          release();
#pragma unroll
          for (int h = 0; h < kPer; ++h) emit(v[h], egrp + h * kEG, res0, std::false_type{});
        } else if constexpr (kPrefetch) {
          {
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + (uint32_t)(slot * TN + egrp * 32), v);
            tmem_wait_ld();
            if (kPer == 1) release();
            emit(v, egrp, res0, std::true_type{});
          }
#pragma unroll 1
          for (int h = 1; h < kPer; ++h) {
            const int c = egrp + h * kEG;
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + (uint32_t)(slot * TN + c * 32), v);
            tmem_wait_ld();
            if (h == kPer - 1) release();
            emit(v, c, res0, std::false_type{});
          }
        } else {
#pragma unroll 1
          for (int h = 0; h < kPer; ++h) {
            const int c = egrp + h * kEG;
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + (uint32_t)(slot * TN + c * 32), v);
            tmem_wait_ld();
            if (h == kPer - 1) release();
            if (vt_warp) {
              emit_vt(v, c);
            } else {
              emit(v, c, res0, std::false_type{});
            }
          }
        }
        if (te) {
          const unsigned long long c1 = clock64();
          e_work += c1 - ce;
          ce = c1;
        }
      }
      if (++acc == C::kNAcc) {
        acc = 0;
        accphase ^= 1;
      }
    }
  epi_done:
    // scattered rows may sit in another GPU's memory: make them visible
    // there before the kernel's completion is
    if (EPI == EPI_STORE && p.scatter > 0) __threadfence_system();
    if (te) {
      tr[TR_EPI_WAIT] = e_wait;
      tr[TR_EPI_WORK] = e_work;
      tr[TR_EPI_DONE] = clock64();
    }
  }

  tc_fence_before();
  __syncthreads();

  if (!PAIR && p.splits > 1) {
    // One cluster per output tile, one CTA per K split (cluster rank ==
    // split).  Each CTA reduces a band of token rows across the cluster's
    // partials through DSMEM, in rank order, and stores the bf16 result.
    cluster_sync_all();
    int mt, nt, kb0, kb1;
    decode_tile(p, blockIdx.x, mt, nt, kb0, kb1);
    const int crank = (int)cluster_ctarank();
    const int per = (TN + p.splits - 1) / p.splits;
    const int r0 = crank * per;
    const int r1 = min(TN, r0 + per);
    const uint32_t red = smem_u32(s_x);
    for (int idx = threadIdx.x; idx < (r1 - r0) * (C::kBM / 4); idx += blockDim.x) {
      const int jl = r0 + idx / (C::kBM / 4);
      const int c4 = (idx % (C::kBM / 4)) * 4;
      const int j = mt * TN + jl;
      const int n = nt * C::kBM + c4;
      if (j >= p.M || n >= p.N) continue;
      const uint32_t off = (uint32_t)((jl * C::kBM + c4) * 4);
      float4 v[8];
#pragma unroll
      for (int sp = 0; sp < 8; ++sp)
        if (sp < p.splits) v[sp] = ld_dsmem_f4(mapa_shared(red + off, (uint32_t)sp));
      float4 sum = v[0];
#pragma unroll
      for (int sp = 1; sp < 8; ++sp) {
        if (sp < p.splits) {
          sum.x += v[sp].x;
          sum.y += v[sp].y;
          sum.z += v[sp].z;
          sum.w += v[sp].w;
        }
      }
      __nv_bfloat16* yrow = out_row<EPI>(p, j);
      auto site = [&](float a, float b, int nn) {
        float2 bias = make_float2(0.0f, 0.0f), g = make_float2(0.0f, 0.0f);
        uint32_t res = 0u;
        if (p.bias != nullptr) {
          const __nv_bfloat162 bb = *reinterpret_cast<const __nv_bfloat162*>(p.bias + nn);
          bias = make_float2(__bfloat162float(bb.x), __bfloat162float(bb.y));
        }
        if constexpr (EPI == EPI_GATED_RES) {
          g = *reinterpret_cast<const float2*>(p.gate + nn);
          res = *reinterpret_cast<const uint32_t*>(yrow + nn);
        }
        *reinterpret_cast<uint32_t*>(yrow + nn) =
            epi_pair<EPI>(a, b, p.bias != nullptr, bias, g, res);
      };
      site(sum.x, sum.y, n);
      if (n + 2 < p.N) site(sum.z, sum.w, n + 2);   // N is even, not always % 4
    }
    // Peers may still be reading this CTA's partial: leave together.
    cluster_sync_all();
  }
  if constexpr (PAIR) {
    // The leader's MMAs read this CTA's shared memory and write its TMEM;
    // they have drained, and no remote arrive is left in flight after this.
    cluster_sync_all();
  }
  if (tr != nullptr && threadIdx.x == 0) tr[TR_REDUCED] = clock64();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem, 512);
    } else {
      tmem_dealloc(tmem, 512);
    }
    if (tr != nullptr && lane == 0) tr[TR_END] = clock64();
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

template <int MODE, int TN, int EPI, bool PAIR, int WB>
int launch_t(const GemmLaunch& L, cudaStream_t stream)
{
  using C = GemmCfg<MODE, TN, PAIR, WB>;
  CUtensorMap tx, tw, tsz;
  memset(&tsz, 0, sizeof(tsz));
  GemmParams p = L.p;
  static const int group_m = [] {
    const char* e = getenv("LTX25_GROUP_M");
    const int g = e != nullptr ? atoi(e) : 0;
    return g > 0 ? g : 0;
  }();
  if (p.group_m == 0) p.group_m = group_m;
  // Two-block pairs: 16 token tiles per weight sweep (each weight tile
  // read from DRAM half as often as with 8; measured 1-2 % faster on the
  // M = 8160 video shapes, 32 no better than 8).
  if (p.group_m == 0 && WB == 2) p.group_m = 16;
  static const int krot = [] {
    const char* e = getenv("LTX25_KROT");   // A/B: 0 = every tile walks K in order
    return (e != nullptr && e[0] == '0') ? 0 : 1;
  }();
  p.krot = krot;
  if (MODE == MODE_I8) {
    if (!encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.x, p.K, p.M, L.ldx,
                   128, C::kXRows, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
    if (!encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.w, p.K, p.N, p.K,
                   128, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
  } else {
    if (!encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, L.x, p.K, p.M,
                   (uint64_t)L.ldx * 2, 64, C::kXRows, CU_TENSOR_MAP_SWIZZLE_128B))
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
  // The extension maps: the adapter's B [N][ext_k] beside the weight and
  // r [M][ext_k] beside the activations, same boxes; copies of the main
  // maps when there is no extension (never read then).
  CUtensorMap tew = tw, tex = tx;
  if (L.ext_k > 0) {
    if (MODE != MODE_BF16 || L.ext_k % 8 != 0 || L.ld_ext < L.ext_k || L.ld_ext % 8 != 0 ||
        L.ext_w == nullptr || L.ext_x == nullptr)
      return -1;
    if (!encode_2d(&tew, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, L.ext_w, L.ext_k, p.N,
                   (uint64_t)L.ext_k * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&tex, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, L.ext_x, L.ext_k, p.M,
                   (uint64_t)L.ld_ext * 2, 64, C::kXRows, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
  }
  auto kern = gemm_tc_kernel<MODE, TN, EPI, PAIR, WB>;
  static std::atomic<unsigned long long> attr_done{0};
  if (!smem_limit_once(kern, C::kSmemBytes, attr_done)) return -2;
  // Tail split (two weight blocks per CTA): when the tiles past the last
  // full wave of pairs fit the pairs twice over, they run as half units of
  // one weight block each, so the last wave takes half a tile's time
  // instead of a whole one (e.g. 256 tiles on 74 pairs: 3.5 tile times,
  // not 4).
  static const bool tail_split = [] {
    const char* e = getenv("LTX25_TAIL_SPLIT");   // A/B: 0 = whole tiles only
    return !(e != nullptr && e[0] == '0');
  }();
  p.full_units = p.num_tiles;
  p.num_units = p.num_tiles;
  if (WB == 2 && tail_split) {
    const int pairs = L.num_sms / 2;
    const int rem = p.num_tiles % pairs;
    if (rem > 0 && 2 * rem <= pairs) {
      p.full_units = p.num_tiles - rem;
      p.num_units = p.full_units + 2 * rem;
    }
  }
  int cluster = 1;
  int grid = p.num_tiles < L.num_sms ? p.num_tiles : L.num_sms;
  if (PAIR) {
    // One cluster of two CTAs per work unit, persistent over units.
    if (p.splits != 1) return -5;
    const int pairs = p.num_units < L.num_sms / 2 ? p.num_units : L.num_sms / 2;
    grid = 2 * pairs;
    cluster = 2;
  } else if (p.splits > 1) {
    // One cluster of `splits` CTAs per output tile, one unit per CTA.
    if (p.num_tiles > L.num_sms || p.splits > 8) return -5;
    grid = p.num_tiles;
    cluster = p.splits;
  }
  launch_k(kern, dim3(grid), dim3(C::kThreads), C::kSmemBytes, stream, cluster, tx, tw, tsz,
           tew, tex, p);
  return launched() == 0 ? 0 : -3;
}

template <int MODE, int TN, bool PAIR, int WB = 1>
int launch_epi(const GemmLaunch& L, cudaStream_t stream)
{
  switch (L.epi) {
    case EPI_STORE: return launch_t<MODE, TN, EPI_STORE, PAIR, WB>(L, stream);
    case EPI_GELU: return launch_t<MODE, TN, EPI_GELU, PAIR, WB>(L, stream);
    case EPI_GATED_RES: return launch_t<MODE, TN, EPI_GATED_RES, PAIR, WB>(L, stream);
  }
  return -4;
}

template <int MODE>
int launch_tn(const GemmLaunch& L, cudaStream_t stream)
{
  if constexpr (MODE == MODE_BF16) {
    if (L.pair && L.wb == 2) return L.tn == 256 ? launch_epi<MODE, 256, true, 2>(L, stream) : -4;
  }
  if (L.wb != 1) return -4;
  if constexpr (MODE == MODE_W8G64 || MODE == MODE_BF16) {
    if (L.pair) return L.tn == 256 ? launch_epi<MODE, 256, true>(L, stream) : -4;
  } else {
    if (L.pair) return -4;
  }
  switch (L.tn) {
    case 128: return launch_epi<MODE, 128, false>(L, stream);
    case 256: return launch_epi<MODE, 256, false>(L, stream);
  }
  return -4;
}

}  // namespace

int gemm_smem_bytes(int mode, int tn)
{
  switch (mode * 1000 + tn) {
    case MODE_W8G64 * 1000 + 128: return GemmCfg<MODE_W8G64, 128>::kSmemBytes;
    case MODE_W8G64 * 1000 + 256: return GemmCfg<MODE_W8G64, 256>::kSmemBytes;
    case MODE_BF16 * 1000 + 128: return GemmCfg<MODE_BF16, 128>::kSmemBytes;
    case MODE_BF16 * 1000 + 256: return GemmCfg<MODE_BF16, 256>::kSmemBytes;
    case MODE_I8 * 1000 + 128: return GemmCfg<MODE_I8, 128>::kSmemBytes;
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
