// attention_tc.cu -- flash attention on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA) for head_dim 128: the video stream's self and text
// cross attention, >95 % of the block's attention FLOPs.
//
// Same math as attention.cu (src/ltx25-block-ref.cc:49-127):
//   o[t][h] = softmax(q k^T / sqrt(D)) v  *  2 sigmoid(g[t][h]).
//
// One CTA owns 128 query rows of one head and streams 128-key tiles:
//   warp 0      TMA: Q once, then K and V^T tiles into a 3-stage ring
//   warp 1      MMA: S_j = Q K_j^T into one of two TMEM S buffers, then
//               O += P_{j-1} V_{j-1} with P read from TMEM (the TS form)
//   warps 4-7   softmax: thread i owns query row i (TMEM lane i): reads its
//               S row, online max / exp2 / sum, writes P (bf16) over the
//               S buffer it read, and at the end normalizes and gates O.
// The S MMA of tile j+1 runs while the softmax works on tile j.  O is
// rescaled in TMEM only when a row's running max grows by more than 2^8
// (exp2 domain); until then P is computed against the older max, whose
// values stay below 2^8 -- exact in f32 accumulation and in bf16 P.
//
// V is consumed K-major: a small kernel first writes V^T ([head*D + d][key])
// so that every operand is a 128-byte-row, 128B-swizzled TMA tile, the
// layout the GEMM in gemm_tc.cu already uses.  Every wait is bounded; a
// timeout sets the context's error word and the CTA drains and exits.
#include <cuda.h>

#include <cstdlib>
#include <cstring>

#include "block_ops.h"
#include "kernels.h"
#include "ptx.cuh"

namespace ltx {

namespace {

constexpr int kFaBQ = 128;        // query rows per CTA = TMEM lanes
constexpr int kFaBK = 128;        // keys per tile
constexpr int kFaStages = 3;
constexpr int kFaThreads = 256;   // warp 0 TMA, 1 MMA, 4-7 softmax
constexpr float kRescale = 8.0f;  // log2 of the largest P before O is rescaled

enum : int {
  FERR_PRODUCER = 0x61,
  FERR_MMA = 0x62,
  FERR_SOFTMAX = 0x63,
  FERR_DRAIN = 0x64,
};

template <int D, bool I8>
struct FaCfg {
  static constexpr int kAtom = 128 * 128;             // 128 rows x 128 B
  // Q and K tiles: bf16 [128][D] in D/64 atoms, or int8 [128][128 B] (D
  // padded to 128 bytes) in one atom.
  static constexpr int kQKAtoms = I8 ? 1 : D / 64;
  static constexpr int kQBytes = kQKAtoms * kAtom;
  static constexpr int kKBytes = kQKAtoms * kAtom;
  static constexpr int kVAtom = D * 128;              // V^T: D rows x 64 keys
  static constexpr int kVBytes = 2 * kVAtom;          // 128 keys
  static constexpr int kStageBytes = kKBytes + kVBytes;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmem = 1024 + kQBytes + kFaStages * kStageBytes + kBarBytes;
  static constexpr uint32_t kOCol = 0;                // O: D f32 columns
  static constexpr uint32_t kSCol = D;                // S0, S1: 128 columns each
  static_assert(D + 2 * kFaBK <= 512, "TMEM columns");
};

struct FaParams {
  __nv_bfloat16* o;
  const __nv_bfloat16* gate;
  int ldo, ldg;
  int tq, tk, ntiles;
  float scale_log2;
  int* err;
  // int8 QK (sage): per-block scales sq[head][query block], sk[head][key
  // block]; the int8 tiles are head-major with tq_pad / tk_pad rows a head.
  const float* sq;
  const float* sk;
  int nqb, tq_pad, tk_pad;
  // split-KV (grid z > 1): each CTA covers key tiles [z n / splits,
  // (z+1) n / splits) and leaves its unnormalized O and (max, sum) in
  // part_o [split][tq][heads][D] / part_ml [split][tq][heads][2] (f32).
  int splits;
  float* part_o;
  float* part_ml;
  int heads;
};

__device__ __forceinline__ float fast_exp2(float x)
{
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100 three-input max).
__device__ __forceinline__ float max3f(float a, float b, float c)
{
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Packed f32 pairs (sm_100 f32x2): d = a * b + c and d = a + b, lane-wise.
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b,
                                                    unsigned long long c)
{
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ unsigned long long fadd2(unsigned long long a, unsigned long long b)
{
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ unsigned long long pair2(uint32_t lo, uint32_t hi)
{
  return ((unsigned long long)hi << 32) | lo;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi)
{
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int D, bool I8>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                 const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_vt, FaParams p)
{
  using C = FaCfg<D, I8>;
  constexpr int S = kFaStages;
  constexpr int kQAtoms = C::kQKAtoms;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = base;
  uint8_t* s_kv = s_q + C::kQBytes;   // stage i: K at +i*stage, V^T after K
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_kv + S * C::kStageBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + S;
  uint64_t* empty = v_full + S;
  uint64_t* s_full = empty + S;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * kFaBQ;
  const int h = blockIdx.y;
  // key tiles [jb, jb + n) of p.ntiles (all of them unless split)
  const int jb = (int)((long long)blockIdx.z * p.ntiles / p.splits);
  const int n = (int)((long long)(blockIdx.z + 1) * p.ntiles / p.splits) - jb;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < S; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_vt);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // prologue done (barriers, TMEM): wait for the previous kernel, let the
  // next one start its own prologue
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------- TMA
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      mbar_arrive_expect_tx(q_full, C::kQBytes);
      for (int a = 0; a < kQAtoms; ++a) {
        if constexpr (I8)
          tma_load_2d(&tm_q, q_full, s_q, 0, h * p.tq_pad + q0);
        else
          tma_load_2d(&tm_q, q_full, s_q + a * C::kAtom, h * D + a * 64, q0);
      }
      for (int j = 0; j < n; ++j) {
        const int st = j % S;
        const uint32_t ph = (uint32_t)(j / S) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, s_abort, p.err, FERR_PRODUCER)) break;
        uint8_t* sk = s_kv + st * C::kStageBytes;
        uint8_t* sv = sk + C::kKBytes;
        mbar_arrive_expect_tx(&k_full[st], C::kKBytes);
        const int jg = jb + j;   // global key tile
        for (int a = 0; a < kQAtoms; ++a) {
          if constexpr (I8)
            tma_load_2d(&tm_k, &k_full[st], sk, 0, h * p.tk_pad + jg * kFaBK);
          else
            tma_load_2d(&tm_k, &k_full[st], sk + a * C::kAtom, h * D + a * 64, jg * kFaBK);
        }
        mbar_arrive_expect_tx(&v_full[st], C::kVBytes);
        for (int a = 0; a < 2; ++a)
          tma_load_2d(&tm_vt, &v_full[st], sv + a * C::kVAtom, jg * kFaBK + a * 64, h * D);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      // Every load lands before the CTA may exit.
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, p.err, FERR_DRAIN);
      for (int st = 0; st < S; ++st) {
        if (armed & (1u << st)) {
          mbar_wait(&k_full[st], (armed_par >> st) & 1u, &no_abort, p.err, FERR_DRAIN);
          mbar_wait(&v_full[st], (armed_par >> st) & 1u, &no_abort, p.err, FERR_DRAIN);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc_s = I8 ? idesc_s8(kFaBQ, kFaBK) : idesc_bf16(kFaBQ, kFaBK);
      constexpr uint32_t idesc_o = idesc_bf16(kFaBQ, D);
      bool ok = mbar_wait(q_full, 0, s_abort, p.err, FERR_MMA);
      for (int j = 0; ok && j <= n; ++j) {
        if (j < n) {
          const int st = j % S;
          if (!mbar_wait(&k_full[st], (uint32_t)(j / S) & 1u, s_abort, p.err, FERR_MMA)) break;
          tc_fence_after();
          const uint32_t sk = smem_u32(s_kv + st * C::kStageBytes);
          const uint32_t d = tmem + C::kSCol + (uint32_t)(j & 1) * kFaBK;
          if constexpr (I8) {
            // int8 rows of 128 B: K = 32 per instruction, D/32 of them.
#pragma unroll
            for (int kk = 0; kk < D / 32; ++kk)
              umma_i8_ss(d, sdesc_k128_sw128(smem_u32(s_q)) + (uint64_t)(2 * kk),
                         sdesc_k128_sw128(sk) + (uint64_t)(2 * kk), idesc_s,
                         kk > 0 ? 1u : 0u);
          } else {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (uint32_t)((kk >> 2) * C::kAtom);
              umma_f16_ss(d, sdesc_k128_sw128(smem_u32(s_q) + off) + (uint64_t)(2 * (kk & 3)),
                          sdesc_k128_sw128(sk + off) + (uint64_t)(2 * (kk & 3)), idesc_s,
                          kk > 0 ? 1u : 0u);
            }
          }
          umma_commit(&s_full[j & 1]);
        }
        if (j >= 1) {
          const int i = j - 1;
          const int st = i % S;
          if (!mbar_wait(&p_full[i & 1], (uint32_t)(i >> 1) & 1u, s_abort, p.err, FERR_MMA) ||
              !mbar_wait(&v_full[st], (uint32_t)(i / S) & 1u, s_abort, p.err, FERR_MMA))
            break;
          tc_fence_after();
          const uint32_t sv = smem_u32(s_kv + st * C::kStageBytes + C::kKBytes);
          const uint32_t pa = tmem + C::kSCol + (uint32_t)(i & 1) * kFaBK;
#pragma unroll
          for (int kk = 0; kk < kFaBK / 16; ++kk) {
            umma_f16_ts(tmem + C::kOCol, pa + (uint32_t)(kk * 8),
                        sdesc_k128_sw128(sv + (uint32_t)((kk >> 2) * C::kVAtom)) +
                            (uint64_t)(2 * (kk & 3)),
                        idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[st]);
          umma_commit(o_done);
        }
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.err, FERR_DRAIN);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------- softmax
    const int q = warp & 3;
    const int r = q * 32 + (int)lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const float c0 = p.scale_log2 * (I8 ? p.sq[h * p.nqb + blockIdx.x] : 1.0f);
    float m_run = 0.0f, l_run = 0.0f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int sb = i & 1;
      if (!mbar_wait(&s_full[sb], (uint32_t)(i >> 1) & 1u, s_abort, p.err, FERR_SOFTMAX)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t scol = tmem + lane_base + C::kSCol + (uint32_t)sb * kFaBK;
      float s[kFaBK];
#pragma unroll
      for (int c4 = 0; c4 < kFaBK / 32; ++c4) {
        uint32_t v[32];
        tmem_ld32(scol + (uint32_t)(c4 * 32), v);
#pragma unroll
        for (int e = 0; e < 32; ++e)
          s[c4 * 32 + e] = I8 ? (float)(int)v[e] : __uint_as_float(v[e]);
      }
      tmem_wait_ld();
      // exp2-domain factor of this tile's raw scores (the int8 path folds
      // in the key block's scale; the scales are positive)
      const float c = I8 ? c0 * p.sk[h * p.ntiles + jb + i] : c0;
      const int valid = p.tk - (jb + i) * kFaBK;
      float mx = -3.0e38f;
#pragma unroll
      for (int e = 0; e < kFaBK; ++e) {
        if (e >= valid) s[e] = -3.0e38f;
        mx = fmaxf(mx, s[e]);
      }
      const float m_tile = mx * c;
      if (i == 0) m_run = m_tile;
      // tcgen05.ld/st are warp-collective: the warp rescales together when
      // any of its rows needs it (rows that do not use a factor of 1).
      const bool need = i > 0 && m_tile > m_run + kRescale;
      if (__any_sync(0xffffffffu, need)) {
        // O holds P V up to tile i-1 against m_run: wait for it, rescale.
        const float m_new = need ? m_tile : m_run;
        const float f = fast_exp2(m_run - m_new);
        l_run *= f;
        if (!mbar_wait(o_done, (uint32_t)(i - 1) & 1u, s_abort, p.err, FERR_SOFTMAX)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c4 = 0; c4 < D / 32; ++c4) {
          uint32_t v[32];
          const uint32_t oc = tmem + lane_base + C::kOCol + (uint32_t)(c4 * 32);
          tmem_ld32(oc, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * f);
          tmem_st32(oc, v);
        }
        m_run = m_new;
      }
      float sum = 0.0f;
#pragma unroll
      for (int c4 = 0; c4 < kFaBK / 64; ++c4) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float p0 = fast_exp2(fmaf(s[c4 * 64 + 2 * e], c, -m_run));
          const float p1 = fast_exp2(fmaf(s[c4 * 64 + 2 * e + 1], c, -m_run));
          sum += p0 + p1;
          pk[e] = pack_bf16(p0, p1);
        }
        tmem_st32(scol + (uint32_t)(c4 * 32), pk);
      }
      l_run += sum;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    if (ok && n > 0 && p.splits > 1 &&
        mbar_wait(o_done, (uint32_t)(n - 1) & 1u, s_abort, p.err, FERR_SOFTMAX)) {
      // split-KV partial: unnormalized O and this split's (max, sum)
      tc_fence_after();
      const int row = q0 + r;
      const size_t site = ((size_t)blockIdx.z * p.tq + row) * p.heads + h;
      float* po = p.part_o + site * D;
#pragma unroll
      for (int c4 = 0; c4 < D / 32; ++c4) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + C::kOCol + (uint32_t)(c4 * 32), v);
        tmem_wait_ld();
        if (row < p.tq) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            *reinterpret_cast<uint4*>(po + c4 * 32 + 4 * e) =
                make_uint4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
        }
      }
      if (row < p.tq) *reinterpret_cast<float2*>(p.part_ml + site * 2) = make_float2(m_run, l_run);
    } else if (ok && n > 0 &&
        mbar_wait(o_done, (uint32_t)(n - 1) & 1u, s_abort, p.err, FERR_SOFTMAX)) {
      tc_fence_after();
      const int row = q0 + r;
      float g = 1.0f / l_run;
      if (p.gate != nullptr && row < p.tq)
        g *= 2.0f / (1.0f + __expf(-__bfloat162float(p.gate[(size_t)row * p.ldg + h])));
      __nv_bfloat16* orow = p.o + (size_t)row * p.ldo + h * D;
#pragma unroll
      for (int c4 = 0; c4 < D / 32; ++c4) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + C::kOCol + (uint32_t)(c4 * 32), v);
        tmem_wait_ld();
        if (row < p.tq) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(v[8 * e + 0]) * g, __uint_as_float(v[8 * e + 1]) * g);
            w.y = pack_bf16(__uint_as_float(v[8 * e + 2]) * g, __uint_as_float(v[8 * e + 3]) * g);
            w.z = pack_bf16(__uint_as_float(v[8 * e + 4]) * g, __uint_as_float(v[8 * e + 5]) * g);
            w.w = pack_bf16(__uint_as_float(v[8 * e + 6]) * g, __uint_as_float(v[8 * e + 7]) * g);
            *reinterpret_cast<uint4*>(orow + c4 * 32 + 8 * e) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ---- two query tiles per CTA (head_dim 128, bf16) ---------------------
//
// The same tile math as fa_tc_kernel, with 256 query rows per CTA in two
// 128-row tiles, each with its own softmax warpgroup and its own O and S in
// TMEM (O0 | O1 | S0 | S1 = 512 columns).  The MMA warp interleaves them:
//   S0_0 S1_0 | PV0_0 S0_1 PV1_0 S1_1 | PV0_1 S0_2 PV1_1 S1_2 | ...
// so while one warpgroup runs its softmax the tensor core computes the
// other tile's P V and next S -- in steady state four MMAs per key tile
// against two softmaxes, neither waiting on the other.  K (3 stages) and V^T
// (2 stages) have separate rings and producers.  The softmax reads each S
// row twice from TMEM (max, then exp) to stay within 168 registers.
constexpr int kFa2Threads = 384;   // w0 Q/K TMA, w1 MMA, w2 V TMA, w4-7 / w8-11 softmax
constexpr int kFa2KStages = 3;
constexpr int kFa2VStages = 2;

struct Fa2Cfg {
  static constexpr int D = 128;
  static constexpr int kAtom = 128 * 128;
  static constexpr int kQTile = 2 * kAtom;            // 128 rows x 128 dims
  static constexpr int kKStage = 2 * kAtom;
  static constexpr int kVStage = 2 * kAtom;           // 128 dims x 128 keys
  static constexpr int kSmem =
      1024 + 2 * kQTile + kFa2KStages * kKStage + kFa2VStages * kVStage + 256;
  static constexpr uint32_t kOCol = 0;                 // O_t at t * 128
  static constexpr uint32_t kSCol = 256;               // S_t at 256 + t * 128
};

__global__ void __launch_bounds__(kFa2Threads, 1)
    fa2_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                  const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_vt, FaParams p)
{
  using C = Fa2Cfg;
  constexpr int D = C::D;
  constexpr int SK = kFa2KStages, SV = kFa2VStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = base;                                 // tile t at t * kQTile
  uint8_t* s_k = s_q + 2 * C::kQTile;
  uint8_t* s_v = s_k + SK * C::kKStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_v + SV * C::kVStage);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + SK;
  uint64_t* v_full = k_empty + SK;
  uint64_t* v_empty = v_full + SV;
  uint64_t* s_full = v_empty + SV;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * 2 * kFaBQ;
  const int h = blockIdx.y;
  const int n = p.ntiles;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < SK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < SV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_vt);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // prologue done (barriers, TMEM): wait for the previous kernel, let the
  // next one start its own prologue
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ----------------------------------------------------------- Q, K TMA
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      mbar_arrive_expect_tx(q_full, 2 * C::kQTile);
      for (int t = 0; t < 2; ++t)
        for (int a = 0; a < 2; ++a)
          tma_load_2d(&tm_q, q_full, s_q + t * C::kQTile + a * C::kAtom, h * D + a * 64,
                      q0 + t * kFaBQ);
      for (int j = 0; j < n; ++j) {
        const int st = j % SK;
        const uint32_t ph = (uint32_t)(j / SK) & 1u;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, s_abort, p.err, FERR_PRODUCER)) break;
        mbar_arrive_expect_tx(&k_full[st], C::kKStage);
        for (int a = 0; a < 2; ++a)
          tma_load_2d(&tm_k, &k_full[st], s_k + st * C::kKStage + a * C::kAtom,
                      h * D + a * 64, j * kFaBK);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, p.err, FERR_DRAIN);
      for (int st = 0; st < SK; ++st)
        if (armed & (1u << st))
          mbar_wait(&k_full[st], (armed_par >> st) & 1u, &no_abort, p.err, FERR_DRAIN);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------- V TMA
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j % SV;
        const uint32_t ph = (uint32_t)(j / SV) & 1u;
        if (!mbar_wait(&v_empty[st], ph ^ 1u, s_abort, p.err, FERR_PRODUCER)) break;
        mbar_arrive_expect_tx(&v_full[st], C::kVStage);
        for (int a = 0; a < 2; ++a)
          tma_load_2d(&tm_vt, &v_full[st], s_v + st * C::kVStage + a * (D * 128),
                      j * kFaBK + a * 64, h * D);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      volatile int no_abort = 0;
      for (int st = 0; st < SV; ++st)
        if (armed & (1u << st))
          mbar_wait(&v_full[st], (armed_par >> st) & 1u, &no_abort, p.err, FERR_DRAIN);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(kFaBQ, kFaBK);
      constexpr uint32_t idesc_o = idesc_bf16(kFaBQ, D);
      auto issue_s = [&](int t, int j) {
        const uint32_t sk = smem_u32(s_k + (j % SK) * C::kKStage);
        const uint32_t sq = smem_u32(s_q + t * C::kQTile);
        const uint32_t d = tmem + C::kSCol + (uint32_t)t * kFaBK;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * C::kAtom);
          umma_f16_ss(d, sdesc_k128_sw128(sq + off) + (uint64_t)(2 * (kk & 3)),
                      sdesc_k128_sw128(sk + off) + (uint64_t)(2 * (kk & 3)), idesc_s,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t sv = smem_u32(s_v + (j % SV) * C::kVStage);
        const uint32_t pa = tmem + C::kSCol + (uint32_t)t * kFaBK;
#pragma unroll
        for (int kk = 0; kk < kFaBK / 16; ++kk)
          umma_f16_ts(tmem + C::kOCol + (uint32_t)t * D, pa + (uint32_t)(kk * 8),
                      sdesc_k128_sw128(sv + (uint32_t)((kk >> 2) * (D * 128))) +
                          (uint64_t)(2 * (kk & 3)),
                      idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_done[t]);
      };
      bool ok = mbar_wait(q_full, 0, s_abort, p.err, FERR_MMA) &&
                mbar_wait(&k_full[0], 0, s_abort, p.err, FERR_MMA);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < n; ++j) {
        const bool more = j + 1 < n;
        // tile 0: P V, then its next S (in-order: the S MMA overwrites
        // S0 only after this P V has read P0 from it)
        if (!mbar_wait(&p_full[0], (uint32_t)j & 1u, s_abort, p.err, FERR_MMA) ||
            !mbar_wait(&v_full[j % SV], (uint32_t)(j / SV) & 1u, s_abort, p.err, FERR_MMA))
          break;
        tc_fence_after();
        issue_pv(0, j);
        if (more) {
          if (!mbar_wait(&k_full[(j + 1) % SK], (uint32_t)((j + 1) / SK) & 1u, s_abort, p.err,
                         FERR_MMA))
            break;
          tc_fence_after();
          issue_s(0, j + 1);
        }
        if (!mbar_wait(&p_full[1], (uint32_t)j & 1u, s_abort, p.err, FERR_MMA)) break;
        tc_fence_after();
        issue_pv(1, j);
        umma_commit(&v_empty[j % SV]);
        if (more) {
          issue_s(1, j + 1);
          umma_commit(&k_empty[(j + 1) % SK]);
        }
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.err, FERR_DRAIN);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int t = (warp - 4) >> 2;                      // query tile
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t scol = tmem + lane_base + C::kSCol + (uint32_t)t * kFaBK;
    const uint32_t ocol = tmem + lane_base + C::kOCol + (uint32_t)t * D;
    const float c = p.scale_log2;
    float m_run = 0.0f, l_run = 0.0f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      if (!mbar_wait(&s_full[t], (uint32_t)i & 1u, s_abort, p.err, FERR_SOFTMAX)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int valid = p.tk - i * kFaBK;
      const bool full = valid >= kFaBK;        // warp-uniform: no masking
      float mx;
      {
        // row max: two 64-column reads, four independent max chains
        float m4[4] = {-3.0e38f, -3.0e38f, -3.0e38f, -3.0e38f};
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint32_t a[32], b[32];
          tmem_ld32(scol + (uint32_t)(h2 * 64), a);
          tmem_ld32(scol + (uint32_t)(h2 * 64 + 32), b);
          tmem_wait_ld();
          if (full) {
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              m4[0] = max3f(m4[0], __uint_as_float(a[e]), __uint_as_float(a[e + 1]));
              m4[1] = max3f(m4[1], __uint_as_float(a[e + 2]), __uint_as_float(a[e + 3]));
              m4[2] = max3f(m4[2], __uint_as_float(b[e]), __uint_as_float(b[e + 1]));
              m4[3] = max3f(m4[3], __uint_as_float(b[e + 2]), __uint_as_float(b[e + 3]));
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (h2 * 64 + e < valid) m4[0] = fmaxf(m4[0], __uint_as_float(a[e]));
              if (h2 * 64 + 32 + e < valid) m4[1] = fmaxf(m4[1], __uint_as_float(b[e]));
            }
          }
        }
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      }
      const float m_tile = mx * c;
      if (i == 0) m_run = m_tile;
      const bool need = i > 0 && m_tile > m_run + kRescale;
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? m_tile : m_run;
        const float f = fast_exp2(m_run - m_new);
        l_run *= f;
        if (!mbar_wait(&o_done[t], (uint32_t)(i - 1) & 1u, s_abort, p.err, FERR_SOFTMAX)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c4 = 0; c4 < D / 32; ++c4) {
          uint32_t v[32];
          tmem_ld32(ocol + (uint32_t)(c4 * 32), v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * f);
          tmem_st32(ocol + (uint32_t)(c4 * 32), v);
        }
        m_run = m_new;
      }
      float sum = 0.0f;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        // keys [64 h2, 64 h2 + 64) -> P columns [32 h2, 32 h2 + 32); the S
        // columns this overwrites were read above or in the previous half
        uint32_t a[32], b[32], pk[32];
        tmem_ld32(scol + (uint32_t)(h2 * 64), a);
        tmem_ld32(scol + (uint32_t)(h2 * 64 + 32), b);
        tmem_wait_ld();
        if (!full) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            if (h2 * 64 + e >= valid) a[e] = __float_as_uint(-3.0e38f);
            if (h2 * 64 + 32 + e >= valid) b[e] = __float_as_uint(-3.0e38f);
          }
        }
        // exponent arguments two at a time (f32x2 FMA), sums likewise
        const unsigned long long c2 = pair2(__float_as_uint(c), __float_as_uint(c));
        const unsigned long long nm2 = pair2(__float_as_uint(-m_run), __float_as_uint(-m_run));
        unsigned long long sa = 0ull, sb = 0ull;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const unsigned long long xa = ffma2(pair2(a[2 * e], a[2 * e + 1]), c2, nm2);
          const unsigned long long xb = ffma2(pair2(b[2 * e], b[2 * e + 1]), c2, nm2);
          const float p0 = fast_exp2(__uint_as_float((uint32_t)xa));
          const float p1 = fast_exp2(__uint_as_float((uint32_t)(xa >> 32)));
          const float p2 = fast_exp2(__uint_as_float((uint32_t)xb));
          const float p3 = fast_exp2(__uint_as_float((uint32_t)(xb >> 32)));
          sa = fadd2(sa, pair2(__float_as_uint(p0), __float_as_uint(p1)));
          sb = fadd2(sb, pair2(__float_as_uint(p2), __float_as_uint(p3)));
          pk[e] = pack_bf16(p0, p1);
          pk[16 + e] = pack_bf16(p2, p3);
        }
        const unsigned long long st2 = fadd2(sa, sb);
        sum += __uint_as_float((uint32_t)st2) + __uint_as_float((uint32_t)(st2 >> 32));
        tmem_st32(scol + (uint32_t)(h2 * 32), pk);
      }
      l_run += sum;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok && n > 0 &&
        mbar_wait(&o_done[t], (uint32_t)(n - 1) & 1u, s_abort, p.err, FERR_SOFTMAX)) {
      tc_fence_after();
      const int row = q0 + t * kFaBQ + q * 32 + (int)lane;
      float g = 1.0f / l_run;
      if (p.gate != nullptr && row < p.tq)
        g *= 2.0f / (1.0f + __expf(-__bfloat162float(p.gate[(size_t)row * p.ldg + h])));
      __nv_bfloat16* orow = p.o + (size_t)row * p.ldo + h * D;
#pragma unroll
      for (int c4 = 0; c4 < D / 32; ++c4) {
        uint32_t v[32];
        tmem_ld32(ocol + (uint32_t)(c4 * 32), v);
        tmem_wait_ld();
        if (row < p.tq) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(v[8 * e + 0]) * g, __uint_as_float(v[8 * e + 1]) * g);
            w.y = pack_bf16(__uint_as_float(v[8 * e + 2]) * g, __uint_as_float(v[8 * e + 3]) * g);
            w.z = pack_bf16(__uint_as_float(v[8 * e + 4]) * g, __uint_as_float(v[8 * e + 5]) * g);
            w.w = pack_bf16(__uint_as_float(v[8 * e + 6]) * g, __uint_as_float(v[8 * e + 7]) * g);
            *reinterpret_cast<uint4*>(orow + c4 * 32 + 8 * e) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// The 64 exponentials of one half row: p = 2^(s c - m), packed to bf16 pairs
// (low half = even column) and summed in two f32x2 chains.
__device__ __forceinline__ void fa3_exp(const uint32_t (&a)[32], const uint32_t (&b)[32],
                                        unsigned long long c2, unsigned long long nm2,
                                        uint32_t (&pk)[32], unsigned long long& sa,
                                        unsigned long long& sb)
{
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const unsigned long long xa = ffma2(pair2(a[2 * e], a[2 * e + 1]), c2, nm2);
    const unsigned long long xb = ffma2(pair2(b[2 * e], b[2 * e + 1]), c2, nm2);
    const float p0 = fast_exp2(__uint_as_float((uint32_t)xa));
    const float p1 = fast_exp2(__uint_as_float((uint32_t)(xa >> 32)));
    const float p2 = fast_exp2(__uint_as_float((uint32_t)xb));
    const float p3 = fast_exp2(__uint_as_float((uint32_t)(xb >> 32)));
    sa = fadd2(sa, pair2(__float_as_uint(p0), __float_as_uint(p1)));
    sb = fadd2(sb, pair2(__float_as_uint(p2), __float_as_uint(p3)));
    pk[e] = pack_bf16(p0, p1);
    pk[16 + e] = pack_bf16(p2, p3);
  }
}

// ---- two query tiles, each row's scores split over two warps -----------
//
// fa2_tc_kernel's schedule with 16 softmax warps instead of 8: the two
// warps that share a TMEM lane quarter split a row's 128 scores (64 each,
// one TMEM read per tile), combine the row max through shared memory behind
// a per-tile named barrier, and each rescale / normalize half of O.  Four
// softmax warps per SM sub-partition hide the TMEM-read latency that bounds
// the eight-warp version.
constexpr int kFa3Threads = 640;   // w0 Q/K TMA, w1 MMA, w2 V TMA, w4-11 / w12-19 softmax
constexpr int kFa3KStages = 2;     // one K stage fewer: room for the row-max exchange

struct Fa3Cfg : Fa2Cfg {
  static constexpr int kSmem =
      1024 + 2 * kQTile + kFa3KStages * kKStage + kFa2VStages * kVStage + 256;
};

__global__ void __launch_bounds__(kFa3Threads, 1)
    fa3_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                  const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_vt, FaParams p)
{
  using C = Fa3Cfg;
  constexpr int D = C::D;
  constexpr int SK = kFa3KStages, SV = kFa2VStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_q = base;                                 // tile t at t * kQTile
  uint8_t* s_k = s_q + 2 * C::kQTile;
  uint8_t* s_v = s_k + SK * C::kKStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_v + SV * C::kVStage);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + SK;
  uint64_t* v_full = k_empty + SK;
  uint64_t* v_empty = v_full + SV;
  uint64_t* s_full = v_empty + SV;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  // row-max exchange between the two half-row warps: [tile][parity][half][row]
  __shared__ float s_mx[2][2][2][kFaBQ];

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * 2 * kFaBQ;
  const int h = blockIdx.y;
  const int n = p.ntiles;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < SK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < SV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_vt);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  // prologue done (barriers, TMEM): wait for the previous kernel, let the
  // next one start its own prologue
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ----------------------------------------------------------- Q, K TMA
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      mbar_arrive_expect_tx(q_full, 2 * C::kQTile);
      for (int t = 0; t < 2; ++t)
        for (int a = 0; a < 2; ++a)
          tma_load_2d(&tm_q, q_full, s_q + t * C::kQTile + a * C::kAtom, h * D + a * 64,
                      q0 + t * kFaBQ);
      for (int j = 0; j < n; ++j) {
        const int st = j % SK;
        const uint32_t ph = (uint32_t)(j / SK) & 1u;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, s_abort, p.err, FERR_PRODUCER)) break;
        mbar_arrive_expect_tx(&k_full[st], C::kKStage);
        for (int a = 0; a < 2; ++a)
          tma_load_2d(&tm_k, &k_full[st], s_k + st * C::kKStage + a * C::kAtom,
                      h * D + a * 64, j * kFaBK);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, p.err, FERR_DRAIN);
      for (int st = 0; st < SK; ++st)
        if (armed & (1u << st))
          mbar_wait(&k_full[st], (armed_par >> st) & 1u, &no_abort, p.err, FERR_DRAIN);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------- V TMA
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j % SV;
        const uint32_t ph = (uint32_t)(j / SV) & 1u;
        if (!mbar_wait(&v_empty[st], ph ^ 1u, s_abort, p.err, FERR_PRODUCER)) break;
        mbar_arrive_expect_tx(&v_full[st], C::kVStage);
        for (int a = 0; a < 2; ++a)
          tma_load_2d(&tm_vt, &v_full[st], s_v + st * C::kVStage + a * (D * 128),
                      j * kFaBK + a * 64, h * D);
        armed |= 1u << st;
        armed_par = (armed_par & ~(1u << st)) | (ph << st);
      }
      volatile int no_abort = 0;
      for (int st = 0; st < SV; ++st)
        if (armed & (1u << st))
          mbar_wait(&v_full[st], (armed_par >> st) & 1u, &no_abort, p.err, FERR_DRAIN);
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(kFaBQ, kFaBK);
      constexpr uint32_t idesc_o = idesc_bf16(kFaBQ, D);
      auto issue_s = [&](int t, int j) {
        const uint32_t sk = smem_u32(s_k + (j % SK) * C::kKStage);
        const uint32_t sq = smem_u32(s_q + t * C::kQTile);
        const uint32_t d = tmem + C::kSCol + (uint32_t)t * kFaBK;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * C::kAtom);
          umma_f16_ss(d, sdesc_k128_sw128(sq + off) + (uint64_t)(2 * (kk & 3)),
                      sdesc_k128_sw128(sk + off) + (uint64_t)(2 * (kk & 3)), idesc_s,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t sv = smem_u32(s_v + (j % SV) * C::kVStage);
        const uint32_t pa = tmem + C::kSCol + (uint32_t)t * kFaBK;
#pragma unroll
        for (int kk = 0; kk < kFaBK / 16; ++kk)
          umma_f16_ts(tmem + C::kOCol + (uint32_t)t * D, pa + (uint32_t)(kk * 8),
                      sdesc_k128_sw128(sv + (uint32_t)((kk >> 2) * (D * 128))) +
                          (uint64_t)(2 * (kk & 3)),
                      idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_done[t]);
      };
      bool ok = mbar_wait(q_full, 0, s_abort, p.err, FERR_MMA) &&
                mbar_wait(&k_full[0], 0, s_abort, p.err, FERR_MMA);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < n; ++j) {
        const bool more = j + 1 < n;
        // tile 0: P V, then its next S (in-order: the S MMA overwrites
        // S0 only after this P V has read P0 from it)
        if (!mbar_wait(&p_full[0], (uint32_t)j & 1u, s_abort, p.err, FERR_MMA) ||
            !mbar_wait(&v_full[j % SV], (uint32_t)(j / SV) & 1u, s_abort, p.err, FERR_MMA))
          break;
        tc_fence_after();
        issue_pv(0, j);
        if (more) {
          if (!mbar_wait(&k_full[(j + 1) % SK], (uint32_t)((j + 1) / SK) & 1u, s_abort, p.err,
                         FERR_MMA))
            break;
          tc_fence_after();
          issue_s(0, j + 1);
        }
        if (!mbar_wait(&p_full[1], (uint32_t)j & 1u, s_abort, p.err, FERR_MMA)) break;
        tc_fence_after();
        issue_pv(1, j);
        umma_commit(&v_empty[j % SV]);
        if (more) {
          issue_s(1, j + 1);
          umma_commit(&k_empty[(j + 1) % SK]);
        }
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, p.err, FERR_DRAIN);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    // warps 4-11: tile 0, 12-19: tile 1; within a tile the first four take
    // score columns [0, 64), the next four [64, 128) of the same rows.
    const int t = (warp - 4) >> 3;
    const int hh = ((warp - 4) >> 2) & 1;
    const int q = warp & 3;
    const int r = q * 32 + (int)lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t scol = tmem + lane_base + C::kSCol + (uint32_t)t * kFaBK;
    const uint32_t ocol = tmem + lane_base + C::kOCol + (uint32_t)t * D + (uint32_t)hh * (D / 2);
    const float c = p.scale_log2;
    float m_run = 0.0f, l_run = 0.0f;
    bool ok = true;
    // Every warp of a tile takes the same n + 1 named barriers, also after an
    // abort (which then only skips the TMEM work), so none is left waiting.
    for (int i = 0; i < n; ++i) {
      ok = __all_sync(0xffffffffu,
                      ok && mbar_wait(&s_full[t], (uint32_t)i & 1u, s_abort, p.err, FERR_SOFTMAX));
      // after an abort the reads below see whatever TMEM holds (still
      // allocated); only the mbarrier traffic is skipped
      uint32_t a[32], b[32];
      float m4[4] = {-3.0e38f, -3.0e38f, -3.0e38f, -3.0e38f};
      tc_fence_after();
      const int valid = p.tk - i * kFaBK - hh * 64;   // valid columns of this half
      tmem_ld32(scol + (uint32_t)(hh * 64), a);
      tmem_ld32(scol + (uint32_t)(hh * 64 + 32), b);
      tmem_wait_ld();
      if (valid < 64) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (e >= valid) a[e] = __float_as_uint(-3.0e38f);
          if (32 + e >= valid) b[e] = __float_as_uint(-3.0e38f);
        }
      }
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        m4[0] = max3f(m4[0], __uint_as_float(a[e]), __uint_as_float(a[e + 1]));
        m4[1] = max3f(m4[1], __uint_as_float(a[e + 2]), __uint_as_float(a[e + 3]));
        m4[2] = max3f(m4[2], __uint_as_float(b[e]), __uint_as_float(b[e + 1]));
        m4[3] = max3f(m4[3], __uint_as_float(b[e + 2]), __uint_as_float(b[e + 3]));
      }
      // the row's max over both halves: exchange through shared memory (both
      // halves have their scores in registers after this barrier, so either
      // may then overwrite the TMEM columns with P)
      s_mx[t][i & 1][hh][r] = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      named_bar_sync(1 + t, 256);
      if (!ok) continue;
      const float mx = fmaxf(s_mx[t][i & 1][0][r], s_mx[t][i & 1][1][r]);
      const float m_tile = mx * c;
      if (i == 0) m_run = m_tile;
      const bool need = i > 0 && m_tile > m_run + kRescale;
      // the O rescale waits until P is in TMEM, so the scores' registers are
      // free by then (P must only land before p_full is signalled)
      const bool rescale = __any_sync(0xffffffffu, need);
      float f = 1.0f;
      if (rescale) {
        const float m_new = need ? m_tile : m_run;
        f = fast_exp2(m_run - m_new);
        l_run *= f;
        m_run = m_new;
      }
      const unsigned long long c2 = pair2(__float_as_uint(c), __float_as_uint(c));
      const unsigned long long nm2 = pair2(__float_as_uint(-m_run), __float_as_uint(-m_run));
      unsigned long long sa = 0ull, sb = 0ull;
      uint32_t pk[32];
      fa3_exp(a, b, c2, nm2, pk, sa, sb);
      tmem_st32(scol + (uint32_t)(hh * 32), pk);
      const unsigned long long st2 = fadd2(sa, sb);
      l_run += __uint_as_float((uint32_t)st2) + __uint_as_float((uint32_t)(st2 >> 32));
      if (rescale)
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&o_done[t], (uint32_t)(i - 1) & 1u, s_abort, p.err,
                                  FERR_SOFTMAX));
      if (rescale && ok) {
        tc_fence_after();
#pragma unroll
        for (int c4 = 0; c4 < D / 64; ++c4) {
          uint32_t v[32];
          tmem_ld32(ocol + (uint32_t)(c4 * 32), v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * f);
          tmem_st32(ocol + (uint32_t)(c4 * 32), v);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&p_full[t]);
    }
    // the row's sum over both halves (parity slot 0/1 of tile i are free now)
    s_mx[t][n & 1][hh][r] = l_run;
    named_bar_sync(1 + t, 256);
    const float l_row = s_mx[t][n & 1][0][r] + s_mx[t][n & 1][1][r];
    if (ok && n > 0 &&
        mbar_wait(&o_done[t], (uint32_t)(n - 1) & 1u, s_abort, p.err, FERR_SOFTMAX)) {
      tc_fence_after();
      const int row = q0 + t * kFaBQ + r;
      float g = 1.0f / l_row;
      if (p.gate != nullptr && row < p.tq)
        g *= 2.0f / (1.0f + __expf(-__bfloat162float(p.gate[(size_t)row * p.ldg + h])));
      __nv_bfloat16* orow = p.o + (size_t)row * p.ldo + h * D + hh * (D / 2);
#pragma unroll
      for (int c4 = 0; c4 < D / 64; ++c4) {
        uint32_t v[32];
        tmem_ld32(ocol + (uint32_t)(c4 * 32), v);
        tmem_wait_ld();
        if (row < p.tq) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(v[8 * e + 0]) * g, __uint_as_float(v[8 * e + 1]) * g);
            w.y = pack_bf16(__uint_as_float(v[8 * e + 2]) * g, __uint_as_float(v[8 * e + 3]) * g);
            w.z = pack_bf16(__uint_as_float(v[8 * e + 4]) * g, __uint_as_float(v[8 * e + 5]) * g);
            w.w = pack_bf16(__uint_as_float(v[8 * e + 6]) * g, __uint_as_float(v[8 * e + 7]) * g);
            *reinterpret_cast<uint4*>(orow + c4 * 32 + 8 * e) = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// Merge split-KV partials: for each (row, head), weights 2^(m_s - max m),
// o = sum_s w_s O_s / sum_s w_s l_s, times the gate; 4 columns per thread.
__global__ void fa_combine_kernel(const float* __restrict__ part_o,
                                  const float* __restrict__ part_ml, int splits, int tq,
                                  int heads, int D, __nv_bfloat16* __restrict__ o, int ldo,
                                  const __nv_bfloat16* __restrict__ gate, int ldg)
{
  pdl_wait();
  pdl_trigger();
  const int d4 = D / 4;
  const size_t total = (size_t)tq * heads * d4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % d4) * 4;
    const size_t rh = i / d4;                 // row * heads + h
    const int h = (int)(rh % heads), row = (int)(rh / heads);
    float mx = -3.0e38f;
    for (int sp = 0; sp < splits; ++sp)
      mx = fmaxf(mx, part_ml[((size_t)sp * tq * heads + rh) * 2]);
    float l = 0.0f, a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (int sp = 0; sp < splits; ++sp) {
      const size_t site = (size_t)sp * tq * heads + rh;
      const float2 ml = *reinterpret_cast<const float2*>(part_ml + site * 2);
      const float w = fast_exp2(ml.x - mx);
      l += w * ml.y;
      const float4 v = *reinterpret_cast<const float4*>(part_o + site * D + c);
      a0 += w * v.x;
      a1 += w * v.y;
      a2 += w * v.z;
      a3 += w * v.w;
    }
    float g = 1.0f / l;
    if (gate != nullptr)
      g *= 2.0f / (1.0f + __expf(-__bfloat162float(gate[(size_t)row * ldg + h])));
    uint2 out;
    out.x = pack_bf16(a0 * g, a1 * g);
    out.y = pack_bf16(a2 * g, a3 * g);
    *reinterpret_cast<uint2*>(o + (size_t)row * ldo + h * D + c) = out;
  }
}

// vt[c][t] = v[t][c]: c < cols (= heads * D), t < tk.  64 x 64 tiles.
__global__ void __launch_bounds__(256)
    transpose_kernel(const __nv_bfloat16* __restrict__ v, int ldv, int tk, int cols,
                     __nv_bfloat16* __restrict__ vt, int ldvt)
{
  pdl_wait();
  pdl_trigger();
  // A 128-token x 64-column tile a CTA, four 16-byte loads and stores a
  // thread.  Rows of 66 elements (33 words) put the load phase's element
  // stores and the store phase's column reads on distinct banks; each
  // column's 16 tokens of a store step are one 32-byte sector of vt.
  __shared__ __nv_bfloat16 tile[128][66];
  const int t0 = blockIdx.x * 128, c0 = blockIdx.y * 64;
  for (int i = threadIdx.x; i < 128 * 8; i += 256) {
    const int rr = i >> 3, cc = (i & 7) * 8;
    uint4 w = make_uint4(0, 0, 0, 0);
    if (t0 + rr < tk && c0 + cc < cols)
      w = *reinterpret_cast<const uint4*>(v + (size_t)(t0 + rr) * ldv + c0 + cc);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[rr][cc + k] = e[k];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 128 * 8; i += 256) {
    const int j = i & 127;
    const int cc = j >> 1, rr = (i >> 7) * 16 + (j & 1) * 8;
    if (c0 + cc >= cols || t0 + rr >= tk) continue;
    __align__(16) __nv_bfloat16 e[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] = tile[rr + k][cc];
    __nv_bfloat16* dst = vt + (size_t)(c0 + cc) * ldvt + t0 + rr;
    if (t0 + rr + 8 <= ldvt) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(e);
    } else {
      for (int k = 0; k < 8 && t0 + rr + k < ldvt; ++k) dst[k] = e[k];
    }
  }
}

// mean[c] = (1/tk) sum_t k[t][c] for c < cols: the per-channel key mean the
// sage tier subtracts (each thread one column pair, a CTA 64 token slices).
__global__ void __launch_bounds__(256)
    col_mean_kernel(const __nv_bfloat16* __restrict__ k, int ldk, int tk, int cols,
                    float* __restrict__ mean)
{
  pdl_wait();
  pdl_trigger();
  __shared__ float part[8][64];
  const int c = blockIdx.x * 64 + (threadIdx.x & 63);
  const int slice = threadIdx.x >> 6;           // 4 token slices
  float acc = 0.0f;
  if (c < cols)
    for (int t = slice; t < tk; t += 4) acc += __bfloat162float(k[(size_t)t * ldk + c]);
  part[slice][threadIdx.x & 63] = acc;
  __syncthreads();
  if (slice == 0 && c < cols)
    mean[c] = (part[0][threadIdx.x] + part[1][threadIdx.x] + part[2][threadIdx.x] +
               part[3][threadIdx.x]) / (float)tk;
}

// One 128-token block of one head to int8 with one scale: x (minus the
// channel mean, when given) / (absmax / 127), rounded to nearest even,
// into rows of 128 bytes (D <= 128; the rest of the row and the rows past
// `tokens` are zero).  out: [head][tpad][128], scale: [head][tpad / 128].
// Thread pair (2r, 2r+1) owns row r, 64 bytes each.
template <int D>
__global__ void __launch_bounds__(256)
    quant_block_i8_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int tokens,
                          const float* __restrict__ mean, int8_t* __restrict__ out,
                          float* __restrict__ scale, int tpad)
{
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8];
  const int b = blockIdx.x, h = blockIdx.y;
  const int nb = tpad / 128;
  const int r = threadIdx.x >> 1;
  const int c0 = (threadIdx.x & 1) * 64;
  const int t = b * 128 + r;
  float v[64];
  float amax = 0.0f;
#pragma unroll
  for (int e8 = 0; e8 < 8; ++e8) {
    const int c = c0 + e8 * 8;
    if (c < D && t < tokens) {
      const uint4 w = *reinterpret_cast<const uint4*>(x + (size_t)t * ldx + h * D + c);
      const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(hw[i]);
        v[e8 * 8 + 2 * i] = f.x;
        v[e8 * 8 + 2 * i + 1] = f.y;
      }
      if (mean != nullptr) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[e8 * 8 + i] -= mean[h * D + c + i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[e8 * 8 + i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[e8 * 8 + i]));
  }
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) m = fmaxf(m, red[w]);
  const float sc = m > 0.0f ? m / 127.0f : 1.0f;
  if (threadIdx.x == 0) scale[h * nb + b] = sc;
  uint32_t words[16];
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int q = __float2int_rn(__fdiv_rn(v[4 * w + e], sc));
      q = q > 127 ? 127 : (q < -127 ? -127 : q);
      word |= (uint32_t)(q & 0xff) << (8 * e);
    }
    words[w] = word;
  }
  uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)h * tpad + (size_t)t) * 128 + c0);
#pragma unroll
  for (int w = 0; w < 4; ++w)
    dst[w] = make_uint4(words[4 * w], words[4 * w + 1], words[4 * w + 2], words[4 * w + 3]);
}

PFN_encodeTiled g_fa_encode = nullptr;

bool fa_encode(CUtensorMap* map, const void* gaddr, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16)
{
  if (g_fa_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) !=
            cudaSuccess ||
        fn == nullptr)
      return false;
    g_fa_encode = reinterpret_cast<PFN_encodeTiled>(fn);
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return g_fa_encode(map, dt, 2, const_cast<void*>(gaddr), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


template <int D, bool I8>
int launch_fa(const CUtensorMap& tq_map, const CUtensorMap& tk_map, const CUtensorMap& tv_map,
              const FaParams& prm, int heads, cudaStream_t s)
{
  using C = FaCfg<D, I8>;
  static std::atomic<unsigned long long> attr{0};
  if (!smem_limit_once(fa_tc_kernel<D, I8>, C::kSmem, attr)) return -1;
  launch_k(fa_tc_kernel<D, I8>, dim3(dim3((prm.tq + kFaBQ - 1) / kFaBQ, heads, prm.splits)), dim3(kFaThreads), C::kSmem, s, 1, tq_map, tk_map, tv_map, prm);
  return launched();
}

FaParams fa_params(__nv_bfloat16* o, int ldo, const __nv_bfloat16* gate, int ldg, int tq,
                   int tk, int D, int* err)
{
  FaParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.o = o;
  prm.gate = gate;
  prm.ldo = ldo;
  prm.ldg = ldg;
  prm.tq = tq;
  prm.tk = tk;
  prm.ntiles = (tk + kFaBK - 1) / kFaBK;
  prm.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
  prm.err = err;
  prm.splits = 1;
  return prm;
}

// V^T into the scratch and its tensor map.
int prepare_vt(const __nv_bfloat16* v, int ldv, int tk, int cols, int D, __nv_bfloat16* vt,
               CUtensorMap* map, cudaStream_t s)
{
  const int ldvt = (tk + 7) / 8 * 8;
  launch_k(transpose_kernel, dim3(dim3((tk + 127) / 128, (cols + 63) / 64)), dim3(256), 0, s, 1, v, ldv, tk, cols, vt, ldvt);
  if (launched() != 0) return -1;
  return fa_encode(map, vt, (uint64_t)tk, (uint64_t)cols, (uint64_t)ldvt * 2, 64, D) ? 0 : -1;
}

bool aligned16(const void* a) { return (reinterpret_cast<uintptr_t>(a) & 15u) == 0; }

}  // namespace

size_t attention_tc_scratch(int tk, int heads, int head_dim)
{
  const size_t ldvt = ((size_t)tk + 7) / 8 * 8;
  return ldvt * (size_t)heads * head_dim;
}

int attention_tc_splits(int tq, int tk, int heads)
{
  const int ctas = (tq + kFaBQ - 1) / kFaBQ * heads;
  const int n = (tk + kFaBK - 1) / kFaBK;
  if (ctas >= 148 || n < 4) return 1;
  int sp = (2 * 148 + ctas - 1) / ctas;
  sp = sp > n / 2 ? n / 2 : sp;
  return sp > 32 ? 32 : (sp < 1 ? 1 : sp);
}

size_t attention_tc_part(int tq, int tk, int heads, int head_dim)
{
  const int sp = attention_tc_splits(tq, tk, heads);
  return sp > 1 ? (size_t)sp * tq * heads * (head_dim + 2) : 0;
}

int launch_attention_tc(const __nv_bfloat16* q, int ldq, const __nv_bfloat16* k, int ldk,
                        const __nv_bfloat16* v, int ldv, __nv_bfloat16* vt,
                        size_t vt_elems, __nv_bfloat16* o, int ldo,
                        const __nv_bfloat16* gate, int ldg, int tq, int tk, int heads,
                        int head_dim, int* err, cudaStream_t s, float* part,
                        size_t part_elems, bool vt_ready)
{
  if (tq <= 0 || tk <= 0 || heads <= 0) return 0;
  if (head_dim != 128 && head_dim != 64) return -2;
  if ((ldq | ldk | ldv) % 8 != 0 || ldo % 8 != 0 || !aligned16(q) || !aligned16(k) ||
      !aligned16(v) || !aligned16(o))
    return -2;
  if (vt_elems < attention_tc_scratch(tk, heads, head_dim)) return -3;
  const int D = head_dim;
  const int cols = heads * D;
  CUtensorMap tq_map, tk_map, tv_map;
  if (vt_ready) {
    // V^T written by its producer ([cols][ldvt], keys contiguous)
    const uint64_t ldvt = ((uint64_t)tk + 7) / 8 * 8;
    if (!aligned16(vt) || !fa_encode(&tv_map, vt, (uint64_t)tk, (uint64_t)cols, ldvt * 2, 64, D))
      return -1;
  } else if (prepare_vt(v, ldv, tk, cols, D, vt, &tv_map, s) != 0) {
    return -1;
  }
  if (!fa_encode(&tq_map, q, (uint64_t)cols, (uint64_t)tq, (uint64_t)ldq * 2, 64, kFaBQ) ||
      !fa_encode(&tk_map, k, (uint64_t)cols, (uint64_t)tk, (uint64_t)ldk * 2, 64, kFaBK))
    return -1;
  FaParams prm = fa_params(o, ldo, gate, ldg, tq, tk, D, err);
  const int splits = attention_tc_splits(tq, tk, heads);
  if (splits > 1) {
    // few query tiles, many keys (video->audio): split the keys, merge after
    if (part == nullptr || part_elems < attention_tc_part(tq, tk, heads, D)) return -3;
    prm.splits = splits;
    prm.heads = heads;
    prm.part_o = part;
    prm.part_ml = part + (size_t)splits * tq * heads * D;
    const int rc = D == 128 ? launch_fa<128, false>(tq_map, tk_map, tv_map, prm, heads, s)
                            : launch_fa<64, false>(tq_map, tk_map, tv_map, prm, heads, s);
    if (rc != 0) return rc;
    const size_t total = (size_t)tq * heads * (D / 4);
    size_t grid = (total + 255) / 256;
    if (grid > 148 * 8) grid = 148 * 8;
    launch_k(fa_combine_kernel, dim3((unsigned)grid), dim3(256), 0, s, 1, prm.part_o, prm.part_ml, splits, tq, heads, D, o, ldo, gate, ldg);
    return launched();
  }
  if (D == 64) return launch_fa<64, false>(tq_map, tk_map, tv_map, prm, heads, s);
  static const int two_tiles = [] {
    const char* e = getenv("LTX25_FA_TILES");
    return (e != nullptr && e[0] == '1') ? 0 : 1;
  }();
  if (tq <= kFaBQ || !two_tiles) return launch_fa<128, false>(tq_map, tk_map, tv_map, prm, heads, s);
  // kernel for tq > 128: split rows (default) or whole rows a softmax warp
  // (LTX25_FA_KIND=2)
  static const int kind = [] {
    const char* e = getenv("LTX25_FA_KIND");
    return (e != nullptr && e[0] == '2') ? 2 : 3;
  }();
  const dim3 grid2((tq + 2 * kFaBQ - 1) / (2 * kFaBQ), heads);
  if (kind == 3) {
    static std::atomic<unsigned long long> attr3{0};
    if (!smem_limit_once(fa3_tc_kernel, Fa3Cfg::kSmem, attr3)) return -1;
    launch_k(fa3_tc_kernel, grid2, dim3(kFa3Threads), Fa3Cfg::kSmem, s, 1, tq_map, tk_map,
             tv_map, prm);
    return launched();
  }
  static std::atomic<unsigned long long> attr2{0};
  if (!smem_limit_once(fa2_tc_kernel, Fa2Cfg::kSmem, attr2)) return -1;
  launch_k(fa2_tc_kernel, grid2, dim3(kFa2Threads), Fa2Cfg::kSmem, s, 1, tq_map, tk_map, tv_map,
           prm);
  return launched();
}

SageScratch sage_scratch_need(int tq, int tk, int heads, int head_dim)
{
  SageScratch n;
  const size_t tqp = ((size_t)tq + 127) / 128 * 128, tkp = ((size_t)tk + 127) / 128 * 128;
  n.qi8 = (size_t)heads * tqp * 128;
  n.ki8 = (size_t)heads * tkp * 128;
  n.scales = (size_t)heads * (tqp + tkp) / 128;
  n.mean = (size_t)heads * head_dim;
  n.vt = attention_tc_scratch(tk, heads, head_dim);
  return n;
}

int launch_sage_tc(const __nv_bfloat16* q, int ldq, const __nv_bfloat16* k, int ldk,
                   const __nv_bfloat16* v, int ldv, const SageBuffers& sb,
                   __nv_bfloat16* o, int ldo, const __nv_bfloat16* gate, int ldg, int tq,
                   int tk, int heads, int head_dim, int* err, cudaStream_t s)
{
  if (tq <= 0 || tk <= 0 || heads <= 0) return 0;
  if (head_dim != 128 && head_dim != 64) return -2;
  if ((ldq | ldk | ldv) % 8 != 0 || ldo % 8 != 0 || !aligned16(v) || !aligned16(o))
    return -2;
  const SageScratch need = sage_scratch_need(tq, tk, heads, head_dim);
  if (sb.cap.qi8 < need.qi8 || sb.cap.ki8 < need.ki8 || sb.cap.scales < need.scales ||
      sb.cap.mean < need.mean || sb.cap.vt < need.vt)
    return -3;
  const int D = head_dim;
  const int cols = heads * D;
  const int tqp = (tq + 127) / 128 * 128, tkp = (tk + 127) / 128 * 128;
  float* sq = sb.scales;
  float* sk = sb.scales + (size_t)heads * (tqp / 128);
  // K - mean(K) over tokens (exact under softmax), then per-block int8.
  launch_k(col_mean_kernel, dim3((cols + 63) / 64), dim3(256), 0, s, 1, k, ldk, tk, cols, sb.mean);
  if (launched() != 0) return -1;
  if (D == 128) {
    launch_k(quant_block_i8_kernel<128>, dim3(dim3(tqp / 128, heads)), dim3(256), 0, s, 1, q, ldq, tq, nullptr, sb.qi8, sq, tqp);
    if (launched() != 0) return -1;
    launch_k(quant_block_i8_kernel<128>, dim3(dim3(tkp / 128, heads)), dim3(256), 0, s, 1, k, ldk, tk, sb.mean, sb.ki8, sk, tkp);
  } else {
    launch_k(quant_block_i8_kernel<64>, dim3(dim3(tqp / 128, heads)), dim3(256), 0, s, 1, q, ldq, tq, nullptr, sb.qi8, sq, tqp);
    if (launched() != 0) return -1;
    launch_k(quant_block_i8_kernel<64>, dim3(dim3(tkp / 128, heads)), dim3(256), 0, s, 1, k, ldk, tk, sb.mean, sb.ki8, sk, tkp);
  }
  if (launched() != 0) return -1;
  CUtensorMap tq_map, tk_map, tv_map;
  if (prepare_vt(v, ldv, tk, cols, D, sb.vt, &tv_map, s) != 0) return -1;
  if (!fa_encode(&tq_map, sb.qi8, 128, (uint64_t)heads * tqp, 128, 128, kFaBQ,
                 CU_TENSOR_MAP_DATA_TYPE_UINT8) ||
      !fa_encode(&tk_map, sb.ki8, 128, (uint64_t)heads * tkp, 128, 128, kFaBK,
                 CU_TENSOR_MAP_DATA_TYPE_UINT8))
    return -1;
  FaParams prm = fa_params(o, ldo, gate, ldg, tq, tk, D, err);
  prm.sq = sq;
  prm.sk = sk;
  prm.nqb = tqp / 128;
  prm.tq_pad = tqp;
  prm.tk_pad = tkp;
  return D == 128 ? launch_fa<128, true>(tq_map, tk_map, tv_map, prm, heads, s)
                  : launch_fa<64, true>(tq_map, tk_map, tv_map, prm, heads, s);
}

}  // namespace ltx
