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

template <int D>
struct FaCfg {
  static constexpr int kAtom = 128 * 128;             // 128 rows x 128 B
  static constexpr int kQBytes = kFaBQ * D * 2;       // D/64 atoms
  static constexpr int kKBytes = kFaBK * D * 2;       // D/64 atoms
  static constexpr int kVAtom = D * 128;              // D rows x 64 keys
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
};

__device__ __forceinline__ float fast_exp2(float x)
{
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi)
{
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int D>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                 const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_vt, FaParams p)
{
  using C = FaCfg<D>;
  constexpr int S = kFaStages;
  constexpr int kQAtoms = D / 64;
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
  const int n = p.ntiles;

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

  if (warp == 0) {
    // ------------------------------------------------------------- TMA
    if (lane == 0) {
      uint32_t armed = 0, armed_par = 0;
      mbar_arrive_expect_tx(q_full, C::kQBytes);
      for (int a = 0; a < kQAtoms; ++a)
        tma_load_2d(&tm_q, q_full, s_q + a * C::kAtom, h * D + a * 64, q0);
      for (int j = 0; j < n; ++j) {
        const int st = j % S;
        const uint32_t ph = (uint32_t)(j / S) & 1u;
        if (!mbar_wait(&empty[st], ph ^ 1u, s_abort, p.err, FERR_PRODUCER)) break;
        uint8_t* sk = s_kv + st * C::kStageBytes;
        uint8_t* sv = sk + C::kKBytes;
        mbar_arrive_expect_tx(&k_full[st], C::kKBytes);
        for (int a = 0; a < kQAtoms; ++a)
          tma_load_2d(&tm_k, &k_full[st], sk + a * C::kAtom, h * D + a * 64, j * kFaBK);
        mbar_arrive_expect_tx(&v_full[st], C::kVBytes);
        for (int a = 0; a < 2; ++a)
          tma_load_2d(&tm_vt, &v_full[st], sv + a * C::kVAtom, j * kFaBK + a * 64, h * D);
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
      constexpr uint32_t idesc_s = idesc_bf16(kFaBQ, kFaBK);
      constexpr uint32_t idesc_o = idesc_bf16(kFaBQ, D);
      bool ok = mbar_wait(q_full, 0, s_abort, p.err, FERR_MMA);
      for (int j = 0; ok && j <= n; ++j) {
        if (j < n) {
          const int st = j % S;
          if (!mbar_wait(&k_full[st], (uint32_t)(j / S) & 1u, s_abort, p.err, FERR_MMA)) break;
          tc_fence_after();
          const uint32_t sk = smem_u32(s_kv + st * C::kStageBytes);
          const uint32_t d = tmem + C::kSCol + (uint32_t)(j & 1) * kFaBK;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (uint32_t)((kk >> 2) * C::kAtom);
            umma_f16_ss(d, sdesc_k128_sw128(smem_u32(s_q) + off) + (uint64_t)(2 * (kk & 3)),
                        sdesc_k128_sw128(sk + off) + (uint64_t)(2 * (kk & 3)), idesc_s,
                        kk > 0 ? 1u : 0u);
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
    const float c = p.scale_log2;
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
        for (int e = 0; e < 32; ++e) s[c4 * 32 + e] = __uint_as_float(v[e]);
      }
      tmem_wait_ld();
      const int valid = p.tk - i * kFaBK;
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
    if (ok && n > 0 &&
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

// vt[c][t] = v[t][c]: c < cols (= heads * D), t < tk.  64 x 64 tiles.
__global__ void __launch_bounds__(256)
    transpose_kernel(const __nv_bfloat16* __restrict__ v, int ldv, int tk, int cols,
                     __nv_bfloat16* __restrict__ vt, int ldvt)
{
  __shared__ __nv_bfloat16 tile[64][64 + 8];
  const int t0 = blockIdx.x * 64, c0 = blockIdx.y * 64;
  // load: 64 rows x 64 columns, 8 columns (16 B) per thread
  for (int i = threadIdx.x; i < 64 * 8; i += 256) {
    const int rr = i >> 3, cc = (i & 7) * 8;
    uint4 w = make_uint4(0, 0, 0, 0);
    if (t0 + rr < tk && c0 + cc < cols)
      w = *reinterpret_cast<const uint4*>(v + (size_t)(t0 + rr) * ldv + c0 + cc);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[rr][cc + k] = e[k];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 64 * 8; i += 256) {
    const int cc = i >> 3, rr = (i & 7) * 8;
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

PFN_encodeTiled g_fa_encode = nullptr;

bool fa_encode(CUtensorMap* map, const void* gaddr, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer)
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
  return g_fa_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(gaddr), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t attention_tc_scratch(int tk, int heads, int head_dim)
{
  const size_t ldvt = ((size_t)tk + 7) / 8 * 8;
  return ldvt * (size_t)heads * head_dim;
}

int launch_attention_tc(const __nv_bfloat16* q, int ldq, const __nv_bfloat16* k, int ldk,
                        const __nv_bfloat16* v, int ldv, __nv_bfloat16* vt,
                        size_t vt_elems, __nv_bfloat16* o, int ldo,
                        const __nv_bfloat16* gate, int ldg, int tq, int tk, int heads,
                        int head_dim, int* err, cudaStream_t s)
{
  if (tq <= 0 || tk <= 0 || heads <= 0) return 0;
  if (head_dim != 128) return -2;
  if ((ldq | ldk | ldv) % 8 != 0 || ldo % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) % 16 != 0)
    return -2;
  if (vt_elems < attention_tc_scratch(tk, heads, head_dim)) return -3;
  constexpr int D = 128;
  using C = FaCfg<D>;
  const int cols = heads * D;
  const int ldvt = (tk + 7) / 8 * 8;
  transpose_kernel<<<dim3((tk + 63) / 64, (cols + 63) / 64), 256, 0, s>>>(v, ldv, tk, cols, vt,
                                                                         ldvt);
  if (launched() != 0) return -1;
  CUtensorMap tq_map, tk_map, tv_map;
  if (!fa_encode(&tq_map, q, (uint64_t)cols, (uint64_t)tq, (uint64_t)ldq * 2, 64, kFaBQ) ||
      !fa_encode(&tk_map, k, (uint64_t)cols, (uint64_t)tk, (uint64_t)ldk * 2, 64, kFaBK) ||
      !fa_encode(&tv_map, vt, (uint64_t)tk, (uint64_t)cols, (uint64_t)ldvt * 2, 64, D))
    return -1;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(fa_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmem) != cudaSuccess)
      return -1;
    attr = true;
  }
  FaParams prm;
  prm.o = o;
  prm.gate = gate;
  prm.ldo = ldo;
  prm.ldg = ldg;
  prm.tq = tq;
  prm.tk = tk;
  prm.ntiles = (tk + kFaBK - 1) / kFaBK;
  prm.scale_log2 = 1.4426950408889634f / sqrtf((float)D);
  prm.err = err;
  fa_tc_kernel<D><<<dim3((tq + kFaBQ - 1) / kFaBQ, heads), kFaThreads, C::kSmem, s>>>(
      tq_map, tk_map, tv_map, prm);
  return launched();
}

}  // namespace ltx
