// gemm_tc.cuh -- the tcgen05 GEMM behind every projection of the LTX-2.5
// block:  y[M][N] = x[M][K] . W[N][K]^T (+ bias) with a fused epilogue.
//
// One persistent kernel per (mode, token-tile, epilogue):
//
//   MODE_W8G64  W is the group-affine u8 pack (4 codes per u32 word, low
//               bits first; one bf16 scale and zero-point per 64 K).  The
//               codes are TMA-staged into shared memory and DEQUANTIZED BY
//               FOUR WARPS STRAIGHT INTO TENSOR MEMORY, where tcgen05.mma
//               reads them as its A operand.  The dequantized weight never
//               touches shared memory, so the only smem operand stream is the
//               activation tile.
//   MODE_BF16   W is dense bf16 (the dequant-once arm, the gate logits).
//   MODE_I8     x and W are int8 (the i8_gemm tier), s32 accumulate,
//               per-token x scale and per-channel W scale in the epilogue.
//
// The MMA is issued TRANSPOSED: its M dimension (128 lanes of TMEM) is the
// weight's output-feature tile and its N dimension is the TOKEN tile (TN).
// Small token counts (the 126-token audio stream) therefore cost a 128-wide
// MMA instead of padding 126 rows up to a 128-row M tile, and the epilogue
// thread that owns TMEM lane n owns output feature n for every token.
//
// Warp roles (576 threads):
//   warp 0       TMA producer (one elected lane)
//   warp 1       TMEM allocator + MMA issuer (one elected lane)
//   warps 2-9    dequant (MODE_W8G64): two groups of four, one warp per
//                TMEM lane quarter (warp % 4), alternating k-blocks; on
//                the dense path (MODE_BF16) these eight join the epilogue
//   warps 10-17  epilogue: groups of four (two, or four with warps 2-9),
//                alternating 32-column chunks;
//                TMEM -> registers -> bias/act/residual -> global
//
// Large token counts run as CTA PAIRS (cta_group::2, a cluster of two):
// one M = 256 MMA spans 256 weight rows, each CTA dequantizing its 128 into
// its own TMEM and holding half of the 256-token activation tile, so each
// SM streams half the activation bytes per FLOP of a single-CTA tile.
// A dense pair may also hold TWO weight blocks per CTA (WB = 2: 512 weight
// rows x 256 tokens per pair, both accumulators filling all 512 TMEM
// columns): each activation stage then feeds two MMAs, so an SM takes in
// 48 KB per 2 x 128x256x64 MMA instead of 32 KB per one.  Without a second
// accumulator set, the epilogue pulls its chunks out of TMEM and releases
// the accumulator before storing (or, for the gated residual, prefetches
// the first chunk's residual during the wait), and the tiles of a last,
// partial wave run as half tiles of one weight block each.
//
// Besides y, the store epilogue has two output forms: a ROW SCATTER (each
// token row to the receive slot of the tensor-parallel rank that owns it,
// possibly another GPU's memory: the reduce-scatter fused into the GEMM)
// and TRANSPOSED columns (an attention's V^T written by the K/V projection).
//
// K is split across CTAs (`splits` > 1, at most 8) for the small-M,
// bandwidth-bound shapes.  The splits of one output tile are launched as
// one thread-block cluster; each parks its f32 partial in its own shared
// memory and the cluster reduces them through distributed shared memory in
// rank order, so the result is deterministic and never leaves the SMs
// before it is final.
#pragma once

#include "ptx.cuh"

namespace ltx {

enum GemmMode : int { MODE_W8G64 = 0, MODE_BF16 = 1, MODE_I8 = 2 };
enum EpiMode : int { EPI_STORE = 0, EPI_GELU = 1, EPI_GATED_RES = 2 };

// Error codes written into GemmParams::err by a kernel that gave up.
enum KernelErr : int {
  KERR_NONE = 0,
  KERR_WAIT_PRODUCER = 1,
  KERR_WAIT_MMA = 2,
  KERR_WAIT_DEQUANT = 3,
  KERR_WAIT_EPILOGUE = 4,
  KERR_DRAIN = 5,
};

struct GemmParams {
  int M, N, K;             // tokens, output features, input features
  int m_tiles, n_tiles;    // ceil(M/TN), ceil(N/128)
  int splits;              // K splits (1 = no split)
  int kblocks;             // K blocks in all (main + extension)
  // K blocks of x.W^T; the blocks after them read the extension maps (a
  // low-rank adapter's r.B^T, MODE_BF16 only) into the same accumulator.
  // 0 or == kblocks: no extension.
  int kblocks_main;
  int num_tiles;           // m_tiles * n_tiles * splits
  // Work units of the persistent loop.  Units below full_units are whole
  // tiles; with two weight blocks per CTA the tiles past full_units (the
  // last, partial wave) run as two half units of one weight block each,
  // unit full_units + 2 h + b taking block b of tile full_units + h.
  // Without a tail split both equal num_tiles.
  int full_units, num_units;
  int ldy;                 // row stride of y, elements
  const __nv_bfloat16* bias;   // [N] or null
  const float* gate;           // [N] f32, EPI_GATED_RES only
  union {
    __nv_bfloat16* y;               // [M][ldy]
    __nv_bfloat16* const* ys;       // row scatter: see scatter_rows
  };
  const float* sx;             // MODE_I8: [M] token scales
  union {
    const float* sw;             // MODE_I8: [N] channel scales
    // The other modes, EPI_STORE, one K split: columns n >= vt_col0 are
    // written TRANSPOSED, vt[(n - vt_col0) * ldvt + j] (an attention's V^T,
    // keys contiguous), and not to y; null = off.  vt_col0 % 32 == 0.
    __nv_bfloat16* vt;
  };
  int* err;                    // device error word (0 = ok)
  int group_m;                 // raster: token tiles per weight sweep (0 = 8)
  int krot;                    // 1: rotate each tile's K start (one token tile)
  // Diagnostics (null = off): kTraceSlots u64 per CTA for the first
  // `trace_ctas` CTAs -- phase timestamps (clock64) and the MMA issuer's
  // cumulative wait cycles per barrier kind.
  unsigned long long* trace;
  int trace_ctas;
  // Row scatter (the fused tensor-parallel reduce-scatter), EPI_STORE, one
  // K split, packed as rows * 8 + slot (0 = off; slot < 8): token row j is
  // stored at ys[j / rows] + (slot * rows + j % rows) * ldy instead of
  // y + j * ldy -- the receive slot of the rank that owns row j, which may be
  // another GPU's memory mapped into this one (plain stores over NVLink),
  // followed by a system-scope fence before the kernel ends.  `ys` (a device
  // array of the owners' buffers) takes the place of y.
  int scatter;
  // Transposed columns (see vt), packed as (vt_col0 / 32) << 20 | ldvt / 8
  // (0 = off).  Both switches fit the 8 bytes added to this block: a larger
  // parameter block made ptxas spill in the gated-residual variants, which
  // use neither.
  int vt_spec;
};

// The packed switches: rows < 2^28 and slot < 8; col0 % 32 == 0 and
// col0 < 65536, ld % 8 == 0 and ld < 2^23 (the host checks the ranges).
__host__ __device__ inline int pack_scatter(int rows, int slot) { return rows * 8 + slot; }
__host__ __device__ inline int pack_vt(int col0, int ld) { return ((col0 / 32) << 20) | (ld / 8); }
__host__ __device__ inline int scatter_rows(const GemmParams& p) { return p.scatter >> 3; }
__host__ __device__ inline int scatter_slot(const GemmParams& p) { return p.scatter & 7; }
__host__ __device__ inline int vt_col0(const GemmParams& p) { return (p.vt_spec >> 20) * 32; }
__host__ __device__ inline int vt_ld(const GemmParams& p) { return (p.vt_spec & 0xFFFFF) * 8; }

constexpr int kTraceSlots = 24;
enum TraceSlot : int {
  TR_ENTRY = 0, TR_SETUP, TR_FIRST_TMA, TR_LAST_TMA, TR_FIRST_FULL_DEQ,
  TR_FIRST_MMA, TR_LAST_COMMIT, TR_FIRST_ACC, TR_EPI_DONE, TR_REDUCED,
  TR_END, TR_TILES, TR_MMA_WAIT_FULL, TR_MMA_WAIT_A, TR_MMA_WAIT_ACC,
  TR_PROD_WAIT_EMPTY,
  // dequant warp 2, lane 0: cumulative cycles
  TR_DEQ_WAIT_FULL, TR_DEQ_LOAD, TR_DEQ_MATH, TR_DEQ_WAIT_ST,
  TR_DEQ_WAIT_AEMPTY, TR_DEQ_BLOCKS,
  // first epilogue warp, lane 0: cumulative cycles waiting / working
  TR_EPI_WAIT, TR_EPI_WORK
};

template <int MODE, int TN, bool PAIR = false, int WB = 1>
struct GemmCfg {
  static constexpr int kBM = 128;                       // weight rows / block
  // Weight blocks of kBM rows per CTA: a dense pair may hold two, so one
  // activation stage feeds two M = 256 MMAs (512 weight rows per pair).
  static constexpr int kWB = WB;
  // Activation rows per CTA: a pair splits the TN-token tile between its
  // two CTAs (each holds half of the MMA's B operand).
  static constexpr int kXRows = PAIR ? TN / 2 : TN;
  static constexpr int kXStage = kXRows * 128;           // 128 B of K per row
  static constexpr int kWStage = MODE == MODE_W8G64 ? kBM * 64 : WB * kBM * 128;
  static constexpr int kSZStage = MODE == MODE_W8G64 ? kBM * 4 : 0;
  static constexpr int kStageBytes = kXStage + kWStage + kSZStage;
  static constexpr int kStages =
      (224 * 1024) / kStageBytes > 8 ? 8 : (224 * 1024) / kStageBytes;
  // Accumulator sets in TMEM (double buffering across tiles); a set is WB
  // accumulators of TN columns.
  static constexpr int kNAcc =
      MODE == MODE_W8G64 ? (2 * TN + 4 * 32 <= 512 ? 2 : 1) : (WB == 2 ? 1 : 2);
  static constexpr int kASlotsRaw = (512 - kNAcc * WB * TN) / 32;
  static constexpr int kASlots =
      MODE == MODE_W8G64 ? (kASlotsRaw > 8 ? 8 : kASlotsRaw) : 0;
  static constexpr int kACol0 = kNAcc * WB * TN;         // first A column
  static constexpr int kKPerStage = MODE == MODE_I8 ? 128 : 64;  // elements
  static constexpr int kThreads = 576;   // 18 warps, see the role table
  // Epilogue warps: on the dense path the eight dequant warps join them
  // (the int8 path keeps eight: its rescale needs the registers).
  static constexpr int kEpiWarps = MODE == MODE_BF16 ? 16 : 8;
  static constexpr int kEpiWarp0 = 18 - kEpiWarps;
  static constexpr int kNumBars =
      3 * kStages + 2 * (kASlots > 0 ? kASlots : 1) + 2 * 2 + 1;
  static constexpr int kSmemBytes =
      1024 + kStages * kStageBytes + kNumBars * 8 + 64;
  static_assert(TN % 16 == 0 && TN >= 16 && TN <= 256, "MMA N");
  static_assert(WB == 1 || (WB == 2 && PAIR && MODE == MODE_BF16 && TN == 256),
                "two weight blocks: dense 256-token pairs only");
  static_assert(kNAcc * WB <= 2, "accumulator barriers");
  static_assert(TN / 32 >= kEpiWarps / 4, "every epilogue group drains a chunk");
  static_assert(kNAcc * WB * TN + kASlots * 32 <= 512, "TMEM budget");
  static_assert(MODE != MODE_W8G64 || kASlots >= 2, "A pipeline depth");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

}  // namespace ltx
