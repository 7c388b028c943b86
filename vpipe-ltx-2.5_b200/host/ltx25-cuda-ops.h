// ltx25-cuda-ops.h -- the op vocabulary of the LTX-2.5 block on B200.
//
// The CUDA counterpart of the reference's MetalOps (src/ltx25-metal-ops.h):
// one object per device, owning the scratch arena and the tier switches,
// with each op one (or a few) kernel launches on a caller-supplied stream.
// Buffers are caller-owned device memory; nothing here allocates on a hot
// call once reserve() has sized the arena.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>

#include "ltx25-comm.h"
#include "../csrc/block_ops.h"

namespace ltx25 {

// One linear's weights, dense or w8g64 group-affine (src/ltx25-metal-ops.h:
// 45-57).  The pack stays bit-exact: `codes` is the reference's u32 words
// viewed as bytes (little-endian, so code k of a row is byte k).  The
// scale/zero-point pairs are stored per K group as one u32 each, bf16
// scale low / bf16 zero-point high, [K/64][N].
struct QWeight {
  uint8_t* codes = nullptr;        // [N][K]
  uint32_t* sz = nullptr;          // [K/64][N]
  __nv_bfloat16* w = nullptr;      // dense [N][K] when !quantized
  int8_t* wq = nullptr;            // int8 tier: per-channel requantized
  float* sw = nullptr;             // int8 tier: [N] channel scales
  int N = 0, K = 0, bits = 0, group = 0;
  bool quantized = false;
  int device = 0;
};

// A low-rank adapter riding on one linear (the reference's LoraPair and
// lora_add, src/ltx25-lora.h:48-56, src/ltx25-metal-ops.cc:986-1000):
// y = epilogue(x.W^T + bias + (x.A^T).B^T).  The delta is contracted in the
// linear's own accumulator (extra K blocks of the tcgen05 GEMM), so it
// lands before the epilogue's GELU / gated residual exactly where the
// reference adds it (between the linear and its consumer).
struct LoraExt {
  const __nv_bfloat16* a = nullptr;   // [r][K], the scale folded in
  const __nv_bfloat16* b = nullptr;   // [N][r]
  int r = 0;                          // rank padded to a multiple of 8
  __nv_bfloat16* rbuf = nullptr;      // [M][r] scratch: x.A^T
};

// Where a linear's output rows go under the fused tensor-parallel
// reduce-scatter: row j to dst[j / rows] + (slot * rows + j % rows) * ldy,
// the receive slot of the rank owning row j (up to 8 ranks; the owners'
// buffers may be other GPUs' memory mapped into this process).  `dst` is a
// device array of the owners' buffers (what the kernel reads).
struct RowScatter {
  __nv_bfloat16* const* dst = nullptr;
  int owners = 0;  // entries of dst
  int rows = 0;    // rows per owner
  int slot = 0;    // this rank's slot in every owner's buffer
};

// A linear's columns [col0, N) written TRANSPOSED, vt[(n - col0) * ld + j]
// (an attention's V^T, keys contiguous), instead of to y: col0 % 32 == 0,
// ld % 8 == 0, vt 16-byte aligned; not on the int8 tier.
struct VtOut {
  __nv_bfloat16* vt = nullptr;
  int col0 = 0;
  int ld = 0;
};

// One module's uploaded adapter pair (src/ltx25-lora.h:48-56): a [r8][k]
// with the scale folded in, b [n][r8], the rank padded to r8 (a multiple of
// 8, so every row is 16-byte aligned for TMA) with zero rows / columns.
struct LoraPair {
  __nv_bfloat16* a = nullptr;
  __nv_bfloat16* b = nullptr;
  int rank = 0, r8 = 0, k = 0, n = 0;
  int device = 0;
};

enum class Route { Fused = 0, DequantOnce = 1, Auto = 2 };

// A/B overrides of the GEMM tile plan (the reference's tile knob,
// src/ltx25-metal-ops.h:793-795): CTA pairs on/off, the token tile, the
// K split.  -1 = the planner's own choice.
struct PlanKnobs {
  int pair = -1, tn = -1, splits = -1;   // pair: -1 auto, 0, 1, 2 (two weight blocks)
};

class CudaOps {
public:
  ~CudaOps();

  // False (with `err`) when the device is missing or not sm_100.
  bool init(int device, std::string* err);

  // Grow the shared scratch to cover calls up to these sizes.
  bool reserve(int max_tokens, int max_n, int max_k, std::string* err);
  // Bytes of device scratch the context holds now (it grows on demand).
  size_t scratch_bytes() const;

  // y[M][N] = x[M][K] . W^T (+ bias), epilogue per ltx::EpiMode.
  // `lora` (optional): a low-rank adapter on this linear, contracted in
  // the same accumulator (see LoraExt).  A linear carrying one runs the
  // bf16 route whatever its M and tier.
  bool linear(cudaStream_t s, const __nv_bfloat16* x, int ldx,
              const QWeight& w, const __nv_bfloat16* bias, __nv_bfloat16* y,
              int ldy, int M, int K, int N, int epi,
              const float* gate, std::string* err, const LoraExt* lora = nullptr,
              const RowScatter* scatter = nullptr, const VtOut* vto = nullptr);

  // Ltx25Dit's patchify (src/ltx25-dit.cc:1509-1540): x[T][dim] =
  // latent . W^T + bias (+ adapter), then `prefix` [dim] added to rows
  // [0, prefix_rows) (the keyframe position embedding).  `latent` is
  // token-major [T][z], or channel-major [z][T] when channel_major (packed
  // on the device first, the DiT's inline pack).
  bool patchify(cudaStream_t s, const QWeight& w, const __nv_bfloat16* bias,
                const LoraPair* lora, const __nv_bfloat16* latent, bool channel_major,
                const __nv_bfloat16* prefix, int prefix_rows, __nv_bfloat16* x, int T, int z,
                int dim, std::string* err);
  // Ltx25Dit's output head (src/ltx25-dit.cc:2000-2045): LayerNorm (no
  // affine, eps 1e-6), x * (1 + scale) + shift with shift_scale f32 [2][dim]
  // (shift row first), then proj_out (+ bias, + adapter) -> out [T][out_ch],
  // or [out_ch][T] when channel_major.
  bool output_head(cudaStream_t s, const __nv_bfloat16* x, const float* shift_scale,
                   const QWeight& w, const __nv_bfloat16* bias, const LoraPair* lora,
                   __nv_bfloat16* out, bool channel_major, int T, int dim, int out_ch,
                   std::string* err);

  // MetalOps::lora_add (src/ltx25-metal-ops.cc:986-1000) on its own:
  // y[M][N] += (x[M][K].A^T).B^T for a y that already holds the linear.
  // The add is the second GEMM's epilogue (gated residual at gate 1), so
  // no [M][N] delta is written; `lora.rbuf` holds x.A^T.
  bool lora_add(cudaStream_t s, const __nv_bfloat16* x, int ldx, const LoraExt& lora,
                __nv_bfloat16* y, int ldy, int M, int K, int N, std::string* err);

  void set_route(Route r) { _route = r; }
  void set_plan_knobs(const PlanKnobs& k) { _knobs = k; }
  const PlanKnobs& plan_knobs() const { return _knobs; }
  Route route() const { return _route; }

  void set_i8_gemm(bool on) { _i8 = on; }
  bool i8_on() const { return _i8; }
  bool i8_takes(int M, int K, int N) const;

  void set_sage(bool on, int dense_layers)
  {
    _sage = on;
    _sage_dense = dense_layers;
  }
  bool sage_on() const { return _sage; }
  int sage_dense_layers() const { return _sage_dense; }

  // Per-channel int8 copy of a quantized weight for the int8 tier; made
  // once per weight, on first use or here.
  bool prepare_i8(QWeight& w, cudaStream_t s, std::string* err) const;

  // The int8 tier's quantize + kind::i8 GEMM on caller-given scratch (xq:
  // M*K codes, sx: M scales) and allocating nothing: the weight must
  // already hold its int8 copy (made by the tier's first linear on it).
  bool linear_i8_scratch(cudaStream_t s, const __nv_bfloat16* x, const QWeight& w,
                         const __nv_bfloat16* bias, __nv_bfloat16* y, int M,
                         int K, int N, int8_t* xq, float* sx,
                         std::string* err);

  int device() const { return _dev; }
  int num_sms() const { return _sms; }
  int* err_word() const { return _err_word; }

  // Multi-GPU: blocks finalized after this either shard their weights over
  // the group (tensor parallel) or keep them whole and shard the video
  // tokens (sequence parallel, `sequence` true); null comm = one GPU.
  void set_comm(std::unique_ptr<Comm> c, bool sequence = false,
                std::unique_ptr<Comm> side = nullptr)
  {
    _comm = std::move(c);
    _comm_side = std::move(side);
    _sequence = sequence;
  }
  const Comm* comm() const { return _comm.get(); }
  // Grow the tensor-parallel communicator's peer-mapped buffers to `bytes`
  // each (collective over the group; see Comm::share_buffers).
  bool share_peer_buffers(size_t bytes, std::string* err)
  {
    return _comm == nullptr || _comm->share_buffers(bytes, nullptr, err);
  }
  // The communicator for collectives on the side stream (null: none).
  const Comm* side_comm() const { return _comm_side.get(); }
  bool sequence_parallel() const { return _comm != nullptr && _sequence; }

  // Diagnostics: every following GEMM writes per-CTA phase timestamps into
  // `buf` (16 u64 per CTA, first `ctas` CTAs); null turns it off.
  void set_trace(unsigned long long* buf, int ctas)
  {
    _trace = buf;
    _trace_ctas = ctas;
  }

  // Reads and clears the device error word.  0 when clean.
  int check(cudaStream_t s, std::string* err) const;

  // Softmax attention (ltx_attention): head_dim 128 runs the tcgen05 flash
  // kernel (with its V^T scratch), head_dim 64 the warp-MMA kernel.  With
  // the sage tier on and `layer` >= sage_dense_layers, both widths take the
  // int8-QK kernel instead (sdpa_steel's sage_layer, src/ltx25-metal-ops.cc:
  // 1243-1289).  layer < 0: never sage.
  bool attention(cudaStream_t s, const __nv_bfloat16* q, int ldq,
                 const __nv_bfloat16* k, int ldk, const __nv_bfloat16* v, int ldv,
                 __nv_bfloat16* o, int ldo, const __nv_bfloat16* gate, int ldg,
                 int tq, int tk, int heads, int head_dim, std::string* err,
                 int layer = -1, const __nv_bfloat16* vt_ready = nullptr);
  // Whether attention() with these arguments reads V through the main
  // stream's V^T scratch (the tcgen05 path), so that a producer should
  // write V^T there itself (vt_scratch, VtOut) and pass it as vt_ready;
  // false under LTX25_VT_OUT=0.
  bool attention_reads_vt(cudaStream_t s, int tq, int tk, int heads, int head_dim,
                          int layer = -1) const;
  // That scratch, grown to tk keys x width columns ([width][round8(tk)]).
  __nv_bfloat16* vt_scratch(int tk, int width, std::string* err);
  // MetalOps::sage_takes (src/ltx25-metal-ops.cc:897-905): the widths the
  // int8 twin exists for, while the tier is on.
  bool sage_takes(int head_dim) const
  {
    return _sage && (head_dim == 64 || head_dim == 128);
  }
  bool sage_for(int layer, int head_dim) const
  {
    return layer >= 0 && layer >= _sage_dense && sage_takes(head_dim);
  }
  bool reserve_sage(int tq, int tk, int heads, int head_dim, std::string* err);
  // A second stream (highest priority) and events for running a block's
  // audio stream beside its video stream.  fork(a, b, i): b waits for what
  // a has issued so far (event slot i).
  cudaStream_t aux_stream(std::string* err);
  bool fork(cudaStream_t from, cudaStream_t to, int slot, std::string* err);
  // A stream for collectives issued beside the compute stream (tensor
  // parallel), and its own events: cfork(a, b, i) makes b wait for what a
  // has issued so far.
  cudaStream_t comm_stream(std::string* err);
  bool cfork(cudaStream_t from, cudaStream_t to, int slot, std::string* err);
  // The two halves of cfork: record event `slot` on `from`; make `to` wait
  // for it.
  bool crecord(cudaStream_t from, int slot, std::string* err);
  bool cwait(cudaStream_t to, int slot, std::string* err);
  // True when an audio stream of this geometry launches nothing that uses
  // the context's scratch (fused GEMMs only, warp-MMA attentions, no tier).
  bool audio_side_ok(int tokens, int text_tokens, int heads, int head_dim, int layer) const;
  // Pre-size the split-KV partials for an attention of this shape.
  bool reserve_split(int tq, int tk, int heads, int head_dim, std::string* err);
  // Pre-size the attention scratch for up to `keys` keys x `width` columns.
  bool reserve_attention(int keys, int width, std::string* err);
  // The same for attentions issued on the side (audio) stream.
  bool reserve_attention_side(int keys, int width, std::string* err);

private:
  bool ensure_(size_t i8_bytes, size_t deq_bytes, std::string* err);
  bool gemm_(cudaStream_t s, int mode, const void* x, int ldx,
             const void* wptr, const uint32_t* sz, const __nv_bfloat16* bias,
             __nv_bfloat16* y, int ldy, int M, int K, int N, int epi,
             const float* gate, const float* sx, const float* sw,
             std::string* err, const LoraExt* ext = nullptr,
             const RowScatter* scatter = nullptr, const VtOut* vto = nullptr);
  // f32 ones [n] (the gate of lora_add's accumulate), grown on demand
  const float* ones_(int n, cudaStream_t s, std::string* err);
public:
  // The context's x.A^T scratch for the standalone adapter calls, >= elems.
  __nv_bfloat16* lora_rbuf(size_t elems, std::string* err);
  // f32 ones [>= n]: the gate of a plain residual through the gated-residual
  // epilogue (y += 1 * (x W^T + b)).
  const float* ones(int n, cudaStream_t s, std::string* err) { return ones_(n, s, err); }
private:

  float* _ones = nullptr;
  int _ones_n = 0;
  __nv_bfloat16* _lora_r = nullptr;
  size_t _lora_r_elems = 0;
  // the trunk's scratch: packed latents / normalized rows, token-major out
  __nv_bfloat16* _tr[2] = {nullptr, nullptr};
  size_t _tr_elems[2] = {0, 0};
  __nv_bfloat16* trunk_buf_(int i, size_t elems, std::string* err);
  int _dev = -1;
  int _sms = 148;
  Route _route = Route::Auto;
  PlanKnobs _knobs;
  bool _i8 = false;
  bool _sage = false;
  int _sage_dense = 0;

  // Scratch arena: the int8 tier's quantized activations and the
  // dequant-once expansion.
  int8_t* _xq = nullptr;
  float* _sx = nullptr;
  size_t _xq_bytes = 0;
  __nv_bfloat16* _deq = nullptr;
  size_t _deq_bytes = 0;
  __nv_bfloat16* _vt = nullptr;    // attention: V^T
  size_t _vt_elems = 0;
  __nv_bfloat16* _vt_side = nullptr;   // the side (audio) stream's V^T
  size_t _vt_side_elems = 0;
  cudaStream_t _aux = nullptr;
  cudaStream_t _cstream = nullptr;
  cudaEvent_t _cev[8] = {};
  cudaEvent_t _ev[4] = {};
  float* _part = nullptr;          // attention: split-KV partials
  size_t _part_elems = 0;
  ltx::SageBuffers _sb;            // sage tier: int8 Q/K, scales, key mean
  int _attn_mode = 1;              // LTX25_ATTN=mma: 0 = always warp-MMA
  bool _attn64_tc = false;         // 64-wide unsplit on tcgen05 (LTX25_ATTN64=tc), else warp-MMA
  bool _vt_out = true;             // V^T from the K/V projection (LTX25_VT_OUT=0: copy kernel)
  int* _err_word = nullptr;
  std::unique_ptr<Comm> _comm;
  std::unique_ptr<Comm> _comm_side;
  bool _sequence = false;
  unsigned long long* _trace = nullptr;
  int _trace_ctas = 0;
};

// Upload helpers (the ltx25-dit-weights bind path, src/ltx25-dit-weights.cc:
// 352-403): validate, copy once into HBM, relayout scale/zero-point pairs.
bool upload_qweight(const CudaOps& ops, const uint32_t* codes,
                    const void* scales, const void* biases, int sb_dtype,
                    int N, int K, int bits, int group, bool on_device,
                    QWeight* out, std::string* err);
bool upload_dweight(const CudaOps& ops, const uint16_t* w, int N, int K,
                    bool on_device, QWeight* out, std::string* err);
void free_qweight(QWeight* w);
// LoraAdapter::load's per-module bind (src/ltx25-lora.cc:56-124): a [rank][k]
// and b [n][rank] bf16; a' = bf16(f32(a) * scale), one rounding.
bool upload_lora(const CudaOps& ops, const uint16_t* a, const uint16_t* b, int rank, int k,
                 int n, float scale, bool on_device, LoraPair* out, std::string* err);
void free_lora(LoraPair* p);

}  // namespace ltx25
