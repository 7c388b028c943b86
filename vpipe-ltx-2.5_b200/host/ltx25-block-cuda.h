// ltx25-block-cuda.h -- one BasicAVTransformerBlock on B200.
//
// The CUDA counterpart of the reference's MetalBlock (src/ltx25-block-metal.h)
// with the math of its CPU reference block_forward (src/ltx25-block-ref.cc:
// 308-389): the same order, adaLN row slices and pre-cross semantics.  Where
// the two differ it is by fusion, never by result:
//   * q/k/v of a self-attention are ONE GEMM over a fused [3*inner][dim]
//     pack, k/v of a cross-attention one GEMM over [2*inner][dim];
//   * bias, GELU and the gated residual ride in the GEMM epilogues;
//   * the a2v/v2a "pre-cross snapshot" is realised by computing all four
//     ada_zero operands before either residual update, so nothing is copied;
//   * the per-head gate is applied in the attention's output step.
// Weights come in under the reference's parameter names (load_block_weights,
// src/ltx25-block-ref.cc:424-523); the 28 block linears are w8g64 packs, the
// gate logits stay dense (the quant recipe's exclusion list,
// src/ltx25-quant-family.cc:50-71).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "ltx25-cuda-ops.h"

namespace ltx25 {

// One GEMM site's adapters (src/ltx25-lora.h:58-76): the pairs of the
// modules the GEMM computes, A stacked [r][K] and B block-diagonal [N][r]
// over the site's output rows, sharded like the base weight.  r == 0: none.
struct LoraSite {
  __nv_bfloat16* a = nullptr;
  __nv_bfloat16* b = nullptr;
  int r = 0;
};

struct CudaAttn {
  QWeight qkv;        // fused [q; k; v] (self-attention)
  QWeight q, kv;      // q and fused [k; v] (cross-attentions)
  QWeight o;
  QWeight gate;       // dense bf16 [heads][query_dim]
  __nv_bfloat16* qkv_b = nullptr;   // [3*inner] (self) or q_b [inner]
  __nv_bfloat16* kv_b = nullptr;    // [2*inner] (cross)
  __nv_bfloat16* o_b = nullptr;
  __nv_bfloat16* gate_b = nullptr;
  float* q_norm = nullptr;
  float* k_norm = nullptr;
  bool self = false;
  // heads/inner are this rank's share under tensor parallelism; head0 is
  // its first head and norm_width the full inner width the q/k RMSNorm
  // spans (== inner on one GPU).
  int heads = 0, head_dim = 0, inner = 0, qdim = 0, kvdim = 0, odim = 0;
  int head0 = 0, norm_width = 0;
  LoraSite l_qkv, l_q, l_kv, l_o, l_gate;   // adapters of the sites above
};

struct CudaStreamW {
  CudaAttn attn1, attn2;
  QWeight ff_in, ff_out;
  __nv_bfloat16* ff_in_b = nullptr;
  __nv_bfloat16* ff_out_b = nullptr;
  float* scale_shift = nullptr;         // 9 * dim
  float* prompt_scale_shift = nullptr;  // 2 * dim
  float* cross_table = nullptr;         // 5 * dim
  int dim = 0, heads = 0, ff_hidden = 0;
  LoraSite l_ff_in, l_ff_out;
};

// One stream's per-forward inputs (device pointers; see ltx_stream_io).
struct StreamIO {
  __nv_bfloat16* x = nullptr;
  const __nv_bfloat16* context = nullptr;
  const __nv_bfloat16* timesteps = nullptr;
  const __nv_bfloat16* cross_scale_shift = nullptr;
  const __nv_bfloat16* cross_gate = nullptr;
  const __nv_bfloat16* prompt_timestep = nullptr;
  const float* pe_cos = nullptr;
  const float* pe_sin = nullptr;
  const float* cpe_cos = nullptr;
  const float* cpe_sin = nullptr;
  int tokens = 0, text_tokens = 0;
  bool present = true;
  // Sequence parallel: x holds tokens [tok0, tok0 + tokens) of tokens_all,
  // which index the RoPE tables (0: this io is the whole sequence).
  int tok0 = 0, tokens_all = 0;
};

// A RoPE table view: [heads][tbl_tokens][half] f32, rows read from tok0 on.
struct RopeRef {
  const float* cos = nullptr;
  const float* sin = nullptr;
  int tbl_tokens = 0, tok0 = 0;
};

// The scratch ONE block forward needs, shared by every block of a stack
// (the reference's BlockScratch, src/ltx25-block-metal.h:140-240): the stack
// runs strictly in sequence, so 48 private arenas would only cost memory.
struct BlockArena {
  __nv_bfloat16 *normed = nullptr, *qkv = nullptr, *qn = nullptr,
                *kn = nullptr, *att = nullptr, *glog = nullptr,
                *ctxmod = nullptr, *kvp = nullptr, *ff = nullptr,
                *qv = nullptr, *kva = nullptr, *qa = nullptr, *kvv = nullptr;
  float* mods = nullptr;      // adaLN rows, f32
  __nv_bfloat16* part = nullptr;   // row-split partial sums (tensor parallel)
  float* ssq = nullptr;            // per-token q/k sums of squares (tensor parallel)
  __nv_bfloat16* sp_send = nullptr;   // all-to-all staging (sequence parallel)
  __nv_bfloat16* sp_recv = nullptr;
  __nv_bfloat16* lr = nullptr;        // an adapter site's x.A^T
  size_t cap[19] = {};        // element capacity of each buffer above
  std::shared_ptr<BlockArena> side;    // the audio stream's own buffers (side stream)
  size_t video = 0, audio = 0, text = 0;   // reserved token maxima
  ~BlockArena();
  // Grow buffer i (in the order declared) to at least n elements.
  bool ensure(int i, size_t n, std::string* err);
};

class CudaBlock {
public:
  CudaBlock(CudaOps* ops, int vdim, int vheads, int adim, int aheads)
      : _ops(ops), _vdim(vdim), _vheads(vheads), _adim(adim), _aheads(aheads)
  {
  }
  ~CudaBlock();

  // Stage one tensor under its reference name.  Quantized linears arrive as
  // w8g64 packs; every other tensor as f32 (host or device).
  bool set_qlinear(const std::string& name, const uint32_t* codes,
                   const void* scales, const void* biases, int sb_dtype, int N,
                   int K, bool on_device, std::string* err);
  bool set_tensor(const std::string& name, const float* data, int rows,
                  int cols, bool on_device, std::string* err);

  // Assemble the block: every required tensor must be present (the
  // reference refuses a partial map, src/ltx25-block-ref.cc:424-432), fuse
  // the q/k/v and k/v packs, upload the rest.  Frees the staged parts.
  // Attach one module's low-rank adapter (MetalBlock::lora_, src/
  // ltx25-block-metal.cc:404-420) under the reference's module name
  // ("attn1.to_q", "audio_ff.net.2", ...; src/ltx25-lora.cc:328-360).
  // Before finalize, which checks the pair against the base linear's widths
  // and copies it (sharded like the base weight); the pair may be freed
  // after finalize.  An unknown module name is refused.
  bool set_lora(const std::string& module, const LoraPair& pair, std::string* err);
  bool finalize(std::string* err);

  // Size the scratch arena once for the largest geometry.  `share`, when
  // given, is adopted (and grown if this block needs more): every block of
  // a stack uses the same arena.
  bool reserve(int max_video, int max_audio, int max_text, std::string* err,
               std::shared_ptr<BlockArena> share = nullptr);
  const std::shared_ptr<BlockArena>& arena() const { return _arp; }

  // Run the block; video.x / audio.x are updated in place.  Sequence
  // parallel: every rank passes the whole x and gets the whole x back.
  bool forward(cudaStream_t s, StreamIO& video, StreamIO& audio,
               std::string* err);
  // Sequence parallel, for a stack: `video` is this rank's token shard
  // (see shard_io); the caller gathers x once after the last block.
  bool forward_shard(cudaStream_t s, StreamIO& video, StreamIO& audio, std::string* err);
  bool sequence_parallel() const { return _sp; }
  // Whether a forward over `tokens` video tokens shards the video rows over
  // the group: always under sequence parallelism; under tensor parallelism
  // when the tokens split evenly over the ranks (the residual stream is then
  // kept by token rows between the row-split and column-split products --
  // reduce-scatter / all-gather instead of all-reduce -- and the per-token
  // work runs on 1/world of the rows); never on one GPU.
  bool shards_video(int tokens) const;
  // This rank's shard of a whole-sequence video io; false (with err) when
  // the tokens do not split evenly.
  bool shard_io(const StreamIO& whole, StreamIO* shard, std::string* err) const;
  // All-gather the video x shards back into the whole x on every rank.
  bool gather_video(cudaStream_t s, const StreamIO& whole, std::string* err) const;

  bool finalized() const { return _final; }
  CudaOps* ops() const { return _ops; }
  // The block's index in its stack: the sage tier leaves blocks below
  // sage_dense_layers dense (MetalBlock::forward's layer argument,
  // src/ltx25-block-metal.h:307-311).
  void set_layer(int layer) { _layer = layer; }
  int layer() const { return _layer; }
  bool same_widths(const CudaBlock& o) const
  {
    return _vdim == o._vdim && _vheads == o._vheads && _adim == o._adim &&
           _aheads == o._aheads && _video.ff_hidden == o._video.ff_hidden &&
           _audio.ff_hidden == o._audio.ff_hidden;
  }

private:
  struct Staged {
    QWeight q;          // quantized linear
    std::vector<float> host;
    float* dev_f32 = nullptr;   // caller's device pointer (on_device)
    int rows = 0, cols = 0;
    bool quant = false;
  };
  bool build_attn_(const std::string& prefix, bool self, int qdim, int kvdim,
                   int heads, int head_dim, int odim, CudaAttn& a,
                   std::string* err);
  bool build_stream_(bool audio, CudaStreamW& w, std::string* err);
  bool attend_(cudaStream_t s, const CudaAttn& a, const __nv_bfloat16* xq,
               int tq, const __nv_bfloat16* xkv, int tkv, const RopeRef& qr,
               const RopeRef& kr, __nv_bfloat16* out, std::string* err);
  // Sequence parallel: the video self-attention over the whole sequence
  // (all-to-all to heads and back) and v2a (video keys to heads, outputs
  // gathered); inputs are this rank's token rows.
  bool attend_self_sp_(cudaStream_t s, const CudaAttn& a, const __nv_bfloat16* xq, int tl,
                       const RopeRef& r, __nv_bfloat16* out, std::string* err);
  bool attend_v2a_sp_(cudaStream_t s, const CudaAttn& a, const __nv_bfloat16* xq, int tq,
                      const RopeRef& qr, const __nv_bfloat16* xkv, int tl,
                      const RopeRef& kr, __nv_bfloat16* out, std::string* err);
  bool forward_impl_(cudaStream_t s, StreamIO& video, StreamIO& audio, std::string* err);
  bool first_half_(cudaStream_t s, const CudaStreamW& w, StreamIO& io,
                   std::string* err);
  bool ff_(cudaStream_t s, const CudaStreamW& w, StreamIO& io,
           std::string* err);
  // The row-sharded feed-forward in two chunks with its collectives on the
  // communication stream, overlapped with the other chunk's GEMMs.
  bool ff_rows_chunked_(cudaStream_t s, const CudaStreamW& w, StreamIO& io, const float* mods,
                        std::string* err);
  // Upload tensor `name` (count elements in all) as f32 / bf16, keeping
  // elements [off, off + n) (n = 0: all).
  bool take_f32_(const std::string& name, size_t count, float** out,
                 std::string* err, bool required = true, size_t off = 0,
                 size_t n = 0);
  bool take_bf16_(const std::string& name, size_t count, __nv_bfloat16** out,
                  std::string* err, bool required = true, size_t off = 0,
                  size_t n = 0);
  // A block of a w8g64 pack: rows [r0, r0 + rows) and K columns
  // [k0, k0 + kcols) (kcols = 0: all of K).
  struct Part {
    const QWeight* q;
    int r0, rows, k0, kcols;
  };
  bool fuse_(const std::vector<Part>& parts, QWeight* out, std::string* err);
  // One adapter site from its modules' pairs (null: not adapted): rows
  // [r0, r0 + rows) of each pair's B in site order, A columns [k0, k0 + K).
  struct LPart {
    const LoraPair* p;
    int r0, rows, k0;
  };
  bool build_lora_(const std::vector<LPart>& parts, int K, LoraSite* out, std::string* err);
  const LoraPair* lora_of_(const std::string& module, int k, int n, std::string* err) const;
  // The extension for a site, x.A^T into the current arena's scratch.
  const LoraExt* lx_(const LoraSite& site, LoraExt* tmp) const;
  // x += gate * (att . Wo^T + bias), row-split and reduced under tensor
  // parallelism.
  // With n_all > n (row-sharded residual), `in` holds all n_all token rows
  // and x this rank's n: the partial is reduce-scattered to those rows.
  bool out_proj_(cudaStream_t s, const __nv_bfloat16* in, int k, const QWeight& w,
                 const __nv_bfloat16* bias, __nv_bfloat16* x, int n, int d,
                 const float* gate, std::string* err, const LoraSite* lora = nullptr,
                 int n_all = 0);
  // The fused reduce-scatter's availability for a row-split product over
  // n_all rows of width d on the current communicator.
  bool scatter_ok_(int n_all, int d) const;
  // All-gather this rank's n rows (in place at rank * n * d) of a
  // [world * n][d] buffer on the current stream's communicator.
  bool gather_rows_(cudaStream_t s, __nv_bfloat16* buf, int n, int d, std::string* err) const;

  CudaOps* _ops;
  int _vdim, _vheads, _adim, _aheads;
  const Comm* _comm = nullptr;   // set at finalize when the context is sharded
  const Comm* _comm_side = nullptr;   // the side stream's (tensor parallel)
  const Comm* _ccur = nullptr;        // the communicator of the stream being issued
  int _tp_rank = 0, _tp_world = 1;
  bool _tp_rows = true;          // tensor parallel: shard the residual by rows
  bool _tp_ff_chunks = false;    // ... and run the feed-forward in two chunks
  bool _tp_scatter = false;      // ... and fuse the row-split products' reduce-scatter
  bool _sp = false;              // sequence parallel (weights whole)
  int _sp_rank = 0, _sp_world = 1;
  std::map<std::string, Staged> _staged;
  std::map<std::string, LoraPair> _lora;   // attached pairs, until finalize
  int _lora_rmax = 0;                      // widest site (arena sizing)
  bool _audio_lora = false;                // an audio-stream site is adapted
  std::vector<void*> _owned;   // device buffers this block frees
  CudaStreamW _video, _audio;
  CudaAttn _a2v, _v2a;
  bool _final = false;
  int _layer = 0;

  std::shared_ptr<BlockArena> _arp;
  BlockArena* _cur = nullptr;    // the buffers the stream being issued uses
};

}  // namespace ltx25
