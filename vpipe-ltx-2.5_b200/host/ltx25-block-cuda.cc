// ltx25-block-cuda.cc -- CudaBlock (see ltx25-block-cuda.h).
#include "ltx25-block-cuda.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "../csrc/block_ops.h"
#include "../csrc/kernels.h"

namespace ltx25 {

namespace {

constexpr float kEps = 1e-6f;   // norm_eps, src/ltx25-block-ref.h:74

bool cuda_ok(cudaError_t e, const char* what, std::string* err)
{
  if (e == cudaSuccess) return true;
  if (err) *err = std::string(what) + ": " + cudaGetErrorString(e);
  return false;
}

bool fail(std::string* err, const std::string& m)
{
  if (err) *err = m;
  return false;
}

// Offsets (in units of the stream width) of the f32 adaLN rows in a stream's
// region of the modulation scratch.
enum ModRow : int {
  MOD_MSA = 0,      // self-attn shift, scale, gate   (table rows 0..2)
  MOD_CA = 3,       // text cross shift, scale, gate   (rows 6..8)
  MOD_PROMPT = 6,   // K/V shift, scale                 (prompt table)
  MOD_MLP = 8,      // ff shift, scale, gate            (rows 3..5)
  MOD_AV = 11,      // a2v/v2a scale, shift, scale, shift (cross rows 0..3)
  MOD_AVG = 15,     // a2v/v2a gate                      (cross row 4)
  MOD_ROWS = 16
};

}  // namespace

CudaBlock::~CudaBlock()
{
  for (auto& kv : _staged)
    if (kv.second.quant) free_qweight(&kv.second.q);
  for (CudaAttn* a : {&_video.attn1, &_video.attn2, &_audio.attn1,
                      &_audio.attn2, &_a2v, &_v2a}) {
    free_qweight(&a->qkv);
    free_qweight(&a->q);
    free_qweight(&a->kv);
    free_qweight(&a->o);
    free_qweight(&a->gate);
  }
  for (CudaStreamW* w : {&_video, &_audio}) {
    free_qweight(&w->ff_in);
    free_qweight(&w->ff_out);
  }
  for (void* p : _owned) cudaFree(p);
}

bool CudaBlock::set_qlinear(const std::string& name, const uint32_t* codes,
                            const void* scales, const void* biases,
                            int sb_dtype, int N, int K, bool on_device,
                            std::string* err)
{
  if (_final) return fail(err, "block already finalized");
  Staged st;
  st.quant = true;
  if (!upload_qweight(*_ops, codes, scales, biases, sb_dtype, N, K, 8, 64,
                      on_device, &st.q, err))
    return false;
  st.rows = N;
  st.cols = K;
  auto it = _staged.find(name);
  if (it != _staged.end() && it->second.quant) free_qweight(&it->second.q);
  _staged[name] = std::move(st);
  return true;
}

bool CudaBlock::set_tensor(const std::string& name, const float* data,
                           int rows, int cols, bool on_device,
                           std::string* err)
{
  if (_final) return fail(err, "block already finalized");
  if (data == nullptr || rows <= 0) return fail(err, "set_tensor: null or empty " + name);
  Staged st;
  st.rows = rows;
  st.cols = cols > 0 ? cols : 1;
  const size_t n = (size_t)st.rows * st.cols;
  if (on_device) {
    st.dev_f32 = const_cast<float*>(data);
  } else {
    st.host.assign(data, data + n);
  }
  auto it = _staged.find(name);
  if (it != _staged.end() && it->second.quant) free_qweight(&it->second.q);
  _staged[name] = std::move(st);
  return true;
}

bool CudaBlock::take_f32_(const std::string& name, size_t count, float** out,
                          std::string* err, bool required, size_t off, size_t n)
{
  *out = nullptr;
  auto it = _staged.find(name);
  if (it == _staged.end() || it->second.quant) {
    if (!required) return true;
    return fail(err, "missing tensor '" + name + "'");
  }
  const Staged& st = it->second;
  if ((size_t)st.rows * st.cols != count)
    return fail(err, "tensor '" + name + "' has " +
                         std::to_string((size_t)st.rows * st.cols) +
                         " elements, want " + std::to_string(count));
  if (n == 0) n = count - off;
  if (off + n > count) return fail(err, "tensor '" + name + "': slice outside the tensor");
  float* d = nullptr;
  if (!cuda_ok(cudaMalloc(&d, n * sizeof(float)), "cudaMalloc", err)) return false;
  _owned.push_back(d);
  const cudaError_t e =
      st.dev_f32 ? cudaMemcpy(d, st.dev_f32 + off, n * 4, cudaMemcpyDeviceToDevice)
                 : cudaMemcpy(d, st.host.data() + off, n * 4, cudaMemcpyHostToDevice);
  if (!cuda_ok(e, "upload", err)) return false;
  *out = d;
  return true;
}

bool CudaBlock::take_bf16_(const std::string& name, size_t count,
                           __nv_bfloat16** out, std::string* err,
                           bool required, size_t off, size_t n)
{
  *out = nullptr;
  float* f = nullptr;
  if (!take_f32_(name, count, &f, err, required, off, n)) return false;
  if (f == nullptr) return true;
  if (n == 0) n = count - off;
  __nv_bfloat16* d = nullptr;
  if (!cuda_ok(cudaMalloc(&d, n * 2), "cudaMalloc", err)) return false;
  _owned.push_back(d);
  if (ltx::launch_f32_to_bf16(f, d, n, nullptr) != 0 ||
      !cuda_ok(cudaDeviceSynchronize(), "convert", err))
    return fail(err, "f32 -> bf16 conversion failed for " + name);
  *out = d;
  return true;
}

// Concatenate blocks of quantized linears along N (rows of the weight):
// codes row blocks back to back, scale/zero-point pairs side by side per K
// group.  Each part may also keep only a K range (a row-split shard): its
// codes columns and the matching scale groups.
bool CudaBlock::fuse_(const std::vector<Part>& parts, QWeight* out,
                      std::string* err)
{
  const int K = parts[0].kcols > 0 ? parts[0].kcols : parts[0].q->K;
  int N = 0;
  for (const Part& pt : parts) {
    const int kc = pt.kcols > 0 ? pt.kcols : pt.q->K;
    if (!pt.q->quantized || kc != K || pt.k0 % 64 != 0 || kc % 64 != 0 ||
        pt.k0 + kc > pt.q->K || pt.r0 < 0 || pt.r0 + pt.rows > pt.q->N)
      return fail(err, "fuse: mismatched parts");
    N += pt.rows;
  }
  QWeight f;
  f.N = N;
  f.K = K;
  f.bits = 8;
  f.group = 64;
  f.quantized = true;
  f.device = _ops->device();
  const int G = K / 64;
  if (!cuda_ok(cudaMalloc(&f.codes, (size_t)N * K), "cudaMalloc(fused codes)", err) ||
      !cuda_ok(cudaMalloc(&f.sz, (size_t)N * G * 4), "cudaMalloc(fused sz)", err)) {
    free_qweight(&f);
    return false;
  }
  int n0 = 0;
  for (const Part& pt : parts) {
    const QWeight* q = pt.q;
    const uint8_t* src_codes = q->codes + (size_t)pt.r0 * q->K + pt.k0;
    const uint32_t* src_sz = q->sz + (size_t)(pt.k0 / 64) * q->N + pt.r0;
    if (!cuda_ok(cudaMemcpy2D(f.codes + (size_t)n0 * K, K, src_codes, q->K, K,
                              pt.rows, cudaMemcpyDeviceToDevice), "fuse codes", err) ||
        !cuda_ok(cudaMemcpy2D(f.sz + n0, (size_t)N * 4, src_sz, (size_t)q->N * 4,
                              (size_t)pt.rows * 4, G, cudaMemcpyDeviceToDevice),
                 "fuse sz", err)) {
      free_qweight(&f);
      return false;
    }
    n0 += pt.rows;
  }
  *out = f;
  return true;
}

namespace {

// The modules an adapter may name, as the reference's loader binds them
// (src/ltx25-lora.cc:328-360).
bool known_module(const std::string& m)
{
  for (const char* a : {"attn1", "attn2", "audio_attn1", "audio_attn2",
                        "audio_to_video_attn", "video_to_audio_attn"})
    for (const char* s : {".to_q", ".to_k", ".to_v", ".to_out.0", ".to_gate_logits"})
      if (m == std::string(a) + s) return true;
  for (const char* f : {"ff.net.0.proj", "ff.net.2", "audio_ff.net.0.proj", "audio_ff.net.2"})
    if (m == f) return true;
  return false;
}

}  // namespace

bool CudaBlock::set_lora(const std::string& module, const LoraPair& pair, std::string* err)
{
  if (_final) return fail(err, "block already finalized (attach adapters before finalize)");
  if (!known_module(module))
    return fail(err, "adapter names '" + module + "', which this block does not apply "
                     "(not run by this build)");
  if (pair.a == nullptr || pair.b == nullptr || pair.rank <= 0)
    return fail(err, "adapter '" + module + "': null pair");
  _lora[module] = pair;
  return true;
}

const LoraPair* CudaBlock::lora_of_(const std::string& module, int k, int n,
                                    std::string* err) const
{
  auto it = _lora.find(module);
  if (it == _lora.end()) return nullptr;
  const LoraPair& p = it->second;
  if (p.k != k || p.n != n) {
    if (err && err->empty())
      *err = "adapter '" + module + "' is [" + std::to_string(p.n) + "][" +
             std::to_string(p.rank) + "] x [" + std::to_string(p.rank) + "][" +
             std::to_string(p.k) + "], the base linear reads " + std::to_string(k) +
             " and writes " + std::to_string(n) + " (shape)";
    return nullptr;
  }
  return &p;
}

bool CudaBlock::build_lora_(const std::vector<LPart>& parts, int K, LoraSite* out,
                            std::string* err)
{
  int r = 0, N = 0;
  for (const LPart& pt : parts) {
    if (pt.p != nullptr) r += pt.p->r8;
    N += pt.rows;
  }
  *out = LoraSite{};
  if (r == 0) return true;
  __nv_bfloat16 *a = nullptr, *b = nullptr;
  if (!cuda_ok(cudaMalloc(&a, (size_t)r * K * 2), "cudaMalloc(adapter a)", err)) return false;
  _owned.push_back(a);
  if (!cuda_ok(cudaMalloc(&b, (size_t)N * r * 2), "cudaMalloc(adapter b)", err)) return false;
  _owned.push_back(b);
  if (!cuda_ok(cudaMemset(b, 0, (size_t)N * r * 2), "adapter b", err)) return false;
  int ro = 0, n0 = 0;
  for (const LPart& pt : parts) {
    if (pt.p != nullptr) {
      const LoraPair& p = *pt.p;
      if (pt.k0 + K > p.k || pt.r0 + pt.rows > p.n)
        return fail(err, "adapter shard out of range");
      if (!cuda_ok(cudaMemcpy2D(a + (size_t)ro * K, (size_t)K * 2, p.a + pt.k0, (size_t)p.k * 2,
                                (size_t)K * 2, p.r8, cudaMemcpyDeviceToDevice),
                   "adapter a", err) ||
          !cuda_ok(cudaMemcpy2D(b + (size_t)n0 * r + ro, (size_t)r * 2,
                                p.b + (size_t)pt.r0 * p.r8, (size_t)p.r8 * 2, (size_t)p.r8 * 2,
                                pt.rows, cudaMemcpyDeviceToDevice),
                   "adapter b", err))
        return false;
      ro += p.r8;
    }
    n0 += pt.rows;
  }
  out->a = a;
  out->b = b;
  out->r = r;
  _lora_rmax = std::max(_lora_rmax, r);
  return true;
}

const LoraExt* CudaBlock::lx_(const LoraSite& site, LoraExt* tmp) const
{
  if (site.r == 0) return nullptr;
  tmp->a = site.a;
  tmp->b = site.b;
  tmp->r = site.r;
  tmp->rbuf = _cur->lr;
  return tmp;
}

bool CudaBlock::build_attn_(const std::string& p, bool self, int qdim,
                            int kvdim, int heads, int head_dim, int odim,
                            CudaAttn& a, std::string* err)
{
  const int inner = heads * head_dim;
  // Tensor parallelism (Megatron): q/k/v and the gate logits are split by
  // heads (column split), the output projection by its K columns (row
  // split); the out bias is added once, after the partial sums are reduced.
  const int W = _tp_world, R = _tp_rank;
  if (heads % W != 0)
    return fail(err, p + ": " + std::to_string(heads) + " heads do not split over " +
                         std::to_string(W) + " ranks (shape)");
  const int hl = heads / W, il = hl * head_dim, c0 = R * il;
  if (W > 1 && il % 64 != 0)
    return fail(err, p + ": per-rank width " + std::to_string(il) +
                         " is not a multiple of 64 (shape)");
  a.self = self;
  a.heads = hl;
  a.head_dim = head_dim;
  a.inner = il;
  a.qdim = qdim;
  a.kvdim = kvdim;
  a.odim = odim;
  a.head0 = R * hl;
  a.norm_width = inner;
  auto qlin = [&](const std::string& n, int N, int K) -> const QWeight* {
    auto it = _staged.find(p + n);
    if (it == _staged.end() || !it->second.quant) {
      fail(err, "missing quantized tensor '" + p + n + "'");
      return nullptr;
    }
    if (it->second.q.N != N || it->second.q.K != K) {
      fail(err, "tensor '" + p + n + "' is [" + std::to_string(it->second.q.N) +
                    "][" + std::to_string(it->second.q.K) + "], want [" +
                    std::to_string(N) + "][" + std::to_string(K) + "]");
      return nullptr;
    }
    return &it->second.q;
  };
  const QWeight* wq = qlin(".to_q.weight", inner, qdim);
  if (!wq) return false;
  const QWeight* wk = qlin(".to_k.weight", inner, kvdim);
  if (!wk) return false;
  const QWeight* wv = qlin(".to_v.weight", inner, kvdim);
  if (!wv) return false;
  const QWeight* wo = qlin(".to_out.0.weight", odim, inner);
  if (!wo) return false;

  // Biases: this rank's q/k/v columns, concatenated to match the fused
  // GEMM's output columns.
  std::vector<float> bcat;
  for (const char* bn : {".to_q.bias", ".to_k.bias", ".to_v.bias"}) {
    auto it = _staged.find(p + bn);
    if (it == _staged.end() || it->second.quant || (size_t)it->second.rows * it->second.cols != (size_t)inner)
      return fail(err, "missing tensor '" + p + bn + "'");
    std::vector<float> h(inner);
    if (it->second.dev_f32) {
      if (!cuda_ok(cudaMemcpy(h.data(), it->second.dev_f32, inner * 4, cudaMemcpyDeviceToHost), "bias", err))
        return false;
    } else {
      h = it->second.host;
    }
    bcat.insert(bcat.end(), h.begin() + c0, h.begin() + c0 + il);
  }
  const std::string tmpq = p + ".__qkv_bias", tmpkv = p + ".__kv_bias";
  if (self) {
    if (!fuse_({{wq, c0, il, 0, 0}, {wk, c0, il, 0, 0}, {wv, c0, il, 0, 0}}, &a.qkv, err))
      return false;
    if (!set_tensor(tmpq, bcat.data(), 3 * il, 0, false, err) ||
        !take_bf16_(tmpq, (size_t)3 * il, &a.qkv_b, err))
      return false;
  } else {
    if (!fuse_({{wq, c0, il, 0, 0}}, &a.q, err) ||
        !fuse_({{wk, c0, il, 0, 0}, {wv, c0, il, 0, 0}}, &a.kv, err))
      return false;
    if (!set_tensor(tmpq, bcat.data(), il, 0, false, err) ||
        !take_bf16_(tmpq, (size_t)il, &a.qkv_b, err))
      return false;
    if (!set_tensor(tmpkv, bcat.data() + il, 2 * il, 0, false, err) ||
        !take_bf16_(tmpkv, (size_t)2 * il, &a.kv_b, err))
      return false;
  }
  _staged.erase(tmpq);
  _staged.erase(tmpkv);
  if (!fuse_({{wo, 0, odim, W > 1 ? c0 : 0, W > 1 ? il : 0}}, &a.o, err)) return false;
  if (!take_bf16_(p + ".to_out.0.bias", odim, &a.o_b, err) ||
      !take_f32_(p + ".q_norm.weight", inner, &a.q_norm, err, true, c0, il) ||
      !take_f32_(p + ".k_norm.weight", inner, &a.k_norm, err, true, c0, il))
    return false;
  // Gate logits: dense (excluded from quantization), [heads][qdim]; this
  // rank's rows.
  float* gw = nullptr;
  if (!take_f32_(p + ".to_gate_logits.weight", (size_t)heads * qdim, &gw, err, false,
                 (size_t)R * hl * qdim, (size_t)hl * qdim))
    return false;
  if (gw != nullptr) {
    __nv_bfloat16* gwb = nullptr;
    if (!cuda_ok(cudaMalloc(&gwb, (size_t)hl * qdim * 2), "cudaMalloc", err)) return false;
    if (ltx::launch_f32_to_bf16(gw, gwb, (size_t)hl * qdim, nullptr) != 0 ||
        !cuda_ok(cudaDeviceSynchronize(), "convert", err))
      return false;
    const bool ok = upload_dweight(*_ops, reinterpret_cast<const uint16_t*>(gwb),
                                   hl, qdim, true, &a.gate, err);
    cudaFree(gwb);
    if (!ok) return false;
    if (!take_bf16_(p + ".to_gate_logits.bias", heads, &a.gate_b, err, false,
                    (size_t)R * hl, (size_t)hl))
      return false;
  }
  // Adapters, sharded like the weights they ride on: q/k/v and gate rows
  // of this rank's heads; the output projection's A keeps this rank's K
  // columns (its partial products are summed with the base's).
  std::string lerr;
  const LoraPair* lq = lora_of_(p + ".to_q", qdim, inner, &lerr);
  const LoraPair* lk = lora_of_(p + ".to_k", kvdim, inner, &lerr);
  const LoraPair* lv = lora_of_(p + ".to_v", kvdim, inner, &lerr);
  const LoraPair* lo = lora_of_(p + ".to_out.0", inner, odim, &lerr);
  const LoraPair* lg = lora_of_(p + ".to_gate_logits", qdim, heads, &lerr);
  if (!lerr.empty()) return fail(err, lerr);
  if (lg != nullptr && a.gate.N == 0)
    return fail(err, p + ".to_gate_logits: adapter on a block without gate logits");
  if (self) {
    if (!build_lora_({{lq, c0, il, 0}, {lk, c0, il, 0}, {lv, c0, il, 0}}, qdim, &a.l_qkv, err))
      return false;
  } else {
    if (!build_lora_({{lq, c0, il, 0}}, qdim, &a.l_q, err) ||
        !build_lora_({{lk, c0, il, 0}, {lv, c0, il, 0}}, kvdim, &a.l_kv, err))
      return false;
  }
  return build_lora_({{lo, 0, odim, W > 1 ? c0 : 0}}, W > 1 ? il : inner, &a.l_o, err) &&
         build_lora_({{lg, R * hl, hl, 0}}, qdim, &a.l_gate, err);
}

bool CudaBlock::build_stream_(bool audio, CudaStreamW& w, std::string* err)
{
  const std::string pre = audio ? "audio_" : "";
  const int d = audio ? _adim : _vdim;
  const int h = audio ? _aheads : _vheads;
  w.dim = d;
  w.heads = h;
  if (d % h != 0) return fail(err, "stream width is not a multiple of the heads");
  if (!build_attn_(pre + "attn1", true, d, d, h, d / h, d, w.attn1, err) ||
      !build_attn_(pre + "attn2", false, d, d, h, d / h, d, w.attn2, err))
    return false;
  auto fi = _staged.find(pre + "ff.net.0.proj.weight");
  auto fo = _staged.find(pre + "ff.net.2.weight");
  if (fi == _staged.end() || !fi->second.quant)
    return fail(err, "missing quantized tensor '" + pre + "ff.net.0.proj.weight'");
  if (fo == _staged.end() || !fo->second.quant)
    return fail(err, "missing quantized tensor '" + pre + "ff.net.2.weight'");
  const int hidden = fi->second.q.N;
  if (fi->second.q.K != d || fo->second.q.N != d || fo->second.q.K != hidden)
    return fail(err, "feed-forward shapes disagree with the stream width");
  // Column-split ff.net.0 (GELU is per column), row-split ff.net.2.
  const int W = _tp_world, R = _tp_rank;
  if (hidden % (64 * W) != 0)
    return fail(err, pre + "ff: hidden width " + std::to_string(hidden) +
                         " does not split over " + std::to_string(W) + " ranks (shape)");
  const int fl = hidden / W, f0 = R * fl;
  w.ff_hidden = fl;
  if (!fuse_({{&fi->second.q, f0, fl, 0, 0}}, &w.ff_in, err) ||
      !fuse_({{&fo->second.q, 0, d, W > 1 ? f0 : 0, W > 1 ? fl : 0}}, &w.ff_out, err))
    return false;
  std::string lerr;
  const LoraPair* lfi = lora_of_(pre + "ff.net.0.proj", d, hidden, &lerr);
  const LoraPair* lfo = lora_of_(pre + "ff.net.2", hidden, d, &lerr);
  if (!lerr.empty()) return fail(err, lerr);
  if (!build_lora_({{lfi, f0, fl, 0}}, d, &w.l_ff_in, err) ||
      !build_lora_({{lfo, 0, d, W > 1 ? f0 : 0}}, W > 1 ? fl : hidden, &w.l_ff_out, err))
    return false;
  // Video ff has no bias, audio ff does (src/ltx25-dit-weights.cc:482-486).
  if (!take_bf16_(pre + "ff.net.0.proj.bias", hidden, &w.ff_in_b, err, false, f0, fl) ||
      !take_bf16_(pre + "ff.net.2.bias", d, &w.ff_out_b, err, false))
    return false;
  if (!take_f32_(pre + "scale_shift_table", (size_t)9 * d, &w.scale_shift, err) ||
      !take_f32_(pre + "prompt_scale_shift_table", (size_t)2 * d,
                 &w.prompt_scale_shift, err) ||
      !take_f32_(audio ? "scale_shift_table_a2v_ca_audio"
                       : "scale_shift_table_a2v_ca_video",
                 (size_t)5 * d, &w.cross_table, err))
    return false;
  return true;
}

bool CudaBlock::finalize(std::string* err)
{
  if (_final) return true;
  _comm = _ops->comm();
  _comm_side = _ops->side_comm();
  _ccur = _comm;
  _sp = _ops->sequence_parallel();
  _sp_world = _sp ? _comm->world() : 1;
  _sp_rank = _sp ? _comm->rank() : 0;
  // Tensor parallel shards the weights; sequence parallel keeps them whole.
  _tp_world = (_comm && !_sp) ? _comm->world() : 1;
  _tp_rank = (_comm && !_sp) ? _comm->rank() : 0;
  // A/B switches for the tensor-parallel residual layout (LTX25_TP_ROWS=0:
  // whole x on every rank, all-reduced products) and for the feed-forward's
  // two overlapped chunks (LTX25_TP_FF_CHUNKS=0 / 1), read once per block.
  // The chunks pay ~0.06-0.2 ms of smaller GEMMs and extra launches a block
  // (measured with the collectives stubbed out) to hide half of the
  // feed-forward's gather and reduce-scatter, which grow toward 2 x 67 MB a
  // block as the group does: on from 8 ranks by default.
  _tp_ff_chunks = _tp_world >= 8;
  if (const char* e = std::getenv("LTX25_TP_ROWS")) _tp_rows = e[0] != '0';
  if (const char* e = std::getenv("LTX25_TP_FF_CHUNKS")) _tp_ff_chunks = e[0] != '0';
  // The fused reduce-scatter of the row-split products (peer stores from
  // the GEMM's epilogue, up to 8 ranks; on by default, LTX25_TP_SCATTER=0
  // restores the NCCL reduce-scatter).  Measured on 2 GPUs: 178.1 ms a
  // 48-block step against 184.4-188.3 with the NCCL reduce-scatter.
  _tp_scatter = true;
  if (const char* e = std::getenv("LTX25_TP_SCATTER")) _tp_scatter = e[0] != '0';
  _tp_scatter = _tp_scatter && _tp_world > 1 && _tp_world <= 8 && _tp_rows && !_sp;
  if (_sp && (_vheads % _sp_world != 0 || _aheads % _sp_world != 0))
    return fail(err, "sequence parallel shape: heads do not split over the ranks");
  if (!build_stream_(false, _video, err) || !build_stream_(true, _audio, err))
    return false;
  // Both cross-attentions run at the AUDIO head count and head width
  // (src/ltx25-block-ref.cc:510-519).
  const int ahd = _adim / _aheads;
  if (!build_attn_("audio_to_video_attn", false, _vdim, _adim, _aheads, ahd,
                   _vdim, _a2v, err) ||
      !build_attn_("video_to_audio_attn", false, _adim, _vdim, _aheads, ahd,
                   _adim, _v2a, err))
    return false;
  for (auto& kv : _staged)
    if (kv.second.quant) free_qweight(&kv.second.q);
  _staged.clear();
  _lora.clear();   // copied into the sites; the caller's pairs are free now
  _audio_lora = false;
  for (const CudaAttn* at : {&_audio.attn1, &_audio.attn2})
    for (const LoraSite* ls : {&at->l_qkv, &at->l_q, &at->l_kv, &at->l_o, &at->l_gate})
      _audio_lora = _audio_lora || ls->r > 0;
  _audio_lora = _audio_lora || _audio.l_ff_in.r > 0 || _audio.l_ff_out.r > 0;
  _final = true;
  return true;
}

BlockArena::~BlockArena()
{
  for (void* p : {(void*)normed, (void*)qkv, (void*)qn, (void*)kn, (void*)att,
                  (void*)glog, (void*)ctxmod, (void*)kvp, (void*)ff, (void*)qv,
                  (void*)kva, (void*)qa, (void*)kvv, (void*)mods, (void*)part,
                  (void*)ssq, (void*)sp_send, (void*)sp_recv, (void*)lr})
    cudaFree(p);
}

bool BlockArena::ensure(int i, size_t n, std::string* err)
{
  void** slots[19] = {(void**)&normed, (void**)&qkv, (void**)&qn, (void**)&kn,
                      (void**)&att, (void**)&glog, (void**)&ctxmod, (void**)&kvp,
                      (void**)&ff, (void**)&qv, (void**)&kva, (void**)&qa,
                      (void**)&kvv, (void**)&mods, (void**)&part, (void**)&ssq,
                      (void**)&sp_send, (void**)&sp_recv, (void**)&lr};
  if (n <= cap[i]) return true;
  const size_t elt = (i == 13 || i == 15) ? sizeof(float) : sizeof(__nv_bfloat16);
  cudaFree(*slots[i]);
  *slots[i] = nullptr;
  cap[i] = 0;
  if (!cuda_ok(cudaMalloc(slots[i], (n + 64) * elt), "cudaMalloc(block arena)", err))
    return false;
  cap[i] = n;
  return true;
}

bool CudaBlock::reserve(int max_video, int max_audio, int max_text,
                        std::string* err, std::shared_ptr<BlockArena> share)
{
  if (!_final) return fail(err, "reserve before finalize");
  const size_t vt = std::max(max_video, 0), at = std::max(max_audio, 0),
               tt = std::max(max_text, 0);
  const size_t vd = _vdim, ad = _adim;
  const size_t ai = ad;   // audio inner (the cross attentions' width too)
  auto mx = [](std::initializer_list<size_t> l) { return std::max(l); };
  const size_t need[19] = {
      mx({vt * vd, at * ad}),                                        // normed
      mx({vt * 3 * vd, at * 3 * ad, vt * vd, vt * ai, at * ai}),     // qkv / q
      mx({vt * vd, at * ad, vt * ai}),                               // qn
      mx({vt * vd, at * ad, tt * vd, tt * ad, vt * ai, at * ai}),    // kn
      mx({vt * vd, at * ad, vt * ai}),                               // att
      mx({vt, at}) * (size_t)std::max(_vheads, _aheads),             // glog
      tt * std::max(vd, ad),                                         // ctxmod
      mx({tt * 2 * vd, tt * 2 * ad, at * 2 * ai, vt * 2 * ai}),      // kv proj
      mx({vt * (size_t)_video.ff_hidden, at * (size_t)_audio.ff_hidden}),  // ff
      vt * vd, at * ad, at * ad, vt * vd,                            // qv kva qa kvv
      (size_t)MOD_ROWS * (vd + ad),                                  // mods
      _tp_world > 1 ? mx({vt * vd, at * ad}) : 0,                    // part
      _tp_world > 1 ? 2 * (vt + at + tt) : 0,                        // ssq
      // sequence parallel: q, k, v of one head group for the whole sequence
      // (the video self-attention), or the v2a keys/values / outputs
      _sp ? 3 * vt * vd / _sp_world + at * ai : 0,                   // sp_send
      _sp ? 3 * vt * vd / _sp_world + at * ai : 0,                   // sp_recv
      mx({vt, at, tt}) * (size_t)_lora_rmax};                        // lr
  _arp = share ? share : std::make_shared<BlockArena>();
  for (int i = 0; i < 19; ++i)
    if (!_arp->ensure(i, need[i], err)) return false;
  // The audio stream's own buffers, so that it can run beside the video
  // stream on a second CUDA stream (shared by the blocks like the rest).
  {
    const size_t na[19] = {
        at * ad, mx({at * 3 * ad, at * ai}), at * ad, mx({at * ad, tt * ad, at * ai}),
        at * ad, at * (size_t)_aheads, tt * ad, mx({tt * 2 * ad, at * 2 * ai}),
        at * (size_t)_audio.ff_hidden, 0, 0, 0, 0, 0,
        _tp_world > 1 ? at * ad : 0, _tp_world > 1 ? 2 * (at + tt) : 0, 0, 0,
        mx({at, tt}) * (size_t)_lora_rmax};
    if (!_arp->side) _arp->side = std::make_shared<BlockArena>();
    for (int i = 0; i < 19; ++i)
      if (!_arp->side->ensure(i, na[i], err)) return false;
  }
  // the fused reduce-scatter's receive slots: world x (rows / world) x width,
  // the video partial's size, on every rank (collective)
  if (_tp_scatter && !_ops->share_peer_buffers(vt * vd * 2, err)) return false;
  _arp->video = std::max(_arp->video, vt);
  _arp->audio = std::max(_arp->audio, at);
  _arp->text = std::max(_arp->text, tt);
  // The attention's V^T scratch for the widest head_dim-128 stream, and the
  // sage tier's when it is on.
  if (!_ops->reserve_attention((int)mx({vt, at, tt}),
                               std::max(_video.attn1.inner, _audio.attn1.inner), err))
    return false;
  // The audio stream's attentions on the side stream have their own V^T.
  if (!_ops->reserve_attention_side((int)mx({at, tt}), _audio.attn1.inner, err)) return false;
  // v2a (audio queries over every video key) splits over the keys.
  if (!_ops->reserve_split((int)at, (int)vt, _v2a.heads, _v2a.head_dim, err)) return false;
  if (_ops->sage_on() &&
      !_ops->reserve_sage((int)mx({vt, at}), (int)mx({vt, at, tt}),
                          std::max(_video.attn1.heads, _audio.attn1.heads), 128, err))
    return false;
  // The GEMMs' own scratch (int8 tier) follows the largest projection.
  return _ops->reserve((int)mx({vt, at, tt}), (int)mx({3 * vd, (size_t)_video.ff_hidden}),
                       (int)mx({vd, (size_t)_video.ff_hidden}), err);
}

bool CudaBlock::attend_(cudaStream_t s, const CudaAttn& a,
                        const __nv_bfloat16* xq, int tq,
                        const __nv_bfloat16* xkv, int tkv, const RopeRef& qr,
                        const RopeRef& kr, __nv_bfloat16* out, std::string* err)
{
  const int I = a.inner;
  const __nv_bfloat16 *qraw, *kraw, *vraw;
  int ldq, ldkv;
  LoraExt lx;
  // Long key sequences (the video keys: 8160) whose attention reads V^T (the
  // tcgen05 path) take V^T straight from the K/V projection's epilogue, which
  // writes those columns transposed into the attention's scratch instead of
  // next to K; the V^T copy kernel then does not run.  Shorter K/V
  // projections (the text's 256 tokens) run K-split GEMMs, which that
  // output form excludes.
  VtOut vo;
  const VtOut* vop = nullptr;
  if (tkv >= 1024 && _ops->attention_reads_vt(s, tq, tkv, a.heads, a.head_dim, _layer) &&
      !_ops->i8_takes(a.self ? tq : tkv, a.self ? a.qdim : a.kvdim, a.self ? 3 * I : 2 * I)) {
    vo.vt = _ops->vt_scratch(tkv, I, err);
    if (vo.vt == nullptr) return false;
    vo.col0 = a.self ? 2 * I : I;
    vo.ld = (tkv + 7) / 8 * 8;
    vop = &vo;
  }
  if (a.self) {
    if (!_ops->linear(s, xq, a.qdim, a.qkv, a.qkv_b, _cur->qkv, 3 * I, tq, a.qdim,
                      3 * I, ltx::EPI_STORE, nullptr, err, lx_(a.l_qkv, &lx), nullptr, vop))
      return false;
    qraw = _cur->qkv;
    kraw = _cur->qkv + I;
    vraw = _cur->qkv + 2 * I;
    ldq = ldkv = 3 * I;
  } else {
    if (!_ops->linear(s, xq, a.qdim, a.q, a.qkv_b, _cur->qkv, I, tq, a.qdim, I,
                      ltx::EPI_STORE, nullptr, err, lx_(a.l_q, &lx)) ||
        !_ops->linear(s, xkv, a.kvdim, a.kv, a.kv_b, _cur->kvp, 2 * I, tkv,
                      a.kvdim, 2 * I, ltx::EPI_STORE, nullptr, err, lx_(a.l_kv, &lx), nullptr,
                      vop))
      return false;
    qraw = _cur->qkv;
    kraw = _cur->kvp;
    vraw = _cur->kvp + I;
    ldq = I;
    ldkv = 2 * I;
  }
  // RMSNorm spans the whole inner width: a rank that holds only some heads
  // reduces the per-token sums of squares (q rows then k rows) first.
  const float *qss = nullptr, *kss = nullptr;
  if (a.norm_width != I) {
    if (ltx::launch_row_sumsq(qraw, ldq, tq, I, _cur->ssq, s) != 0 ||
        ltx::launch_row_sumsq(kraw, ldkv, tkv, I, _cur->ssq + tq, s) != 0)
      return fail(err, "q/k sum-of-squares launch failed");
    if (!_ccur->allreduce_sum(_cur->ssq, (size_t)tq + tkv, 0, s, err)) return false;
    qss = _cur->ssq;
    kss = _cur->ssq + tq;
  }
  if (ltx::launch_qk_norm_rope(qraw, ldq, _cur->qn, I, tq, a.heads, a.head_dim,
                               a.q_norm, qr.cos, qr.sin, kEps, s, qss, a.norm_width,
                               a.head0, qr.tbl_tokens, qr.tok0) != 0 ||
      ltx::launch_qk_norm_rope(kraw, ldkv, _cur->kn, I, tkv, a.heads,
                               a.head_dim, a.k_norm, kr.cos, kr.sin, kEps, s, kss,
                               a.norm_width, a.head0, kr.tbl_tokens, kr.tok0) != 0)
    return fail(err, "q/k norm + rope launch failed");
  const __nv_bfloat16* glog = nullptr;
  if (a.gate.N > 0) {
    if (!_ops->linear(s, xq, a.qdim, a.gate, a.gate_b, _cur->glog, a.heads, tq,
                      a.qdim, a.heads, ltx::EPI_STORE, nullptr, err, lx_(a.l_gate, &lx)))
      return false;
    glog = _cur->glog;
  }
  if (!_ops->attention(s, _cur->qn, I, _cur->kn, I, vraw, ldkv, out, I, glog, a.heads, tq,
                       tkv, a.heads, a.head_dim, err, _layer, vop != nullptr ? vo.vt : nullptr))
    return false;
  return true;
}

bool CudaBlock::attend_self_sp_(cudaStream_t s, const CudaAttn& a, const __nv_bfloat16* xq,
                                int tl, const RopeRef& r, __nv_bfloat16* out,
                                std::string* err)
{
  // Tokens are sharded, weights whole: q, k, v of this rank's tl tokens for
  // ALL heads, then an all-to-all to the whole sequence for this rank's
  // heads, attention, and an all-to-all back (DeepSpeed-Ulysses layout).
  const int I = a.inner, N = _sp_world, Il = I / N, tv = tl * N, hl = a.heads / N;
  LoraExt lx;
  if (!_ops->linear(s, xq, a.qdim, a.qkv, a.qkv_b, _cur->qkv, 3 * I, tl, a.qdim, 3 * I,
                    ltx::EPI_STORE, nullptr, err, lx_(a.l_qkv, &lx)))
    return false;
  if (ltx::launch_qk_norm_rope(_cur->qkv, 3 * I, _cur->qn, I, tl, a.heads, a.head_dim,
                               a.q_norm, r.cos, r.sin, kEps, s, nullptr, 0, 0, r.tbl_tokens,
                               r.tok0) != 0 ||
      ltx::launch_qk_norm_rope(_cur->qkv + I, 3 * I, _cur->kn, I, tl, a.heads, a.head_dim,
                               a.k_norm, r.cos, r.sin, kEps, s, nullptr, 0, 0, r.tbl_tokens,
                               r.tok0) != 0)
    return fail(err, "q/k norm + rope launch failed");
  const size_t blk = (size_t)tv * Il;   // one of q, k, v for this rank's heads
  if (ltx::launch_a2a_pack(_cur->qn, I, tl, N, Il, _cur->sp_send, s) != 0 ||
      ltx::launch_a2a_pack(_cur->kn, I, tl, N, Il, _cur->sp_send + blk, s) != 0 ||
      ltx::launch_a2a_pack(_cur->qkv + 2 * I, 3 * I, tl, N, Il, _cur->sp_send + 2 * blk, s) != 0)
    return fail(err, "all-to-all pack launch failed");
  if (!_comm->alltoall_bf16(_cur->sp_send, _cur->sp_recv, (size_t)tl * Il, 3, blk, s, err))
    return false;
  // gate logits of this rank's tokens, all heads (applied on the way back)
  if (!_ops->linear(s, xq, a.qdim, a.gate, a.gate_b, _cur->glog, a.heads, tl, a.qdim,
                    a.heads, ltx::EPI_STORE, nullptr, err, lx_(a.l_gate, &lx)))
    return false;
  const __nv_bfloat16* qh = _cur->sp_recv;
  if (!_ops->attention(s, qh, Il, qh + blk, Il, qh + 2 * blk, Il, _cur->sp_send, Il, nullptr,
                       0, tv, tv, hl, a.head_dim, err, _layer))
    return false;
  if (!_comm->alltoall_bf16(_cur->sp_send, _cur->sp_recv, (size_t)tl * Il, 1, 0, s, err))
    return false;
  if (ltx::launch_a2a_unpack(_cur->sp_recv, tl, N, Il, out, I, _cur->glog, a.heads,
                             a.head_dim, s) != 0)
    return fail(err, "all-to-all unpack launch failed");
  return true;
}

bool CudaBlock::attend_v2a_sp_(cudaStream_t s, const CudaAttn& a, const __nv_bfloat16* xq,
                               int tq, const RopeRef& qr, const __nv_bfloat16* xkv, int tl,
                               const RopeRef& kr, __nv_bfloat16* out, std::string* err)
{
  // Audio queries (replicated) against the whole video sequence: this
  // rank's video keys/values go to their heads' owners, each rank attends
  // all audio queries for its heads, and the outputs are gathered.
  const int I = a.inner, N = _sp_world, Il = I / N, tv = tl * N, hl = a.heads / N;
  LoraExt lx;
  if (!_ops->linear(s, xq, a.qdim, a.q, a.qkv_b, _cur->qkv, I, tq, a.qdim, I, ltx::EPI_STORE,
                    nullptr, err, lx_(a.l_q, &lx)) ||
      !_ops->linear(s, xkv, a.kvdim, a.kv, a.kv_b, _cur->kvp, 2 * I, tl, a.kvdim, 2 * I,
                    ltx::EPI_STORE, nullptr, err, lx_(a.l_kv, &lx)))
    return false;
  if (ltx::launch_qk_norm_rope(_cur->qkv, I, _cur->qn, I, tq, a.heads, a.head_dim, a.q_norm,
                               qr.cos, qr.sin, kEps, s, nullptr, 0, 0, qr.tbl_tokens,
                               qr.tok0) != 0 ||
      ltx::launch_qk_norm_rope(_cur->kvp, 2 * I, _cur->kn, I, tl, a.heads, a.head_dim,
                               a.k_norm, kr.cos, kr.sin, kEps, s, nullptr, 0, 0, kr.tbl_tokens,
                               kr.tok0) != 0)
    return fail(err, "q/k norm + rope launch failed");
  const size_t blk = (size_t)tv * Il;
  if (ltx::launch_a2a_pack(_cur->kn, I, tl, N, Il, _cur->sp_send, s) != 0 ||
      ltx::launch_a2a_pack(_cur->kvp + I, 2 * I, tl, N, Il, _cur->sp_send + blk, s) != 0)
    return fail(err, "all-to-all pack launch failed");
  if (!_comm->alltoall_bf16(_cur->sp_send, _cur->sp_recv, (size_t)tl * Il, 2, blk, s, err))
    return false;
  if (!_ops->linear(s, xq, a.qdim, a.gate, a.gate_b, _cur->glog, a.heads, tq, a.qdim, a.heads,
                    ltx::EPI_STORE, nullptr, err, lx_(a.l_gate, &lx)))
    return false;
  // this rank's heads of every audio query -> sp_send [rank][tq][Il]
  __nv_bfloat16* mine = _cur->sp_send + (size_t)_sp_rank * tq * Il;
  if (!_ops->attention(s, _cur->qn + (size_t)_sp_rank * Il, I, _cur->sp_recv, Il,
                       _cur->sp_recv + blk, Il, mine, Il, nullptr, 0, tq, tv, hl,
                       a.head_dim, err, _layer))
    return false;
  if (!_comm->allgather_bf16(mine, _cur->sp_send, (size_t)tq * Il, s, err)) return false;
  if (ltx::launch_a2a_unpack(_cur->sp_send, tq, N, Il, out, I, _cur->glog, a.heads,
                             a.head_dim, s) != 0)
    return fail(err, "gather unpack launch failed");
  return true;
}

bool CudaBlock::out_proj_(cudaStream_t s, const __nv_bfloat16* in, int k,
                          const QWeight& w, const __nv_bfloat16* bias,
                          __nv_bfloat16* x, int n, int d, const float* gate,
                          std::string* err, const LoraSite* lora, int n_all)
{
  LoraExt lx;
  const LoraExt* ext = lora != nullptr ? lx_(*lora, &lx) : nullptr;
  if (_tp_world == 1)
    return _ops->linear(s, in, k, w, bias, x, d, n, k, d, ltx::EPI_GATED_RES, gate, err, ext);
  // Row split: this rank's K columns give a partial product (the adapter's
  // too, from its A columns); the sum over ranks, then the bias and the
  // gated residual, once.
  if (n_all > n && scatter_ok_(n_all, d)) {
    // Fused reduce-scatter: the GEMM's epilogue stores each token row's
    // partial into the receive slot of the rank that owns the row (this
    // rank's slot of that rank's buffer, over NVLink for the others); after
    // one ordering collective each rank sums its rows' W slots in rank
    // order, adding the bias and the gated residual in the same pass.
    const int which = _ccur->next_buffer();
    RowScatter sc;
    sc.dst = _ccur->peer_table(which);
    sc.owners = _tp_world;
    sc.rows = n;
    sc.slot = _tp_rank;
    __nv_bfloat16* mine = static_cast<__nv_bfloat16*>(_ccur->peer_buffer(_tp_rank, which));
    if (!_ops->linear(s, in, k, w, nullptr, mine, d, n_all, k, d, ltx::EPI_STORE, nullptr, err,
                      ext, &sc) ||
        !_ccur->barrier(s, err))
      return false;
    if (ltx::launch_gated_residual(x, d, mine, bias, gate, n, d, s, _tp_world,
                                   (size_t)n * d) != 0)
      return fail(err, "gated residual launch failed");
    return true;
  }
  if (n_all > n) {
    // Row-sharded residual: the partial covers all n_all tokens; the
    // reduce-scatter leaves this rank the sum for its own n rows only.
    __nv_bfloat16* mine = _cur->part + (size_t)_tp_rank * n * d;
    if (!_ops->linear(s, in, k, w, nullptr, _cur->part, d, n_all, k, d, ltx::EPI_STORE,
                      nullptr, err, ext) ||
        !_ccur->reduce_scatter_bf16(_cur->part, (size_t)n * d, s, err))
      return false;
    if (ltx::launch_gated_residual(x, d, mine, bias, gate, n, d, s) != 0)
      return fail(err, "gated residual launch failed");
    return true;
  }
  if (!_ops->linear(s, in, k, w, nullptr, _cur->part, d, n, k, d, ltx::EPI_STORE,
                    nullptr, err, ext) ||
      !_ccur->allreduce_sum(_cur->part, (size_t)n * d, 1, s, err))
    return false;
  if (ltx::launch_gated_residual(x, d, _cur->part, bias, gate, n, d, s) != 0)
    return fail(err, "gated residual launch failed");
  return true;
}

bool CudaBlock::scatter_ok_(int n_all, int d) const
{
  return _tp_scatter && _ccur == _comm && _comm != nullptr &&
         _comm->shared_bytes() >= (size_t)n_all * d * 2;
}

bool CudaBlock::gather_rows_(cudaStream_t s, __nv_bfloat16* buf, int n, int d,
                             std::string* err) const
{
  return _ccur->allgather_bf16(buf + (size_t)_tp_rank * n * d, buf, (size_t)n * d, s, err);
}

bool CudaBlock::first_half_(cudaStream_t s, const CudaStreamW& w, StreamIO& io,
                            std::string* err)
{
  // src/ltx25-block-ref.cc:196-262
  const int n = io.tokens, d = w.dim;
  // Tensor parallel with the residual sharded by token rows: this rank
  // holds rows [tok0, tok0 + n) of x; each modulated input is formed for
  // those rows into their place of a whole-sequence buffer and gathered, the
  // projections see all n_all rows, and the row-split products are
  // reduce-scattered back to the rank's rows.
  const bool rows = &w == &_video && _tp_world > 1 && io.tokens_all > n;
  const int nf = rows ? io.tokens_all : n;
  const size_t off = rows ? (size_t)_tp_rank * n * d : 0;
  float* mods = _arp->mods + (&w == &_audio ? (size_t)MOD_ROWS * _vdim : 0);
  if (ltx::launch_vec_add(w.scale_shift, io.timesteps, mods + MOD_MSA * d, 3 * d, s) ||
      ltx::launch_vec_add(w.scale_shift + 6 * d, io.timesteps ? io.timesteps + 6 * d : nullptr,
                          mods + MOD_CA * d, 3 * d, s) ||
      ltx::launch_vec_add(w.prompt_scale_shift, io.prompt_timestep,
                          mods + MOD_PROMPT * d, 2 * d, s))
    return fail(err, "adaLN rows launch failed");
  // normed = rms_norm(x) * (1 + scale) + shift;  x += gate * attn1(normed)
  if (ltx::launch_ada_zero(io.x, d, _cur->normed + off, d, n, d, mods + (MOD_MSA + 1) * d,
                           mods + MOD_MSA * d, kEps, true, s))
    return fail(err, "ada_zero launch failed");
  if (rows && !gather_rows_(s, _cur->normed, n, d, err)) return false;
  const RopeRef self_r = rows ? RopeRef{io.pe_cos, io.pe_sin, nf, 0}
                              : RopeRef{io.pe_cos, io.pe_sin,
                                        io.tokens_all > 0 ? io.tokens_all : n, io.tok0};
  const bool sp = _sp && &w == &_video;
  if (sp ? !attend_self_sp_(s, w.attn1, _cur->normed, n, self_r, _cur->att, err)
         : !attend_(s, w.attn1, _cur->normed, nf, _cur->normed, nf, self_r, self_r, _cur->att,
                    err))
    return false;
  if (!out_proj_(s, _cur->att, w.attn1.inner, w.attn1.o, w.attn1.o_b, io.x, n, d,
                 mods + (MOD_MSA + 2) * d, err, &w.attn1.l_o, nf))
    return false;
  // Text cross-attention: query = mod(rms_norm(x)) (= ada_zero with the
  // cross rows), key/value = context modulated by the prompt table + driver.
  if (ltx::launch_ada_zero(io.x, d, _cur->normed + off, d, n, d, mods + (MOD_CA + 1) * d,
                           mods + MOD_CA * d, kEps, true, s) ||
      ltx::launch_ada_zero(io.context, d, _cur->ctxmod, d, io.text_tokens, d,
                           mods + (MOD_PROMPT + 1) * d, mods + MOD_PROMPT * d,
                           kEps, false, s))
    return fail(err, "modulation launch failed");
  if (rows && !gather_rows_(s, _cur->normed, n, d, err)) return false;
  if (!attend_(s, w.attn2, _cur->normed, nf, _cur->ctxmod, io.text_tokens, RopeRef{},
               RopeRef{}, _cur->att, err))
    return false;
  return out_proj_(s, _cur->att, w.attn2.inner, w.attn2.o, w.attn2.o_b, io.x, n, d,
                   mods + (MOD_CA + 2) * d, err, &w.attn2.l_o, nf);
}

bool CudaBlock::ff_(cudaStream_t s, const CudaStreamW& w, StreamIO& io,
                    std::string* err)
{
  // src/ltx25-block-ref.cc:264-281
  const int n = io.tokens, d = w.dim;
  const bool rows = &w == &_video && _tp_world > 1 && io.tokens_all > n;
  const int nf = rows ? io.tokens_all : n;
  const size_t off = rows ? (size_t)_tp_rank * n * d : 0;
  float* mods = _arp->mods + (&w == &_audio ? (size_t)MOD_ROWS * _vdim : 0);
  if (ltx::launch_vec_add(w.scale_shift + 3 * d, io.timesteps ? io.timesteps + 3 * d : nullptr,
                          mods + MOD_MLP * d, 3 * d, s) ||
      ltx::launch_ada_zero(io.x, d, _cur->normed + off, d, n, d, mods + (MOD_MLP + 1) * d,
                           mods + MOD_MLP * d, kEps, true, s))
    return fail(err, "ff pre-norm launch failed");
  if (rows && _tp_ff_chunks && n % 2 == 0 && !scatter_ok_(nf, d))
    return ff_rows_chunked_(s, w, io, mods, err);
  if (rows && !gather_rows_(s, _cur->normed, n, d, err)) return false;
  LoraExt lx;
  return _ops->linear(s, _cur->normed, d, w.ff_in, w.ff_in_b, _cur->ff, w.ff_hidden, nf,
                      d, w.ff_hidden, ltx::EPI_GELU, nullptr, err, lx_(w.l_ff_in, &lx)) &&
         out_proj_(s, _cur->ff, w.ff_hidden, w.ff_out, w.ff_out_b, io.x, n, d,
                   mods + (MOD_MLP + 2) * d, err, &w.l_ff_out, nf);
}

bool CudaBlock::ff_rows_chunked_(cudaStream_t s, const CudaStreamW& w, StreamIO& io,
                                 const float* mods, std::string* err)
{
  // The feed-forward is token-local, so with the residual sharded by rows it
  // runs in two chunks: each rank's first and second halves of its rows.
  // The collectives go on the communication stream in one fixed order --
  // all-gather chunk 0, all-gather chunk 1, reduce-scatter chunk 0,
  // reduce-scatter chunk 1 -- each chunk's products waiting only for its own
  // gather, each reduce-scatter only for its own products: the second
  // gather runs under the first chunk's GEMMs and the first reduce-scatter
  // under the second's.  Every rank issues the same collectives in the same
  // order, and the compute stream waits for the last one before anything
  // after the feed-forward can touch the communicator.
  const int n = io.tokens, d = w.dim, h = n / 2, W = _tp_world, R = _tp_rank;
  const int nfh = h * W;                         // gathered rows of one chunk
  cudaStream_t cs = _ops->comm_stream(err);
  if (cs == nullptr) return false;
  __nv_bfloat16* G[2] = {_cur->normed, _cur->normed + (size_t)nfh * d};
  __nv_bfloat16* H[2] = {_cur->ff, _cur->ff + (size_t)nfh * w.ff_hidden};
  __nv_bfloat16* P[2] = {_cur->part, _cur->part + (size_t)nfh * d};
  for (int c = 0; c < 2; ++c)
    if (ltx::launch_ada_zero(io.x + (size_t)c * h * d, d, G[c] + (size_t)R * h * d, d, h, d,
                             mods + (MOD_MLP + 1) * d, mods + MOD_MLP * d, kEps, true, s))
      return fail(err, "ff pre-norm launch failed");
  // the communication stream starts after everything issued on s so far
  if (!_ops->cfork(s, cs, 0, err)) return false;
  for (int c = 0; c < 2; ++c)
    if (!_comm->allgather_bf16(G[c] + (size_t)R * h * d, G[c], (size_t)h * d, cs, err) ||
        !_ops->crecord(cs, 1 + c, err))          // event 1 + c: chunk c gathered
      return false;
  LoraExt lx;
  for (int c = 0; c < 2; ++c) {
    if (!_ops->cwait(s, 1 + c, err) ||
        !_ops->linear(s, G[c], d, w.ff_in, w.ff_in_b, H[c], w.ff_hidden, nfh, d, w.ff_hidden,
                      ltx::EPI_GELU, nullptr, err, lx_(w.l_ff_in, &lx)) ||
        !_ops->linear(s, H[c], w.ff_hidden, w.ff_out, nullptr, P[c], d, nfh, w.ff_hidden, d,
                      ltx::EPI_STORE, nullptr, err, lx_(w.l_ff_out, &lx)) ||
        !_ops->cfork(s, cs, 3 + c, err) ||       // cs: chunk c's products done
        !_comm->reduce_scatter_bf16(P[c], (size_t)h * d, cs, err))
      return false;
  }
  if (!_ops->cfork(cs, s, 5, err)) return false;   // s: both reduce-scatters done
  for (int c = 0; c < 2; ++c)
    if (ltx::launch_gated_residual(io.x + (size_t)c * h * d, d, P[c] + (size_t)R * h * d,
                                   w.ff_out_b, mods + (MOD_MLP + 2) * d, h, d, s) != 0)
      return fail(err, "gated residual launch failed");
  return true;
}

bool CudaBlock::shards_video(int tokens) const
{
  if (_sp) return true;
  return _tp_world > 1 && _tp_rows && tokens > 0 && tokens % _tp_world == 0;
}

bool CudaBlock::shard_io(const StreamIO& whole, StreamIO* shard, std::string* err) const
{
  *shard = whole;
  if (!whole.present || whole.tokens <= 0 || !shards_video(whole.tokens)) {
    if (_sp && whole.present && whole.tokens > 0)
      return fail(err, "sequence parallel shape: " + std::to_string(whole.tokens) +
                           " video tokens do not split over " + std::to_string(_sp_world) +
                           " ranks");
    return true;
  }
  const int world = _sp ? _sp_world : _tp_world, rank = _sp ? _sp_rank : _tp_rank;
  if (whole.tokens % world != 0)
    return fail(err, "sequence parallel shape: " + std::to_string(whole.tokens) +
                         " video tokens do not split over " + std::to_string(world) +
                         " ranks");
  const int tl = whole.tokens / world;
  shard->x = whole.x + (size_t)rank * tl * _vdim;
  shard->tokens = tl;
  shard->tok0 = rank * tl;
  shard->tokens_all = whole.tokens;
  return true;
}

bool CudaBlock::gather_video(cudaStream_t s, const StreamIO& whole, std::string* err) const
{
  if (!whole.present || whole.tokens <= 0 || !shards_video(whole.tokens)) return true;
  const int world = _sp ? _sp_world : _tp_world, rank = _sp ? _sp_rank : _tp_rank;
  const size_t cnt = (size_t)(whole.tokens / world) * _vdim;
  return _comm->allgather_bf16(whole.x + (size_t)rank * cnt, whole.x, cnt, s, err);
}

bool CudaBlock::forward(cudaStream_t s, StreamIO& v, StreamIO& a, std::string* err)
{
  if (!shards_video(v.present ? v.tokens : 0)) return forward_impl_(s, v, a, err);
  StreamIO vl;
  return shard_io(v, &vl, err) && forward_impl_(s, vl, a, err) && gather_video(s, v, err);
}

bool CudaBlock::forward_shard(cudaStream_t s, StreamIO& v, StreamIO& a, std::string* err)
{
  return forward_impl_(s, v, a, err);
}

bool CudaBlock::forward_impl_(cudaStream_t s, StreamIO& v, StreamIO& a, std::string* err)
{
  if (!_final) return fail(err, "forward before finalize");
  if (!_arp) return fail(err, "forward before reserve");
  const bool rv = v.present && v.tokens > 0;
  const bool ra = a.present && a.tokens > 0;
  if (!rv && !ra) return fail(err, "neither stream is present");
  const bool too_big =
      (rv && ((size_t)v.tokens > _arp->video || (size_t)v.text_tokens > _arp->text)) ||
      (ra && ((size_t)a.tokens > _arp->audio || (size_t)a.text_tokens > _arp->text));
  if (too_big)
    return fail(err, "geometry exceeds the reserved arena");
  for (const StreamIO* io : {&v, &a}) {
    const bool on = io == &v ? rv : ra;
    if (on && (io->x == nullptr || io->context == nullptr || io->timesteps == nullptr))
      return fail(err, "stream input missing x, context or timesteps");
  }
  // The audio stream runs beside the video one on the context's second
  // CUDA stream while they are independent (first halves, feed-forwards),
  // when nothing it launches shares scratch or a communicator with video.
  // An adapted audio linear takes the bf16 route and expands its pack into
  // the context's one dequant scratch, so such blocks keep audio in line.
  const bool conc = rv && ra && (_tp_world == 1 || _comm_side != nullptr) && !_audio_lora &&
                    _ops->audio_side_ok(a.tokens, a.text_tokens, _aheads, _adim / _aheads, _layer);
  cudaStream_t sa = conc ? _ops->aux_stream(err) : s;
  if (conc && sa == nullptr) return false;
  if (conc && !_ops->fork(s, sa, 0, err)) return false;
  _cur = conc ? _arp->side.get() : _arp.get();
  _ccur = conc ? _comm_side : _comm;
  if (ra && !first_half_(sa, _audio, a, err)) return false;
  _cur = _arp.get();
  _ccur = _comm;
  if (rv && !first_half_(s, _video, v, err)) return false;
  if (conc && !_ops->fork(sa, s, 1, err)) return false;

  if (rv && ra) {
    // src/ltx25-block-ref.cc:336-385.  Both directions read the PRE-cross
    // state: all four ada_zero operands are formed before either update.
    const int vd = _vdim, ad = _adim;
    float* vm = _arp->mods;
    float* am = _arp->mods + (size_t)MOD_ROWS * _vdim;
    if (ltx::launch_vec_add(_video.cross_table, v.cross_scale_shift, vm + MOD_AV * vd, 4 * vd, s) ||
        ltx::launch_vec_add(_video.cross_table + 4 * vd, v.cross_gate, vm + MOD_AVG * vd, vd, s) ||
        ltx::launch_vec_add(_audio.cross_table, a.cross_scale_shift, am + MOD_AV * ad, 4 * ad, s) ||
        ltx::launch_vec_add(_audio.cross_table + 4 * ad, a.cross_gate, am + MOD_AVG * ad, ad, s))
      return fail(err, "cross adaLN launch failed");
    // Row-sharded residual (tensor parallel): x's rows are gathered once
    // (into the idle `normed` buffer) and both video modulations formed on
    // all rows, one all-gather instead of two.
    const bool vrows = _tp_world > 1 && v.tokens_all > v.tokens;
    const int vn = v.tokens, vnf = vrows ? v.tokens_all : vn;
    const __nv_bfloat16* vxs = v.x;
    if (vrows) {
      if (!_comm->allgather_bf16(v.x, _arp->normed, (size_t)vn * vd, s, err)) return false;
      vxs = _arp->normed;
    }
    // av rows: [scale(lo=0), shift(lo=0), scale(lo=2), shift(lo=2)]
    if (ltx::launch_ada_zero(vxs, vd, _arp->qv, vd, vnf, vd, vm + (MOD_AV + 0) * vd,
                             vm + (MOD_AV + 1) * vd, kEps, true, s) ||
        ltx::launch_ada_zero(a.x, ad, _arp->kva, ad, a.tokens, ad, am + (MOD_AV + 0) * ad,
                             am + (MOD_AV + 1) * ad, kEps, true, s) ||
        ltx::launch_ada_zero(a.x, ad, _arp->qa, ad, a.tokens, ad, am + (MOD_AV + 2) * ad,
                             am + (MOD_AV + 3) * ad, kEps, true, s) ||
        ltx::launch_ada_zero(vxs, vd, _arp->kvv, vd, vnf, vd, vm + (MOD_AV + 2) * vd,
                             vm + (MOD_AV + 3) * vd, kEps, true, s))
      return fail(err, "cross ada_zero launch failed");
    // a2v: video queries, audio keys/values
    const RopeRef vc = vrows ? RopeRef{v.cpe_cos, v.cpe_sin, vnf, 0}
                             : RopeRef{v.cpe_cos, v.cpe_sin,
                                       v.tokens_all > 0 ? v.tokens_all : v.tokens, v.tok0};
    const RopeRef ac{a.cpe_cos, a.cpe_sin, a.tokens, 0};
    if (!attend_(s, _a2v, _arp->qv, vnf, _arp->kva, a.tokens, vc, ac, _arp->att, err) ||
        !out_proj_(s, _arp->att, _a2v.inner, _a2v.o, _a2v.o_b, v.x, vn, vd,
                   vm + MOD_AVG * vd, err, &_a2v.l_o, vnf))
      return false;
    // v2a: audio queries, video keys/values
    if ((_sp ? !attend_v2a_sp_(s, _v2a, _arp->qa, a.tokens, ac, _arp->kvv, v.tokens, vc,
                               _arp->att, err)
             : !attend_(s, _v2a, _arp->qa, a.tokens, _arp->kvv, vnf, ac, vc, _arp->att,
                        err)) ||
        !out_proj_(s, _arp->att, _v2a.inner, _v2a.o, _v2a.o_b, a.x, a.tokens, ad,
                   am + MOD_AVG * ad, err, &_v2a.l_o))
      return false;
  }

  if (conc && !_ops->fork(s, sa, 2, err)) return false;
  _cur = conc ? _arp->side.get() : _arp.get();
  _ccur = conc ? _comm_side : _comm;
  if (ra && !ff_(sa, _audio, a, err)) return false;
  _cur = _arp.get();
  _ccur = _comm;
  if (rv && !ff_(s, _video, v, err)) return false;
  if (conc && !_ops->fork(sa, s, 3, err)) return false;
  return true;
}

}  // namespace ltx25
