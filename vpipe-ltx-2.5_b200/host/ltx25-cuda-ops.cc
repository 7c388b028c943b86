// ltx25-cuda-ops.cc -- CudaOps: routing, tile planning and the scratch
// arena around the tcgen05 GEMM (see ltx25-cuda-ops.h).
#include "ltx25-cuda-ops.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "../../include/ltx25_cuda.h"
#include "../csrc/block_ops.h"
#include "../csrc/kernels.h"

namespace ltx25 {

namespace {

bool cuda_ok(cudaError_t e, const char* what, std::string* err)
{
  if (e == cudaSuccess) return true;
  if (err) *err = std::string(what) + ": " + cudaGetErrorString(e);
  return false;
}

bool aligned(const void* p, size_t a)
{
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

struct Plan {
  int tn = 256;
  bool pair = false;
  int wb = 1;          // weight blocks per CTA (2: 512 weight rows per pair tile)
  int splits = 1;
  int m_tiles = 1, n_tiles = 1, kblocks = 1;
};

// Token tile and K split for one GEMM.  Large token counts take the
// 256-token tile (the widest MMA N, least dequant per FLOP); the audio and
// text shapes (M <= 128 / small tile counts) split K until the grid covers
// the SMs, because those shapes are bound by reading the weight, not by
// the tensor pipe.
// Dense pairs hold two weight blocks per CTA unless LTX25_PAIR_WB=1.
const bool g_wb2_default = [] {
  const char* e = std::getenv("LTX25_PAIR_WB");
  return !(e != nullptr && e[0] == '1');
}();

Plan plan_gemm(int mode, int M, int N, int K, int epi, int sms, const PlanKnobs& kn)
{
  Plan p;
  const int kpb = mode == ltx::MODE_I8 ? 128 : 64;
  // a K tail past the last full block reads as zeros (TMA fill)
  p.kblocks = (K + kpb - 1) / kpb;
  p.tn = M <= 128 ? 128 : 256;
  // CTA pairs (M = 256 MMA over two SMs) halve the activation bytes each SM
  // streams per FLOP.  The dense path pairs by default once there are
  // enough tiles; the fused w8g64 path measured slower paired (the
  // cross-CTA hand-off of dequantized A slots), so opt-in there.
  p.pair = mode == ltx::MODE_BF16 && M >= 1024 && N % 256 == 0 &&
           ((M + 255) / 256) * (N / 256) >= sms / 2;
  // ... except a gated residual over a short K: with at most 32 k-blocks a
  // tile's main loop is not much longer than that epilogue (residual loads
  // included), which single CTAs hide behind their second accumulator and
  // a two-block pair cannot (a2v out, 8160 x 2048 -> 4096: 132-144 us single
  // against 148-161 paired, same box, arms interleaved).
  if (epi == ltx::EPI_GATED_RES && K <= 2048) p.pair = false;
  if (kn.pair >= 0) {
    p.pair = (mode == ltx::MODE_W8G64 || mode == ltx::MODE_BF16) && kn.pair != 0 &&
             M > 128 && N % 256 == 0;
  }
  if (p.pair) p.tn = 256;
  // Two weight blocks per CTA: one activation stage feeds two MMAs, 48 KB
  // per 2 x 128x256x64 MMA taken in by each SM instead of 32 KB per one.
  if ((kn.pair == 2 || (kn.pair < 0 && g_wb2_default)) && p.pair && mode == ltx::MODE_BF16 &&
      N % 512 == 0)
    p.wb = 2;
  if (kn.tn >= 0) {
    if (!p.pair && (kn.tn == 128 || kn.tn == 256)) p.tn = kn.tn;
  }
  const int wrows = (p.pair ? 256 : 128) * p.wb;   // weight rows per tile
  p.n_tiles = (N + wrows - 1) / wrows;
  p.m_tiles = (M + p.tn - 1) / p.tn;
  const int tiles = p.m_tiles * p.n_tiles;
  p.splits = 1;
  // Split K over a cluster until ~128 CTAs stream the weight.  Measured on
  // B200 (M = 126, 16-64 weight tiles): clusters of up to 6 CTAs and grids
  // of <= 128 CTAs win; 8-CTA clusters and 3-way splits of 48 tiles place
  // poorly across the GPCs and run a second wave (24.6 vs 36.9 us at
  // K=8192 N=2048; 21.3 vs 31.6 us at K=2048 N=6144).
  if (!p.pair && tiles * 2 <= 128 && p.kblocks >= 4) {
    p.splits = std::min(std::min(128 / tiles, p.kblocks / 2), 6);
    if (p.splits < 1) p.splits = 1;
  }
  // A/B override of the K split (the reference's tile knobs,
  // src/ltx25-metal-ops.cc:164-231).  Ignored when out of range.
  if (kn.splits >= 0) {
    const int sp = kn.splits;
    if (!p.pair && sp >= 1 && sp <= 8 && sp <= p.kblocks && (sp == 1 || tiles * sp <= sms))
      p.splits = sp;
  }
  return p;
}

}  // namespace

CudaOps::~CudaOps()
{
  if (_dev < 0) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(_dev);
  cudaFree(_xq);
  cudaFree(_sx);
  cudaFree(_deq);
  for (cudaEvent_t e : _ev)
    if (e != nullptr) cudaEventDestroy(e);
  if (_aux != nullptr) cudaStreamDestroy(_aux);
  for (cudaEvent_t e : _cev)
    if (e != nullptr) cudaEventDestroy(e);
  if (_cstream != nullptr) cudaStreamDestroy(_cstream);
  cudaFree(_vt);
  cudaFree(_vt_side);
  cudaFree(_part);
  cudaFree(_sb.qi8);
  cudaFree(_sb.ki8);
  cudaFree(_sb.scales);
  cudaFree(_sb.mean);
  cudaFree(_err_word);
  cudaFree(_ones);
  cudaFree(_lora_r);
  cudaFree(_tr[0]);
  cudaFree(_tr[1]);
  cudaSetDevice(prev);
}

bool CudaOps::init(int device, std::string* err)
{  // the tile plan's and the attention's A/B overrides start from the
  // environment, read here once (LTX25_FORCE_PAIR, LTX25_FORCE_TN,
  // LTX25_FORCE_SPLITS, LTX25_ATTN, LTX25_ATTN64)
  if (const char* e = std::getenv("LTX25_FORCE_PAIR")) {
    const int v = std::atoi(e);
    _knobs.pair = v == 2 ? 2 : v != 0 ? 1 : 0;
  }
  if (const char* e = std::getenv("LTX25_FORCE_TN")) _knobs.tn = std::atoi(e);
  if (const char* e = std::getenv("LTX25_FORCE_SPLITS")) _knobs.splits = std::atoi(e);
  // attention kernel choice (A/B switches): LTX25_ATTN=mma runs every
  // attention on the warp-MMA kernel.  The unsplit 64-wide attentions (126-256
  // keys: the audio stream's, and the video queries over the audio keys) run
  // the warp-MMA kernel; LTX25_ATTN64=tc selects the tcgen05 one, measured
  // slower on all of them (8160 x 126: 74 vs 60 us; 126 x 126: 26 vs 19 us)
  // and, on the side stream beside the video GEMMs, 5 % slower a block.
  if (const char* e = std::getenv("LTX25_ATTN")) _attn_mode = std::strcmp(e, "mma") == 0 ? 0 : 1;
  if (const char* e = std::getenv("LTX25_ATTN64")) _attn64_tc = std::strcmp(e, "tc") == 0;
  // V^T from the K/V projection's epilogue (on by default; LTX25_VT_OUT=0
  // keeps the V^T copy kernel)
  if (const char* e = std::getenv("LTX25_VT_OUT")) _vt_out = e[0] != '0';

  int n = 0;
  if (!cuda_ok(cudaGetDeviceCount(&n), "cudaGetDeviceCount", err)) return false;
  if (device < 0 || device >= n) {
    if (err) *err = "no CUDA device " + std::to_string(device);
    return false;
  }
  cudaDeviceProp prop;
  if (!cuda_ok(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties", err))
    return false;
  if (prop.major != 10 || prop.minor != 0) {
    if (err)
      *err = std::string("device ") + prop.name + " is sm_" +
             std::to_string(prop.major) + std::to_string(prop.minor) +
             "; this library is built for sm_100a (B200) only";
    return false;
  }
  if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice", err)) return false;
  _dev = device;
  _sms = prop.multiProcessorCount;
  if (!cuda_ok(cudaMalloc(&_err_word, sizeof(int)), "cudaMalloc(err)", err))
    return false;
  return cuda_ok(cudaMemset(_err_word, 0, sizeof(int)), "cudaMemset", err);
}

bool CudaOps::ensure_(size_t i8_bytes, size_t deq_bytes, std::string* err)
{
  if (i8_bytes > _xq_bytes) {
    cudaFree(_xq);
    cudaFree(_sx);
    _xq = nullptr;
    _sx = nullptr;
    _xq_bytes = 0;
    if (!cuda_ok(cudaMalloc(&_xq, i8_bytes), "cudaMalloc(int8 activations)", err))
      return false;
    if (!cuda_ok(cudaMalloc(&_sx, i8_bytes / 64 * sizeof(float) + 1024), "cudaMalloc(int8 scales)", err))
      return false;
    _xq_bytes = i8_bytes;
  }
  if (deq_bytes > _deq_bytes) {
    cudaFree(_deq);
    _deq = nullptr;
    _deq_bytes = 0;
    if (!cuda_ok(cudaMalloc(&_deq, deq_bytes), "cudaMalloc(dequant scratch)", err))
      return false;
    _deq_bytes = deq_bytes;
  }
  return true;
}

size_t CudaOps::scratch_bytes() const
{
  size_t b = 0;
  if (_xq_bytes > 0) b += _xq_bytes + _xq_bytes / 64 * sizeof(float) + 1024;
  b += _deq_bytes + (_vt_elems + _vt_side_elems) * sizeof(__nv_bfloat16) +
       _part_elems * sizeof(float);
  b += _sb.cap.qi8 + _sb.cap.ki8 + (_sb.cap.scales + _sb.cap.mean) * sizeof(float);
  b += (size_t)_ones_n * sizeof(float) + _lora_r_elems * sizeof(__nv_bfloat16);
  if (_tr_elems[0] > 0) b += _tr_elems[0] * 2 + 256;
  if (_tr_elems[1] > 0) b += _tr_elems[1] * 2 + 256;
  return b;
}

bool CudaOps::reserve(int max_tokens, int max_n, int max_k, std::string* err)
{
  if (max_tokens <= 0 || max_n <= 0 || max_k <= 0) {
    if (err) *err = "reserve: sizes must be positive";
    return false;
  }
  // The split-K partials live in shared memory; only the int8 tier's
  // quantized activations and the dequant-once expansion need HBM scratch.
  const size_t i8 = _i8 ? (size_t)max_tokens * max_k : 0;
  const bool expand = _route == Route::DequantOnce ||
                      (_route == Route::Auto && max_tokens >= LTX_DEQUANT_MIN_M);
  const size_t deq = expand ? (size_t)max_n * max_k * 2 : 0;
  return ensure_(i8, deq, err);
}

bool CudaOps::i8_takes(int M, int K, int N) const
{
  // The reference's gates (src/ltx25-metal-ops.cc:381-391): the int8 tier
  // pays back its quantize passes only on tall, deep GEMMs.  K must fill
  // whole 128-byte int8 K tiles here.
  return _i8 && M >= 1024 && K >= 1024 && K % 128 == 0 && N % 4 == 0;
}

bool CudaOps::prepare_i8(QWeight& w, cudaStream_t s, std::string* err) const
{
  if (w.wq != nullptr) return true;
  if (!w.quantized) {
    if (err) *err = "int8 tier: weight is not quantized";
    return false;
  }
  const size_t nk = (size_t)w.N * w.K;
  __nv_bfloat16* tmp = nullptr;
  if (!cuda_ok(cudaMalloc(&tmp, nk * 2), "cudaMalloc(i8 prep)", err)) return false;
  if (!cuda_ok(cudaMalloc(&w.wq, nk), "cudaMalloc(i8 weight)", err)) {
    cudaFree(tmp);
    return false;
  }
  if (!cuda_ok(cudaMalloc(&w.sw, (size_t)w.N * sizeof(float)), "cudaMalloc(i8 scales)", err)) {
    cudaFree(tmp);
    return false;
  }
  bool ok = ltx::launch_dequant_w8(w.codes, w.sz, w.N, w.K, tmp, s) == 0 &&
            ltx::launch_quant_rows_i8(tmp, w.N, w.K, w.K, w.K, w.wq, w.sw, s) == 0;
  ok = ok && cuda_ok(cudaStreamSynchronize(s), "i8 weight prep", err);
  cudaFree(tmp);
  if (!ok && err && err->empty()) *err = "i8 weight prep launch failed";
  return ok;
}

bool CudaOps::gemm_(cudaStream_t s, int mode, const void* x, int ldx,
                    const void* wptr, const uint32_t* sz,
                    const __nv_bfloat16* bias, __nv_bfloat16* y, int ldy,
                    int M, int K, int N, int epi, const float* gate,
                    const float* sx, const float* sw, std::string* err,
                    const LoraExt* ext, const RowScatter* scatter, const VtOut* vto)
{
  // An extension adds ceil(r / 64) K blocks after the main K.
  const int ext_k = (ext != nullptr) ? ext->r : 0;
  const int ext_kb = (ext_k + 63) / 64;
  Plan pl = plan_gemm(mode, M, N, K + 64 * ext_kb, epi, _sms, _knobs);
  if (scatter != nullptr) {
    // scattered rows are stored by the tile epilogue itself: one K split
    if (epi != ltx::EPI_STORE || scatter->dst == nullptr || scatter->rows <= 0 ||
        scatter->rows >= (1 << 28) || scatter->slot < 0 || scatter->slot >= 8 ||
        (M + scatter->rows - 1) / scatter->rows > scatter->owners) {
      if (err) *err = "row scatter: store epilogue, an owner for every row";
      return false;
    }
    pl.splits = 1;
  }
  if (vto != nullptr) {
    // transposed columns are stored by the tile epilogue itself: one K split
    if (mode == ltx::MODE_I8 || epi != ltx::EPI_STORE || scatter != nullptr ||
        vto->vt == nullptr || !aligned(vto->vt, 16) || vto->col0 < 0 || vto->col0 % 32 != 0 ||
        vto->col0 / 32 >= 2048 || vto->ld <= 0 || vto->ld % 8 != 0 || vto->ld / 8 >= (1 << 20)) {
      if (err) *err = "V^T output: store epilogue, no int8 tier, col0 % 32, ld % 8, aligned";
      return false;
    }
    pl.splits = 1;
  }
  ltx::GemmLaunch L;
  L.mode = mode;
  L.tn = pl.tn;
  L.pair = pl.pair;
  L.wb = pl.wb;
  L.epi = epi;
  L.num_sms = _sms;
  L.x = x;
  L.ldx = ldx;
  L.w = wptr;
  L.sz = sz;
  ltx::GemmParams& p = L.p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.m_tiles = pl.m_tiles;
  p.n_tiles = pl.n_tiles;
  p.splits = pl.splits;
  p.kblocks = pl.kblocks;
  p.kblocks_main = pl.kblocks - ext_kb;
  if (ext_k > 0) {
    L.ext_w = ext->b;
    L.ext_x = ext->rbuf;
    L.ext_k = ext_k;
    L.ld_ext = ext_k;
  }
  p.num_tiles = pl.m_tiles * pl.n_tiles * pl.splits;
  p.ldy = ldy;
  p.bias = bias;
  p.gate = gate;
  p.y = y;
  p.sx = sx;
  p.sw = sw;
  p.err = _err_word;
  p.trace = _trace;
  p.trace_ctas = _trace_ctas;
  if (scatter != nullptr) {
    p.ys = scatter->dst;
    p.scatter = ltx::pack_scatter(scatter->rows, scatter->slot);
  }
  if (vto != nullptr) {
    p.vt = vto->vt;
    p.vt_spec = ltx::pack_vt(vto->col0, vto->ld);
  }
  const int rc = ltx::gemm_launch(L, s);
  if (rc != 0) {
    if (err)
      *err = "gemm launch failed (" + std::to_string(rc) + "): " +
             cudaGetErrorString(cudaGetLastError());
    return false;
  }
  return true;
}

bool CudaOps::linear(cudaStream_t s, const __nv_bfloat16* x, int ldx,
                     const QWeight& w, const __nv_bfloat16* bias,
                     __nv_bfloat16* y, int ldy, int M, int K, int N, int epi,
                     const float* gate, std::string* err, const LoraExt* lora,
                     const RowScatter* sc, const VtOut* vto)
{
  if (x == nullptr || y == nullptr) {
    if (err) *err = "linear: null x or y";
    return false;
  }
  if (M <= 0 || K != w.K || N != w.N) {
    if (err)
      *err = "linear: shape (M=" + std::to_string(M) + ", K=" + std::to_string(K) +
             ", N=" + std::to_string(N) + ") disagrees with the weight [" +
             std::to_string(w.N) + "][" + std::to_string(w.K) + "]";
    return false;
  }
  if (!aligned(x, 16) || ldx % 8 != 0 || ldx < K || !aligned(y, 4) ||
      ldy % 2 != 0 || ldy < N || (bias && !aligned(bias, 4)) ||
      (gate && !aligned(gate, 8))) {
    if (err) *err = "linear: x must be 16-byte aligned with ldx % 8 == 0; y, bias 4-byte, gate 8-byte aligned";
    return false;
  }
  if (epi == ltx::EPI_GATED_RES && gate == nullptr) {
    if (err) *err = "linear: gated residual needs a gate";
    return false;
  }
  if (lora != nullptr && lora->r > 0) {
    // r = x.A^T, then the linear with r.B^T contracted after its own K.
    // The int8 tier's s32 accumulator cannot hold the bf16 delta and the
    // fused w8g64 kernel's A operand is dequantized in TMEM, so an adapted
    // linear takes the bf16 route: the dense weight, or the pack expanded
    // once into the scratch.
    if (lora->a == nullptr || lora->b == nullptr || lora->rbuf == nullptr ||
        lora->r % 8 != 0 || !aligned(lora->a, 16) || !aligned(lora->b, 16) ||
        !aligned(lora->rbuf, 16)) {
      if (err) *err = "linear: adapter needs a, b, r scratch (16-byte aligned) and rank % 8 == 0";
      return false;
    }
    if (!gemm_(s, ltx::MODE_BF16, x, ldx, lora->a, nullptr, nullptr, lora->rbuf, lora->r, M,
               K, lora->r, ltx::EPI_STORE, nullptr, nullptr, nullptr, err))
      return false;
    const void* wb = w.w;
    if (w.quantized) {
      if (!ensure_(0, (size_t)N * K * 2, err)) return false;
      if (ltx::launch_dequant_w8(w.codes, w.sz, N, K, _deq, s) != 0) {
        if (err) *err = "dequant launch failed";
        return false;
      }
      wb = _deq;
    }
    return gemm_(s, ltx::MODE_BF16, x, ldx, wb, nullptr, bias, y, ldy, M, K, N, epi, gate,
                 nullptr, nullptr, err, lora, sc, vto);
  }
  if (!w.quantized) {
    return gemm_(s, ltx::MODE_BF16, x, ldx, w.w, nullptr, bias, y, ldy, M, K,
                 N, epi, gate, nullptr, nullptr, err, nullptr, sc, vto);
  }
  if (i8_takes(M, K, N)) {
    if (vto != nullptr) {
      if (err) *err = "linear: V^T output is not on the int8 tier";
      return false;
    }
    if (!prepare_i8(const_cast<QWeight&>(w), s, err)) return false;
    if (!ensure_((size_t)M * K, 0, err)) return false;
    if (ltx::launch_quant_rows_i8(x, M, K, ldx, K, _xq, _sx, s) != 0) {
      if (err) *err = "int8 activation quantize launch failed";
      return false;
    }
    return gemm_(s, ltx::MODE_I8, _xq, K, w.wq, nullptr, bias, y, ldy, M, K,
                 N, epi, gate, _sx, w.sw, err, nullptr, sc);
  }
  if (_route == Route::DequantOnce || (_route == Route::Auto && M >= LTX_DEQUANT_MIN_M)) {
    if (!ensure_(0, (size_t)N * K * 2, err)) return false;
    if (ltx::launch_dequant_w8(w.codes, w.sz, N, K, _deq, s) != 0) {
      if (err) *err = "dequant launch failed";
      return false;
    }
    return gemm_(s, ltx::MODE_BF16, x, ldx, _deq, nullptr, bias, y, ldy, M,
                 K, N, epi, gate, nullptr, nullptr, err, nullptr, sc, vto);
  }
  return gemm_(s, ltx::MODE_W8G64, x, ldx, w.codes, w.sz, bias, y, ldy, M, K,
               N, epi, gate, nullptr, nullptr, err, nullptr, sc, vto);
}

__nv_bfloat16* CudaOps::lora_rbuf(size_t elems, std::string* err)
{
  if (elems <= _lora_r_elems) return _lora_r;
  cudaFree(_lora_r);
  _lora_r = nullptr;
  _lora_r_elems = 0;
  if (!cuda_ok(cudaMalloc(&_lora_r, elems * 2), "cudaMalloc(lora scratch)", err))
    return nullptr;
  _lora_r_elems = elems;
  return _lora_r;
}

__nv_bfloat16* CudaOps::trunk_buf_(int i, size_t elems, std::string* err)
{
  if (elems <= _tr_elems[i]) return _tr[i];
  cudaFree(_tr[i]);
  _tr[i] = nullptr;
  _tr_elems[i] = 0;
  if (!cuda_ok(cudaMalloc(&_tr[i], elems * 2 + 256), "cudaMalloc(trunk scratch)", err))
    return nullptr;
  _tr_elems[i] = elems;
  return _tr[i];
}

bool CudaOps::patchify(cudaStream_t s, const QWeight& w, const __nv_bfloat16* bias,
                       const LoraPair* lora, const __nv_bfloat16* latent, bool channel_major,
                       const __nv_bfloat16* prefix, int prefix_rows, __nv_bfloat16* x, int T,
                       int z, int dim, std::string* err)
{
  if (latent == nullptr || x == nullptr) {
    if (err) *err = "patchify: null latent or x";
    return false;
  }
  if (T <= 0 || prefix_rows < 0 || prefix_rows > T || (prefix_rows > 0 && prefix == nullptr)) {
    if (err) *err = "patchify shape: T, prefix_rows (need a prefix vector for prefix rows)";
    return false;
  }
  const __nv_bfloat16* in = latent;
  if (channel_major) {
    __nv_bfloat16* packed = trunk_buf_(0, (size_t)T * z, err);
    if (packed == nullptr) return false;
    if (ltx::launch_transpose_bf16(latent, T, packed, z, z, T, s) != 0) {
      if (err) *err = "patchify pack launch failed";
      return false;
    }
    in = packed;
  }
  LoraExt ext;
  if (lora != nullptr) {
    if (lora->k != z || lora->n != dim) {
      if (err) *err = "patchify adapter shape: pair widths disagree with the projection";
      return false;
    }
    ext.a = lora->a;
    ext.b = lora->b;
    ext.r = lora->r8;
    ext.rbuf = lora_rbuf((size_t)T * lora->r8, err);
    if (ext.rbuf == nullptr) return false;
  }
  if (!linear(s, in, z, w, bias, x, dim, T, z, dim, ltx::EPI_STORE, nullptr, err,
              lora != nullptr ? &ext : nullptr))
    return false;
  if (prefix_rows > 0 && ltx::launch_add_row_prefix(x, dim, prefix, prefix_rows, dim, s) != 0) {
    if (err) *err = "keyframe embedding launch failed";
    return false;
  }
  return true;
}

bool CudaOps::output_head(cudaStream_t s, const __nv_bfloat16* x, const float* shift_scale,
                          const QWeight& w, const __nv_bfloat16* bias, const LoraPair* lora,
                          __nv_bfloat16* out, bool channel_major, int T, int dim, int out_ch,
                          std::string* err)
{
  if (x == nullptr || shift_scale == nullptr || out == nullptr) {
    if (err) *err = "output head: null x, shift/scale table or out";
    return false;
  }
  if (T <= 0 || dim % 8 != 0 || !aligned(shift_scale, 16)) {
    if (err) *err = "output head shape: dim % 8, table 16-byte aligned";
    return false;
  }
  __nv_bfloat16* tmp = trunk_buf_(0, (size_t)T * dim, err);
  if (tmp == nullptr) return false;
  if (ltx::launch_layer_norm_mod(x, dim, tmp, dim, T, dim, shift_scale, shift_scale + dim,
                                 1e-6f, s) != 0) {
    if (err) *err = "output head norm launch failed";
    return false;
  }
  __nv_bfloat16* y = out;
  if (channel_major) {
    y = trunk_buf_(1, (size_t)T * out_ch, err);
    if (y == nullptr) return false;
  }
  LoraExt ext;
  if (lora != nullptr) {
    if (lora->k != dim || lora->n != out_ch) {
      if (err) *err = "output head adapter shape: pair widths disagree with proj_out";
      return false;
    }
    ext.a = lora->a;
    ext.b = lora->b;
    ext.r = lora->r8;
    ext.rbuf = lora_rbuf((size_t)T * lora->r8, err);
    if (ext.rbuf == nullptr) return false;
  }
  if (!linear(s, tmp, dim, w, bias, y, out_ch, T, dim, out_ch, ltx::EPI_STORE, nullptr, err,
              lora != nullptr ? &ext : nullptr))
    return false;
  if (channel_major && ltx::launch_transpose_bf16(y, out_ch, out, T, T, out_ch, s) != 0) {
    if (err) *err = "output head unpack launch failed";
    return false;
  }
  return true;
}

const float* CudaOps::ones_(int n, cudaStream_t s, std::string* err)
{
  if (n <= _ones_n) return _ones;
  cudaFree(_ones);
  _ones = nullptr;
  _ones_n = 0;
  if (!cuda_ok(cudaMalloc(&_ones, (size_t)n * sizeof(float)), "cudaMalloc(ones)", err))
    return nullptr;
  if (ltx::launch_fill_f32(_ones, 1.0f, n, s) != 0) {
    if (err) *err = "fill launch failed";
    return nullptr;
  }
  _ones_n = n;
  return _ones;
}

bool CudaOps::lora_add(cudaStream_t s, const __nv_bfloat16* x, int ldx, const LoraExt& lora,
                       __nv_bfloat16* y, int ldy, int M, int K, int N, std::string* err)
{
  if (M <= 0 || K <= 0 || N <= 0 || lora.r <= 0) return true;   // nothing to add
  if (x == nullptr || y == nullptr || lora.a == nullptr || lora.b == nullptr ||
      lora.rbuf == nullptr) {
    if (err) *err = "lora_add: null operand";
    return false;
  }
  if (K % 8 != 0 || lora.r % 8 != 0 || !aligned(x, 16) || ldx % 8 != 0 || ldx < K ||
      !aligned(y, 4) || ldy % 2 != 0 || ldy < N || !aligned(lora.rbuf, 16)) {
    if (err) *err = "lora_add: K % 8, rank % 8, x 16-byte aligned (ldx % 8), y 4-byte aligned";
    return false;
  }
  const float* one = ones_(N, s, err);
  if (one == nullptr) return false;
  // r = x.A^T; y = y + 1 * (r.B^T): the gated-residual epilogue reads y
  // and writes it once, so the delta never exists as its own [M][N].
  return gemm_(s, ltx::MODE_BF16, x, ldx, lora.a, nullptr, nullptr, lora.rbuf, lora.r, M, K,
               lora.r, ltx::EPI_STORE, nullptr, nullptr, nullptr, err) &&
         gemm_(s, ltx::MODE_BF16, lora.rbuf, lora.r, lora.b, nullptr, nullptr, y, ldy, M,
               lora.r, N, ltx::EPI_GATED_RES, one, nullptr, nullptr, err);
}

bool CudaOps::linear_i8_scratch(cudaStream_t s, const __nv_bfloat16* x,
                                const QWeight& w, const __nv_bfloat16* bias,
                                __nv_bfloat16* y, int M, int K, int N,
                                int8_t* xq, float* sx, std::string* err)
{
  if (x == nullptr || y == nullptr) {
    if (err) *err = "linear: null x or y";
    return false;
  }
  if (M <= 0 || K != w.K || N != w.N) {
    if (err)
      *err = "linear: shape (M=" + std::to_string(M) + ", K=" + std::to_string(K) +
             ", N=" + std::to_string(N) + ") disagrees with the weight [" +
             std::to_string(w.N) + "][" + std::to_string(w.K) + "]";
    return false;
  }
  if (K % 128 != 0 || N % 4 != 0) {
    if (err) *err = "int8 tier shape: K must be a multiple of 128, N of 4";
    return false;
  }
  if (!w.quantized || w.wq == nullptr) {
    if (err) *err = "int8 tier state: the weight has no int8 copy yet";
    return false;
  }
  if (!aligned(x, 16) || !aligned(y, 4) || (bias && !aligned(bias, 4))) {
    if (err) *err = "linear: x must be 16-byte aligned; y, bias 4-byte aligned";
    return false;
  }
  if (ltx::launch_quant_rows_i8(x, M, K, K, K, xq, sx, s) != 0) {
    if (err) *err = "int8 activation quantize launch failed";
    return false;
  }
  return gemm_(s, ltx::MODE_I8, xq, K, w.wq, nullptr, bias, y, N, M, K, N,
               ltx::EPI_STORE, nullptr, sx, w.sw, err);
}

bool CudaOps::reserve_attention(int keys, int width, std::string* err)
{
  const size_t need = ltx::attention_tc_scratch(keys, 1, width);
  if (need <= _vt_elems) return true;
  cudaFree(_vt);
  _vt = nullptr;
  _vt_elems = 0;
  if (!cuda_ok(cudaMalloc(&_vt, need * sizeof(__nv_bfloat16)), "cudaMalloc(attention scratch)", err))
    return false;
  _vt_elems = need;
  return true;
}

bool CudaOps::reserve_attention_side(int keys, int width, std::string* err)
{
  const size_t need = ltx::attention_tc_scratch(keys, 1, width);
  if (need <= _vt_side_elems) return true;
  cudaFree(_vt_side);
  _vt_side = nullptr;
  _vt_side_elems = 0;
  if (!cuda_ok(cudaMalloc(&_vt_side, need * sizeof(__nv_bfloat16)),
               "cudaMalloc(side attention scratch)", err))
    return false;
  _vt_side_elems = need;
  return true;
}

bool CudaOps::reserve_sage(int tq, int tk, int heads, int head_dim, std::string* err)
{
  const ltx::SageScratch need = ltx::sage_scratch_need(tq, tk, heads, head_dim);
  auto grow = [&](void** ptr, size_t* cap, size_t n, size_t elt) {
    if (n <= *cap) return true;
    cudaFree(*ptr);
    *ptr = nullptr;
    *cap = 0;
    if (!cuda_ok(cudaMalloc(ptr, n * elt), "cudaMalloc(sage scratch)", err)) return false;
    *cap = n;
    return true;
  };
  if (!grow((void**)&_sb.qi8, &_sb.cap.qi8, need.qi8, 1) ||
      !grow((void**)&_sb.ki8, &_sb.cap.ki8, need.ki8, 1) ||
      !grow((void**)&_sb.scales, &_sb.cap.scales, need.scales, sizeof(float)) ||
      !grow((void**)&_sb.mean, &_sb.cap.mean, need.mean, sizeof(float)))
    return false;
  if (!reserve_attention(tk, heads * head_dim, err)) return false;
  _sb.vt = _vt;
  _sb.cap.vt = _vt_elems;
  return true;
}

cudaStream_t CudaOps::aux_stream(std::string* err)
{
  if (_aux != nullptr) return _aux;
  int lo = 0, hi = 0;
  cudaDeviceGetStreamPriorityRange(&lo, &hi);
  if (!cuda_ok(cudaStreamCreateWithPriority(&_aux, cudaStreamNonBlocking, hi), "aux stream", err))
    return nullptr;
  for (cudaEvent_t& e : _ev)
    if (!cuda_ok(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "aux events", err))
      return nullptr;
  return _aux;
}

cudaStream_t CudaOps::comm_stream(std::string* err)
{
  if (_cstream != nullptr) return _cstream;
  if (!cuda_ok(cudaStreamCreateWithFlags(&_cstream, cudaStreamNonBlocking), "comm stream", err))
    return nullptr;
  for (cudaEvent_t& e : _cev)
    if (!cuda_ok(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "comm events", err))
      return nullptr;
  return _cstream;
}

bool CudaOps::cfork(cudaStream_t from, cudaStream_t to, int slot, std::string* err)
{
  return cuda_ok(cudaEventRecord(_cev[slot], from), "event record", err) &&
         cuda_ok(cudaStreamWaitEvent(to, _cev[slot], 0), "stream wait", err);
}

bool CudaOps::crecord(cudaStream_t from, int slot, std::string* err)
{
  return cuda_ok(cudaEventRecord(_cev[slot], from), "event record", err);
}

bool CudaOps::cwait(cudaStream_t to, int slot, std::string* err)
{
  return cuda_ok(cudaStreamWaitEvent(to, _cev[slot], 0), "stream wait", err);
}

bool CudaOps::fork(cudaStream_t from, cudaStream_t to, int slot, std::string* err)
{
  return cuda_ok(cudaEventRecord(_ev[slot], from), "event record", err) &&
         cuda_ok(cudaStreamWaitEvent(to, _ev[slot], 0), "stream wait", err);
}

bool CudaOps::audio_side_ok(int tokens, int text_tokens, int heads, int head_dim,
                            int layer) const
{
  static const bool off = [] {
    const char* e = getenv("LTX25_SIDE_STREAM");
    return e != nullptr && e[0] == '0';
  }();
  if (off) return false;
  const int m = std::max(tokens, text_tokens);
  if (m >= LTX_DEQUANT_MIN_M || (_i8 && m >= 1024) || _route == Route::DequantOnce) return false;
  if (sage_for(layer, head_dim)) return false;
  // only 64-wide heads (this model's audio stream) go to the side stream
  if (head_dim == 128) return false;
  return ltx::attention_tc_splits(tokens, tokens, heads) == 1 &&
         ltx::attention_tc_splits(tokens, text_tokens, heads) == 1;
}

bool CudaOps::reserve_split(int tq, int tk, int heads, int head_dim, std::string* err)
{
  const size_t part = ltx::attention_tc_part(tq, tk, heads, head_dim);
  if (part <= _part_elems) return true;
  cudaFree(_part);
  _part = nullptr;
  _part_elems = 0;
  if (!cuda_ok(cudaMalloc(&_part, part * sizeof(float)), "cudaMalloc(attention partials)", err))
    return false;
  _part_elems = part;
  return true;
}

bool CudaOps::attention_reads_vt(cudaStream_t s, int tq, int tk, int heads, int head_dim,
                                 int layer) const
{
  const bool on_side = _aux != nullptr && s == _aux;
  const int splits = ltx::attention_tc_splits(tq, tk, heads);
  return _vt_out && !on_side && _attn_mode == 1 && !sage_for(layer, head_dim) &&
         (head_dim == 128 || (head_dim == 64 && (splits > 1 || _attn64_tc)));
}

__nv_bfloat16* CudaOps::vt_scratch(int tk, int width, std::string* err)
{
  return reserve_attention(tk, width, err) ? _vt : nullptr;
}

bool CudaOps::attention(cudaStream_t s, const __nv_bfloat16* q, int ldq,
                        const __nv_bfloat16* k, int ldk, const __nv_bfloat16* v,
                        int ldv, __nv_bfloat16* o, int ldo, const __nv_bfloat16* gate,
                        int ldg, int tq, int tk, int heads, int head_dim,
                        std::string* err, int layer, const __nv_bfloat16* vt_ready)
{
  int rc;
  const bool on_side = _aux != nullptr && s == _aux;
  const int splits = ltx::attention_tc_splits(tq, tk, heads);
  // tcgen05 for head_dim 128 and the key-split 64-wide attentions (the
  // unsplit 64-wide ones too with LTX25_ATTN64=tc); the key-split form needs
  // the main stream's partials scratch
  const bool tc = _attn_mode == 1 && !(on_side && splits > 1) &&
                  (head_dim == 128 || (head_dim == 64 && (splits > 1 || _attn64_tc)));
  const bool sage = sage_for(layer, head_dim);
  if (vt_ready != nullptr && (sage || !tc || on_side)) {
    // the producer left V out of its buffer: only the path that reads V^T may run
    if (err) *err = "attention: a ready V^T was given to a path that reads V";
    return false;
  }
  if (sage) {
    if (!reserve_sage(tq, tk, heads, head_dim, err)) return false;
    rc = ltx::launch_sage_tc(q, ldq, k, ldk, v, ldv, _sb, o, ldo, gate, ldg, tq, tk, heads,
                             head_dim, _err_word, s);
  } else if (tc) {
    // tcgen05 kernel.  On the side (audio) stream, beside the video stream,
    // its V^T copy has a buffer of its own; the key-split form (partials
    // scratch) stays on the main stream.
    const bool side = on_side;
    __nv_bfloat16* vt = nullptr;
    size_t vt_elems = 0;
    if (side) {
      if (!reserve_attention_side(tk, heads * head_dim, err)) return false;
      vt = _vt_side;
      vt_elems = _vt_side_elems;
    } else {
      if (!reserve_attention(tk, heads * head_dim, err)) return false;
      if (!reserve_split(tq, tk, heads, head_dim, err)) return false;
      vt = vt_ready != nullptr ? const_cast<__nv_bfloat16*>(vt_ready) : _vt;
      vt_elems = vt_ready != nullptr ? ltx::attention_tc_scratch(tk, heads, head_dim) : _vt_elems;
    }
    rc = ltx::launch_attention_tc(q, ldq, k, ldk, v, ldv, vt, vt_elems, o, ldo, gate, ldg,
                                  tq, tk, heads, head_dim, _err_word, s,
                                  side ? nullptr : _part, side ? 0 : _part_elems,
                                  vt_ready != nullptr);
  } else {
    rc = ltx::launch_attention(q, ldq, k, ldk, v, ldv, o, ldo, gate, ldg, tq, tk, heads,
                               head_dim, s);
  }
  if (rc == -2) {
    if (err) *err = "attention shape: head_dim must be 64 or 128, strides % 8, 16-byte aligned";
    return false;
  }
  if (rc != 0) {
    if (err) *err = "attention launch failed";
    return false;
  }
  return true;
}

int CudaOps::check(cudaStream_t s, std::string* err) const
{
  int h = 0;
  if (!cuda_ok(cudaMemcpyAsync(&h, _err_word, sizeof(int), cudaMemcpyDeviceToHost, s), "check", err))
    return -1;
  if (!cuda_ok(cudaStreamSynchronize(s), "check", err)) return -1;
  if (h != 0) {
    cudaMemsetAsync(_err_word, 0, sizeof(int), s);
    cudaStreamSynchronize(s);
    if (err) *err = "a kernel gave up on a bounded wait (code " + std::to_string(h) + ")";
  }
  return h;
}

// ---- upload ---------------------------------------------------------------

bool upload_qweight(const CudaOps& ops, const uint32_t* codes,
                    const void* scales, const void* biases, int sb_dtype,
                    int N, int K, int bits, int group, bool on_device,
                    QWeight* out, std::string* err)
{
  if (codes == nullptr || scales == nullptr || biases == nullptr || out == nullptr) {
    if (err) *err = "upload: null tensor";
    return false;
  }
  if (bits != 8 || group != 64) {
    if (err)
      *err = "upload: w" + std::to_string(bits) + "g" + std::to_string(group) +
             " is not run by this build (only the w8g64 pack)";
    return false;
  }
  if (N <= 0 || K <= 0 || K % 64 != 0 || N % 4 != 0) {
    if (err) *err = "upload: need K % 64 == 0 and N % 4 == 0, got N=" +
                    std::to_string(N) + " K=" + std::to_string(K);
    return false;
  }
  if (sb_dtype < 0 || sb_dtype > 2) {
    if (err) *err = "upload: unknown scale dtype";
    return false;
  }
  const int G = K / 64;
  const size_t sb_elt = sb_dtype == 2 ? 4 : 2;
  QWeight w;
  w.N = N;
  w.K = K;
  w.bits = 8;
  w.group = 64;
  w.quantized = true;
  w.device = ops.device();
  const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  void* d_s = nullptr;
  void* d_b = nullptr;
  bool ok = cuda_ok(cudaMalloc(&w.codes, (size_t)N * K), "cudaMalloc(codes)", err) &&
            cuda_ok(cudaMalloc(&w.sz, (size_t)N * G * 4), "cudaMalloc(sz)", err) &&
            cuda_ok(cudaMemcpy(w.codes, codes, (size_t)N * K, kind), "upload codes", err);
  if (ok && !on_device) {
    ok = cuda_ok(cudaMalloc(&d_s, (size_t)N * G * sb_elt), "cudaMalloc", err) &&
         cuda_ok(cudaMalloc(&d_b, (size_t)N * G * sb_elt), "cudaMalloc", err) &&
         cuda_ok(cudaMemcpy(d_s, scales, (size_t)N * G * sb_elt, kind), "upload scales", err) &&
         cuda_ok(cudaMemcpy(d_b, biases, (size_t)N * G * sb_elt, kind), "upload zero-points", err);
  }
  if (ok) {
    ok = ltx::launch_pack_sz(on_device ? scales : d_s, on_device ? biases : d_b,
                             sb_dtype, N, G, w.sz, nullptr) == 0 &&
         cuda_ok(cudaDeviceSynchronize(), "pack scales", err);
  }
  cudaFree(d_s);
  cudaFree(d_b);
  if (!ok) {
    free_qweight(&w);
    return false;
  }
  *out = w;
  return true;
}

bool upload_dweight(const CudaOps& ops, const uint16_t* wsrc, int N, int K,
                    bool on_device, QWeight* out, std::string* err)
{
  if (wsrc == nullptr || out == nullptr) {
    if (err) *err = "upload: null tensor";
    return false;
  }
  if (N <= 0 || K <= 0 || K % 64 != 0 || N % 2 != 0) {
    if (err) *err = "upload: dense weight needs K % 64 == 0 and N % 2 == 0";
    return false;
  }
  QWeight w;
  w.N = N;
  w.K = K;
  w.quantized = false;
  w.device = ops.device();
  const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (!cuda_ok(cudaMalloc(&w.w, (size_t)N * K * 2), "cudaMalloc(w)", err) ||
      !cuda_ok(cudaMemcpy(w.w, wsrc, (size_t)N * K * 2, kind), "upload w", err)) {
    free_qweight(&w);
    return false;
  }
  *out = w;
  return true;
}

bool upload_lora(const CudaOps& ops, const uint16_t* a, const uint16_t* b, int rank, int k,
                 int n, float scale, bool on_device, LoraPair* out, std::string* err)
{
  if (a == nullptr || b == nullptr || out == nullptr) {
    if (err) *err = "lora upload: null tensor";
    return false;
  }
  if (rank <= 0 || k <= 0 || n <= 0 || k % 8 != 0 || n % 2 != 0) {
    if (err)
      *err = "lora upload shape: rank " + std::to_string(rank) + ", k " + std::to_string(k) +
             " (multiple of 8), n " + std::to_string(n) + " (even)";
    return false;
  }
  LoraPair p;
  p.rank = rank;
  p.r8 = (rank + 7) / 8 * 8;
  p.k = k;
  p.n = n;
  p.device = ops.device();
  const cudaMemcpyKind kind = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  const size_t na = (size_t)p.r8 * k, nb = (size_t)n * p.r8;
  bool ok = cuda_ok(cudaMalloc(&p.a, na * 2), "cudaMalloc(lora a)", err) &&
            cuda_ok(cudaMalloc(&p.b, nb * 2), "cudaMalloc(lora b)", err) &&
            cuda_ok(cudaMemset(p.a, 0, na * 2), "lora a", err) &&
            cuda_ok(cudaMemset(p.b, 0, nb * 2), "lora b", err) &&
            cuda_ok(cudaMemcpy(p.a, a, (size_t)rank * k * 2, kind), "upload lora a", err) &&
            cuda_ok(cudaMemcpy2D(p.b, (size_t)p.r8 * 2, b, (size_t)rank * 2, (size_t)rank * 2, n,
                                 kind),
                    "upload lora b", err);
  if (ok && scale != 1.0f) {
    ok = ltx::launch_scale_bf16(p.a, p.a, scale, (size_t)rank * k, nullptr) == 0 &&
         cuda_ok(cudaDeviceSynchronize(), "lora scale", err);
    if (!ok && err && err->empty()) *err = "lora scale launch failed";
  }
  if (!ok) {
    free_lora(&p);
    return false;
  }
  *out = p;
  return true;
}

void free_lora(LoraPair* p)
{
  if (p == nullptr) return;
  cudaFree(p->a);
  cudaFree(p->b);
  *p = LoraPair{};
}

void free_qweight(QWeight* w)
{
  if (w == nullptr) return;
  cudaFree(w->codes);
  cudaFree(w->sz);
  cudaFree(w->w);
  cudaFree(w->wq);
  cudaFree(w->sw);
  *w = QWeight{};
}

}  // namespace ltx25
