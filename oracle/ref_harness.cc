// ref_harness.cc -- C entry points over the REFERENCE's own CPU code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file against the
// reference tree (-I<reference>/src): it #includes the reference's
// src/ltx25-block-ref.cc so the file-static `linear_` (block-ref.cc:13-29)
// is reachable, links src/ltx25-rope.cc unmodified, and includes the packer
// functions that extract_ref_packer.py lifted verbatim from
// tests/ltx25-qlinear-test.cc:66-141.  The result, oracle/_ref/
// libref_oracle.so, pins the restatement in ltx_oracle.c / block_np.py and
// serves as the reference CPU baseline.  Nothing in the product loads it.

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <unordered_map>
#include <vector>

#include "ltx25-block-ref.cc"   // reference source, compiled as-is
#include "ltx25-rope.h"

namespace refpack {
#include "ref_packer.inc"        // reference test helpers, verbatim
}  // namespace refpack

// The host adaLN chain's helpers of src/ltx25-dit.cc:30-135, verbatim, over
// shims of the two vpipe types they read (a bf16 buffer's contents() /
// empty(), an adapter pair's widths and buffers).
namespace refdit {
struct SharedBuffer {
  const void* p = nullptr;
  const void* contents() const { return p; }
  bool empty() const { return p == nullptr; }
};
struct LoraPair {
  SharedBuffer a, b;
  int rank = 0, k = 0, n = 0;
  bool valid() const { return rank > 0 && a.p != nullptr && b.p != nullptr; }
};
#include "ref_dit.inc"
}  // namespace refdit

// The adapter test's CPU fold (tests/ltx25-lora-apply-test.cc:330-366) and
// the bf16 rounding src/ltx25-lora.cc's scaled_ folds the factor with
// (lines 27-47), verbatim.
namespace reflora {
#include "ref_lora_test.inc"
#include "ref_lora_bits.inc"
}  // namespace reflora

namespace {

void put_err(char* err, int errlen, const std::string& m)
{
  if (err != nullptr && errlen > 0) {
    std::snprintf(err, (size_t)errlen, "%s", m.c_str());
  }
}

struct BlockHandle {
  std::unordered_map<std::string, ltx25::NamedTensor> tensors;
  ltx25::BlockWeights w;
  bool loaded = false;
};

ltx25::RopeTable table_from(const float* c, const float* s, int heads,
                            int tokens, int half)
{
  ltx25::RopeTable t;
  t.heads = heads;
  t.tokens = tokens;
  t.half = half;
  t.cos.assign(c, c + t.size());
  t.sin.assign(s, s + t.size());
  return t;
}

void table_out(const ltx25::RopeTable& t, float* c, float* s)
{
  std::memcpy(c, t.cos.data(), t.size() * sizeof(float));
  std::memcpy(s, t.sin.data(), t.size() * sizeof(float));
}

}  // namespace

extern "C" {

// One stream's inputs, mirrored by ctypes in oracle/ref.py.
struct ref_stream {
  float* x;
  int tokens;
  int dim;
  const float* ctx;
  int text_tokens;
  const float* ts;
  int ts_n;
  const float* css;
  int css_n;
  const float* cg;
  int cg_n;
  const float* pts;
  int pts_n;
  const float* pe_cos;
  const float* pe_sin;
  int pe_heads;
  int pe_half;
  const float* cpe_cos;
  const float* cpe_sin;
  int cpe_heads;
  int cpe_half;
  int present;
};

int ref_pack(const float* w, int N, int K, int bits, int group,
             uint32_t* codes, uint16_t* scales, uint16_t* biases, float* deq)
{
  std::vector<float> wv(w, w + (size_t)N * K);
  std::vector<std::uint32_t> c;
  std::vector<std::uint16_t> s, b;
  std::vector<float> d;
  refpack::quantize(wv, N, K, bits, group, c, s, b, d);
  std::memcpy(codes, c.data(), c.size() * 4);
  std::memcpy(scales, s.data(), s.size() * 2);
  std::memcpy(biases, b.data(), b.size() * 2);
  if (deq != nullptr) std::memcpy(deq, d.data(), d.size() * 4);
  return 0;
}

uint16_t ref_to_bf16(float v) { return refpack::to_bf16(v); }

void ref_linear(const float* x, const float* w, const float* b, float* out,
                int M, int K, int N)
{
  ltx25::Mat xm, wm, om;
  xm.rows = M; xm.cols = K; xm.v.assign(x, x + (size_t)M * K);
  wm.rows = N; wm.cols = K; wm.v.assign(w, w + (size_t)N * K);
  std::vector<float> bv;
  if (b != nullptr) bv.assign(b, b + N);
  ltx25::linear_(xm, wm, bv, om);
  std::memcpy(out, om.v.data(), (size_t)M * N * sizeof(float));
}

void* ref_block_new(void) { return new BlockHandle(); }
void ref_block_free(void* h) { delete static_cast<BlockHandle*>(h); }

int ref_block_put(void* h, const char* name, const float* data, int rows,
                  int cols)
{
  auto* bh = static_cast<BlockHandle*>(h);
  ltx25::NamedTensor t;
  const size_t n = (size_t)rows * (size_t)(cols > 0 ? cols : 1);
  t.data.assign(data, data + n);
  if (cols > 0) t.shape = {rows, cols};
  else t.shape = {rows};
  bh->tensors[name] = std::move(t);
  return 0;
}

int ref_block_load(void* h, int vdim, int vheads, int adim, int aheads,
                   char* err, int errlen)
{
  auto* bh = static_cast<BlockHandle*>(h);
  std::string e;
  if (!ltx25::load_block_weights(bh->tensors, vdim, vheads, adim, aheads,
                                 bh->w, &e)) {
    put_err(err, errlen, e);
    return -1;
  }
  bh->loaded = true;
  return 0;
}

int ref_block_forward(void* h, ref_stream* v, ref_stream* a, char* err,
                      int errlen)
{
  auto* bh = static_cast<BlockHandle*>(h);
  if (!bh->loaded) {
    put_err(err, errlen, "weights not loaded");
    return -1;
  }
  ltx25::RopeTable tabs[4];
  ltx25::StreamInput in[2];
  ref_stream* ss[2] = {v, a};
  for (int i = 0; i < 2; ++i) {
    ref_stream* s = ss[i];
    ltx25::StreamInput& o = in[i];
    o.present = s->present != 0;
    o.x.rows = s->tokens;
    o.x.cols = s->dim;
    o.x.v.assign(s->x, s->x + (size_t)s->tokens * s->dim);
    o.context.rows = s->text_tokens;
    o.context.cols = s->dim;
    if (s->ctx != nullptr)
      o.context.v.assign(s->ctx, s->ctx + (size_t)s->text_tokens * s->dim);
    if (s->ts) o.timesteps.assign(s->ts, s->ts + s->ts_n);
    if (s->css) o.cross_scale_shift.assign(s->css, s->css + s->css_n);
    if (s->cg) o.cross_gate.assign(s->cg, s->cg + s->cg_n);
    if (s->pts) o.prompt_timestep.assign(s->pts, s->pts + s->pts_n);
    if (s->pe_cos != nullptr) {
      tabs[2 * i] = table_from(s->pe_cos, s->pe_sin, s->pe_heads, s->tokens,
                               s->pe_half);
      o.pe = &tabs[2 * i];
    }
    if (s->cpe_cos != nullptr) {
      tabs[2 * i + 1] = table_from(s->cpe_cos, s->cpe_sin, s->cpe_heads,
                                   s->tokens, s->cpe_half);
      o.cross_pe = &tabs[2 * i + 1];
    }
  }
  std::string e;
  if (!ltx25::block_forward(bh->w, in[0], in[1], &e)) {
    put_err(err, errlen, e);
    return -1;
  }
  for (int i = 0; i < 2; ++i) {
    if (ss[i]->present) {
      std::memcpy(ss[i]->x, in[i].x.v.data(), in[i].x.v.size() * 4);
    }
  }
  return 0;
}

// ---- RoPE builders (src/ltx25-rope.cc) ----------------------------------

int ref_build_video_rope(int frames, int height, int width,
                         const int* max_pos3, int inner_dim, int heads,
                         int scale_t, int scale_h, int scale_w, double fps,
                         int causal_fix, float* cos_out, float* sin_out)
{
  ltx25::RopeGeometry geo{scale_t, scale_h, scale_w, fps, causal_fix != 0};
  const ltx25::RopeTable t = ltx25::build_video_rope(
      frames, height, width, {max_pos3[0], max_pos3[1], max_pos3[2]},
      inner_dim, heads, geo);
  if (t.size() == 0) return -1;
  table_out(t, cos_out, sin_out);
  return 0;
}

int ref_build_audio_rope(int tokens, int max_pos, int inner_dim, int heads,
                         float* cos_out, float* sin_out)
{
  const ltx25::RopeTable t =
      ltx25::build_audio_rope(tokens, {max_pos}, inner_dim, heads);
  if (t.size() == 0) return -1;
  table_out(t, cos_out, sin_out);
  return 0;
}

int ref_build_index_rope(int tokens, int max_pos, int inner_dim, int heads,
                         float* cos_out, float* sin_out)
{
  const ltx25::RopeTable t =
      ltx25::build_index_rope(tokens, {max_pos}, inner_dim, heads);
  if (t.size() == 0) return -1;
  table_out(t, cos_out, sin_out);
  return 0;
}

int ref_build_cross_rope(const double* starts, const double* ends, int n,
                         int max_pos, int inner_dim, int heads,
                         float* cos_out, float* sin_out)
{
  std::vector<double> s(starts, starts + n), e(ends, ends + n);
  const ltx25::RopeTable t =
      ltx25::build_cross_rope(s, e, max_pos, inner_dim, heads);
  if (t.size() == 0) return -1;
  table_out(t, cos_out, sin_out);
  return 0;
}

void ref_video_time_seconds(int frames, int scale_t, double fps,
                            int causal_fix, double* out)
{
  ltx25::RopeGeometry geo{scale_t, 32, 32, fps, causal_fix != 0};
  const std::vector<double> v = ltx25::video_time_seconds(frames, geo);
  std::memcpy(out, v.data(), v.size() * sizeof(double));
}

void ref_audio_time_seconds(int tokens, double* out)
{
  const std::vector<double> v = ltx25::audio_time_seconds(tokens);
  std::memcpy(out, v.data(), v.size() * sizeof(double));
}

// Ltx25Dit::adaln_ (src/ltx25-dit.cc:137-160) without adapters, driven
// through the reference's own helpers: sinusoid(t) -> linear_1 -> SiLU ->
// linear_2 (= embedded) -> SiLU -> linear.  Weights and biases bf16 bits
// ([out][in]); bias pointers may be null.
int ref_adaln_chain(double t, const uint16_t* w1, const uint16_t* b1, const uint16_t* w2,
                    const uint16_t* b2, const uint16_t* w3, const uint16_t* b3, int dim,
                    int out_dim, float* out, float* embedded)
{
  using refdit::SharedBuffer;
  const SharedBuffer W1{w1}, B1{b1}, W2{w2}, B2{b2}, W3{w3}, B3{b3};
  std::vector<float> proj = refdit::timestep_sinusoid_(t, 256);
  std::vector<float> h1, h2, o;
  refdit::gemv_host_(proj, W1, B1, 256, dim, h1);
  refdit::silu_(h1);
  refdit::gemv_host_(h1, W2, B2, dim, dim, h2);
  if (embedded != nullptr) std::memcpy(embedded, h2.data(), h2.size() * sizeof(float));
  std::vector<float> act = h2;
  refdit::silu_(act);
  refdit::gemv_host_(act, W3, B3, dim, out_dim, o);
  std::memcpy(out, o.data(), o.size() * sizeof(float));
  return 0;
}

// y[n] += B (A x): the reference's host adapter GEMV (lora_gemv_host_,
// src/ltx25-dit.cc:77-103); a [rank][k], b [n][rank] bf16 bits.
void ref_lora_gemv(const float* x, const uint16_t* a, const uint16_t* b, int rank, int k,
                   int n, float* y)
{
  refdit::LoraPair p;
  p.a.p = a;
  p.b.p = b;
  p.rank = rank;
  p.k = k;
  p.n = n;
  std::vector<float> xv(x, x + k), yv(y, y + n);
  refdit::lora_gemv_host_(xv, p, yv);
  std::memcpy(y, yv.data(), (size_t)n * sizeof(float));
}

// W[n][k] += B A with the adapter test's fold (f32 values).
void ref_lora_fold(float* w, const float* a, const float* b, int rank, int k, int n)
{
  ltx25::Mat m;
  m.rows = n;
  m.cols = k;
  m.v.assign(w, w + (size_t)n * k);
  reflora::HostPair p;
  p.a.assign(a, a + (size_t)rank * k);
  p.b.assign(b, b + (size_t)n * rank);
  p.rank = rank;
  p.k = k;
  p.n = n;
  reflora::fold(m, p);
  std::memcpy(w, m.v.data(), (size_t)n * k * sizeof(float));
}

// The factor folded into A as scaled_ does it (src/ltx25-lora.cc:63):
// d = f32_to_bf16_(bf16_to_f32_(s) * (float)factor), element by element.
void ref_lora_scale(const uint16_t* s, uint16_t* d, size_t n, double factor)
{
  for (size_t i = 0; i < n; ++i)
    d[i] = reflora::f32_to_bf16_(reflora::bf16_to_f32_(s[i]) * (float)factor);
}

}  // extern "C"
