// ltx25-adaln.cc -- see ltx25-adaln.h.
#include "ltx25-adaln.h"
#include "ltx25-threads.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace ltx25 {

namespace {

float bf16f(uint16_t h)
{
  const uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// sum_i x[i] w[i] for one weight row: x f64 (widened from f32), w bf16
// bits, f64 products and sums as sixteen interleaved partial sums (element i
// into sum i % 16) added pairwise at the end.  The product of an f32 value
// and a bf16 value has at most 32 significant bits, so it is exact in f64:
// the vector form's fused multiply-add rounds exactly like the scalar
// multiply-then-add, and both forms return the same bits.
constexpr int kParts = 16;

double combine(const double (&s)[kParts])
{
  double t[8];
  for (int j = 0; j < 8; ++j) t[j] = s[j] + s[j + 8];
  return ((t[0] + t[4]) + (t[2] + t[6])) + ((t[1] + t[5]) + (t[3] + t[7]));
}

double dot_scalar(const double* x, const uint16_t* w, int n)
{
  double s[kParts] = {};
  int i = 0;
  for (; i + kParts <= n; i += kParts)
    for (int j = 0; j < kParts; ++j) s[j] += x[i + j] * (double)bf16f(w[i + j]);
  for (int j = 0; i + j < n; ++j) s[j] += x[i + j] * (double)bf16f(w[i + j]);
  return combine(s);
}

#if defined(__x86_64__)
__attribute__((target("avx2,fma"))) double dot_avx2(const double* x, const uint16_t* w,
                                                    int n)
{
  // v[q] holds sums 4q .. 4q + 3: four independent multiply-add chains
  __m256d v[4] = {_mm256_setzero_pd(), _mm256_setzero_pd(), _mm256_setzero_pd(),
                  _mm256_setzero_pd()};
  int i = 0;
  for (; i + kParts <= n; i += kParts) {
    for (int h = 0; h < 2; ++h) {
      // eight bf16 -> f32 (the bits in the upper half) -> two f64 quads
      const __m256 f = _mm256_castsi256_ps(_mm256_slli_epi32(
          _mm256_cvtepu16_epi32(
              _mm_loadu_si128(reinterpret_cast<const __m128i*>(w + i + 8 * h))),
          16));
      v[2 * h] = _mm256_fmadd_pd(_mm256_loadu_pd(x + i + 8 * h),
                                 _mm256_cvtps_pd(_mm256_castps256_ps128(f)), v[2 * h]);
      v[2 * h + 1] = _mm256_fmadd_pd(_mm256_loadu_pd(x + i + 8 * h + 4),
                                     _mm256_cvtps_pd(_mm256_extractf128_ps(f, 1)),
                                     v[2 * h + 1]);
    }
  }
  double s[kParts];
  for (int q = 0; q < 4; ++q) _mm256_storeu_pd(s + 4 * q, v[q]);
  for (int j = 0; i + j < n; ++j) s[j] += x[i + j] * (double)bf16f(w[i + j]);
  return combine(s);
}
#endif

using DotFn = double (*)(const double*, const uint16_t*, int);

// The vector form where the host has AVX2 + FMA, unless LTX25_HOST_SIMD=0.
DotFn dot_fn()
{
  static const DotFn fn = [] {
    const char* e = std::getenv("LTX25_HOST_SIMD");
    const bool off = e != nullptr && e[0] == '0';
#if defined(__x86_64__)
    if (!off && __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma"))
      return static_cast<DotFn>(dot_avx2);
#endif
    (void)off;
    return static_cast<DotFn>(dot_scalar);
  }();
  return fn;
}

// y[o] = b[o] + sum_i x[i] w[o][i] for rows [o0, o1), f64 products and sums
// stored f32 (gemv_host_, src/ltx25-dit.cc:51-67): each row summed by the
// dot above in a fixed order, then the bias, so the result does not depend
// on how the rows are split over threads.
void gemv_rows(const double* xd, const std::vector<uint16_t>& w,
               const std::vector<uint16_t>& b, int in_dim, int o0, int o1, float* y)
{
  const DotFn dot = dot_fn();
  for (int o = o0; o < o1; ++o) {
    const double acc = dot(xd, w.data() + (size_t)o * in_dim, in_dim);
    y[o] = (float)((b.empty() ? 0.0 : (double)bf16f(b[(size_t)o])) + acc);
  }
}

float silu1(float z) { return z / (1.0f + std::exp(-z)); }

}  // namespace

void timestep_sinusoid(double t, int channels, float* out)
{
  const int half = channels / 2;
  const double log_period = std::log(10000.0);
  for (int i = 0; i < half; ++i) {
    const double a = t * std::exp(-log_period * (double)i / (double)half);
    out[i] = (float)std::cos(a);
    out[half + i] = (float)std::sin(a);
  }
}

void adaln_run_many(const AdaLNChain* const* chains, const double* t, float* const* out,
                    float* const* embedded, int count, int threads)
{
  if (count <= 0) return;
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  threads = std::min(threads, 64);
  // Per chain: the sinusoid and the three linears' inputs in f64 (SiLU
  // applied), and h1 / h2 in f32 (h2 is `embedded`).  Every stage's rows,
  // over all chains, are split evenly over the threads; the stages run one
  // after another (each reads the whole previous output of its own chain).
  struct Work {
    const AdaLNChain* c;
    std::vector<double> x1, x2, x3;
    std::vector<float> h1, h2;
  };
  std::vector<Work> w((size_t)count);
  long long rows[3] = {0, 0, 0};
  for (int i = 0; i < count; ++i) {
    Work& k = w[(size_t)i];
    k.c = chains[i];
    std::vector<float> proj(256);
    timestep_sinusoid(t[i], 256, proj.data());
    k.x1.assign(proj.begin(), proj.end());
    k.x2.resize((size_t)k.c->dim);
    k.x3.resize((size_t)k.c->dim);
    k.h1.resize((size_t)k.c->dim);
    k.h2.resize((size_t)k.c->dim);
    rows[0] += k.c->dim;
    rows[1] += k.c->dim;
    rows[2] += k.c->out_dim;
  }
  const long long most = std::max(rows[0], rows[2]);
  const int nt = (int)std::max(1LL, std::min((long long)threads, most / 64));
  // rows [g0, g1) of stage `stage`, numbered across the chains in order
  auto stage_rows = [&](int stage, long long g0, long long g1) {
    long long base = 0;
    for (Work& k : w) {
      const int n = stage == 2 ? k.c->out_dim : k.c->dim;
      const long long lo = std::max(g0, base), hi = std::min(g1, base + n);
      if (lo < hi) {
        const int a = (int)(lo - base), b = (int)(hi - base);
        if (stage == 0) {
          gemv_rows(k.x1.data(), k.c->w1, k.c->b1, 256, a, b, k.h1.data());
          for (int o = a; o < b; ++o) k.x2[(size_t)o] = (double)silu1(k.h1[(size_t)o]);
        } else if (stage == 1) {
          gemv_rows(k.x2.data(), k.c->w2, k.c->b2, k.c->dim, a, b, k.h2.data());
          for (int o = a; o < b; ++o) k.x3[(size_t)o] = (double)silu1(k.h2[(size_t)o]);
        } else {
          gemv_rows(k.x3.data(), k.c->w3, k.c->b3, k.c->dim, a, b, out[&k - w.data()]);
        }
      }
      base += n;
    }
  };
  for (int stage = 0; stage < 3; ++stage)
    run_parts(nt, [&](int k) {
      stage_rows(stage, rows[stage] * k / nt, rows[stage] * (k + 1) / nt);
    });
  for (int i = 0; i < count; ++i)
    if (embedded != nullptr && embedded[i] != nullptr)
      std::memcpy(embedded[i], w[(size_t)i].h2.data(), (size_t)w[(size_t)i].c->dim * 4);
}

void adaln_run(const AdaLNChain& c, double t, float* out, float* embedded, int threads)
{
  const AdaLNChain* cs[1] = {&c};
  float* outs[1] = {out};
  float* embs[1] = {embedded};
  adaln_run_many(cs, &t, outs, embs, 1, threads);
}

}  // namespace ltx25
