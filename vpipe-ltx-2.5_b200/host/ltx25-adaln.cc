// ltx25-adaln.cc -- see ltx25-adaln.h.
#include "ltx25-adaln.h"

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <mutex>
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

// A reusable barrier for one chain's threads (C++17 has no std::barrier).
class StageBarrier {
public:
  explicit StageBarrier(int n) : _n(n) {}
  void wait()
  {
    std::unique_lock<std::mutex> lk(_m);
    const unsigned gen = _gen;
    if (++_count == _n) {
      _count = 0;
      ++_gen;
      _cv.notify_all();
      return;
    }
    _cv.wait(lk, [&] { return _gen != gen; });
  }

private:
  std::mutex _m;
  std::condition_variable _cv;
  int _n;
  int _count = 0;
  unsigned _gen = 0;
};

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

void adaln_run(const AdaLNChain& c, double t, float* out, float* embedded, int threads)
{
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  threads = std::min(threads, 64);
  const int dim = c.dim, od = c.out_dim;
  std::vector<float> proj(256);
  timestep_sinusoid(t, 256, proj.data());
  const std::vector<double> x1(proj.begin(), proj.end());
  // The three linears' inputs in f64 (silu applied), and h2 itself for
  // `embedded`.  Each thread owns a row range of every stage; the stages
  // are separated by a barrier, since each reads the whole previous output.
  std::vector<double> x2((size_t)dim), x3((size_t)dim);
  std::vector<float> h1((size_t)dim), h2((size_t)dim);
  const int nt = std::max(1, std::min(threads, std::max(dim, od) / 64));
  StageBarrier bar(nt);
  auto part = [](int n, int k, int parts) { return (int)((long long)n * k / parts); };
  auto work = [&](int k) {
    int a = part(dim, k, nt), b = part(dim, k + 1, nt);
    gemv_rows(x1.data(), c.w1, c.b1, 256, a, b, h1.data());
    for (int o = a; o < b; ++o) x2[(size_t)o] = (double)silu1(h1[(size_t)o]);
    bar.wait();
    gemv_rows(x2.data(), c.w2, c.b2, dim, a, b, h2.data());
    for (int o = a; o < b; ++o) x3[(size_t)o] = (double)silu1(h2[(size_t)o]);
    bar.wait();
    gemv_rows(x3.data(), c.w3, c.b3, dim, part(od, k, nt), part(od, k + 1, nt), out);
  };
  if (nt == 1) {
    work(0);
  } else {
    std::vector<std::thread> pool;
    pool.reserve((size_t)nt - 1);
    for (int k = 1; k < nt; ++k) pool.emplace_back(work, k);
    work(0);
    for (auto& th : pool) th.join();
  }
  if (embedded != nullptr) std::memcpy(embedded, h2.data(), (size_t)dim * 4);
}

}  // namespace ltx25
