// ltx25-adaln.cc -- see ltx25-adaln.h.
#include "ltx25-adaln.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>

namespace ltx25 {

namespace {

float bf16f(uint16_t h)
{
  const uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// y[o] = b[o] + sum_i x[i] w[o][i], f64 sums stored f32 (gemv_host_,
// src/ltx25-dit.cc:51-67); rows split over threads, each row's sum in
// index order on one thread.
void gemv(const std::vector<float>& x, const std::vector<uint16_t>& w,
          const std::vector<uint16_t>& b, int in_dim, int out_dim, float* y, int threads)
{
  auto rows = [&](int o0, int o1) {
    for (int o = o0; o < o1; ++o) {
      const uint16_t* row = w.data() + (size_t)o * in_dim;
      double acc = b.empty() ? 0.0 : (double)bf16f(b[(size_t)o]);
      for (int i = 0; i < in_dim; ++i) acc += (double)x[(size_t)i] * (double)bf16f(row[i]);
      y[o] = (float)acc;
    }
  };
  const int nt = std::max(1, std::min(threads, out_dim / 64));
  if (nt == 1) {
    rows(0, out_dim);
    return;
  }
  std::vector<std::thread> pool;
  for (int t = 0; t < nt; ++t)
    pool.emplace_back(rows, (int)((long long)out_dim * t / nt),
                      (int)((long long)out_dim * (t + 1) / nt));
  for (auto& th : pool) th.join();
}

void silu(std::vector<float>& v)
{
  for (float& z : v) z = z / (1.0f + std::exp(-z));
}

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
  std::vector<float> proj(256), h1((size_t)c.dim), h2((size_t)c.dim);
  timestep_sinusoid(t, 256, proj.data());
  gemv(proj, c.w1, c.b1, 256, c.dim, h1.data(), threads);
  silu(h1);
  gemv(h1, c.w2, c.b2, c.dim, c.dim, h2.data(), threads);
  if (embedded != nullptr) std::memcpy(embedded, h2.data(), (size_t)c.dim * 4);
  silu(h2);
  gemv(h2, c.w3, c.b3, c.dim, c.out_dim, out, threads);
}

}  // namespace ltx25
