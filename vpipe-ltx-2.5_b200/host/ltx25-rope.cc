// ltx25-rope.cc -- LTX-2.5's RoPE tables on the host (built once per
// generation; the per-step rotation runs on the GPU in qk_norm_rope).
//
// Follows the reference's src/ltx25-rope.cc:
//   * frequencies theta ** linspace(0, 1, n) * pi/2, n = inner/(2*axes),
//     built in double and narrowed to f32 (frequencies_precision "float64");
//   * a token's position on an axis is the MIDPOINT of its (start, end) span
//     divided by the axis' max_pos, mapped to [-1, 1];
//   * the row is front-padded with cos 1 / sin 0 to heads * head_dim/2 and
//     laid out (freq, axis) with the axis fastest, then split per head into
//     [heads][tokens][head_dim/2];
//   * video positions are pixels on h/w and SECONDS on t (scale factors
//     8/32/32, causal first frame), audio positions are seconds of mel
//     frames (hop 160 at 16 kHz, 4 mel frames per latent, causal).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/ltx25_cuda.h"
#include "ltx25-threads.h"

namespace {

std::vector<float> ladder(double theta, int n_axes, int inner, int f64)
{
  const int n = inner / (2 * n_axes);
  std::vector<float> out;
  for (int i = 0; i < n; ++i) {
    if (f64) {
      const double t = n == 1 ? 0.0 : (double)i / (double)(n - 1);
      out.push_back((float)(std::pow(theta, t) * 3.14159265358979323846 / 2.0));
    } else {
      const float step = n == 1 ? 0.0f : 1.0f / (float)(n - 1);
      float v = std::pow((float)theta, (float)i * step);
      v = v * 3.14159265358979323846f;
      out.push_back(v / 2.0f);
    }
  }
  return out;
}

// Host threads for a table of `tokens` rows: the host's count, or
// LTX25_HOST_THREADS when set, at most one per 256 tokens.  Every element
// is computed the same way on any thread, so the table does not depend on
// the count.
int table_threads(int tokens)
{
  static const int cap = [] {
    const char* e = std::getenv("LTX25_HOST_THREADS");
    int n = e != nullptr ? std::atoi(e) : 0;
    if (n <= 0) n = (int)std::thread::hardware_concurrency();
    return std::max(1, std::min(n, 64));
  }();
  return std::max(1, std::min(cap, tokens / 256));
}

}  // namespace

extern "C" {

int ltx_rope_table(const double* starts, const double* ends, int n_axes,
                   int tokens, const int* max_pos, int inner_dim, int heads,
                   double theta, int f64_precision, float* cos_out,
                   float* sin_out)
{
  if (starts == nullptr || ends == nullptr || max_pos == nullptr ||
      cos_out == nullptr || sin_out == nullptr)
    return LTX_E_NULL;
  if (n_axes <= 0 || tokens <= 0 || heads <= 0 || inner_dim <= 0 ||
      inner_dim % heads != 0 || (inner_dim / heads) % 2 != 0)
    return LTX_E_SHAPE;
  const int half = inner_dim / heads / 2;
  const std::vector<float> lad = ladder(theta, n_axes, inner_dim, f64_precision);
  const int n_freq = (int)lad.size();
  const int used = n_freq * n_axes;
  const int pad = half * heads - used;
  if (pad < 0) return LTX_E_SHAPE;
  // tokens [t0, t1): one padded row at a time in the thread's own scratch,
  // then split per head
  auto rows = [&](int t0, int t1) {
    std::vector<float> rc((size_t)(pad + used)), rs((size_t)(pad + used));
    for (int i = 0; i < pad; ++i) {
      rc[(size_t)i] = 1.0f;
      rs[(size_t)i] = 0.0f;
    }
    for (int t = t0; t < t1; ++t) {
      for (int f = 0; f < n_freq; ++f) {
        for (int a = 0; a < n_axes; ++a) {
          const size_t idx = (size_t)a * tokens + t;
          const float mid = (float)((starts[idx] + ends[idx]) * 0.5);
          const float frac = mid / (float)max_pos[a];
          const float ang = lad[(size_t)f] * (frac * 2.0f - 1.0f);
          const size_t k = (size_t)pad + (size_t)f * n_axes + a;
          rc[k] = std::cos(ang);
          rs[k] = std::sin(ang);
        }
      }
      for (int h = 0; h < heads; ++h) {
        const size_t dst = ((size_t)h * tokens + t) * half;
        std::memcpy(cos_out + dst, rc.data() + (size_t)h * half, half * sizeof(float));
        std::memcpy(sin_out + dst, rs.data() + (size_t)h * half, half * sizeof(float));
      }
    }
  };
  const int nt = table_threads(tokens);
  ltx25::run_parts(nt, [&](int k) {
    rows((int)((long long)tokens * k / nt), (int)((long long)tokens * (k + 1) / nt));
  });
  return LTX_OK;
}

int ltx_rope_video_spans(int frames, int height, int width, int scale_t,
                         int scale_h, int scale_w, double fps, int causal_fix,
                         double* starts, double* ends)
{
  if (starts == nullptr || ends == nullptr) return LTX_E_NULL;
  if (frames <= 0 || height <= 0 || width <= 0 || fps <= 0.0) return LTX_E_SHAPE;
  const size_t T = (size_t)frames * height * width;
  size_t i = 0;
  for (int f = 0; f < frames; ++f) {
    double t = (double)(f * scale_t), e = (double)((f + 1) * scale_t);
    if (causal_fix) {
      t = t + 1.0 - scale_t;
      e = e + 1.0 - scale_t;
      if (t < 0.0) t = 0.0;
      if (e < 0.0) e = 0.0;
    }
    for (int hh = 0; hh < height; ++hh) {
      for (int ww = 0; ww < width; ++ww, ++i) {
        starts[i] = t / fps;
        ends[i] = e / fps;
        starts[T + i] = (double)(hh * scale_h);
        ends[T + i] = (double)((hh + 1) * scale_h);
        starts[2 * T + i] = (double)(ww * scale_w);
        ends[2 * T + i] = (double)((ww + 1) * scale_w);
      }
    }
  }
  return LTX_OK;
}

int ltx_rope_audio_seconds(int tokens, double* starts, double* ends)
{
  if (starts == nullptr || ends == nullptr) return LTX_E_NULL;
  if (tokens <= 0) return LTX_E_SHAPE;
  const double per = 160.0 / 16000.0;
  auto sec = [&](int t) {
    double mel = (double)(t * 4) + 1.0 - 4.0;
    return (mel < 0.0 ? 0.0 : mel) * per;
  };
  for (int t = 0; t < tokens; ++t) {
    starts[t] = sec(t);
    ends[t] = sec(t + 1);
  }
  return LTX_OK;
}

}  // extern "C"
