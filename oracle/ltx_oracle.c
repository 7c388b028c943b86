/*
 * ltx_oracle.c -- CPU restatement of the reference's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY (see ltx_oracle.h).  Compiled with
 * -ffp-contract=off so every multiply and add rounds on its own, as the
 * reference's x86 build does.
 */
#include "ltx_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

uint16_t ltxo_f32_to_bf16(float v)
{
  /* tests/ltx25-qlinear-test.cc:66-73: add 0x7fff plus the kept LSB, then
   * truncate -- round to nearest, ties to even. */
  uint32_t u;
  memcpy(&u, &v, 4);
  const uint32_t r = ((u >> 16) & 1u) + 0x7fffu;
  return (uint16_t)((u + r) >> 16);
}

float ltxo_bf16_to_f32(uint16_t h)
{
  const uint32_t u = (uint32_t)h << 16;
  float v;
  memcpy(&v, &u, 4);
  return v;
}

void ltxo_f32_to_bf16_n(const float* src, uint16_t* dst, size_t n)
{
  for (size_t i = 0; i < n; ++i) dst[i] = ltxo_f32_to_bf16(src[i]);
}

void ltxo_bf16_to_f32_n(const uint16_t* src, float* dst, size_t n)
{
  for (size_t i = 0; i < n; ++i) dst[i] = ltxo_bf16_to_f32(src[i]);
}

int ltxo_pack_affine(const float* w, int N, int K, int bits, int group,
                     uint32_t* codes, uint16_t* scales, uint16_t* biases,
                     float* deq)
{
  /* tests/ltx25-qlinear-test.cc:94-141 */
  if (N <= 0 || K <= 0 || (bits != 4 && bits != 8) || group <= 0 ||
      K % group != 0 || (K * bits) % 32 != 0) {
    return -1;
  }
  const int per_word = 32 / bits;
  const int gcols = K / group;
  const int wcols = K / per_word;
  const float qmax = (float)((1 << bits) - 1);

  memset(codes, 0, sizeof(uint32_t) * (size_t)N * wcols);
  for (int n = 0; n < N; ++n) {
    const float* row = w + (size_t)n * K;
    for (int g = 0; g < gcols; ++g) {
      const int k0 = g * group;
      float lo = row[k0], hi = lo;
      for (int j = 1; j < group; ++j) {
        lo = fminf(lo, row[k0 + j]);
        hi = fmaxf(hi, row[k0 + j]);
      }
      const float sc = (hi - lo) / qmax;
      const uint16_t sc_b = ltxo_f32_to_bf16(sc);
      const uint16_t lo_b = ltxo_f32_to_bf16(lo);
      const float scr = ltxo_bf16_to_f32(sc_b);
      const float lor = ltxo_bf16_to_f32(lo_b);
      scales[(size_t)n * gcols + g] = sc_b;
      biases[(size_t)n * gcols + g] = lo_b;
      for (int j = 0; j < group; ++j) {
        const int k = k0 + j;
        int q = scr > 0.0f ? (int)lroundf((row[k] - lor) / scr) : 0;
        q = q < 0 ? 0 : (q > (int)qmax ? (int)qmax : q);
        if (deq != NULL) {
          const float p = scr * (float)q;
          deq[(size_t)n * K + k] = p + lor;
        }
        codes[(size_t)n * wcols + k / per_word] |= ((uint32_t)q)
                                                   << (bits * (k % per_word));
      }
    }
  }
  return 0;
}

/* Round an exactly-representable double to bf16, nearest-even.  The value
 * s*q + z formed in double is exact for bf16 s, z and q < 2^8, so this is
 * the single correctly-rounded result the GPU's fma.rn.bf16x2 returns. */
static uint16_t bf16_from_double_rne(double d)
{
  /* d -> f32 may round; do it by hand to avoid double rounding. */
  if (d == 0.0) {
    return signbit(d) ? 0x8000u : 0u;
  }
  int e;
  const double m = frexp(fabs(d), &e); /* |d| = m * 2^e, m in [0.5, 1) */
  /* bf16 keeps 8 significant bits: scale so the kept bits are integral. */
  double scaled = ldexp(m, 8);         /* in [128, 256) */
  double fl = floor(scaled);
  const double rem = scaled - fl;
  if (rem > 0.5 || (rem == 0.5 && fmod(fl, 2.0) != 0.0)) fl += 1.0;
  const double r = ldexp(fl, e - 8);
  const float f = (float)r;            /* exact: r has 8 significant bits */
  uint32_t u;
  memcpy(&u, &f, 4);
  uint16_t h = (uint16_t)(u >> 16);
  if (d < 0) h |= 0x8000u;
  return h;
}

int ltxo_dequant_bf16(const uint32_t* codes, const uint16_t* scales,
                      const uint16_t* biases, int N, int K, int bits,
                      int group, uint16_t* out)
{
  if ((bits != 4 && bits != 8) || group <= 0 || K % group != 0) return -1;
  const int per_word = 32 / bits;
  const int wcols = K / per_word;
  const int gcols = K / group;
  const uint32_t mask = (1u << bits) - 1u;
  for (int n = 0; n < N; ++n) {
    for (int k = 0; k < K; ++k) {
      const uint32_t word = codes[(size_t)n * wcols + k / per_word];
      const uint32_t q = (word >> (bits * (k % per_word))) & mask;
      const double s = ltxo_bf16_to_f32(scales[(size_t)n * gcols + k / group]);
      const double z = ltxo_bf16_to_f32(biases[(size_t)n * gcols + k / group]);
      out[(size_t)n * K + k] = bf16_from_double_rne(s * (double)q + z);
    }
  }
  return 0;
}

/* ---- dense linear, src/ltx25-block-ref.cc:13-29 ----------------------- */

typedef struct {
  const float *x, *w, *b;
  float* out;
  int K, N, r0, r1;
} linear_job;

static void* linear_rows(void* p)
{
  const linear_job* j = (const linear_job*)p;
  for (int r = j->r0; r < j->r1; ++r) {
    const float* xr = j->x + (size_t)r * j->K;
    float* o = j->out + (size_t)r * j->N;
    for (int c = 0; c < j->N; ++c) {
      const float* wr = j->w + (size_t)c * j->K;
      double acc = j->b == NULL ? 0.0 : (double)j->b[c];
      for (int i = 0; i < j->K; ++i) acc += (double)xr[i] * wr[i];
      o[c] = (float)acc;
    }
  }
  return NULL;
}

void ltxo_linear_f64(const float* x, const float* w, const float* b,
                     float* out, int M, int K, int N, int threads)
{
  if (threads < 1) threads = 1;
  if (threads > M) threads = M > 0 ? M : 1;
  if (threads == 1) {
    linear_job j = {x, w, b, out, K, N, 0, M};
    linear_rows(&j);
    return;
  }
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  linear_job* jobs = (linear_job*)malloc(sizeof(linear_job) * (size_t)threads);
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (linear_job){x, w, b, out, K, N, (int)((long)M * t / threads),
                           (int)((long)M * (t + 1) / threads)};
    pthread_create(&th[t], NULL, linear_rows, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
  free(jobs);
  free(th);
}

/* ---- int8 tier (parity unpinned; see the header) ---------------------- */

int ltxo_quant_rows_i8(const uint16_t* x_bf16, int rows, int K, int group,
                       int8_t* q, float* scale)
{
  if (group <= 0 || K % group != 0) return -1;
  const int gcols = K / group;
  for (int r = 0; r < rows; ++r) {
    for (int g = 0; g < gcols; ++g) {
      const uint16_t* xs = x_bf16 + (size_t)r * K + (size_t)g * group;
      float amax = 0.0f;
      for (int j = 0; j < group; ++j) {
        const float a = fabsf(ltxo_bf16_to_f32(xs[j]));
        amax = a > amax ? a : amax;
      }
      const float sc = amax / 127.0f;
      scale[(size_t)r * gcols + g] = sc;
      int8_t* qs = q + (size_t)r * K + (size_t)g * group;
      for (int j = 0; j < group; ++j) {
        if (amax == 0.0f) {
          qs[j] = 0;
          continue;
        }
        float v = rintf(ltxo_bf16_to_f32(xs[j]) / sc);
        v = v > 127.0f ? 127.0f : (v < -127.0f ? -127.0f : v);
        qs[j] = (int8_t)v;
      }
    }
  }
  return 0;
}

typedef struct {
  const int8_t *xq, *wq;
  const float *sx, *sw, *bias;
  float* y;
  int K, N, group, r0, r1;
} i8_job;

static void* i8_rows(void* p)
{
  const i8_job* j = (const i8_job*)p;
  const int gcols = j->K / j->group;
  for (int m = j->r0; m < j->r1; ++m) {
    for (int n = 0; n < j->N; ++n) {
      double acc = j->bias == NULL ? 0.0 : (double)j->bias[n];
      for (int g = 0; g < gcols; ++g) {
        int32_t p32 = 0;
        const int8_t* xa = j->xq + (size_t)m * j->K + (size_t)g * j->group;
        const int8_t* wa = j->wq + (size_t)n * j->K + (size_t)g * j->group;
        for (int k = 0; k < j->group; ++k) p32 += (int32_t)xa[k] * (int32_t)wa[k];
        acc += (double)j->sx[(size_t)m * gcols + g] *
               (double)j->sw[(size_t)n * gcols + g] * (double)p32;
      }
      j->y[(size_t)m * j->N + n] = (float)acc;
    }
  }
  return NULL;
}

void ltxo_i8_gemm(const int8_t* xq, const float* sx, const int8_t* wq,
                  const float* sw, const float* bias, float* y, int M, int K,
                  int N, int group, int threads)
{
  if (threads < 1) threads = 1;
  if (threads > M) threads = M > 0 ? M : 1;
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  i8_job* jobs = (i8_job*)malloc(sizeof(i8_job) * (size_t)threads);
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (i8_job){xq, wq, sx, sw, bias, y, K, N, group,
                       (int)((long)M * t / threads),
                       (int)((long)M * (t + 1) / threads)};
    pthread_create(&th[t], NULL, i8_rows, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
  free(jobs);
  free(th);
}
