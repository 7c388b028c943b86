/*
 * ltx_oracle.h -- CPU restatement of the reference's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library, its
 * C ABI, the host mirror) links, calls or loads this code.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * legs use it, and only as the checker or the timed CPU baseline.
 *
 * Parity status:
 *   - w8g64 pack (ltxo_pack_affine): PINNED bit-exact against the
 *     reference's own packer (tests/ltx25-qlinear-test.cc:94-141), compiled
 *     from the reference source by oracle/Makefile into oracle/_ref/ and
 *     frozen into tests/golden/ by tests/golden/make_golden.py.
 *   - dense linear (ltxo_linear_f64): PINNED against the reference's
 *     linear_ (src/ltx25-block-ref.cc:13-29) compiled the same way.
 *   - int8 tier (ltxo_quant_rows_i8, ltxo_i8_gemm): PARITY UNPINNED.  The
 *     reference's I8GemmContext lives in the uninstalled vpipe toolkit; this
 *     restates the method its header describes (src/ltx25-metal-ops.h:
 *     810-824) with the grouping made a parameter.  The int8 codes are the
 *     bit-exact contract between this file and the GPU kernels.
 */
#ifndef LTX_ORACLE_H
#define LTX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* bf16 <-> f32, round to nearest even (tests/ltx25-qlinear-test.cc:66-81). */
uint16_t ltxo_f32_to_bf16(float v);
float ltxo_bf16_to_f32(uint16_t h);
void ltxo_f32_to_bf16_n(const float* src, uint16_t* dst, size_t n);
void ltxo_bf16_to_f32_n(const uint16_t* src, float* dst, size_t n);

/*
 * Group-affine quantizer, MLX layout (tests/ltx25-qlinear-test.cc:94-141):
 * per (row n, group g): lo = min, hi = max, sc = (hi-lo)/(2^bits-1), both
 * rounded to bf16; q = clamp(lround((w - lo_b)/sc_b), 0, 2^bits-1) (0 when
 * sc_b <= 0); codes packed low bits first, 32/bits per u32 word.
 * `deq` (may be NULL) receives sc_b*q + lo_b in f32, as the reference test
 * computes it.  Returns 0, or -1 on a shape the layout cannot hold.
 */
int ltxo_pack_affine(const float* w, int N, int K, int bits, int group,
                     uint32_t* codes, uint16_t* scales, uint16_t* biases,
                     float* deq);

/*
 * The dequantized weight as the GPU kernels form it: bf16 correctly rounded
 * from the exact value s*q + z (one rounding).  `out` is [N][K] bf16.
 * Only bits=8 (the w8g64 pack) and bits=4 are accepted.
 */
int ltxo_dequant_bf16(const uint32_t* codes, const uint16_t* scales,
                      const uint16_t* biases, int N, int K, int bits,
                      int group, uint16_t* out);

/*
 * out[r][o] = sum_i x[r][i] * w[o][i] + b[o], accumulated in double and
 * narrowed once (src/ltx25-block-ref.cc:13-29).  `b` may be NULL.
 * `threads` > 1 splits rows across that many POSIX threads (each row is
 * still computed exactly as the single-threaded loop does).
 */
void ltxo_linear_f64(const float* x, const float* w, const float* b,
                     float* out, int M, int K, int N, int threads);

/*
 * Symmetric int8 quantization of rows of a bf16 matrix, one scale per
 * (row, group of `group` columns): absmax over the group, scale =
 * absmax / 127 (f32, correctly rounded), q = clamp(rint(x / scale),
 * -127, 127) with round-half-even, q = 0 when absmax == 0.
 * `group` == K gives one scale per row (per-token).  `scale` is
 * [rows][K/group] f32.  Returns 0, or -1 when K % group != 0.
 */
int ltxo_quant_rows_i8(const uint16_t* x_bf16, int rows, int K, int group,
                       int8_t* q, float* scale);

/*
 * The int8 tier's product: y[m][n] = sum_g sx[m][g] * sw[n][g] *
 * sum_{k in g} xq[m][k] * wq[n][k] (+ bias[n]), int32 within a group,
 * f64 across groups.  Activation and weight share the group size.
 */
void ltxo_i8_gemm(const int8_t* xq, const float* sx, const int8_t* wq,
                  const float* sw, const float* bias, float* y, int M, int K,
                  int N, int group, int threads);

#ifdef __cplusplus
}
#endif

#endif /* LTX_ORACLE_H */
