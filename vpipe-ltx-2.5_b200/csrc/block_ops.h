// block_ops.h -- launchers for the block's row ops and attention (internal).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "pdl.cuh"

namespace ltx {

// Status of the kernel launch just issued (0 or -1), counting it when it
// went in: the library's launch tally, read by ltx_launch_count.
int launched();
unsigned long long launch_count();

int launch_f32_to_bf16(const float* a, __nv_bfloat16* out, size_t n,
                       cudaStream_t s);
// out[i] = v
int launch_fill_f32(float* out, float v, size_t n, cudaStream_t s);
// x[t] = regs[t % R] for n_valid <= t < T (rows of dim elements)
int launch_fill_registers(__nv_bfloat16* x, int ldx, const __nv_bfloat16* regs, int dim, int R,
                          int n_valid, int T, cudaStream_t s);
// out = LayerNorm(x) (no affine, population variance) * (1 + scale) + shift;
// dim % 8 == 0, dim <= 8192, shift / scale f32 [dim]
int launch_layer_norm_mod(const __nv_bfloat16* x, int ldx, __nv_bfloat16* out, int ldo,
                          int rows, int dim, const float* shift, const float* scale, float eps,
                          cudaStream_t s);
// x[r][c] += vec[c], r < rows
int launch_add_row_prefix(__nv_bfloat16* x, int ldx, const __nv_bfloat16* vec, int rows,
                          int cols, cudaStream_t s);
// dst[c][r] = src[r][c]
int launch_transpose_bf16(const __nv_bfloat16* src, int lds, __nv_bfloat16* dst, int ldd,
                          int rows, int cols, cudaStream_t s);
// out[i] = bf16(f32(in[i]) * scale), round to nearest even; in == out is fine
int launch_scale_bf16(const __nv_bfloat16* in, __nv_bfloat16* out, float scale, size_t n,
                      cudaStream_t s);

// out[i] = a[i] + b[i] (b bf16, may be null), f32.
int launch_vec_add(const float* a, const __nv_bfloat16* b, float* out, int n,
                   cudaStream_t s);

// out = (norm ? rms_norm(x) : x) * (1 + scale) + shift; scale/shift f32 [dim]
// or null.  dim % 8 == 0, dim <= 8192.
int launch_ada_zero(const __nv_bfloat16* x, int ldx, __nv_bfloat16* out,
                    int ldo, int rows, int dim, const float* scale,
                    const float* shift, float eps, bool norm, cudaStream_t s);

// RMSNorm over the whole heads*head_dim row with gain (f32, may be null),
// then split-half RoPE with [heads][rows][head_dim/2] f32 tables (may be
// null; token t reads table row tok0 + t of tbl_tokens).  in: row stride
// ldi; out: row stride ldo.  Tensor-parallel form:
// the row holds heads [head0, head0 + heads) of a wider row whose per-token
// sum of squares (over norm_width columns) is given in sumsq.
int launch_qk_norm_rope(const __nv_bfloat16* in, int ldi, __nv_bfloat16* out,
                        int ldo, int rows, int heads, int head_dim,
                        const float* gain, const float* cosb,
                        const float* sinb, float eps, cudaStream_t s,
                        const float* sumsq = nullptr, int norm_width = 0,
                        int head0 = 0, int tbl_tokens = 0, int tok0 = 0);

// All-to-all regrouping (sequence parallel): pack [rows][ranks * cpr] into
// [ranks][rows][cpr]; unpack the reverse, optionally times the per-head
// gate 2 sigmoid(gate[t][head]).  cpr % 8 == 0.
int launch_a2a_pack(const __nv_bfloat16* src, int ld, int rows, int ranks, int cpr,
                    __nv_bfloat16* dst, cudaStream_t s);
int launch_a2a_unpack(const __nv_bfloat16* src, int rows, int ranks, int cpr,
                      __nv_bfloat16* dst, int ldd, const __nv_bfloat16* gate, int ldg,
                      int head_dim, cudaStream_t s);

// out[r] = sum of squares of row r's first `cols` values, f32.
int launch_row_sumsq(const __nv_bfloat16* in, int ldi, int rows, int cols,
                     float* out, cudaStream_t s);

// x[r] += gate * (part[r] + bias) (part [rows][dim] dense, bias may be null).
// With nslot > 1, part holds nslot such partials slot_stride elements apart
// (one per source rank) and their sum, taken in slot order in f32, stands for
// part[r].
int launch_gated_residual(__nv_bfloat16* x, int ldx, const __nv_bfloat16* part,
                          const __nv_bfloat16* bias, const float* gate, int rows,
                          int dim, cudaStream_t s, int nslot = 1, size_t slot_stride = 0);

// Non-causal attention, token-major q [tq][ldq], k/v [tk][ld], head h at
// columns [h*D, (h+1)*D); o [tq][ldo]; optional gate logits [tq][ldg]
// (o *= 2 sigmoid(gate[t][h])).  head_dim 64 or 128.
int launch_attention(const __nv_bfloat16* q, int ldq, const __nv_bfloat16* k,
                     int ldk, const __nv_bfloat16* v, int ldv,
                     __nv_bfloat16* o, int ldo, const __nv_bfloat16* gate,
                     int ldg, int tq, int tk, int heads, int head_dim,
                     cudaStream_t s);

// tcgen05 flash attention for head_dim 128 / 64 (attention_tc.cu): the same
// contract as launch_attention plus a V^T scratch of
// attention_tc_scratch(tk, heads, head_dim) elements and the context's error
// word for bounded waits.  q, k, v, o 16-byte aligned, strides % 8 == 0.
size_t attention_tc_scratch(int tk, int heads, int head_dim);
// Key splits the kernel will use (few query tiles and many keys: > 1, with
// f32 partials of attention_tc_part elements merged by a second kernel).
int attention_tc_splits(int tq, int tk, int heads);
size_t attention_tc_part(int tq, int tk, int heads, int head_dim);
int launch_attention_tc(const __nv_bfloat16* q, int ldq, const __nv_bfloat16* k, int ldk,
                        const __nv_bfloat16* v, int ldv, __nv_bfloat16* vt,
                        size_t vt_elems, __nv_bfloat16* o, int ldo,
                        const __nv_bfloat16* gate, int ldg, int tq, int tk, int heads,
                        int head_dim, int* err, cudaStream_t s, float* part = nullptr,
                        size_t part_elems = 0, bool vt_ready = false);

// The sage tier (int8 QK^T, one scale per 128-token block, K smoothed by
// its per-channel mean; P V in bf16): scratch sizes in elements and the
// buffers, then the launch (head_dim 64 or 128).
struct SageScratch {
  size_t qi8 = 0, ki8 = 0, scales = 0, mean = 0, vt = 0;
};
struct SageBuffers {
  int8_t* qi8 = nullptr;
  int8_t* ki8 = nullptr;
  float* scales = nullptr;
  float* mean = nullptr;
  __nv_bfloat16* vt = nullptr;
  SageScratch cap;
};
SageScratch sage_scratch_need(int tq, int tk, int heads, int head_dim);
int launch_sage_tc(const __nv_bfloat16* q, int ldq, const __nv_bfloat16* k, int ldk,
                   const __nv_bfloat16* v, int ldv, const SageBuffers& sb,
                   __nv_bfloat16* o, int ldo, const __nv_bfloat16* gate, int ldg, int tq,
                   int tk, int heads, int head_dim, int* err, cudaStream_t s);

}  // namespace ltx
