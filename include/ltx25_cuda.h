/*
 * ltx25_cuda.h -- C ABI of the B200 (sm_100a) implementation of LTX-2.5's
 * quantized-linear hot path and the joint audio-video DiT block.
 *
 * It replaces, for this path, the reference plugin's ltx25-metal-ops,
 * ltx25-block-metal and ltx25-kernels.metal (tgo-app-dev/vpipe-ltx-2.5).
 * Every entry point names the reference interface it stands in for.
 *
 * Conventions
 *   - Plain pointers and sizes only.  Activations, outputs and biases are
 *     DEVICE pointers to bf16 (uint16 bit patterns), caller-owned, row-major.
 *     `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *   - Every call returns LTX_OK (0) or a negative LTX_E_* code; the message
 *     for the last failure on a context is ltx_ctx_last_error().
 *   - Calls on one context are serialized by the caller (the reference's
 *     one-encoder-per-stack discipline, src/ltx25-block-metal.h:162-163).
 *   - A context is bound to the device it was created on.  Every call on a
 *     context, or on a block, stack, connector, weight or adapter made from
 *     one, runs on that device whatever device the calling thread has
 *     selected, and leaves the thread's selection as it found it; so one
 *     thread may drive contexts on several GPUs.  ltx_ctx_create alone
 *     leaves its device selected.  `stream` must belong to that device.
 *   - Nothing is computed on the CPU: without a usable sm_100a device the
 *     context cannot be created and every op fails with LTX_E_CUDA.
 */
#ifndef LTX25_CUDA_H
#define LTX25_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LTX25_ABI_VERSION 1

#if defined(__GNUC__)
#define LTX_API __attribute__((visibility("default")))
#else
#define LTX_API
#endif

enum {
  LTX_OK = 0,
  LTX_E_NULL = -1,        /* a required pointer was NULL */
  LTX_E_SHAPE = -2,       /* sizes disagree with the weight or the layout */
  LTX_E_UNSUPPORTED = -3, /* a pack this build does not run (not w8g64) */
  LTX_E_CUDA = -4,        /* a CUDA runtime call or launch failed */
  LTX_E_OOM = -5,         /* device (or host) allocation failed */
  LTX_E_KERNEL = -6,      /* a kernel gave up on a bounded wait */
  LTX_E_STATE = -7,       /* call out of order (e.g. block not loaded) */
  LTX_E_ALIGN = -8,       /* a pointer is not 16-byte aligned */
  LTX_E_ABORTED = -9,     /* a progress callback asked to stop */
  LTX_E_HOST = -10        /* the library's host code failed (an exception caught
                             at the boundary; no C++ exception leaves the ABI) */
};

/* Data types of a pack's scales / zero-points as they arrive. */
enum { LTX_SB_F16 = 0, LTX_SB_BF16 = 1, LTX_SB_F32 = 2 };

/* qlinear routes for a quantized weight (the reference's
 * VPIPE_LTX25_NO_DEQUANT_MMA A/B, src/ltx25-metal-ops.cc:532-569). */
enum {
  LTX_ROUTE_FUSED = 0,         /* w8g64 dequant-fused tcgen05 GEMM */
  LTX_ROUTE_DEQUANT_ONCE = 1,  /* expand to bf16 scratch, dense GEMM */
  LTX_ROUTE_AUTO = 2           /* DEQUANT_ONCE from LTX_DEQUANT_MIN_M rows, else FUSED */
};

/* Fused epilogues of ltx_qlinear_ex. */
enum {
  LTX_EPI_STORE = 0,     /* y = x W^T + b */
  LTX_EPI_GELU = 1,      /* y = gelu_tanh(x W^T + b) */
  LTX_EPI_GATED_RES = 2  /* y += gate[n] * (x W^T + b), y is the residual */
};

typedef struct ltx_ctx ltx_ctx;
typedef struct ltx_qweight ltx_qweight;

/* ---- context ----------------------------------------------------------
 * Replaces MetalOps::init (src/ltx25-metal-ops.h:68-70): selects the
 * device, checks it is sm_100, and creates the scratch arena. */
LTX_API int ltx_ctx_create(int device, ltx_ctx** out);
LTX_API void ltx_ctx_destroy(ltx_ctx* ctx);
LTX_API const char* ltx_ctx_last_error(const ltx_ctx* ctx);
LTX_API int ltx_abi_version(void);

/* Size the shared scratch once for the largest call that will follow, so
 * the hot calls allocate nothing (BlockScratch / reserve,
 * src/ltx25-block-metal.h:140-240 and 296-299).  A later call that needs
 * more grows the arena outside any graph capture. */
LTX_API int ltx_ctx_reserve(ltx_ctx* ctx, int max_tokens, int max_n, int max_k);

/* Bytes of device scratch the context holds now (what ltx_ctx_reserve and
 * on-demand growth allocated; weights and block arenas are not counted).
 * A host-side read; no device work.  No counterpart in the reference (its
 * arena is sized by the caller, src/ltx25-block-metal.h:140-163). */
LTX_API int ltx_ctx_scratch_bytes(const ltx_ctx* ctx, unsigned long long* bytes);

/* Reads and clears the device-side error word that a kernel sets when one
 * of its bounded waits gave up.  LTX_OK when clean, LTX_E_KERNEL when not
 * (the reference's wait_ok(), src/ltx25-dit.cc:1920-1931). */
LTX_API int ltx_ctx_check(ltx_ctx* ctx, void* stream);

/* Self-test of the failure path above, with no fault: a kernel waits
 * `bound_ms` (1..2000) on a barrier nothing arrives at and gives up the way
 * every pipeline wait does; the next ltx_ctx_check on that stream returns
 * LTX_E_KERNEL, and the context stays usable. */
LTX_API int ltx_ctx_selftest_timeout(ltx_ctx* ctx, int bound_ms, void* stream);

/* Diagnostics (the reference's VPIPE_LTX25_BLOCK_PROFILE role, src/
 * ltx25-dit.cc:1597-1598): every following GEMM launch writes 16 u64 per
 * CTA for its first `max_ctas` CTAs into the device buffer `buf` -- SM
 * clock64 stamps of its phases (entry, setup, first/last TMA, first
 * dequant, first/last MMA, epilogue, end) and the MMA issuer's cumulative
 * wait cycles on loads, on dequantized operands and on the accumulator.
 * NULL turns it off. */
LTX_API int ltx_ctx_set_trace(ltx_ctx* ctx, void* buf, int max_ctas);

/* ---- weights ----------------------------------------------------------
 * Replaces QWeight + bind_qlinear / need_q_ (src/ltx25-metal-ops.h:45-57,
 * src/ltx25-dit-weights.h:170-175, src/ltx25-dit-weights.cc:352-403).
 *
 * codes:   u32 words holding unsigned codes LOW BITS FIRST, [N][K*bits/32]
 * scales:  one per (row, group), [N][K/group], dtype sb_dtype
 * biases:  the group ZERO-POINT (the group minimum), same layout
 * Uploaded once into HBM (scales/zero-points converted to bf16 with RNE,
 * as get_as_bf16_ does, src/ltx25-dit-weights.cc:230-277).
 * `on_device` != 0 means the three pointers are already device memory.
 * Only bits == 8, group == 64 (the w8g64 pack) is accepted; anything else
 * returns LTX_E_UNSUPPORTED.  N must be a multiple of 4, K of 64. */
LTX_API int ltx_qweight_upload(ltx_ctx* ctx, const uint32_t* codes,
                       const void* scales, const void* biases, int sb_dtype,
                       int N, int K, int bits, int group, int on_device,
                       ltx_qweight** out);

/* A dense bf16 weight [N][K] (gate logits and any tensor a pack leaves
 * dense; QWeight with quantized == false).  N even, K a multiple of 64. */
LTX_API int ltx_dweight_upload(ltx_ctx* ctx, const uint16_t* w_bf16, int N, int K,
                       int on_device, ltx_qweight** out);

LTX_API void ltx_qweight_free(ltx_qweight* w);

LTX_API int ltx_qweight_info(const ltx_qweight* w, int* N, int* K, int* bits,
                     int* group, int* quantized);

/* ---- the quantized linear --------------------------------------------
 * Replaces MetalOps::linear(enc, x, QWeight, bias*, y, M, K, N)
 * (src/ltx25-metal-ops.h:100-105, src/ltx25-metal-ops.cc:532-569):
 * y[M][N] = x[M][K] . W[N][K]^T (+ bias[N]).  W is PyTorch's [out][in].
 * bias may be NULL.  x, y, bias: device bf16.  Unlike the reference the
 * bias is fused into the GEMM epilogue instead of a second pass. */
LTX_API int ltx_qlinear(ltx_ctx* ctx, const ltx_qweight* w, const void* x,
                const void* bias, void* y, int M, int K, int N, void* stream);

/* The int8 tier's qlinear (per-token int8 activation codes, kind::i8 GEMM)
 * with its activation scratch in one fixed device array of the library
 * instead of context memory: the call allocates nothing, for callers that
 * may not allocate device memory while they run (a runtime that owns HBM
 * through its own pool and plans every byte ahead).  No counterpart in the
 * reference.
 *   - M*K <= LTX_I8_STATIC_MAX_CODES and M <= LTX_I8_STATIC_MAX_ROWS, else
 *     LTX_E_SHAPE; K a multiple of 128, N of 4.  ldx = K, ldy = N.
 *   - The weight must already hold its int8 copy, which the first int8-tier
 *     ltx_qlinear on it makes (ltx_set_tiers(ctx, 1, ...)); else LTX_E_STATE.
 *   - The array (32 MiB + 64 KiB) is held by every GPU that loads the
 *     library until the process exits.  The first call on a device looks up
 *     its address (cudaGetSymbolAddress, with that device current); make
 *     that first call before any stream capture.  The address is kept for
 *     the life of the process: after cudaDeviceReset (or the primary
 *     context's release and re-creation) the module loads at another
 *     address, so a process that resets a device must not call this entry
 *     point on that device again.
 *   - All calls on a device share the array and it keeps the last call's
 *     contents; calls whose kernels overlap on the GPU race on it. */
#define LTX_I8_STATIC_MAX_CODES 33554432
#define LTX_I8_STATIC_MAX_ROWS 16384
LTX_API int ltx_qlinear_i8_static(ltx_ctx* ctx, const ltx_qweight* w,
                                  const void* x, const void* bias, void* y,
                                  int M, int K, int N, void* stream);

/* The same with explicit row strides and a fused epilogue (LTX_EPI_*).
 * `gate` is [N] f32 for LTX_EPI_GATED_RES (y += gate * (xW^T + b)), the
 * reference's linear + gated_residual pair (src/ltx25-metal-ops.cc:
 * 1047-1059) and linear + gelu (src/ltx25-metal-ops.cc:1062-1070). */
LTX_API int ltx_qlinear_ex(ltx_ctx* ctx, const ltx_qweight* w, const void* x,
                   int ldx, const void* bias, void* y, int ldy, int M, int K,
                   int N, int epilogue, const void* gate, void* stream);

/* ---- low-rank adapters ---------------------------------------------------
 * Replace one module's LoraPair as LoraAdapter::load binds it (src/
 * ltx25-lora.h:48-56, src/ltx25-lora.cc:56-124) and MetalOps::lora_add
 * (src/ltx25-metal-ops.h:107-132, src/ltx25-metal-ops.cc:986-1000).
 * a is [rank][k] and b [n][rank], bf16, both in the [out][in] order the
 * checkpoint stores (neither is transposed).  `scale` -- lora_scale times
 * the adapter's alpha / rank, which the caller reads from its metadata --
 * is folded into a at upload: a' = bf16(f32(a) * scale), one rounding, as
 * the reference's loader does.  k must be a multiple of 8, n even.
 * on_device != 0: a and b are device memory.  The pair is copied; the
 * caller's arrays may be freed after the call. */
typedef struct ltx_lora ltx_lora;
LTX_API int ltx_lora_upload(ltx_ctx* ctx, const uint16_t* a, const uint16_t* b, int rank,
                            int k, int n, float scale, int on_device, ltx_lora** out);
LTX_API void ltx_lora_free(ltx_lora* l);
LTX_API int ltx_lora_info(const ltx_lora* l, int* rank, int* k, int* n);

/* y[M][N] += (x[M][K] . A^T) . B^T for a y that already holds the linear
 * it adapts (MetalOps::lora_add).  K == k, N == n; row strides ldx, ldy in
 * elements.  x.A^T goes to the context's scratch; the add is the second
 * GEMM's epilogue, so no [M][N] delta is written (the reference's
 * matrix-core pair, src/ltx25-metal-ops.h:850-866). */
LTX_API int ltx_lora_add(ltx_ctx* ctx, const ltx_lora* l, const void* x, int ldx, void* y,
                         int ldy, int M, int K, int N, void* stream);

/* ltx_qlinear_ex with an adapter on the linear: y = epilogue(x.W^T + bias
 * + (x.A^T).B^T).  The delta is contracted in the linear's own GEMM
 * accumulator (extra K blocks after the weight's), so it lands before the
 * GELU / gated residual, where the reference's MetalBlock::lora_ puts it
 * (between a linear and its consumer, src/ltx25-block-metal.cc:404-420).
 * An adapted linear takes the bf16 route (the pack expanded once) whatever
 * its M or tier.  l == NULL is ltx_qlinear_ex. */
LTX_API int ltx_qlinear_lora(ltx_ctx* ctx, const ltx_qweight* w, const ltx_lora* l,
                             const void* x, int ldx, const void* bias, void* y, int ldy,
                             int M, int K, int N, int epilogue, const void* gate,
                             void* stream);

/* ---- the trunk around the block loop ------------------------------------
 * Ltx25Dit's patchify (src/ltx25-dit.cc:1509-1540): x[T][dim] = latent .
 * W^T + bias (+ the adapter's delta, l may be NULL), then `prefix` [dim]
 * added to rows [0, prefix_rows) -- the keyframe position embedding on the
 * first latent frame's tokens (NULL / 0: none).  latent is bf16 token-major
 * [T][z], or channel-major [z][T] (the VAE's layout) when channel_major;
 * the pack to token-major (w fastest) runs on the device. */
LTX_API int ltx_patchify(ltx_ctx* ctx, const ltx_qweight* w, const void* bias, const ltx_lora* l,
                         const void* latent, int channel_major, const void* prefix,
                         int prefix_rows, void* x, int T, int z, int dim, void* stream);

/* Ltx25Dit's output head (src/ltx25-dit.cc:2000-2045): LayerNorm over dim
 * (no affine -- NOT an RMSNorm -- eps 1e-6), then x * (1 + scale) + shift,
 * then proj_out (+ bias, + adapter) -> out bf16 [T][out_ch], or the
 * channel-major [out_ch][T] the sampler and VAE take when channel_major.
 * shift_scale: f32 [2][dim], the shift row first: the head's 2-row table
 * with the embedded timestep added to both rows (the caller's adaLN). */
LTX_API int ltx_output_head(ltx_ctx* ctx, const void* x, const float* shift_scale,
                            const ltx_qweight* w, const void* bias, const ltx_lora* l,
                            void* out, int channel_major, int T, int dim, int out_ch,
                            void* stream);

/* Route for quantized weights (LTX_ROUTE_*).  Default AUTO, the reference's
 * own choice (MetalOps::linear -> dequant_mma_, src/ltx25-metal-ops.cc:
 * 343-347, 468-545): a call tall enough to be tensor-bound expands the
 * weight once into the context's bf16 scratch and runs the dense tcgen05
 * GEMM; below it (audio, text) the fused kernel, which reads 1.06 bytes per
 * weight instead of 5.  The crossover on B200 is LTX_DEQUANT_MIN_M rows. */
#define LTX_DEQUANT_MIN_M 1536
LTX_API int ltx_set_route(ltx_ctx* ctx, int route);

/* A/B overrides of the GEMM tile plan, the counterpart of the reference's
 * tile knob (src/ltx25-metal-ops.h:793-795, src/ltx25-metal-ops.cc:223-226,
 * VPIPE_LTX25_MMA_TILE, read once at construction): force_pair 1/0
 * forces CTA pairs (cta_group::2, 256 weight rows over two SMs) on or off,
 * 2 forces pairs holding two weight blocks per CTA (512 weight rows per
 * pair tile; dense bf16 weights with N % 512 == 0, else as 1),
 * force_tn 128/256 the token tile, force_splits 1..8 the K split; -1 leaves
 * each to the planner.  A forced value the shape cannot take is ignored.
 * The context starts from LTX25_FORCE_PAIR / _TN / _SPLITS, read once when
 * it is created. */
LTX_API int ltx_set_tile_plan(ltx_ctx* ctx, int force_pair, int force_tn, int force_splits);

/* ---- acceleration tiers ------------------------------------------------
 * Replaces MetalOps::set_i8_gemm / set_sage (src/ltx25-metal-ops.h:151,
 * 265) fed from the accel bag keys i8_gemm, sage_attn, sage_dense_layers
 * (src/ltx25-generator.cc:297-375). */
LTX_API int ltx_set_tiers(ltx_ctx* ctx, int i8_gemm, int sage_attn,
                  int sage_dense_layers);

/* Will ltx_qlinear take the int8 tier for this shape?  1 / 0.
 * Replaces MetalOps::i8_takes (src/ltx25-metal-ops.cc:761-768). */
LTX_API int ltx_i8_takes(const ltx_ctx* ctx, int M, int K, int N);

/* Whether the sage tier takes an attention of this head width
 * (MetalOps::sage_takes, src/ltx25-metal-ops.cc:897-905): 64 and 128, while
 * the tier is on.  The standalone ltx_attention takes it whenever this says
 * yes; a block's attentions only from layer sage_dense_layers on. */
LTX_API int ltx_sage_takes(const ltx_ctx* ctx, int head_dim);

/* ---- pieces exposed for parity tests -----------------------------------
 * The dequantized weight exactly as the GEMMs see it: out[N][K] bf16 =
 * s*q + z rounded once (the M5 dequant-once expansion,
 * src/ltx25-metal-ops.cc:468-502). */
LTX_API int ltx_dequant(ltx_ctx* ctx, const ltx_qweight* w, void* out, void* stream);

/* Symmetric int8 quantization per (row, group): scale = absmax/127,
 * q = rint(x/scale) in [-127, 127].  group == K is per-token.  q is
 * [rows][K] int8, scale [rows][K/group] f32, both device. */
LTX_API int ltx_quant_rows_i8(ltx_ctx* ctx, const void* x, int rows, int K,
                      int group, void* q, void* scale, void* stream);

/* The w8g64 quantizer itself, on the device: w f32 [N][K] -> codes u32
 * [N][K/4] (low bits first), scales and zero-points bf16 [N][K/64], with
 * the arithmetic of the reference's packer (tests/ltx25-qlinear-test.cc:
 * 94-141) so the pack is bit-identical.  What vpipe's model-quantize
 * writes for a w8g64 tensor, before its F16 storage.  All device pointers;
 * K % 64 == 0. */
LTX_API int ltx_pack_w8g64(ltx_ctx* ctx, const float* w, int N, int K,
                           uint32_t* codes, uint16_t* scales,
                           uint16_t* biases, void* stream);

/* ---- block op vocabulary ---------------------------------------------
 * The row ops and attention of the block, exposed one by one (MetalOps::
 * ada_zero / rms_norm_gain + rope / sdpa_steel + gate_heads,
 * src/ltx25-metal-ops.h:330-560).  bf16 device tensors, f32 vectors. */

/* out = rms_norm(x) * (1 + scale) + shift (normalize != 0) or
 * x * (1 + scale) + shift (normalize == 0); scale, shift f32 [dim] or NULL;
 * eps 1e-6 (src/ltx25-block-ref.cc:134-165). */
LTX_API int ltx_ada_zero(ltx_ctx* ctx, const void* x, void* out, int rows,
                         int dim, const float* scale, const float* shift,
                         int normalize, void* stream);

/* RMSNorm over the whole heads*head_dim row with an f32 gain, then the
 * split-half RoPE per head with f32 tables [heads][rows][head_dim/2] (NULL:
 * no rotation).  in has row stride ld_in; out is compact
 * (src/ltx25-block-ref.cc:31-45, src/ltx25-rope.cc:325-352). */
LTX_API int ltx_qk_norm_rope(ltx_ctx* ctx, const void* in, int ld_in,
                             void* out, int rows, int heads, int head_dim,
                             const float* gain, const float* cos_tab,
                             const float* sin_tab, void* stream);

/* o = softmax(q k^T / sqrt(D)) v per head, times 2 sigmoid(gate[t][h]) when
 * gate_logits != NULL.  Token-major: head h at columns [h*D, (h+1)*D).
 * head_dim 64 or 128 (src/ltx25-block-ref.cc:49-127). */
LTX_API int ltx_attention(ltx_ctx* ctx, const void* q, int ldq, const void* k,
                          int ldk, const void* v, int ldv, void* o, int ldo,
                          const void* gate_logits, int ldg, int tq, int tk,
                          int heads, int head_dim, void* stream);

/* ---- RoPE tables (host, once per generation) ----------------------------
 * The reference's build_rope / video_spans / audio_time_seconds
 * (src/ltx25-rope.cc:74-296), computed on the host into caller buffers; no
 * device or context needed.  starts/ends are [n_axes][tokens] doubles, the
 * tables [heads][tokens][inner_dim/heads/2] f32.  theta 10000 and
 * f64_precision 1 are LTX-2.5's values. */
LTX_API int ltx_rope_table(const double* starts, const double* ends,
                           int n_axes, int tokens, const int* max_pos,
                           int inner_dim, int heads, double theta,
                           int f64_precision, float* cos_out, float* sin_out);

/* Per-token (start, end) of a [frames][height][width] latent in pixels (h,
 * w) and seconds (t), w fastest, causal first frame (video_spans,
 * src/ltx25-rope.cc:180-247).  starts/ends: [3][frames*height*width]. */
LTX_API int ltx_rope_video_spans(int frames, int height, int width,
                                 int scale_t, int scale_h, int scale_w,
                                 double fps, int causal_fix, double* starts,
                                 double* ends);

/* Audio latent token spans in seconds (audio_time_seconds,
 * src/ltx25-rope.cc:262-276): tokens of 4 mel frames, hop 160 at 16 kHz. */
LTX_API int ltx_rope_audio_seconds(int tokens, double* starts, double* ends);

/* ---- the joint audio-video block ---------------------------------------
 * Replaces MetalBlock (src/ltx25-block-metal.h:245-371) with the math of
 * block_forward (src/ltx25-block-ref.cc:308-389). */
typedef struct ltx_block ltx_block;

/* One stream's inputs for a forward (GpuStreamInput,
 * src/ltx25-block-metal.h:70-118).  Device pointers; bf16 unless noted. */
typedef struct {
  void* x;                        /* [tokens][dim], UPDATED in place */
  const void* context;            /* [text_tokens][dim] */
  const void* timesteps;          /* 9 * dim adaLN driver */
  const void* cross_scale_shift;  /* 4 * dim */
  const void* cross_gate;         /* dim */
  const void* prompt_timestep;    /* 2 * dim, or NULL (static table alone) */
  const float* pe_cos;            /* self RoPE [heads][tokens][head_dim/2] */
  const float* pe_sin;
  const float* cross_pe_cos;      /* a2v/v2a RoPE at the AUDIO width */
  const float* cross_pe_sin;
  int tokens;
  int text_tokens;
  int present;                    /* 0: stream absent this forward */
} ltx_stream_io;

LTX_API int ltx_block_create(ltx_ctx* ctx, int video_dim, int video_heads,
                             int audio_dim, int audio_heads, ltx_block** out);
LTX_API void ltx_block_destroy(ltx_block* b);
LTX_API const char* ltx_block_last_error(const ltx_block* b);

/* Stage a tensor under the reference's parameter name
 * (load_block_weights, src/ltx25-block-ref.cc:424-523): the 28 quantized
 * linears (`attn1.to_q.weight`, `audio_ff.net.2.weight`, ...) as w8g64
 * packs (bind_qlinear); every other tensor (biases, q/k norms, gate
 * logits, adaLN tables) as f32 [rows][cols] (cols 0 for a vector). */
LTX_API int ltx_block_set_qlinear(ltx_block* b, const char* name,
                                  const uint32_t* codes, const void* scales,
                                  const void* biases, int sb_dtype, int N,
                                  int K, int on_device);
LTX_API int ltx_block_set_tensor(ltx_block* b, const char* name,
                                 const float* data, int rows, int cols,
                                 int on_device);

/* Attach one module's adapter (MetalBlock::lora_ with the LoraBlock the
 * reference's loader builds, src/ltx25-block-metal.cc:404-420, src/
 * ltx25-lora.h:58-76) under the module's reference name: "attn1.to_q",
 * ".to_k", ".to_v", ".to_out.0", ".to_gate_logits" of attn1, attn2,
 * audio_attn1, audio_attn2, audio_to_video_attn, video_to_audio_attn, and
 * "ff.net.0.proj", "ff.net.2", "audio_ff.net.0.proj", "audio_ff.net.2".
 * Call before ltx_block_finalize, which checks each pair against its base
 * linear (LTX_E_SHAPE), shards it like the base weight under tensor
 * parallelism and copies it; the pair may be freed afterwards.  A name this
 * block does not apply returns LTX_E_UNSUPPORTED, as the reference's loader
 * refuses an adapter naming a module it would not apply; after finalize,
 * LTX_E_STATE.  Each adapted linear contracts its delta in its own GEMM
 * (ltx_qlinear_lora), before the norm / GELU / gated residual that consumes
 * it. */
LTX_API int ltx_block_set_lora(ltx_block* b, const char* module, const ltx_lora* l);

/* Check every required tensor is present (naming the first missing one,
 * as load_block_weights does), fuse the q/k/v and k/v packs, upload. */
LTX_API int ltx_block_finalize(ltx_block* b);

/* Size the block's scratch arena once (MetalBlock::reserve). */
LTX_API int ltx_block_reserve(ltx_block* b, int max_video_tokens,
                              int max_audio_tokens, int max_text_tokens);

/* The block's index in its model (MetalBlock::forward's layer,
 * src/ltx25-block-metal.h:307-311): with the sage tier on, blocks below
 * sage_dense_layers keep dense attention.  Default 0; ltx_stack_add_block
 * sets it to the block's position. */
LTX_API int ltx_block_set_layer(ltx_block* b, int layer);

/* Run the block on `stream`; video->x and audio->x are updated in place
 * (MetalBlock::forward, src/ltx25-block-metal.h:307-311). */
LTX_API int ltx_block_forward(ltx_block* b, const ltx_stream_io* video,
                              const ltx_stream_io* audio, void* stream);

/* Kernels this library has launched in the process so far (all contexts,
 * all devices): bracket a region with two reads to count its launches. */
LTX_API unsigned long long ltx_launch_count(void);

/* ---- tensor parallelism (no reference counterpart) --
 * One process per GPU, one context each.  Rank 0 makes a rendezvous id,
 * the caller ships its LTX_TP_ID_BYTES to every rank by any channel, and
 * every rank joins with ltx_ctx_set_tp before creating blocks.  Blocks
 * finalized on a TP context keep only their rank's shard of the weights
 * they are given in full: q/k/v, the gate logits and ff.net.0 split by
 * heads / hidden columns, the output projections and ff.net.2 by K, with
 * the partial products summed over the group (NCCL all-reduce) before the
 * bias and the gated residual.  Every rank then calls the same forwards
 * with the same (replicated) stream inputs, and each ends with the same x.
 * NCCL is loaded at run time (libnccl.so.2). */
#define LTX_TP_ID_BYTES 128
LTX_API int ltx_tp_unique_id(void* id, int bytes);
LTX_API int ltx_ctx_set_tp(ltx_ctx* ctx, int rank, int world, const void* id);
/* Sequence (head) parallelism instead: blocks keep their weights whole
 * and each rank runs 1/world of the video tokens through the GEMMs, the row
 * ops, the text and audio->video cross attentions and the feed-forward with
 * no communication; the video self-attention and the video->audio keys
 * switch to a head split by all-to-all (DeepSpeed-Ulysses) and back.  The
 * audio stream (126 tokens) is replicated.  Callers still pass and get the
 * WHOLE x on every rank (the stack gathers the shards once, at its end).
 * The video token count must divide by world; heads by world. */
LTX_API int ltx_ctx_set_sp(ltx_ctx* ctx, int rank, int world, const void* id);

/* In-place sum over the group on `stream`; dtype 0 = f32, 1 = bf16. */
LTX_API int ltx_tp_allreduce(ltx_ctx* ctx, void* buf, size_t count, int dtype,
                             void* stream);

/* ---- the block stack ----------------------------------------------------
 * The block loop of Ltx25Dit::forward (src/ltx25-dit.cc:1716-1931): blocks
 * run in order on the same stream inputs, x updated in place, and share ONE
 * scratch arena (the reference's BlockScratch, src/ltx25-block-metal.h:
 * 140-240).  The stack references its blocks without owning them: destroy
 * the stack first. */
typedef struct ltx_stack ltx_stack;

/* Host-side progress hook, called before block `block` of `blocks` is
 * enqueued (the reference's in.progress, src/ltx25-dit.cc:1718-1720).
 * Return 0 to stop: the forward returns LTX_E_ABORTED with the blocks
 * before it enqueued. */
typedef int (*ltx_progress_fn)(int block, int blocks, void* user);

LTX_API int ltx_stack_create(ltx_ctx* ctx, ltx_stack** out);
LTX_API void ltx_stack_destroy(ltx_stack* s);
LTX_API const char* ltx_stack_last_error(const ltx_stack* s);

/* Append a finalized block of the same context and widths. */
LTX_API int ltx_stack_add_block(ltx_stack* s, ltx_block* b);
LTX_API int ltx_stack_size(const ltx_stack* s);

/* Size the shared arena for the largest geometry; call after the last
 * add_block (Ltx25Dit::set_geometry's reserve, src/ltx25-dit.cc:984-1204). */
LTX_API int ltx_stack_reserve(ltx_stack* s, int max_video_tokens,
                              int max_audio_tokens, int max_text_tokens);

/* Run blocks [begin, end) (end < 0: to the last block) on `stream`.
 * progress may be NULL. */
LTX_API int ltx_stack_forward(ltx_stack* s, const ltx_stream_io* video,
                              const ltx_stream_io* audio, int begin, int end,
                              ltx_progress_fn progress, void* user,
                              void* stream);

/* ---- checkpoints ---------------------------------------------------------
 * The on-disk pack reader (the WeightSet the reference binds through,
 * src/ltx25-dit-weights.cc:230-403, src/ltx25-lora.cc:180-300): a
 * safetensors file mapped read-only, its header parsed once -- u64 header
 * length, JSON {name: {dtype, shape, data_offsets}, "__metadata__": {..}},
 * data.  A header that is not the format's (unknown dtype, offsets outside
 * the data or disagreeing with shape x dtype, truncated file, trailing
 * bytes) is refused whole: LTX_E_SHAPE with the reason in `err`; a file
 * that cannot be opened or mapped: LTX_E_STATE. */
typedef struct ltx_st ltx_st;
enum {
  LTX_ST_F32 = 0, LTX_ST_F16 = 1, LTX_ST_BF16 = 2, LTX_ST_U32 = 3, LTX_ST_I32 = 4,
  LTX_ST_U8 = 5, LTX_ST_I8 = 6, LTX_ST_F64 = 7, LTX_ST_I64 = 8, LTX_ST_U16 = 9,
  LTX_ST_I16 = 10, LTX_ST_BOOL = 11
};
LTX_API int ltx_st_open(const char* path, ltx_st** out, char* err, int err_len);
LTX_API void ltx_st_close(ltx_st* f);
LTX_API int ltx_st_count(const ltx_st* f);
LTX_API const char* ltx_st_name(const ltx_st* f, int i);
/* index of `name`, or -1 */
LTX_API int ltx_st_find(const ltx_st* f, const char* name);
/* shape: room for 8 dimensions; data points into the mapping. */
LTX_API int ltx_st_info(const ltx_st* f, int i, int* dtype, int* ndim, int64_t* shape,
                        const void** data, uint64_t* bytes);
/* a __metadata__ string value, or NULL */
LTX_API const char* ltx_st_metadata(const ltx_st* f, const char* key);
/* n elements of a float tensor (F32 / F16 / BF16) from element `off`, as
 * f32 (F16 and BF16 widened exactly); LTX_E_SHAPE for another dtype or a
 * range past the tensor. */
LTX_API int ltx_st_read_f32(const ltx_st* f, int i, uint64_t off, uint64_t n, float* out);

/* Stage every tensor of one block from a checkpoint: the names under
 * `prefix` (e.g. "model.diffusion_model.transformer_blocks.7.") with the
 * prefix stripped.  A quantized linear is the "X.weight" u32 codes +
 * "X.scales" + "X.biases" triplet (need_q_, src/ltx25-dit-weights.cc:
 * 352-403): staged as ltx_block_set_qlinear (F16 / BF16 / F32 scales);
 * every other float tensor as ltx_block_set_tensor.  A pack that closes at
 * another group or bit width returns LTX_E_UNSUPPORTED (this build runs
 * w8g64).  Then ltx_block_finalize as usual. */
LTX_API int ltx_block_load_st(ltx_block* b, const ltx_st* f, const char* prefix);

/* One module's adapter pair from an adapter file: "<module>.lora_A.weight"
 * [rank][k] and "<module>.lora_B.weight" [n][rank] (any float dtype), the
 * rank derived from each against the base widths and cross-checked
 * (bind_pair_, src/ltx25-lora.cc:69-124); the factor is lora_scale times
 * alpha / rank when the file's __metadata__ names lora_alpha and lora_rank
 * (src/ltx25-lora.cc:265-287).  LTX_E_STATE when the module is not
 * adapted. */
LTX_API int ltx_lora_load_st(ltx_ctx* ctx, const ltx_st* f, const char* module, int k, int n,
                             float lora_scale, ltx_lora** out);

/* ---- the embeddings connector ---------------------------------------------
 * Replaces Ltx25Connector (src/ltx25-connector.cc:38-260): the 1-D
 * transformer between the text encoder and the DiT.  Per block: RMSNorm,
 * q / k / v with bias, q / k RMS gain over the whole width and the 1-D
 * index RoPE at the connector's own max_pos (position i spans [i, i + 1)),
 * full attention with the optional per-head gate, out projection with bias
 * and a PLAIN residual; RMSNorm, the biased GELU feed-forward (4x), a plain
 * residual; then an optional RMSNorm (norm_output).  Padded positions
 * (t >= n_valid) are replaced by the learnable registers tiled over the
 * sequence before the first block.  Tensor names are relative to the
 * connector root ("transformer_1d_blocks.{i}.attn1.to_q.weight",
 * "learnable_registers", ...); linears as w8g64 packs or dense f32. */
typedef struct ltx_connector ltx_connector;
LTX_API int ltx_connector_create(ltx_ctx* ctx, int heads, int head_dim, int layers,
                                 int registers, int norm_output, double theta, int max_pos,
                                 int rope_f64, ltx_connector** out);
LTX_API void ltx_connector_destroy(ltx_connector* c);
LTX_API const char* ltx_connector_last_error(const ltx_connector* c);
LTX_API int ltx_connector_set_qlinear(ltx_connector* c, const char* name, const uint32_t* codes,
                                      const void* scales, const void* biases, int sb_dtype,
                                      int N, int K, int on_device);
LTX_API int ltx_connector_set_tensor(ltx_connector* c, const char* name, const float* data,
                                     int rows, int cols, int on_device);
/* every tensor under `root` of a checkpoint (e.g. "model.diffusion_model.
 * video_embeddings_connector.") */
LTX_API int ltx_connector_load_st(ltx_connector* c, const ltx_st* f, const char* root);
LTX_API int ltx_connector_finalize(ltx_connector* c);
/* tokens: a multiple of the register count (LTX_E_SHAPE otherwise) */
LTX_API int ltx_connector_reserve(ltx_connector* c, int tokens);
/* out [tokens][dim] bf16 = connector(in); in == out allowed */
LTX_API int ltx_connector_forward(ltx_connector* c, const void* in, void* out, int tokens,
                                  int n_valid, void* stream);

/* ---- the trunk's adaLN chains (host) --------------------------------------
 * Ltx25Dit::adaln_ (src/ltx25-dit.cc:51-160): the 256-channel timestep
 * sinusoid (max period 10000, no downscale shift, flip_sin_to_cos: the row
 * is [cos | sin]) through emb.timestep_embedder.linear_1 -> SiLU ->
 * linear_2 -> SiLU -> the root `linear`, as host GEMVs over bf16 weights
 * with f64 sums stored f32, split over host threads by output row.  The
 * reference runs them on the host once per denoise level and step; the
 * caller passes the timestep it feeds (sigma times the timestep scale
 * multiplier).  out: [out_dim] (the k*dim modulation driver); embedded:
 * [dim] = the linear_2 output, before the SiLU -- the `embedded_timestep`
 * the output head adds to its table -- or NULL.  threads <= 0: the host's
 * count. */
typedef struct ltx_adaln ltx_adaln;
/* bf16 [dim][256], [dim], [dim][dim], [dim], [out_dim][dim], [out_dim];
 * biases may be NULL.  Copied. */
LTX_API int ltx_adaln_create(const uint16_t* w1, const uint16_t* b1, const uint16_t* w2,
                             const uint16_t* b2, const uint16_t* w3, const uint16_t* b3,
                             int dim, int out_dim, ltx_adaln** out);
/* From a checkpoint: prefix + "emb.timestep_embedder.linear_1", "..._2",
 * "linear" (.weight / .bias), e.g. prefix "model.diffusion_model.
 * adaln_single."; any float dtype, rounded to bf16 as the reference's
 * loader does. */
LTX_API int ltx_adaln_load_st(const ltx_st* f, const char* prefix, ltx_adaln** out, char* err,
                              int err_len);
LTX_API void ltx_adaln_free(ltx_adaln* a);
LTX_API int ltx_adaln_dims(const ltx_adaln* a, int* dim, int* out_dim);
LTX_API int ltx_adaln_run(const ltx_adaln* a, double timestep, float* out, float* embedded,
                          int threads);
/* A denoise step's chains at once (Ltx25Dit::compute_adaln_step_,
 * src/ltx25-dit.cc:178-236, runs them one after another): chains[i] at
 * timesteps[i] into outs[i] (and embedded[i] when embedded and the entry are
 * non-NULL), each stage's rows over all chains split evenly over the host
 * threads.  Same bits as count separate ltx_adaln_run calls. */
LTX_API int ltx_adaln_run_many(const ltx_adaln* const* chains, const double* timesteps,
                               float* const* outs, float* const* embedded, int count,
                               int threads);

#ifdef __cplusplus
}
#endif

#endif /* LTX25_CUDA_H */
