/*
 * levo_oracle.h — CPU restatement of the LeVo2.cpp elementwise / reduction path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * kernels and the timed CPU baseline ("port") of bench.py.  Nothing in the
 * product (levo2.cpp_b200/) links, loads or calls it.
 *
 * Each function restates the reference's arithmetic in the reference's order,
 * one materialised F32 pass per GGML graph node, as GGML's CPU backend runs the
 * graph.  The GGML node semantics themselves live in the (absent) ggml
 * submodule, ggml-org/ggml @ 8846b79e66747bb9f68597420e95114c177315ce; the
 * per-node formulas used here are the published definitions of those ops.
 * `threads` <= 0 means all online CPUs.
 */
#ifndef LEVO_ORACLE_H
#define LEVO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* SnakeBeta, src/levo-audio-ops.cpp:146-151.  params are F32 [C]. */
int oracle_snakebeta_f32(const float *x, const float *alpha_log, const float *beta_log, float *y,
                         int64_t channels, int64_t time, int threads);
/* Same with F16-stored parameters (IEEE half bits), promoted as ggml_cast does. */
int oracle_snakebeta_f16params(const float *x, const uint16_t *alpha_log, const uint16_t *beta_log,
                               float *y, int64_t channels, int64_t time, int threads);

/* add_channel_bias, src/levo-audio-ops.cpp:39-52. */
int oracle_channel_bias_add_f32(const float *in, const float *bias, float *out, int64_t channels,
                                int64_t time, int threads);

/* Fused decoder unit semantics, expressed as the reference's separate nodes:
 * x = residual + (u + bias); y = snake(x) [; tanh].  Any of bias / residual /
 * alpha_log may be NULL; x_out / y_out may be NULL. */
int oracle_fused_unit_f32(const float *u, const float *bias, const float *residual,
                          const float *alpha_log, const float *beta_log, float *x_out, float *y_out,
                          int64_t channels, int64_t time, int tanh_out, int threads);

/* Built-in conv stand-in: out[c][t] = in[c % cin][t / stride]. */
void oracle_conv_standin_f32(const float *in, int64_t cin, int64_t lin, float *out, int64_t cout,
                             int64_t lout, int stride);

/* Decoder stage loop, src/levo-vae.cpp:212-235, with the stand-in convs.
 * topology ints: {latent_dim, audio_channels, entry_width, n_stages,
 * widths[n_stages], strides[n_stages], n_residual} (dilations do not affect the
 * stand-ins).  params packed as levo_vae_param_count documents.
 * audio: [audio_channels][frames * prod(strides)]. */
int oracle_vae_chain_f32(const int32_t *topology, const float *params, const float *latent,
                         int64_t frames, float *audio, int tanh_out, int threads);
/* The same, also copying stage s's output [widths[s]][frames * prod(strides[0..s])]
 * to stages[s] (stages NULL or stages[s] NULL: not copied). */
int oracle_vae_chain_stages_f32(const int32_t *topology, const float *params, const float *latent,
                                int64_t frames, float *audio, int tanh_out, int threads, float *const *stages);

/* Residual add + RMSNorm / LayerNorm on F16 (IEEE half bits) or F32 rows.
 * RMSNorm: src/levo-lm.cpp:131-138, src/levo-kv.cpp:153-170.
 * LayerNorm: src/levo-flow-estimator.cpp:106-109.  r / h_out may be NULL.
 * PARITY UNPINNED against the reference itself: its norms are the GGML nodes
 * ggml_rms_norm / ggml_norm, and GGML (the reference's `ggml` submodule,
 * ggml-org/ggml @ 8846b79e66747bb9f68597420e95114c177315ce as
 * src/levo-vae-model.cpp:132 records it) is absent.  The restatement follows GGML's
 * published CPU algorithm (row statistics accumulated in double, the scale
 * 1/sqrt(stat + eps) in F32, then separate gamma / beta nodes) and is checked
 * against the float64 definitions and against the upstream modules the
 * reference's parity policy gates its norms against (tests/golden/
 * make_norm_golden.py: Transformers' Llama RMSNorm, torch's LayerNorm). */
int oracle_add_rmsnorm_f16(const uint16_t *x, const uint16_t *r, const float *gamma,
                           uint16_t *h_out, uint16_t *y_out, int64_t rows, int64_t dim, float eps,
                           int f16_boundary, int threads);
int oracle_add_rmsnorm_f32(const float *x, const float *r, const float *gamma, float *h_out,
                           float *y_out, int64_t rows, int64_t dim, float eps, int threads);
int oracle_add_layernorm_f16(const uint16_t *x, const uint16_t *r, const float *gamma,
                             const float *beta, uint16_t *h_out, uint16_t *y_out, int64_t rows,
                             int64_t dim, float eps, int f16_boundary, int threads);
int oracle_add_layernorm_f32(const float *x, const float *r, const float *gamma, const float *beta,
                             float *h_out, float *y_out, int64_t rows, int64_t dim, float eps,
                             int threads);

/* Flow block tail, node by node (src/levo-flow-estimator.cpp:89-93,106-109,221-227):
 * h = x*gate[b] + r; y = ((norm(h)*gamma + beta) * (scale[b]*1 + 1)) + shift[b],
 * b = row / batch_rows; gate / r / scale / shift may be NULL. */
int oracle_gated_layernorm_modulate_f32(const float *x, const float *gate, const float *r,
                                        const float *gamma, const float *beta, const float *scale,
                                        const float *shift, int64_t batch_rows, float *h_out,
                                        float *y_out, int64_t rows, int64_t dim, float eps);

/* Weight-norm fold, convert/convert_vae.py:196-199.  norms_out may be NULL.
 * Returns -1 (and still writes w) when a row norm is zero, as the reference
 * raises ValueError. */
int oracle_weightnorm_f32(const float *v, const float *g, float *w, float *norms_out, int64_t rows,
                          int64_t cols, int threads);

/* CFG combine, src/levo-renderer-pattern.cpp:123-135. */
int oracle_cfg_combine_f32(const float *uncond, const float *cond, float *out, int64_t n,
                           float guidance);

/* Euler solve with CFG-combined precomputed velocities, restating
 * solve_flow_euler (src/levo-flow-renderer.cpp:57-120) for one state of
 * `batch` rows: runs steps [first_step, first_step + count) and restores the
 * context prefix when the last step has run.  Like the reference it stops at
 * the first step whose combined velocity (:104, returns -1) or updated state
 * (:106, returns -3) holds a non-finite value, leaving `state` at the checkpoint
 * of the steps completed before it and that step in *failed_step (may be
 * NULL; -1 when every step ran).  -2: invalid arguments or out of memory. */
int oracle_cfg_euler_f32(float *state, const float *noise, const float *context,
                         const float *uncond, const float *cond, int64_t batch, int64_t row,
                         int64_t prefix, int64_t first_step, int64_t count, int64_t steps, int cfg,
                         float guidance, float sigma_min, int64_t *failed_step);

/* Window crossfade assembly, src/levo-renderer-pattern.cpp:137-203, over
 * windows [n][channels][window_samples] -> planar [channels][target]; the
 * reference's sequential copy-then-crossfade loop. */
int oracle_assemble_windows_f32(const float *windows, int64_t n, int64_t channels,
                                int64_t window_samples, int64_t hop, int64_t overlap,
                                int64_t target, float *out);

/* Greedy token per row, restating sample_streams with use_sampling = false
 * (src/levo-sampling.cpp:39-48,75-97,129-152).  Returns -1 when a logit is NaN
 * (the reference throws); the indices are still written. */
int oracle_greedy_tokens_f32(const float *logits, int64_t rows, int64_t vocab, const int64_t *recent,
                             int64_t recent_len, float penalty, int64_t penalty_limit,
                             const int64_t *ignore, int64_t n_ignore, int64_t *out);

/* denormalize_latents + channel_major_latent (src/levo-flow-conditioning.cpp:125-135,
 * src/levo-render.cpp:181-193); mean/stddev NULL: transpose only.  And
 * normalize_latents (src/levo-flow-conditioning.cpp:113-123), frame-major. */
void oracle_latent_to_vae_f32(const float *frame_major, const float *mean, const float *stddev,
                              int64_t frames, int64_t dim, float *channel_major);
void oracle_latent_normalize_f32(const float *raw, const float *mean, const float *stddev, int64_t frames,
                                 int64_t dim, float *normalized);

/* IEEE half <-> float (round to nearest even). */
float oracle_half_to_float(uint16_t h);
uint16_t oracle_float_to_half(float f);

#ifdef __cplusplus
}
#endif

#endif /* LEVO_ORACLE_H */
