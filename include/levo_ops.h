/*
 * levo_ops.h — C ABI of the B200 (sm_100a) elementwise, broadcast and
 * row-reduction layer of LeVo2.cpp.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and
 * returns an `int` status (0 = LEVO_OPS_OK, negative = error).  The last error
 * message of the calling thread is returned by levo_ops_last_error(), in the
 * same way as cantor_engine_last_error() (reference: src/cantor-abi.cpp:55-66).
 *
 * Conventions shared by all entry points
 *   - Tensor pointers are DEVICE pointers unless the name says `_host`.
 *     The caller owns every buffer; the kernels allocate nothing.
 *   - Activation tensors are dense C-order [channels][time] (GGML ne=[T,C]),
 *     or [rows][D] for the row reductions, unless a leading dimension is given.
 *   - `stream` is a cudaStream_t (0 = legacy default stream).  Work is only
 *     enqueued; nothing synchronises unless the name says so.
 *   - Output buffers may alias the input read at the same index (in-place use
 *     is supported and is what the decoder chain does); partial overlap at a
 *     different offset is not supported.
 *   - A size of zero is a successful no-op for the elementwise and norm ops.
 *     The Flow CFG/Euler ops reject empty input, as the reference does
 *     (src/levo-renderer-pattern.cpp:127-128, src/levo-flow-renderer.cpp:30-31).
 *   - Reentrant across streams and devices.  A levo_vae_chain object is not:
 *     like the reference's vae_decoder it serves one decode at a time.
 */
#ifndef LEVO_OPS_H
#define LEVO_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LEVO_OPS_API __attribute__((visibility("default")))
#define LEVO_OPS_ABI 1

/* Identical to cudaStream_t; declared here so the header needs no CUDA include. */
typedef struct CUstream_st *levo_stream_t;

typedef enum {
    LEVO_OPS_OK = 0,
    LEVO_OPS_EINVAL = -1,       /* bad argument: null pointer, bad shape, misaligned pointer */
    LEVO_OPS_ELAUNCH = -2,      /* a kernel launch failed (cudaGetLastError) */
    LEVO_OPS_EUNSUPPORTED = -3, /* valid request outside what this build implements */
    LEVO_OPS_ENONFINITE = -4,   /* a finiteness check failed (Euler state / velocity, VAE latent) */
    LEVO_OPS_ECANCELLED = -5,   /* the cancel callback asked to stop between windows */
    LEVO_OPS_ENOMEM = -6,       /* device or pinned host allocation failed (chain create) */
    LEVO_OPS_ECUDA = -7         /* any other CUDA runtime error */
} levo_ops_status;

typedef enum {
    LEVO_DTYPE_F32 = 0,
    LEVO_DTYPE_F16 = 1,
    /* SnakeBeta parameters already prepared by levo_snake_params_prepare():
     * the alpha pointer holds alpha = exp(alpha_log) and the beta pointer holds
     * 1/beta = 1/(exp(beta_log) + 1e-9), both F32; a bias given with it is F32. */
    LEVO_DTYPE_SNAKE_PREPARED = 2
} levo_dtype;

LEVO_OPS_API uint32_t levo_ops_abi_version(void);
/* Thread-local message of the last failing call on this thread ("" if none). */
LEVO_OPS_API const char *levo_ops_last_error(void);

/* ------------------------------------------------------------------------- */
/* a1  SnakeBeta                                                              */
/* ------------------------------------------------------------------------- */
/*
 * Per-channel SnakeBeta parameter precompute, done once per weight load instead
 * of once per launch: alpha_out[c] = exp(alpha_log[c]) and
 * inv_beta_out[c] = 1 / (exp(beta_log[c]) + 1e-9), F32, with the same device
 * arithmetic the kernels apply to log parameters, so a SnakeBeta launch given
 * the outputs with LEVO_DTYPE_SNAKE_PREPARED is bit-identical to one given the
 * logs.  The reference recomputes exp(alpha_log) and exp(beta_log) + 1e-9 as
 * graph nodes on every call (src/levo-audio-ops.cpp:146-151); it has no
 * separate entry point.  alpha_log / beta_log are F32 or F16 (`param_dtype`).
 * Zero channels is a no-op.
 */
LEVO_OPS_API int levo_snake_params_prepare(const void *alpha_log, const void *beta_log, int param_dtype,
                                           int64_t channels, float *alpha_out, float *inv_beta_out,
                                           levo_stream_t stream);

/*
 * y[c][t] = x[c][t] + sin(x[c][t]*alpha_c)^2 / beta_c
 *   alpha_c = exp(alpha_log[c]),  beta_c = exp(beta_log[c]) + 1e-9
 * Replaces levo::detail::snake_beta (src/levo-audio-ops.h:30-33,
 * src/levo-audio-ops.cpp:125-152) as used by run_snake (src/levo-vae.cpp:80-88).
 * alpha_log / beta_log are [channels] in F32 or F16 (`param_dtype`), promoted to
 * F32 in-kernel as the reference's ggml_cast does (src/levo-audio-ops.cpp:32-37),
 * or LEVO_DTYPE_SNAKE_PREPARED outputs of levo_snake_params_prepare().
 * ldx / ldy are row strides in elements (>= time).  Dense rows use the 256-bit
 * vector path; strided rows use the scalar path.
 */
LEVO_OPS_API int levo_snakebeta_f32(const float *x, int64_t ldx,
                                    const void *alpha_log, const void *beta_log, int param_dtype,
                                    float *y, int64_t ldy,
                                    int64_t channels, int64_t time, levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* a2  per-channel bias add                                                   */
/* ------------------------------------------------------------------------- */
/*
 * out[c][t] = in[c][t] + bias[c]; bias F32 or F16.
 * Replaces add_channel_bias (src/levo-audio-ops.cpp:39-52).
 */
LEVO_OPS_API int levo_channel_bias_add_f32(const float *in, const void *bias, int bias_dtype,
                                           float *out, int64_t channels, int64_t time,
                                           levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* a3  fused decoder unit (bias + residual + SnakeBeta [+ tanh])              */
/* ------------------------------------------------------------------------- */
/*
 * One pass over a dense [channels][time] F32 tensor:
 *   x = (residual ? residual : 0) + (u + bias)     (bias optional)
 *   x_out = x                                       (if x_out != NULL)
 *   y_out = snake(x)  or x when alpha_log == NULL   (if y_out != NULL)
 *   flags & LEVO_FUSED_TANH: y_out = tanh(y_out)
 * Covers every elementwise node of run_residual (src/levo-vae.cpp:90-101) and
 * the stage loop (src/levo-vae.cpp:212-235): conv bias add
 * (src/levo-audio-ops.cpp:39-52), residual add (src/levo-vae.cpp:100) and the
 * SnakeBeta that follows (src/levo-audio-ops.cpp:146-151).  The addition order
 * is the reference graph's: residual + (conv + bias).
 */
#define LEVO_FUSED_TANH 1u
typedef struct {
    const float *u;          /* raw conv output (required) */
    const void *bias;        /* [channels] or NULL */
    const float *residual;   /* [channels][time] or NULL */
    const void *alpha_log;   /* [channels] or NULL: no SnakeBeta */
    const void *beta_log;    /* [channels], required with alpha_log */
    float *x_out;            /* NULL: x is not stored */
    float *y_out;            /* NULL: y is not stored */
    int64_t channels;
    int64_t time;
    int32_t param_dtype;     /* dtype of bias / alpha_log / beta_log (SNAKE_PREPARED: F32 bias) */
    uint32_t flags;
} levo_fused_unit;

LEVO_OPS_API int levo_vae_fused_unit_f32(const levo_fused_unit *unit, levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* a4  decoder elementwise chain driver                                       */
/* ------------------------------------------------------------------------- */
/*
 * Stage table of the Oobleck decoder (src/levo-vae.cpp:212-235,
 * src/levo-vae-model.cpp:172-191).  Convolutions are outside this layer and are
 * delegated to a callback; a NULL callback uses built-in stand-ins (index-map
 * copies for the input, upsample and output convs, identity aliases for the
 * residual convs) so the elementwise chain can be run and measured alone.
 */
#define LEVO_VAE_MAX_STAGES 8
#define LEVO_VAE_MAX_RESIDUALS 4

typedef struct {
    int32_t latent_dim;                          /* 64 */
    int32_t audio_channels;                      /* 2 */
    int32_t entry_width;                         /* 2048: conv_in output channels */
    int32_t n_stages;                            /* 5 */
    int32_t stage_width[LEVO_VAE_MAX_STAGES];    /* output channels: 1024,512,256,128,128 */
    int32_t stage_stride[LEVO_VAE_MAX_STAGES];   /* 10,6,4,4,2 */
    int32_t n_residual;                          /* 3 */
    int32_t dilation[LEVO_VAE_MAX_RESIDUALS];    /* 1,3,9 */
} levo_vae_topology;

/* Fills the reference decoder topology (src/levo-vae.cpp:215-216,
 * src/levo-vae-model.cpp:172-191). */
LEVO_OPS_API int levo_vae_topology_reference(levo_vae_topology *out);

/*
 * Number of F32 values in the packed parameter array, in this order
 * (the reference tensor inventory, src/levo-vae-model.cpp:172-191):
 *   input.bias[E]
 *   per stage s (Cin = previous width, Cout = stage_width[s]):
 *     upsample.activation.alpha_log[Cin], .beta_log[Cin], upsample.bias[Cout],
 *     per residual r: pre.alpha_log[Cout], pre.beta_log[Cout], conv.0.bias[Cout],
 *                     post.alpha_log[Cout], post.beta_log[Cout], conv.1.bias[Cout]
 *   output.alpha_log[last], output.beta_log[last]
 */
LEVO_OPS_API int64_t levo_vae_param_count(const levo_vae_topology *topology);

typedef enum {
    LEVO_CONV_INPUT = 0,     /* k7 pad 3, latent_dim -> entry_width         (src/levo-vae.cpp:212-213) */
    LEVO_CONV_UPSAMPLE = 1,  /* ConvTranspose k=2s stride s pad ceil(s/2)   (src/levo-vae.cpp:220-223) */
    LEVO_CONV_RES0 = 2,      /* k7 dilation d pad 3d                        (src/levo-vae.cpp:95-96) */
    LEVO_CONV_RES1 = 3,      /* k1                                          (src/levo-vae.cpp:98-99) */
    LEVO_CONV_OUTPUT = 4     /* k7 pad 3, no bias, last width -> audio      (src/levo-vae.cpp:234-235) */
} levo_conv_kind;

typedef struct {
    int32_t kind;            /* levo_conv_kind */
    int32_t stage;           /* -1 for INPUT / OUTPUT */
    int32_t unit;            /* residual index, -1 otherwise */
    int32_t kernel, stride, padding, dilation;
    const float *input;      /* dense [in_channels][in_length] */
    int64_t in_channels, in_length;
    float *output;           /* suggested dense [out_channels][out_length] buffer */
    int64_t out_channels, out_length;
    /* Where the raw (bias-free) output lives after the call.  Preset to `output`;
     * a callback may point it at `input` when its conv is an identity.  The
     * chain then writes the fused unit's results in place over it. */
    float *result;
} levo_conv_call;

typedef int (*levo_conv_fn)(void *user, levo_conv_call *call, levo_stream_t stream);
/* Non-zero return stops a multi-window decode (polled before each window). */
typedef int (*levo_cancel_fn)(void *user);

typedef struct levo_vae_chain levo_vae_chain;

/*
 * Creates a chain on `device`: uploads the packed parameters and allocates the
 * activation workspace for windows of up to `max_frames` latent frames (three
 * [max C*L] F32 buffers plus double-buffered window I/O).  Mirrors
 * vae_decoder::create (src/levo-vae.cpp:168-170) with the graph allocation of
 * decode (src/levo-vae.cpp:242-246) done once up front.  On the device each
 * SnakeBeta layer is kept as (alpha, 1/beta), computed once here by
 * levo_snake_params_prepare (bit-identical to exponentiating the log form in
 * every launch); the call waits for that work on the legacy default stream.
 */
LEVO_OPS_API int levo_vae_chain_create(levo_vae_chain **out, const levo_vae_topology *topology,
                                       const float *params_host, int64_t max_frames,
                                       levo_conv_fn conv, void *conv_user, int device);
/*
 * Same, with the packed parameters stored as IEEE F16 (the reference's F16 VAE
 * artifact, tools/levo-quantize.cpp:286-312): they stay F16 in HBM and every
 * fused unit promotes them to F32 in-kernel, as the reference's graph casts
 * each F16 weight to F32 before its node (src/levo-audio-ops.cpp:32-37).
 */
LEVO_OPS_API int levo_vae_chain_create_f16(levo_vae_chain **out, const levo_vae_topology *topology,
                                           const uint16_t *params_host, int64_t max_frames,
                                           levo_conv_fn conv, void *conv_user, int device);
LEVO_OPS_API void levo_vae_chain_destroy(levo_vae_chain *chain);

#define LEVO_CHAIN_TANH 1u    /* tanh epilogue on the audio (BASELINE option; the reference has none) */
#define LEVO_CHAIN_TIMING 2u  /* record CUDA events around each kernel class */

/*
 * Device-resident decode of one window: latent [latent_dim][frames] ->
 * audio [audio_channels][frames * prod(strides)], planar F32.
 * Replaces the elementwise part of vae_decoder::decode (src/levo-vae.cpp:172-276).
 */
LEVO_OPS_API int levo_vae_chain_decode(levo_vae_chain *chain, const float *latent, int64_t frames,
                                       float *audio, uint32_t flags, levo_stream_t stream);

/*
 * Stage capture, vae_decoder::decode's capture_stages (src/levo-vae.cpp:230-231,
 * 271-274): after this call every decode also writes each stage's output
 * x_s [stage_width[s]][frames * prod(strides[0..s])] (the hidden state after
 * the stage's last residual unit, channel-major F32) to stage_out[s].
 * Destinations may be host or device memory (the copies use unified
 * addressing); they must hold the largest frame count decoded.  count must be
 * n_stages; stage_out == NULL or count == 0 turns capture off.  While capture
 * is on, levo_vae_chain_decode_windows takes one window at a time.  Each
 * stage then stores x once more (4 B/elem) and copies it out.
 */
LEVO_OPS_API int levo_vae_chain_set_stage_capture(levo_vae_chain *chain, float *const *stage_out,
                                                  int32_t count);

/*
 * Host-to-host decode of `windows` independent windows: latents_host
 * [windows][latent_dim][frames] -> audio_host [windows][audio_channels][samples].
 * Copies in and out inside the call (pinned host buffers overlap the copies
 * with the next window's kernels), polls `cancel` before each window as the
 * reference DECODE loop does (src/cantor-abi.cpp:901-913,
 * src/levo-render.cpp:442-451) and returns LEVO_OPS_ECANCELLED when it fires.
 * Like vae_decoder::decode (src/levo-vae.cpp:189-191) it rejects a window
 * whose latent holds a non-finite value, before that window's work, with
 * LEVO_OPS_ENONFINITE ("latent payload contains a non-finite value").
 * Synchronous: returns after the last window's audio is in host memory.
 */
LEVO_OPS_API int levo_vae_chain_decode_windows(levo_vae_chain *chain, const float *latents_host,
                                               int64_t windows, int64_t frames, float *audio_host,
                                               uint32_t flags, levo_cancel_fn cancel,
                                               void *cancel_user, levo_stream_t stream);

/*
 * DECODE over several GPUs from one process, for a host like the reference's
 * engine (run_decode, src/cantor-abi.cpp:828-925), whose windows are
 * independent (src/levo-render.cpp:442-451): chains[i] (one per device, one
 * topology) decodes the contiguous block [i*W/n .. (i+1)*W/n) of the W windows
 * (block sizes differ by at most one) on its own host thread and its own
 * stream, writing straight into audio_host.  Each block runs as
 * levo_vae_chain_decode_windows (non-finite latent check included); `cancel`
 * is polled by every thread before each of its windows and must be safe to
 * call from several threads.  Returns after every block is in host memory;
 * on failure, the lowest failing chain's status and message (with its index).
 */
LEVO_OPS_API int levo_vae_chains_decode_windows(levo_vae_chain *const *chains, int32_t n_chains,
                                                const float *latents_host, int64_t windows, int64_t frames,
                                                float *audio_host, uint32_t flags, levo_cancel_fn cancel,
                                                void *cancel_user);

/* Kernel classes timed with LEVO_CHAIN_TIMING. */
typedef enum {
    LEVO_KCLASS_ENTRY = 0,      /* conv_in bias + first SnakeBeta        8 B/elem */
    LEVO_KCLASS_UPSAMPLE = 1,   /* upsample bias, x and pre-SnakeBeta   12 B/elem */
    LEVO_KCLASS_POST = 2,       /* conv.0 bias + post-SnakeBeta          8 B/elem */
    LEVO_KCLASS_RESIDUAL = 3,   /* conv.1 bias + residual + next Snake  16 (12) B/elem */
    LEVO_KCLASS_EPILOGUE = 4,   /* tanh on the audio                     8 B/elem */
    LEVO_KCLASS_CONV = 5,       /* conv callback / built-in stand-ins   (not algorithmic) */
    LEVO_KCLASS_COUNT = 6
} levo_kernel_class;

typedef struct {
    int64_t launches;
    double milliseconds;        /* sum of CUDA-event durations */
    double algorithmic_bytes;   /* sum of bytes the launches must move */
    double elements;
} levo_kernel_timing;

/* Synchronises the chain's events and returns per-class totals accumulated
 * since the last reset (out has LEVO_KCLASS_COUNT entries). */
LEVO_OPS_API int levo_vae_chain_timing(levo_vae_chain *chain, levo_kernel_timing *out, int reset);

/*
 * Allocation-free decode of one window.  This entry point has no counterpart in
 * the reference: it exists for callers that cannot let a library call
 * cudaMalloc, such as a real-time render thread (an allocation can synchronise
 * the whole device) or a host engine that owns a fixed device-memory budget and
 * hands out only its own buffers.
 *
 * Same work and result as levo_vae_chain_decode, but without a levo_vae_chain:
 *   params  device pointer to the packed parameters (levo_vae_param_count floats),
 *   latent  device [latent_dim][frames], audio device [audio_channels][frames * prod(strides)],
 *   conv    optional convolution callback (NULL: built-in stand-ins), as for the chain.
 * The three activation buffers come from one static device array of
 * 3 x 2^21 floats (24 MiB) that every GPU loading this library holds until the
 * process exits; the largest activation tensor of the window must fit in
 * 2^21 floats (the reference topology: frames <= 8), else LEVO_OPS_EINVAL.
 * Nothing is allocated: no cudaMalloc, no cudaFree, no events.
 * Each call made outside stream capture looks up the array's device address
 * (cudaGetSymbolAddress) with the device current, so a device reset leaves no
 * stale address; a call under capture uses the address of the last call outside
 * it, so make the first call on a device before any stream capture.  All calls
 * on a device share the array and it keeps the
 * previous call's contents (the decode writes every value before reading it,
 * so nothing needs clearing); calls that overlap on the GPU (other streams,
 * other threads) race on it.  flags: LEVO_CHAIN_TANH only.
 */
LEVO_OPS_API int levo_vae_decode_noalloc_f32(const levo_vae_topology *topology, const float *params,
                                             const float *latent, int64_t frames, float *audio,
                                             levo_conv_fn conv, void *conv_user, uint32_t flags,
                                             levo_stream_t stream);

/* Built-in conv stand-in: out[c][t] = in[c mod in_channels][t / stride]. */
LEVO_OPS_API int levo_conv_standin_f32(const float *in, int64_t in_channels, int64_t in_length,
                                       float *out, int64_t out_channels, int64_t out_length,
                                       int32_t stride, levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* a5 / a6  residual add + RMSNorm / LayerNorm                                */
/* ------------------------------------------------------------------------- */
/*
 * h = x + r (rounded to the activation type), then
 *   RMSNorm:   y = h / sqrt(mean(h^2) + eps) * gamma
 *   LayerNorm: y = (h - mean) / sqrt(var + eps) * gamma + beta
 * Reductions in F32 over each row of `dim` elements.  `r` may be NULL (plain
 * norm; h_out is then ignored).  h_out may be NULL when the sum is not needed.
 * LEVO_NORM_F16_BOUNDARY (F16 only): the normalised value is rounded to F16
 * before the gamma product, as the F16-activation path does
 * (src/levo-kv.cpp:149-170).
 * RMSNorm replaces rms_norm_weighted + the residual add (src/levo-lm.cpp:131-138,
 * 198-202; src/levo-kv.cpp:153-170,462-472).  LayerNorm replaces layer_norm
 * (src/levo-flow-estimator.cpp:106-109) + its residual add
 * (src/levo-flow-estimator.cpp:221-227).
 * Supported dim: 1..8192 (F16), 1..4096 (F32).
 */
#define LEVO_NORM_F16_BOUNDARY 1u
LEVO_OPS_API int levo_add_rmsnorm_f16(const void *x, const void *r, const float *gamma,
                                      void *h_out, void *y_out, int64_t rows, int64_t dim,
                                      float eps, uint32_t flags, levo_stream_t stream);
LEVO_OPS_API int levo_add_rmsnorm_f32(const float *x, const float *r, const float *gamma,
                                      float *h_out, float *y_out, int64_t rows, int64_t dim,
                                      float eps, uint32_t flags, levo_stream_t stream);
LEVO_OPS_API int levo_add_layernorm_f16(const void *x, const void *r, const float *gamma,
                                        const float *beta, void *h_out, void *y_out,
                                        int64_t rows, int64_t dim, float eps, uint32_t flags,
                                        levo_stream_t stream);
LEVO_OPS_API int levo_add_layernorm_f32(const float *x, const float *r, const float *gamma,
                                        const float *beta, float *h_out, float *y_out,
                                        int64_t rows, int64_t dim, float eps, uint32_t flags,
                                        levo_stream_t stream);

/*
 * Flow block form (next item f2): gated residual + LayerNorm + adaLN modulation
 * in one pass over F32 [rows][dim], rows = batch * batch_rows:
 *   h = r + x * gate[b]                               (src/levo-flow-estimator.cpp:221-227,243-246)
 *   y = (LN(h) * gamma + beta) * (1 + scale[b]) + shift[b]
 *                                                     (src/levo-flow-estimator.cpp:89-93,106-109,209-212)
 * b = row / batch_rows; gate / scale / shift are [batch][dim] (the modulation
 * chunks) and each may be NULL (no gate: h = r + x; r NULL: h = x * gate).
 */
LEVO_OPS_API int levo_gated_layernorm_modulate_f32(const float *x, const float *gate, const float *r,
                                                   const float *gamma, const float *beta,
                                                   const float *scale, const float *shift,
                                                   int64_t batch_rows, float *h_out, float *y_out,
                                                   int64_t rows, int64_t dim, float eps,
                                                   levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* a9  weight-norm fold                                                       */
/* ------------------------------------------------------------------------- */
/*
 * w[o][:] = v[o][:] * (g[o] / ||v[o][:]||_2), the norm over each row of `cols`
 * values (dim=0 weight norm; for a ConvTranspose weight [Cin][Cout][K] the row
 * is the input channel).  Replaces _fold_weight_norm (convert/convert_vae.py:187-199)
 * and _materialize_weight_norm (convert/convert_flow.py:288-293).
 * `norms_out` (optional, [rows] F32): the row norms, so the caller can reject a
 * zero norm as the reference does (convert/convert_vae.py:197-198).
 */
LEVO_OPS_API int levo_weightnorm_f32(const float *v, const float *g, float *w, float *norms_out,
                                     int64_t rows, int64_t cols, levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* a7 / a8  Flow CFG combine + Euler update                                   */
/* ------------------------------------------------------------------------- */
/*
 * out = uncond + guidance * (cond - uncond), elementwise, without FMA
 * contraction.  Replaces combine_renderer_cfg (src/levo-renderer-pattern.cpp:123-135)
 * and the loop in evaluate_velocity (src/levo-flow-renderer.cpp:305-308).
 */
LEVO_OPS_API int levo_cfg_combine_f32(const float *uncond, const float *cond, float *out,
                                      int64_t n, float guidance, levo_stream_t stream);

/*
 * In-context interpolation of the first `prefix` elements of each batch row
 * before a velocity evaluation (src/levo-flow-renderer.cpp:93-101):
 *   state[i] = noise_scale * noise[i] + time * context[i]
 * with time = step * (1/steps) and noise_scale = 1 - (1 - sigma_min) * time
 * computed in F32 exactly as the reference.  state/noise/context are
 * [batch][row] with `row` = frames * latent_dim (frame-major).
 */
LEVO_OPS_API int levo_flow_incontext_f32(float *state, const float *noise, const float *context,
                                         int64_t batch, int64_t row, int64_t prefix,
                                         int64_t step, int64_t steps, float sigma_min,
                                         levo_stream_t stream);

/*
 * One Euler step with the CFG combine fused (src/levo-flow-renderer.cpp:102-106,
 * 301-308):  v = cfg ? uncond + guidance*(cond - uncond) : uncond;  state += dt*v
 * where dt = 1/steps in F32.  `cond` is ignored (may be NULL) when cfg == 0.
 * `status` (optional device int32): bit value 1 is set when a velocity value is
 * not finite, bit value 2 when an updated state value is not finite (the
 * reference's require_finite checks, src/levo-flow-renderer.cpp:104,106).  The
 * caller clears it; the kernel only sets bits.
 */
LEVO_OPS_API int levo_euler_cfg_step_f32(float *state, const float *uncond, const float *cond,
                                         int64_t n, int32_t cfg, float guidance, int64_t steps,
                                         int32_t *status, levo_stream_t stream);

/*
 * Status word of the multi-step solves: the first failing step and its kind,
 *   LEVO_EULER_STATUS(step, kind) = ((LEVO_EULER_STEP_LIMIT - step) << 2) | kind,
 * kind LEVO_EULER_FAIL_VELOCITY (3: a combined velocity was not finite; as in
 * levo_euler_cfg_step_f32 both bits are set, because the state would be too)
 * or LEVO_EULER_FAIL_STATE (2: an updated state was not finite after a finite
 * velocity).  Kernels combine them with atomicMax, so the word keeps the
 * earliest step, and the velocity kind on a tie (the reference checks the
 * velocity first, src/levo-flow-renderer.cpp:104,106).  0 = no failure.
 */
#define LEVO_EULER_STEP_LIMIT 268435456 /* 2^28: steps of a solve must stay below it */
#define LEVO_EULER_FAIL_STATE 2
#define LEVO_EULER_FAIL_VELOCITY 3
#define LEVO_EULER_STATUS(step, kind) ((int32_t)((((int64_t)LEVO_EULER_STEP_LIMIT - (int64_t)(step)) << 2) | (kind)))
#define LEVO_EULER_STATUS_STEP(status) \
    (((status) >> 2) ? (int64_t)LEVO_EULER_STEP_LIMIT - (int64_t)((status) >> 2) : (int64_t)-1)
#define LEVO_EULER_STATUS_KIND(status) ((status) & 3)

/*
 * Fused multi-step solve for velocities known up front (benchmarks, replay of
 * a recorded solve).  Runs steps [first_step, first_step + count) of a
 * `steps`-step solve, reproducing per step the in-context interpolation, the
 * CFG combine and the Euler update, and after the final step (when it is in
 * range) the context restore (src/levo-flow-renderer.cpp:90-118).
 * uncond / cond are [count][batch][row] (velocity of step first_step + k at k).
 * Stopping after `count` steps gives the reference's durable per-step resume
 * boundary (src/levo-flow-renderer.cpp:74-88,107-110).
 * `status` (optional device int32, cleared by the caller): the first failing
 * step and kind as LEVO_EULER_STATUS.  An element whose velocity or state goes
 * non-finite stops there, keeping its state after the last step it completed,
 * and the context restore is skipped for it; elements that did not fail run
 * every step.  levo_cfg_euler_solve_f32 gives the reference's exact checkpoint
 * for the whole state instead.  steps >= LEVO_EULER_STEP_LIMIT:
 * LEVO_OPS_EUNSUPPORTED.
 */
LEVO_OPS_API int levo_cfg_euler_multi_f32(float *state, const float *noise, const float *context,
                                          const float *uncond, const float *cond,
                                          int64_t batch, int64_t row, int64_t prefix,
                                          int64_t first_step, int64_t count, int64_t steps,
                                          int32_t cfg, float guidance, float sigma_min,
                                          int32_t *status, levo_stream_t stream);

/*
 * solve_flow_euler over velocities known up front, with its error semantics
 * (src/levo-flow-renderer.cpp:57-120): runs steps [first_step, first_step +
 * count) as levo_cfg_euler_multi_f32 and, when some step's combined velocity
 * (:104) or updated state (:106) holds a non-finite value, stops where the
 * reference throws: `state` is left at the reference's checkpoint (every
 * element after the steps completed before that step, the checkpoint the
 * reference writes at :107-110), *completed_steps receives that step, and the
 * call returns LEVO_OPS_ENONFINITE with the reference's message ("Euler velocity
 * contains a non-finite value" / "Euler state contains a non-finite value").
 * On success *completed_steps = first_step + count.  All batch rows form one
 * solve: they stop together.  Before any step, like the reference
 * (:71-72,81), it returns LEVO_OPS_ENONFINITE ("Euler noise / in-context
 * latent / resume state contains a non-finite value") with `state` untouched
 * when noise (or, without noise, the starting state at first_step 0), the
 * whole context [batch][row], or the state it resumes from (first_step > 0)
 * holds a non-finite value.
 * checkpoint: caller-owned device scratch of batch * row F32 (the state before
 * the call, kept to replay the completed steps after a failure); status: a
 * caller-owned device int32 (receives LEVO_EULER_STATUS).  Synchronous: the
 * call waits for `stream` before it returns.
 */
LEVO_OPS_API int levo_cfg_euler_solve_f32(float *state, const float *noise, const float *context,
                                          const float *uncond, const float *cond,
                                          int64_t batch, int64_t row, int64_t prefix,
                                          int64_t first_step, int64_t count, int64_t steps,
                                          int32_t cfg, float guidance, float sigma_min,
                                          float *checkpoint, int32_t *status, int64_t *completed_steps,
                                          levo_stream_t stream);

/*
 * Velocity callback of levo_flow_euler_solve_f32 (the estimator evaluation of
 * solve_flow_euler's velocity callback, src/levo-flow-renderer.cpp:102):
 * given the device state the estimator sees at `step` (time = step / steps),
 * returns a device pointer to the velocity, [2][n] F32 (row 0 unconditional,
 * row 1 conditional) when the solve combines CFG, else [n]; NULL reports a
 * failure.  Work it enqueues on `stream` is ordered before the update.
 */
typedef const float *(*levo_velocity_fn)(void *user, const float *state, int64_t step, float time,
                                         levo_stream_t stream);

/*
 * solve_flow_euler (src/levo-flow-renderer.cpp:57-120) on a device state
 * [frames][latent_dim], one velocity evaluation per step: for each step from
 * first_step (a resume point, :76-84) to steps - 1 it polls `cancel`, applies
 * the in-context interpolation (:93-101), calls `velocity`, and runs the fused
 * CFG combine + Euler update with the reference's finiteness checks
 * (:104,106), reading the status back after each step; after the last step it
 * restores the context prefix (:113-114).  Before the first step it checks
 * noise, context (both [frames][latent_dim]) and, when resuming, the state as
 * the reference does (:71-72,81): LEVO_OPS_ENONFINITE with its message and
 * `state` untouched.
 * checkpoint (optional device [frames * latent_dim] F32): the state before each
 * step is kept there, so that on a non-finite velocity or state the solve
 * leaves `state` at the reference's checkpoint (:107-110) and returns
 * LEVO_OPS_ENONFINITE with the reference's message; without it the state is
 * left as the failing step's update wrote it.  status: caller-owned device
 * int32 scratch.  *completed_steps (host) receives the steps completed (the
 * resume point after a failure or a cancellation, `steps` on success).
 * cancel (optional) returning non-zero: LEVO_OPS_ECANCELLED with the state at
 * the last completed step.  Synchronises `stream` once per step.
 */
LEVO_OPS_API int levo_flow_euler_solve_f32(float *state, const float *noise, const float *context,
                                           int64_t frames, int64_t latent_dim, int64_t incontext_frames,
                                           float sigma_min, int64_t steps, int64_t first_step, int32_t cfg,
                                           float guidance, levo_velocity_fn velocity, void *velocity_user,
                                           levo_cancel_fn cancel, void *cancel_user, float *checkpoint,
                                           int32_t *status, int64_t *completed_steps, levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* next (f2)  latent normalisation and the layout change into the VAE         */
/* ------------------------------------------------------------------------- */
/*
 * channel_major[c][f] = frame_major[f][c] * stddev[c] + mean[c]
 * Replaces denormalize_latents (src/levo-flow-conditioning.cpp:125-135)
 * followed by channel_major_latent (src/levo-render.cpp:181-193): the Flow
 * renderer's frame-major [frames][dim] window becomes the VAE's channel-major
 * [dim][frames] input in one pass.  mean and stddev both NULL: transpose only.
 * Not in place.  Bit-identical to the reference (mul then add, no FMA).
 * status (optional device int32, zeroed by the caller): bit 0 set when an
 * input value is non-finite, where the reference throws "normalized latent
 * contains a non-finite value" (:128).
 */
LEVO_OPS_API int levo_latent_to_vae_f32(const float *frame_major, const float *mean, const float *stddev,
                                        int64_t frames, int64_t dim, float *channel_major,
                                        int32_t *status, levo_stream_t stream);
/*
 * normalized[f][c] = (raw[f][c] - mean[c]) / stddev[c], frame-major
 * (normalize_latents, src/levo-flow-conditioning.cpp:113-123).  May run in place.
 * status (optional device int32, zeroed by the caller): bit 0 set when a raw
 * value is non-finite, where the reference throws "raw latent contains a
 * non-finite value" (:116).
 */
LEVO_OPS_API int levo_latent_normalize_f32(const float *raw, const float *mean, const float *stddev,
                                           int64_t frames, int64_t dim, float *normalized, int32_t *status,
                                           levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* next (f3)  greedy next-token selection over LeLM logits                    */
/* ------------------------------------------------------------------------- */
/*
 * Replaces Sampler::sample_streams with use_sampling = false
 * (src/levo-sampling.cpp:129-152, sample_top_k_counted :75-97): for each row
 * (stream) of `vocab` logits (row stride ld),
 *   1. each distinct id of recent[row][0..recent_len) in [0, penalty_limit)
 *      divides its logit once by `penalty` (:39-48; penalty_limit <= 0 means
 *      vocab; the reference passes vocab - 1 so the EOS id is exempt; ids < 0
 *      are skipped, so rows can be padded with -1);
 *   2. row 0 only: ids in ignore[0..n_ignore) become -inf (:146-148);
 *   3. tokens_out[row] = index of the first maximum (std::max_element).
 * Bit-exact with the reference.  recent may be NULL.  status (optional device
 * int32, zeroed by the caller): bit 0 (value 1) set when a logit is NaN, where
 * the reference throws "logits contain NaN" (:81).  vocab <= 131072.
 */
LEVO_OPS_API int levo_greedy_tokens_f32(const float *logits, int64_t rows, int64_t vocab, int64_t ld,
                                        const int64_t *recent, int64_t recent_len, float penalty,
                                        int64_t penalty_limit, const int64_t *ignore, int64_t n_ignore,
                                        int64_t *tokens_out, int32_t *status, levo_stream_t stream);

/* ------------------------------------------------------------------------- */
/* next (f1)  window assembly: crossfade + crop (+ interleave)                */
/* ------------------------------------------------------------------------- */
/*
 * Replaces assemble_renderer_audio (src/levo-renderer-pattern.cpp:137-203) and
 * the L/R interleave of the render result (src/levo-render.cpp:476-480).
 * windows: decoded windows [n_windows][channels][window_samples] (planar, as the
 * decoder writes them).  Window k starts at k*hop_samples; the first
 * overlap_samples of each window after the first are crossfaded linearly into
 * what is already there (alpha = s / (overlap_samples - 1), previous * (1 - alpha)
 * + current * alpha); the song is cropped to target_samples.
 * out: planar [channels][target_samples] (interleaved == 0, the cantor ABI's
 * [L..., R...] layout) or interleaved [target_samples][channels].
 * Requires 2 <= overlap <= hop and hop + overlap <= window (or overlap == 0), as
 * the reference's 750 / 250 / 1000-frame schedule satisfies.  Bit-identical to
 * the reference (same F32 expression order).
 * status (optional device int32, zeroed by the caller): the reference rejects
 * a decoded window holding a non-finite sample (require_finite_audio, :159-160:
 * "decoded left / right channel contains non-finite samples", windows in
 * order, left before right).  Every sample of every window is checked, and the
 * first failing pair is recorded as LEVO_ASSEMBLE_STATUS(window * channels +
 * channel) (0: all finite; the output is then not the reference's, which
 * throws).  n_windows * channels must stay below LEVO_ASSEMBLE_STATUS_LIMIT.
 */
#define LEVO_ASSEMBLE_STATUS_LIMIT 1073741824 /* 2^30 */
#define LEVO_ASSEMBLE_STATUS(pair) (LEVO_ASSEMBLE_STATUS_LIMIT - (pair))
#define LEVO_ASSEMBLE_STATUS_PAIR(word) (LEVO_ASSEMBLE_STATUS_LIMIT - (word))
LEVO_OPS_API int levo_assemble_windows_f32(const float *windows, int64_t n_windows, int64_t channels,
                                           int64_t window_samples, int64_t hop_samples,
                                           int64_t overlap_samples, int64_t target_samples,
                                           float *out, int32_t interleaved, int32_t *status,
                                           levo_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LEVO_OPS_H */
