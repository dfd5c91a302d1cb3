/*
 * levo_oracle.c — CPU restatement of the LeVo2.cpp elementwise / reduction
 * path.  TEST INFRASTRUCTURE ONLY: the parity checker of the CUDA kernels and
 * the timed CPU baseline of bench.py; never linked into the product.
 *
 * The graph-level structure follows the reference files cited per function.
 * Each GGML node is one materialised pass over its tensor, parallelised over
 * rows with pthreads the way GGML's CPU backend splits a node across its
 * thread pool.  Compiled with -ffp-contract=off so every node rounds on its
 * own, as the reference's separate nodes and its ISO C++17 host loops do.
 */
#define _GNU_SOURCE
#include "levo_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* threading                                                                 */
/* ------------------------------------------------------------------------ */

typedef void (*range_fn)(void *ctx, int64_t r0, int64_t r1);

typedef struct {
    range_fn fn;
    void *ctx;
    int64_t r0, r1;
} range_job;

static void *range_main(void *arg) {
    range_job *j = (range_job *)arg;
    if (j->r1 > j->r0) j->fn(j->ctx, j->r0, j->r1);
    return NULL;
}

static int resolve_threads(int threads) {
    if (threads > 0) return threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

/* Splits rows [0, n) into contiguous ranges, one per thread. */
static void parallel_rows(int64_t n, int threads, range_fn fn, void *ctx) {
    threads = resolve_threads(threads);
    if (threads > 256) threads = 256;
    if ((int64_t)threads > n) threads = (int)(n > 0 ? n : 1);
    if (threads <= 1) {
        if (n > 0) fn(ctx, 0, n);
        return;
    }
    pthread_t tid[256];
    range_job jobs[256];
    int started[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].r0 = n * t / threads;
        jobs[t].r1 = n * (t + 1) / threads;
        started[t] = t > 0 && pthread_create(&tid[t], NULL, range_main, &jobs[t]) == 0;
        if (t > 0 && !started[t]) range_main(&jobs[t]);
    }
    range_main(&jobs[0]);
    for (int t = 1; t < threads; ++t)
        if (started[t]) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* half precision                                                            */
/* ------------------------------------------------------------------------ */

float oracle_half_to_float(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

uint16_t oracle_float_to_half(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

/* ------------------------------------------------------------------------ */
/* GGML-style nodes over [rows][len] tensors (rows = channels)               */
/* ------------------------------------------------------------------------ */

enum node_kind {
    NODE_MUL_ROW,   /* out = a * p[row]        (ggml_mul with a [1,C] broadcast)  */
    NODE_SIN,       /* out = sin(a)                                               */
    NODE_SQR,       /* out = a * a                                                */
    NODE_DIV_ROW,   /* out = a / p[row]        (ggml_div broadcast)               */
    NODE_ADD,       /* out = a + b                                                */
    NODE_ADD_ROW,   /* out = a + p[row]        (ggml_add with a [1,C] broadcast)  */
    NODE_TANH       /* out = tanh(a)                                              */
};

typedef struct {
    int kind;
    const float *a;
    const float *b;
    const float *p;
    float *out;
    int64_t len;
} node_job;

static void node_rows(void *ctx, int64_t r0, int64_t r1) {
    const node_job *j = (const node_job *)ctx;
    for (int64_t r = r0; r < r1; ++r) {
        const float *a = j->a + r * j->len;
        const float *b = j->b ? j->b + r * j->len : NULL;
        float *o = j->out + r * j->len;
        const float pv = j->p ? j->p[r] : 0.f;
        switch (j->kind) {
            case NODE_MUL_ROW:
                for (int64_t t = 0; t < j->len; ++t) o[t] = a[t] * pv;
                break;
            case NODE_SIN:
                for (int64_t t = 0; t < j->len; ++t) o[t] = sinf(a[t]);
                break;
            case NODE_SQR:
                for (int64_t t = 0; t < j->len; ++t) o[t] = a[t] * a[t];
                break;
            case NODE_DIV_ROW:
                for (int64_t t = 0; t < j->len; ++t) o[t] = a[t] / pv;
                break;
            case NODE_ADD:
                for (int64_t t = 0; t < j->len; ++t) o[t] = a[t] + b[t];
                break;
            case NODE_ADD_ROW:
                for (int64_t t = 0; t < j->len; ++t) o[t] = a[t] + pv;
                break;
            case NODE_TANH:
                for (int64_t t = 0; t < j->len; ++t) o[t] = tanhf(a[t]);
                break;
        }
    }
}

static void node(int kind, const float *a, const float *b, const float *p, float *out,
                 int64_t rows, int64_t len, int threads) {
    node_job j = {kind, a, b, p, out, len};
    parallel_rows(rows, threads, node_rows, &j);
}

/* SnakeBeta graph of src/levo-audio-ops.cpp:146-151:
 *   alpha = exp(alpha_log); beta = scale_bias(exp(beta_log), 1, 1e-9)
 *   y = x + sqr(sin(x * alpha)) / beta
 * `tmp` holds the intermediate nodes (GGML's allocator reuses one buffer). */
static void snake_graph(const float *x, const float *alog, const float *blog, float *y, float *tmp,
                        int64_t rows, int64_t len, int threads) {
    float *alpha = (float *)malloc(sizeof(float) * (size_t)rows);
    float *beta = (float *)malloc(sizeof(float) * (size_t)rows);
    for (int64_t c = 0; c < rows; ++c) {
        alpha[c] = expf(alog[c]);
        beta[c] = expf(blog[c]) * 1.0f + 1.0e-9f;
    }
    node(NODE_MUL_ROW, x, NULL, alpha, tmp, rows, len, threads);
    node(NODE_SIN, tmp, NULL, NULL, tmp, rows, len, threads);
    node(NODE_SQR, tmp, NULL, NULL, tmp, rows, len, threads);
    node(NODE_DIV_ROW, tmp, NULL, beta, tmp, rows, len, threads);
    node(NODE_ADD, x, tmp, NULL, y, rows, len, threads);
    free(alpha);
    free(beta);
}

int oracle_snakebeta_f32(const float *x, const float *alpha_log, const float *beta_log, float *y,
                         int64_t channels, int64_t time, int threads) {
    if (!x || !alpha_log || !beta_log || !y || channels < 0 || time < 0) return -1;
    if (channels == 0 || time == 0) return 0;
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(channels * time));
    if (!tmp) return -2;
    snake_graph(x, alpha_log, beta_log, y, tmp, channels, time, threads);
    free(tmp);
    return 0;
}

int oracle_snakebeta_f16params(const float *x, const uint16_t *alpha_log, const uint16_t *beta_log,
                               float *y, int64_t channels, int64_t time, int threads) {
    if (!alpha_log || !beta_log || channels < 0) return -1;
    float *a = (float *)malloc(sizeof(float) * (size_t)(channels + 1));
    float *b = (float *)malloc(sizeof(float) * (size_t)(channels + 1));
    for (int64_t c = 0; c < channels; ++c) {
        a[c] = oracle_half_to_float(alpha_log[c]);
        b[c] = oracle_half_to_float(beta_log[c]);
    }
    const int rc = oracle_snakebeta_f32(x, a, b, y, channels, time, threads);
    free(a);
    free(b);
    return rc;
}

int oracle_channel_bias_add_f32(const float *in, const float *bias, float *out, int64_t channels,
                                int64_t time, int threads) {
    if (!in || !bias || !out || channels < 0 || time < 0) return -1;
    node(NODE_ADD_ROW, in, NULL, bias, out, channels, time, threads);
    return 0;
}

int oracle_fused_unit_f32(const float *u, const float *bias, const float *residual,
                          const float *alpha_log, const float *beta_log, float *x_out, float *y_out,
                          int64_t channels, int64_t time, int tanh_out, int threads) {
    if (!u || channels < 0 || time < 0) return -1;
    if ((alpha_log == NULL) != (beta_log == NULL)) return -1;
    if (channels == 0 || time == 0) return 0;
    const size_t n = (size_t)(channels * time);
    float *x = (float *)malloc(sizeof(float) * n);
    float *tmp = (float *)malloc(sizeof(float) * n);
    float *y = (float *)malloc(sizeof(float) * n);
    if (!x || !tmp || !y) return -2;
    if (bias) node(NODE_ADD_ROW, u, NULL, bias, x, channels, time, threads);
    else memcpy(x, u, sizeof(float) * n);
    if (residual) node(NODE_ADD, residual, x, NULL, x, channels, time, threads);
    if (alpha_log) snake_graph(x, alpha_log, beta_log, y, tmp, channels, time, threads);
    else memcpy(y, x, sizeof(float) * n);
    if (tanh_out) node(NODE_TANH, y, NULL, NULL, y, channels, time, threads);
    if (x_out) memcpy(x_out, x, sizeof(float) * n);
    if (y_out) memcpy(y_out, y, sizeof(float) * n);
    free(x);
    free(tmp);
    free(y);
    return 0;
}

void oracle_conv_standin_f32(const float *in, int64_t cin, int64_t lin, float *out, int64_t cout,
                             int64_t lout, int stride) {
    for (int64_t c = 0; c < cout; ++c)
        for (int64_t t = 0; t < lout; ++t) {
            const int64_t st = t / stride;
            out[c * lout + t] = st < lin ? in[(c % cin) * lin + st] : 0.f;
        }
}

/* Stage loop of src/levo-vae.cpp:212-235 with run_residual (src/levo-vae.cpp:90-101).
 * Convs are the stand-ins: the input / upsample / output convs are index-map
 * copies and the residual convs are identities; every conv's bias is a
 * separate add node (src/levo-audio-ops.cpp:39-52). */
int oracle_vae_chain_f32(const int32_t *topo, const float *P, const float *latent, int64_t frames,
                         float *audio, int tanh_out, int threads) {
    return oracle_vae_chain_stages_f32(topo, P, latent, frames, audio, tanh_out, threads, NULL);
}

/* Stage s's output (the hidden state after its residual units, src/levo-vae.cpp:230-231)
 * is copied to stages[s] when stages is non-NULL. */
int oracle_vae_chain_stages_f32(const int32_t *topo, const float *P, const float *latent, int64_t frames,
                                float *audio, int tanh_out, int threads, float *const *stages) {
    if (!topo || !P || !latent || !audio || frames <= 0) return -1;
    const int latent_dim = topo[0], audio_channels = topo[1], entry = topo[2], S = topo[3];
    if (S < 1 || S > 8) return -1;
    const int32_t *widths = topo + 4;
    const int32_t *strides = topo + 4 + S;
    const int R = topo[4 + 2 * S];
    if (R < 0 || R > 4) return -1;

    int64_t maxe = (int64_t)entry * frames, len = frames, cin = entry;
    for (int s = 0; s < S; ++s) {
        len *= strides[s];
        if ((int64_t)widths[s] * len > maxe) maxe = (int64_t)widths[s] * len;
    }
    float *x = (float *)malloc(sizeof(float) * (size_t)maxe);
    float *a = (float *)malloc(sizeof(float) * (size_t)maxe);
    float *b = (float *)malloc(sizeof(float) * (size_t)maxe);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)maxe);
    if (!x || !a || !b || !tmp) {
        free(x);
        free(a);
        free(b);
        free(tmp);
        return -2;
    }

    int64_t off = 0;
    const float *in_bias = P + off;
    off += entry;
    len = frames;
    oracle_conv_standin_f32(latent, latent_dim, frames, x, entry, frames, 1);
    node(NODE_ADD_ROW, x, NULL, in_bias, x, entry, frames, threads);
    cin = entry;
    for (int s = 0; s < S; ++s) {
        const int64_t cout = widths[s], lout = len * strides[s];
        const float *up_a = P + off;
        off += cin;
        const float *up_b = P + off;
        off += cin;
        const float *up_bias = P + off;
        off += cout;
        snake_graph(x, up_a, up_b, a, tmp, cin, len, threads);
        oracle_conv_standin_f32(a, cin, len, x, cout, lout, strides[s]);
        node(NODE_ADD_ROW, x, NULL, up_bias, x, cout, lout, threads);
        for (int r = 0; r < R; ++r) {
            const float *pre_a = P + off;
            off += cout;
            const float *pre_b = P + off;
            off += cout;
            const float *b0 = P + off;
            off += cout;
            const float *post_a = P + off;
            off += cout;
            const float *post_b = P + off;
            off += cout;
            const float *b1 = P + off;
            off += cout;
            snake_graph(x, pre_a, pre_b, a, tmp, cout, lout, threads);      /* pre snake       */
            node(NODE_ADD_ROW, a, NULL, b0, b, cout, lout, threads);         /* conv.0 (id)+b0  */
            snake_graph(b, post_a, post_b, a, tmp, cout, lout, threads);     /* post snake      */
            node(NODE_ADD_ROW, a, NULL, b1, b, cout, lout, threads);         /* conv.1 (id)+b1  */
            node(NODE_ADD, x, b, NULL, x, cout, lout, threads);              /* residual add    */
        }
        if (stages && stages[s]) memcpy(stages[s], x, sizeof(float) * (size_t)(cout * lout));
        cin = cout;
        len = lout;
    }
    const float *out_a = P + off;
    off += cin;
    const float *out_b = P + off;
    snake_graph(x, out_a, out_b, a, tmp, cin, len, threads);
    oracle_conv_standin_f32(a, cin, len, audio, audio_channels, len, 1);
    if (tanh_out) node(NODE_TANH, audio, NULL, NULL, audio, audio_channels, len, threads);
    free(x);
    free(a);
    free(b);
    free(tmp);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* norms                                                                     */
/* ------------------------------------------------------------------------ */

typedef struct {
    const void *x, *r;
    const float *gamma, *beta;
    void *h_out, *y_out;
    int64_t dim;
    float eps;
    int half, layer, f16_boundary;
} norm_job;

static float act_load(const void *p, int64_t i, int half) {
    return half ? oracle_half_to_float(((const uint16_t *)p)[i]) : ((const float *)p)[i];
}
static float act_round(float v, int half) {
    return half ? oracle_half_to_float(oracle_float_to_half(v)) : v;
}
static void act_store(void *p, int64_t i, float v, int half) {
    if (half) ((uint16_t *)p)[i] = oracle_float_to_half(v);
    else ((float *)p)[i] = v;
}

static void norm_rows(void *ctx, int64_t r0, int64_t r1) {
    const norm_job *j = (const norm_job *)ctx;
    float *h = (float *)malloc(sizeof(float) * (size_t)j->dim);
    float *n = (float *)malloc(sizeof(float) * (size_t)j->dim);
    for (int64_t row = r0; row < r1; ++row) {
        const int64_t base = row * j->dim;
        /* residual add node, rounded to the activation type (ggml_add on F16) */
        for (int64_t i = 0; i < j->dim; ++i) {
            float v = act_load(j->x, base + i, j->half);
            if (j->r) v = act_round(v + act_load(j->r, base + i, j->half), j->half);
            h[i] = v;
        }
        if (j->layer) {
            /* ggml_norm: mean, then the centred second moment */
            double sum = 0.0;
            for (int64_t i = 0; i < j->dim; ++i) sum += (double)h[i];
            const float mean = (float)(sum / (double)j->dim);
            double sum2 = 0.0;
            for (int64_t i = 0; i < j->dim; ++i) {
                const float v = h[i] - mean;
                n[i] = v;
                sum2 += (double)(v * v);
            }
            const float variance = (float)(sum2 / (double)j->dim);
            const float scale = 1.0f / sqrtf(variance + j->eps);
            for (int64_t i = 0; i < j->dim; ++i) n[i] = n[i] * scale;
        } else {
            /* ggml_rms_norm */
            double sum = 0.0;
            for (int64_t i = 0; i < j->dim; ++i) sum += (double)(h[i] * h[i]);
            const float mean = (float)(sum / (double)j->dim);
            const float scale = 1.0f / sqrtf(mean + j->eps);
            for (int64_t i = 0; i < j->dim; ++i) n[i] = h[i] * scale;
        }
        for (int64_t i = 0; i < j->dim; ++i) {
            float v = n[i];
            if (j->f16_boundary) v = act_round(v, 1); /* cast F16 before the weight product */
            v = v * j->gamma[i];                      /* ggml_mul by the weight */
            if (j->layer) v = v + j->beta[i];         /* ggml_add of the bias */
            act_store(j->y_out, base + i, v, j->half);
            if (j->h_out && j->r) act_store(j->h_out, base + i, h[i], j->half);
        }
    }
    free(h);
    free(n);
}

static int run_norm(const void *x, const void *r, const float *gamma, const float *beta,
                    void *h_out, void *y_out, int64_t rows, int64_t dim, float eps, int half,
                    int layer, int f16_boundary, int threads) {
    if (!x || !gamma || !y_out || (layer && !beta) || rows < 0 || dim < 0) return -1;
    if (rows == 0 || dim == 0) return 0;
    norm_job j = {x, r, gamma, beta, h_out, y_out, dim, eps, half, layer, f16_boundary};
    parallel_rows(rows, threads, norm_rows, &j);
    return 0;
}

int oracle_add_rmsnorm_f16(const uint16_t *x, const uint16_t *r, const float *gamma,
                           uint16_t *h_out, uint16_t *y_out, int64_t rows, int64_t dim, float eps,
                           int f16_boundary, int threads) {
    return run_norm(x, r, gamma, NULL, h_out, y_out, rows, dim, eps, 1, 0, f16_boundary, threads);
}

int oracle_add_rmsnorm_f32(const float *x, const float *r, const float *gamma, float *h_out,
                           float *y_out, int64_t rows, int64_t dim, float eps, int threads) {
    return run_norm(x, r, gamma, NULL, h_out, y_out, rows, dim, eps, 0, 0, 0, threads);
}

int oracle_add_layernorm_f16(const uint16_t *x, const uint16_t *r, const float *gamma,
                             const float *beta, uint16_t *h_out, uint16_t *y_out, int64_t rows,
                             int64_t dim, float eps, int f16_boundary, int threads) {
    return run_norm(x, r, gamma, beta, h_out, y_out, rows, dim, eps, 1, 1, f16_boundary, threads);
}

int oracle_add_layernorm_f32(const float *x, const float *r, const float *gamma, const float *beta,
                             float *h_out, float *y_out, int64_t rows, int64_t dim, float eps,
                             int threads) {
    return run_norm(x, r, gamma, beta, h_out, y_out, rows, dim, eps, 0, 1, 0, threads);
}

int oracle_gated_layernorm_modulate_f32(const float *x, const float *gate, const float *r,
                                        const float *gamma, const float *beta, const float *scale,
                                        const float *shift, int64_t batch_rows, float *h_out,
                                        float *y_out, int64_t rows, int64_t dim, float eps) {
    if (!x || !gamma || !beta || !y_out || rows < 0 || dim <= 0 || batch_rows <= 0) return -1;
    float *h = (float *)malloc(sizeof(float) * (size_t)(rows * dim));
    if (!h) return -2;
    for (int64_t row = 0; row < rows; ++row) {
        const int64_t b = (row / batch_rows) * dim;
        for (int64_t i = 0; i < dim; ++i) {
            const int64_t e = row * dim + i;
            float v = x[e];
            if (gate) v = v * gate[b + i];      /* ggml_mul(branch, gate chunk) */
            if (r) v = v + r[e];                /* ggml_add(., residual) */
            h[e] = v;
        }
    }
    if (h_out) memcpy(h_out, h, sizeof(float) * (size_t)(rows * dim));
    run_norm(h, NULL, gamma, beta, NULL, y_out, rows, dim, eps, 0, 1, 0, 1);
    for (int64_t row = 0; row < rows; ++row) {
        const int64_t b = (row / batch_rows) * dim;
        for (int64_t i = 0; i < dim; ++i) {
            const int64_t e = row * dim + i;
            float y = y_out[e];
            if (scale) y = y * (scale[b + i] * 1.0f + 1.0f); /* add_scale_shift: mul by 1+scale */
            if (shift) y = y + shift[b + i];                  /* then add shift */
            y_out[e] = y;
        }
    }
    free(h);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* weight norm                                                               */
/* ------------------------------------------------------------------------ */

typedef struct {
    const float *v, *g;
    float *w, *norms;
    int64_t cols;
    int zero;
} wn_job;

static void wn_rows(void *ctx, int64_t r0, int64_t r1) {
    wn_job *j = (wn_job *)ctx;
    for (int64_t o = r0; o < r1; ++o) {
        const float *v = j->v + o * j->cols;
        float *w = j->w + o * j->cols;
        double s = 0.0;
        for (int64_t i = 0; i < j->cols; ++i) s += (double)(v[i] * v[i]); /* np.square in F32 */
        const float norm = sqrtf((float)s);
        if (norm == 0.f) j->zero = 1;
        if (j->norms) j->norms[o] = norm;
        const float scale = j->g[o] / norm; /* weight_g / norm */
        for (int64_t i = 0; i < j->cols; ++i) w[i] = v[i] * scale;
    }
}

int oracle_weightnorm_f32(const float *v, const float *g, float *w, float *norms_out, int64_t rows,
                          int64_t cols, int threads) {
    if (!v || !g || !w || rows < 0 || cols < 0) return -2;
    if (rows == 0 || cols == 0) return 0;
    wn_job j = {v, g, w, norms_out, cols, 0};
    parallel_rows(rows, threads, wn_rows, &j);
    return j.zero ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* Flow CFG + Euler                                                          */
/* ------------------------------------------------------------------------ */

int oracle_cfg_combine_f32(const float *u, const float *c, float *out, int64_t n, float g) {
    if (!u || !c || !out || n <= 0 || !isfinite(g)) return -1;
    for (int64_t i = 0; i < n; ++i) out[i] = u[i] + g * (c[i] - u[i]);
    return 0;
}

int oracle_cfg_euler_f32(float *state, const float *noise, const float *context,
                         const float *uncond, const float *cond, int64_t batch, int64_t row,
                         int64_t prefix, int64_t first_step, int64_t count, int64_t steps, int cfg,
                         float guidance, float sigma_min, int64_t *failed_step) {
    if (!state || batch <= 0 || row <= 0 || steps <= 0 || prefix < 0 || prefix > row) return -2;
    if (first_step < 0 || count < 0 || first_step + count > steps) return -2;
    const int64_t n = batch * row;
    float *v = (float *)malloc(sizeof(float) * (size_t)n);
    float *saved = (float *)malloc(sizeof(float) * (size_t)n);  /* the checkpoint (:85-88, :107-110) */
    if (!v || !saved) {
        free(v);
        free(saved);
        return -2;
    }
    int rc = 0;
    if (failed_step) *failed_step = -1;
    const float dt = 1.0F / (float)steps;                               /* :90  */
    for (int64_t k = 0; k < count && rc == 0; ++k) {
        const int64_t step = first_step + k;
        memcpy(saved, state, sizeof(float) * (size_t)n);
        const float time = (float)step * dt;                            /* :93  */
        const float noise_scale = 1.0F - (1.0F - sigma_min) * time;     /* :94  */
        for (int64_t b = 0; b < batch; ++b)                             /* :95-101 */
            for (int64_t i = 0; i < prefix; ++i) {
                const int64_t e = b * row + i;
                state[e] = noise_scale * noise[e] + time * context[e];
            }
        const float *u = uncond + k * n;
        const float *c = cfg ? cond + k * n : NULL;
        for (int64_t e = 0; e < n; ++e)                                 /* :305-308 */
            v[e] = cfg ? u[e] + guidance * (c[e] - u[e]) : u[e];
        for (int64_t e = 0; e < n && rc == 0; ++e)                      /* :104 */
            if (!isfinite(v[e])) rc = -1;
        if (rc == 0) {
            for (int64_t e = 0; e < n; ++e) state[e] += dt * v[e];      /* :105 */
            for (int64_t e = 0; e < n && rc == 0; ++e)                  /* :106 */
                if (!isfinite(state[e])) rc = -3;
        }
        if (rc != 0) {
            memcpy(state, saved, sizeof(float) * (size_t)n);
            if (failed_step) *failed_step = step;
        }
    }
    if (rc == 0 && first_step + count == steps)                         /* :113-114 */
        for (int64_t b = 0; b < batch; ++b)
            memcpy(state + b * row, context + b * row, sizeof(float) * (size_t)prefix);
    free(v);
    free(saved);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* window assembly                                                           */
/* ------------------------------------------------------------------------ */

int oracle_assemble_windows_f32(const float *windows, int64_t n, int64_t channels,
                                int64_t window_samples, int64_t hop, int64_t overlap,
                                int64_t target, float *out) {
    if (!windows || !out || n <= 0 || channels <= 0 || window_samples <= 0 || hop <= 0) return -1;
    const int64_t assembled = (n - 1) * hop + window_samples;
    if (target > assembled) return -1;
    float *full = (float *)calloc((size_t)(channels * assembled), sizeof(float));
    if (!full) return -2;
    for (int64_t c = 0; c < channels; ++c) {
        float *o = full + c * assembled;
        for (int64_t k = 0; k < n; ++k) {
            const float *d = windows + (k * channels + c) * window_samples;
            const int64_t offset = k * hop;
            if (k == 0) { /* :167-171 */
                memcpy(o + offset, d, sizeof(float) * (size_t)window_samples);
                continue;
            }
            const float denominator = (float)(overlap - 1); /* :184-191 */
            for (int64_t s = 0; s < overlap; ++s) {
                const float alpha = (float)s / denominator;
                o[offset + s] = o[offset + s] * (1.0f - alpha) + d[s] * alpha;
            }
            memcpy(o + offset + overlap, d + overlap, sizeof(float) * (size_t)(window_samples - overlap));
        }
        memcpy(out + c * target, o, sizeof(float) * (size_t)target); /* :198-201 crop */
    }
    free(full);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* greedy token selection                                                    */
/* ------------------------------------------------------------------------ */

int oracle_greedy_tokens_f32(const float *logits, int64_t rows, int64_t vocab, const int64_t *recent,
                             int64_t recent_len, float penalty, int64_t penalty_limit,
                             const int64_t *ignore, int64_t n_ignore, int64_t *out) {
    if (!logits || !out || rows < 0 || vocab <= 0) return -2;
    const int64_t limit = penalty_limit <= 0 ? vocab : (penalty_limit < vocab ? penalty_limit : vocab);
    float *row = (float *)malloc(sizeof(float) * (size_t)vocab);
    unsigned char *seen = (unsigned char *)malloc((size_t)vocab);
    if (!row || !seen) return -2;
    int rc = 0;
    for (int64_t r = 0; r < rows; ++r) {
        memcpy(row, logits + r * vocab, sizeof(float) * (size_t)vocab);
        memset(seen, 0, (size_t)vocab);
        /* unique recent ids, each divided once (:39-48) */
        for (int64_t k = 0; recent && k < recent_len; ++k) {
            const int64_t t = recent[r * recent_len + k];
            if (t >= 0 && t < limit && !seen[t]) {
                seen[t] = 1;
                row[t] /= penalty;
            }
        }
        /* ignore list on the first stream (:146-148) */
        for (int64_t k = 0; r == 0 && ignore && k < n_ignore; ++k)
            if (ignore[k] >= 0 && ignore[k] < vocab) row[ignore[k]] = -INFINITY;
        int64_t best = 0;
        for (int64_t i = 0; i < vocab; ++i) {
            if (isnan(row[i])) rc = -1;
            else if (isnan(row[best]) || row[i] > row[best]) best = i; /* first maximum */
        }
        out[r] = best;
    }
    free(row);
    free(seen);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* latent normalisation / layout                                             */
/* ------------------------------------------------------------------------ */

void oracle_latent_to_vae_f32(const float *frame_major, const float *mean, const float *stddev,
                              int64_t frames, int64_t dim, float *channel_major) {
    for (int64_t f = 0; f < frames; ++f)
        for (int64_t c = 0; c < dim; ++c) {
            float v = frame_major[f * dim + c];
            if (mean && stddev) v = v * stddev[c] + mean[c];
            channel_major[c * frames + f] = v;
        }
}

void oracle_latent_normalize_f32(const float *raw, const float *mean, const float *stddev, int64_t frames,
                                 int64_t dim, float *normalized) {
    for (int64_t f = 0; f < frames; ++f)
        for (int64_t c = 0; c < dim; ++c)
            normalized[f * dim + c] = (raw[f * dim + c] - mean[c]) / stddev[c];
}
