// Streaming elementwise kernels over dense [channels][time] F32 tensors:
// SnakeBeta (a1), per-channel bias add (a2) and the fused decoder unit (a3).
//
// Each is a single HBM pass: every input element is read once with a 256-bit
// load and every output written once with a 256-bit store.  Two vector forms:
//  * rows form (dense rows, 32-byte aligned tensors: the decoder's case; rows
//    that are not a multiple of 8 long get a scalar head and tail around a
//    vector body): the tensor is cut into row chunks of kRowThreads*UNROLL
//    vectors, one CTA per chunk, so the channel is uniform per CTA and its
//    parameters (alpha, 1/beta, bias: promoted to F32 and exponentiated) are
//    computed once in registers.
//  * flat form (any row length, any common 32-byte phase): one CTA per tile of
//    the flat element space; parameters are cached per thread by channel (or
//    staged in shared memory when there are few channels), and a vector that
//    straddles a row boundary selects them per element.
// A scalar form covers strided rows and mismatched alignments.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace levo {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;
// Rows form: 128-thread CTAs, one CTA per chunk.  Measured on the config-4
// chain (sweep of block size 128-256, unroll 1-8 and grid size) on B200:
//  * 1-input units (SnakeBeta, post / upsample units): four vectors per thread
//    per chunk (6.1-6.4 TB/s; a grid of resident CTAs walking chunk ranges
//    reached 5.2-5.5);
//  * 2-input residual unit: two vectors per thread per chunk (6.26 TB/s; one
//    vector with 16x the resident CTAs walking chunk ranges: 6.20).
constexpr int kRowThreads = 128;
// Shortest row length that is not a multiple of 8 the rows form takes: the head
// (< 8) stays inside the row and the body holds at least one vector.
constexpr int64_t kMinRaggedRow = 64;
constexpr int64_t kMaxStagedChannels = 4096;

struct StreamArgs {
    const float *u;
    const void *bias;
    const float *res;
    const void *alog;
    const void *blog;
    float *x_out;
    float *y_out;
    int64_t ldu, ldr, ldx, ldy;  // row strides (scalar path only)
    int64_t rows, len, n;        // n = rows * len
    int64_t head;                // scalar elements before the 32-byte-aligned region
    int64_t nvec;                // full 8-element vectors in the aligned region
    double inv_len;
    int pdtype;
    int has_bias, write_x, write_y, tanh_out, staged;
    // rows form
    int64_t vec_per_row;  // len / 8
    int64_t chunks_per_row;
    int64_t chunks;       // rows * chunks_per_row
    double inv_chunks_per_row;
};

struct ChannelParams {
    float alpha, beta, bias;  // beta holds 1/beta
};

template <bool SNAKE>
__device__ __forceinline__ ChannelParams channel_params(const StreamArgs &a, const float *smem,
                                                        int64_t c) {
    ChannelParams p{0.f, 1.f, 0.f};
    if (a.staged) {
        if (SNAKE) {
            p.alpha = smem[c];
            p.beta = smem[a.rows + c];
        }
        if (a.has_bias) p.bias = smem[2 * a.rows + c];
    } else if constexpr (SNAKE) {
        // The three loads go out together, ahead of the exponentials: a bias load
        // behind the has_bias branch cannot be hoisted (the pointer may be null)
        // and would start one L2 round trip later in every chunk.
        const float bias = load_param(a.has_bias ? a.bias : a.alog, c, a.pdtype);
        p.alpha = snake_alpha_param(a.alog, c, a.pdtype);
        p.beta = snake_inv_beta_param(a.blog, c, a.pdtype);
        if (a.has_bias) p.bias = bias;
    } else {
        if (a.has_bias) p.bias = load_param(a.bias, c, a.pdtype);
    }
    return p;
}

template <bool HAS_RES, bool SNAKE>
__device__ __forceinline__ void unit_eval(const StreamArgs &a, const ChannelParams &p, float u,
                                          float r, float &x, float &y) {
    float v = u;
    if (a.has_bias) v = __fadd_rn(v, p.bias);
    if (HAS_RES) v = __fadd_rn(r, v);
    x = v;
    float w = v;
    if (SNAKE) w = snake_eval(v, p.alpha, p.beta);
    if (a.tanh_out) w = tanhf(w);
    y = w;
}

// 8 values of one channel: bias, residual, SnakeBeta (one range check per
// vector), tanh.  x keeps the pre-activation sum, y the activation.
template <bool HAS_RES, bool SNAKE>
__device__ __forceinline__ void unit_eval8(const StreamArgs &a, const ChannelParams &p, const f32x8 &u,
                                           const f32x8 &r, f32x8 &x, f32x8 &y) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        float v = u.v[k];
        if (a.has_bias) v = __fadd_rn(v, p.bias);
        if (HAS_RES) v = __fadd_rn(r.v[k], v);
        x.v[k] = v;
        y.v[k] = v;
    }
    if (SNAKE) snake_eval8(y.v, p.alpha, p.beta);
    if (a.tanh_out) {
#pragma unroll
        for (int k = 0; k < 8; ++k) y.v[k] = tanhf(y.v[k]);
    }
}

// Rows form: CTA b owns a contiguous share of the chunks (block_range); chunk q covers
// vectors [k*kRowThreads*UNROLL, (k+1)*kRowThreads*UNROLL) of row c, q = c*cpr + k.
// Short-lived CTAs that the block scheduler refills keep HBM busier than a
// persistent grid (a plain 2-in/2-out stream on B200: ~6.8 against ~6.0 TB/s),
// so launch_rows gives every chunk its own CTA (G = chunks).  The loads of a
// chunk are issued before its channel parameters are computed.
template <bool HAS_RES, bool SNAKE, int UNROLL, bool RAGGED>
__global__ void __launch_bounds__(kRowThreads) stream_rows_kernel(const StreamArgs a) {
    pdl_wait();
    pdl_trigger();
    int64_t q0, q1;
    block_range(a.chunks, q0, q1);
    if (q0 >= q1) return;
    int64_t c = row_of(q0, a.chunks_per_row, a.inv_chunks_per_row);
    int64_t k = q0 - c * a.chunks_per_row;
    for (int64_t q = q0; q < q1; ++q) {
        // A row whose length is not a multiple of 8 starts at any 4-byte phase:
        // scalar head up to its first 32-byte boundary, 256-bit body, scalar tail.
        const int64_t row = c * a.len;
        const int64_t head = RAGGED ? ((-row) & 7) : 0;
        const int64_t body = RAGGED ? (a.len - head) >> 3 : a.vec_per_row;
        const size_t base = static_cast<size_t>(row + head);
        const int64_t v0 = k * (kRowThreads * UNROLL) + threadIdx.x;
        f32x8 uu[UNROLL], rr[UNROLL];
#pragma unroll
        for (int j = 0; j < UNROLL; ++j) {
            const int64_t v = v0 + j * kRowThreads;
            if (v < body) {
                uu[j] = ld8(a.u + base + v * 8);
                if (HAS_RES) rr[j] = ld8(a.res + base + v * 8);
            }
        }
        const ChannelParams p = channel_params<SNAKE>(a, nullptr, c);
#pragma unroll
        for (int j = 0; j < UNROLL; ++j) {
            const int64_t v = v0 + j * kRowThreads;
            if (v >= body) continue;
            f32x8 xo, yo;
            unit_eval8<HAS_RES, SNAKE>(a, p, uu[j], rr[j], xo, yo);
            if (a.write_x) st8(a.x_out + base + v * 8, xo);
            if (a.write_y) st8(a.y_out + base + v * 8, yo);
        }
        if (RAGGED && k == 0) {
            // head + tail < 16 <= kRowThreads elements, one per thread
            const int64_t tail = a.len - head - body * 8;
            const int64_t t = threadIdx.x;
            if (t < head + tail) {
                const int64_t e = t < head ? row + t : row + head + body * 8 + (t - head);
                float xs, ys;
                unit_eval<HAS_RES, SNAKE>(a, p, a.u[e], HAS_RES ? a.res[e] : 0.f, xs, ys);
                if (a.write_x) a.x_out[e] = xs;
                if (a.write_y) a.y_out[e] = ys;
            }
        }
        if (++k == a.chunks_per_row) {
            k = 0;
            ++c;
        }
    }
}

// Scalar element e with per-tensor row strides.
template <bool HAS_RES, bool SNAKE>
__device__ __forceinline__ void scalar_element(const StreamArgs &a, const float *smem, int64_t e) {
    const int64_t c = row_of(e, a.len, a.inv_len);
    const int64_t t = e - c * a.len;
    const ChannelParams p = channel_params<SNAKE>(a, smem, c);
    const float u = a.u[c * a.ldu + t];
    const float r = HAS_RES ? a.res[c * a.ldr + t] : 0.f;
    float x, y;
    unit_eval<HAS_RES, SNAKE>(a, p, u, r, x, y);
    if (a.write_x) a.x_out[c * a.ldx + t] = x;
    if (a.write_y) a.y_out[c * a.ldy + t] = y;
}

template <bool HAS_RES, bool SNAKE>
__device__ __forceinline__ void stage_params(const StreamArgs &a, float *smem) {
    if (!a.staged) return;
    for (int64_t c = threadIdx.x; c < a.rows; c += blockDim.x) {
        if (SNAKE) {
            smem[c] = snake_alpha_param(a.alog, c, a.pdtype);
            smem[a.rows + c] = snake_inv_beta_param(a.blog, c, a.pdtype);
        }
        if (a.has_bias) smem[2 * a.rows + c] = load_param(a.bias, c, a.pdtype);
    }
    __syncthreads();
}

// 256-bit vector path: all tensors dense and sharing one 32-byte phase.
template <bool HAS_RES, bool SNAKE>
__global__ void __launch_bounds__(kThreads) stream_vec8_kernel(const StreamArgs a) {
    extern __shared__ float smem[];
    pdl_wait();
    pdl_trigger();
    stage_params<HAS_RES, SNAKE>(a, smem);

    // Ragged head and tail (< 8 elements each) go to block 0.
    if (blockIdx.x == 0) {
        if (threadIdx.x < a.head) scalar_element<HAS_RES, SNAKE>(a, smem, threadIdx.x);
        const int64_t tail0 = a.head + a.nvec * 8;
        if (threadIdx.x < a.n - tail0) scalar_element<HAS_RES, SNAKE>(a, smem, tail0 + threadIdx.x);
    }

    // Each CTA walks one contiguous range of tiles, so a thread's channel
    // changes rarely; its parameters are cached in registers by channel.
    const int64_t tile_vecs = static_cast<int64_t>(kThreads) * kUnroll;
    const int64_t tiles = (a.nvec + tile_vecs - 1) / tile_vecs;
    int64_t t0, t1;
    block_range(tiles, t0, t1);
    int64_t cached_c = -1;
    ChannelParams cached{};
    auto params_for = [&](int64_t c) -> ChannelParams {
        if (c != cached_c) {
            cached = channel_params<SNAKE>(a, smem, c);
            cached_c = c;
        }
        return cached;
    };
    for (int64_t tile = t0 * tile_vecs; tile < t1 * tile_vecs; tile += tile_vecs) {
        f32x8 uu[kUnroll];
        f32x8 rr[kUnroll];
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            const int64_t vi = tile + j * kThreads + threadIdx.x;
            if (vi < a.nvec) {
                const int64_t e = a.head + vi * 8;
                uu[j] = ld8(a.u + e);
                if (HAS_RES) rr[j] = ld8(a.res + e);
            }
        }
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            const int64_t vi = tile + j * kThreads + threadIdx.x;
            if (vi >= a.nvec) continue;
            const int64_t e = a.head + vi * 8;
            f32x8 xo, yo;
            if (a.len >= 8) {
                // At most one row boundary inside the vector.
                const int64_t c0 = row_of(e, a.len, a.inv_len);
                const int64_t boundary = (c0 + 1) * a.len;
                const ChannelParams p0 = params_for(c0);
                if (e + 8 <= boundary) {
                    unit_eval8<HAS_RES, SNAKE>(a, p0, uu[j], rr[j], xo, yo);
                } else {
                    const ChannelParams p1 = channel_params<SNAKE>(a, smem, c0 + 1);
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        unit_eval<HAS_RES, SNAKE>(a, (e + k < boundary) ? p0 : p1, uu[j].v[k],
                                                  HAS_RES ? rr[j].v[k] : 0.f, xo.v[k], yo.v[k]);
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const ChannelParams p =
                        channel_params<SNAKE>(a, smem, row_of(e + k, a.len, a.inv_len));
                    unit_eval<HAS_RES, SNAKE>(a, p, uu[j].v[k], HAS_RES ? rr[j].v[k] : 0.f,
                                              xo.v[k], yo.v[k]);
                }
            }
            if (a.write_x) st8(a.x_out + e, xo);
            if (a.write_y) st8(a.y_out + e, yo);
        }
    }
}

// Scalar path: any row strides, any 4-byte alignment.
template <bool HAS_RES, bool SNAKE>
__global__ void __launch_bounds__(kThreads) stream_scalar_kernel(const StreamArgs a) {
    extern __shared__ float smem[];
    pdl_wait();
    pdl_trigger();
    stage_params<HAS_RES, SNAKE>(a, smem);
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < a.n;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x)
        scalar_element<HAS_RES, SNAKE>(a, smem, e);
}

template <bool HAS_RES, bool SNAKE>
int launch_rows(StreamArgs a, cudaStream_t stream, const char *what) {
    constexpr int kRowUnroll = HAS_RES ? 2 : 4;
    const bool ragged = a.len % 8 != 0;
    auto kernel = ragged ? stream_rows_kernel<HAS_RES, SNAKE, kRowUnroll, true>
                         : stream_rows_kernel<HAS_RES, SNAKE, kRowUnroll, false>;
    a.staged = 0;
    a.vec_per_row = a.len / 8;  // a ragged row's body has vec_per_row or vec_per_row - 1 vectors
    a.chunks_per_row = (a.vec_per_row + kRowThreads * kRowUnroll - 1) / (kRowThreads * kRowUnroll);
    a.chunks = a.rows * a.chunks_per_row;
    a.inv_chunks_per_row = 1.0 / static_cast<double>(a.chunks_per_row);
    // one CTA per chunk; past 2^31 - 1 chunks a CTA takes a contiguous range of them
    const int64_t grid = std::min<int64_t>(a.chunks, 0x7fffffff);
    const cudaError_t err = launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), dim3(kRowThreads), 0, stream, a);
    if (err != cudaSuccess)
        return set_error(LEVO_OPS_ELAUNCH, std::string(what) + ": kernel launch failed: " + cudaGetErrorString(err));
    return check_launch(what);
}

template <bool HAS_RES, bool SNAKE>
int launch_variant(const StreamArgs &a, bool vec, size_t smem_bytes, cudaStream_t stream,
                   const char *what) {
    auto kernel = vec ? stream_vec8_kernel<HAS_RES, SNAKE> : stream_scalar_kernel<HAS_RES, SNAKE>;
    int per_sm = 1;
    if (resident_ctas(reinterpret_cast<const void *>(kernel), kThreads, smem_bytes, &per_sm) != cudaSuccess) {
        cudaGetLastError();
        per_sm = 1;
    }
    const int64_t work_items = vec ? (a.nvec + kUnroll - 1) / kUnroll : a.n;
    const int64_t needed = std::max<int64_t>(1, (work_items + kThreads - 1) / kThreads);
    // vector form: one CTA per tile, as in the rows form; scalar form: persistent grid
    const int64_t grid = vec ? std::min<int64_t>(needed, 0x7fffffff)
                             : std::min<int64_t>(needed, static_cast<int64_t>(sm_count()) * per_sm);
    const cudaError_t err =
        launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem_bytes, stream, a);
    if (err != cudaSuccess)
        return set_error(LEVO_OPS_ELAUNCH, std::string(what) + ": kernel launch failed: " + cudaGetErrorString(err));
    return check_launch(what);
}

// One thread per channel: alpha = exp(alpha_log), 1/beta, with the kernels' own
// device arithmetic (snake_alpha / snake_inv_beta), so prepared and log-form
// launches agree bit for bit.
__global__ void __launch_bounds__(256) snake_params_kernel(const void *alog, const void *blog, int dtype,
                                                          int64_t channels, float *alpha, float *inv_beta) {
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < channels;
         c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        alpha[c] = snake_alpha(load_param(alog, c, dtype));
        inv_beta[c] = snake_inv_beta(load_param(blog, c, dtype));
    }
}

struct StreamRequest {
    const float *u;
    int64_t ldu;
    const void *bias;
    const float *res;
    int64_t ldr;
    const void *alog;
    const void *blog;
    int pdtype;
    float *x_out;
    int64_t ldx;
    float *y_out;
    int64_t ldy;
    int64_t rows, len;
    bool tanh_out;
    bool need_snake;  // the entry point requires SnakeBeta parameters
    bool need_bias;   // the entry point requires a bias
};

int run_stream(const StreamRequest &q, cudaStream_t stream, const char *what) {
    const std::string w(what);
    if (q.rows < 0 || q.len < 0) return set_error(LEVO_OPS_EINVAL, w + ": negative shape");
    if (q.pdtype != LEVO_DTYPE_F32 && q.pdtype != LEVO_DTYPE_F16 && q.pdtype != LEVO_DTYPE_SNAKE_PREPARED)
        return set_error(LEVO_OPS_EINVAL, w + ": parameter dtype must be F32, F16 or SNAKE_PREPARED");
    if (q.rows == 0 || q.len == 0) return LEVO_OPS_OK;  // empty tensors: nothing to read or write
    if (q.u == nullptr) return set_error(LEVO_OPS_EINVAL, w + ": input is null");
    if (q.need_snake && (q.alog == nullptr || q.blog == nullptr))
        return set_error(LEVO_OPS_EINVAL, w + ": SnakeBeta parameters are null");
    if (q.need_bias && q.bias == nullptr) return set_error(LEVO_OPS_EINVAL, w + ": bias is null");
    if ((q.alog == nullptr) != (q.blog == nullptr))
        return set_error(LEVO_OPS_EINVAL, w + ": alpha_log and beta_log must both be given");
    if (q.x_out == nullptr && q.y_out == nullptr)
        return set_error(LEVO_OPS_EINVAL, w + ": no output requested");
    const int64_t lds[4] = {q.ldu, q.res ? q.ldr : q.len, q.x_out ? q.ldx : q.len,
                            q.y_out ? q.ldy : q.len};
    for (int64_t ld : lds)
        if (ld < q.len) return set_error(LEVO_OPS_EINVAL, w + ": row stride smaller than the row");
    const size_t pbytes = q.pdtype == LEVO_DTYPE_F16 ? 2 : 4;
    const void *ptrs[7] = {q.u, q.res, q.x_out, q.y_out, q.bias, q.alog, q.blog};
    for (int i = 0; i < 7; ++i)
        if (ptrs[i] && !aligned_to(ptrs[i], i < 4 ? 4 : pbytes))
            return set_error(LEVO_OPS_EINVAL, w + ": pointer is not aligned to its element size");
    if (q.rows > (int64_t(1) << 40) / q.len)
        return set_error(LEVO_OPS_EINVAL, w + ": tensor too large");

    StreamArgs a{};
    a.u = q.u;
    a.bias = q.bias;
    a.res = q.res;
    a.alog = q.alog;
    a.blog = q.blog;
    a.x_out = q.x_out;
    a.y_out = q.y_out;
    a.ldu = q.ldu;
    a.ldr = q.ldr;
    a.ldx = q.ldx;
    a.ldy = q.ldy;
    a.rows = q.rows;
    a.len = q.len;
    a.n = q.rows * q.len;
    a.inv_len = 1.0 / static_cast<double>(q.len);
    a.pdtype = q.pdtype;
    a.has_bias = q.bias != nullptr;
    a.write_x = q.x_out != nullptr;
    a.write_y = q.y_out != nullptr;
    a.tanh_out = q.tanh_out;
    const bool snake = q.alog != nullptr;

    // The vector path needs dense rows and one common 32-byte phase.
    bool vec = lds[0] == q.len && lds[1] == q.len && lds[2] == q.len && lds[3] == q.len;
    const uintptr_t phase = reinterpret_cast<uintptr_t>(q.u) % 32;
    for (int i = 1; i < 4 && vec; ++i)
        if (ptrs[i] && reinterpret_cast<uintptr_t>(ptrs[i]) % 32 != phase) vec = false;
    if (vec) {
        a.head = std::min<int64_t>(a.n, static_cast<int64_t>(((32 - phase) % 32) / 4));
        a.nvec = (a.n - a.head) / 8;
        if (a.nvec == 0) vec = false;
    }

    // Rows form: dense rows, every tensor 32-byte aligned; rows of a multiple of 8
    // values, or at least kMinRaggedRow (then each row has a scalar head and tail).
    if (vec && a.head == 0 && (q.len % 8 == 0 || q.len >= kMinRaggedRow)) {
        if (q.res)
            return snake ? launch_rows<true, true>(a, stream, what) : launch_rows<true, false>(a, stream, what);
        return snake ? launch_rows<false, true>(a, stream, what) : launch_rows<false, false>(a, stream, what);
    }

    // Stage the per-channel parameters in shared memory only when each CTA has
    // enough elements to amortise exponentiating all of them (a vector-form CTA
    // holds one tile of kThreads*kUnroll*8 values; the stage-0 entry unit, 2048
    // channels, computes them per vector instead).
    const int nparams = (snake ? 2 : 0) + (a.has_bias ? 1 : 0);
    const int64_t per_cta = vec ? static_cast<int64_t>(kThreads) * kUnroll * 8
                                : a.n / (static_cast<int64_t>(sm_count()) * 8);
    a.staged = nparams > 0 && q.rows <= kMaxStagedChannels && q.rows * 64 <= per_cta;
    const size_t smem_bytes = a.staged ? static_cast<size_t>(3 * q.rows) * sizeof(float) : 0;

    if (q.res) {
        return snake ? launch_variant<true, true>(a, vec, smem_bytes, stream, what)
                     : launch_variant<true, false>(a, vec, smem_bytes, stream, what);
    }
    return snake ? launch_variant<false, true>(a, vec, smem_bytes, stream, what)
                 : launch_variant<false, false>(a, vec, smem_bytes, stream, what);
}

}  // namespace

// Used by the chain driver (vae_chain.cu).
int fused_unit(const levo_fused_unit &unit, cudaStream_t stream) {
    StreamRequest q{};
    q.u = unit.u;
    q.ldu = unit.time;
    q.bias = unit.bias;
    q.res = unit.residual;
    q.ldr = unit.time;
    q.alog = unit.alpha_log;
    q.blog = unit.beta_log;
    q.pdtype = unit.param_dtype;
    q.x_out = unit.x_out;
    q.ldx = unit.time;
    q.y_out = unit.y_out;
    q.ldy = unit.time;
    q.rows = unit.channels;
    q.len = unit.time;
    q.tanh_out = (unit.flags & LEVO_FUSED_TANH) != 0;
    if (unit.flags & ~LEVO_FUSED_TANH)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_fused_unit_f32: unknown flag bits");
    return run_stream(q, stream, "levo_vae_fused_unit_f32");
}

}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_snake_params_prepare(const void *alpha_log, const void *beta_log, int param_dtype,
                                           int64_t channels, float *alpha_out, float *inv_beta_out,
                                           levo_stream_t stream) {
    using namespace levo;
    clear_error();
    const std::string w = "levo_snake_params_prepare";
    if (param_dtype != LEVO_DTYPE_F32 && param_dtype != LEVO_DTYPE_F16)
        return set_error(LEVO_OPS_EINVAL, w + ": parameter dtype must be F32 or F16");
    if (channels < 0) return set_error(LEVO_OPS_EINVAL, w + ": negative channel count");
    if (channels == 0) return LEVO_OPS_OK;
    if (!alpha_log || !beta_log || !alpha_out || !inv_beta_out)
        return set_error(LEVO_OPS_EINVAL, w + ": required pointer is null");
    const size_t pbytes = param_dtype == LEVO_DTYPE_F16 ? 2 : 4;
    if (!aligned_to(alpha_log, pbytes) || !aligned_to(beta_log, pbytes) || !aligned_to(alpha_out, 4) ||
        !aligned_to(inv_beta_out, 4))
        return set_error(LEVO_OPS_EINVAL, w + ": pointer is not aligned to its element size");
    const int64_t grid = std::min<int64_t>((channels + 255) / 256, static_cast<int64_t>(sm_count()) * 4);
    snake_params_kernel<<<static_cast<unsigned>(grid), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        alpha_log, beta_log, param_dtype, channels, alpha_out, inv_beta_out);
    return check_launch(w.c_str());
}

LEVO_OPS_API int levo_snakebeta_f32(const float *x, int64_t ldx, const void *alpha_log,
                                    const void *beta_log, int param_dtype, float *y, int64_t ldy,
                                    int64_t channels, int64_t time, levo_stream_t stream) {
    levo::clear_error();
    levo::StreamRequest q{};
    q.need_snake = true;
    q.u = x;
    q.ldu = ldx;
    q.alog = alpha_log;
    q.blog = beta_log;
    q.pdtype = param_dtype;
    q.y_out = y;
    q.ldy = ldy;
    q.rows = channels;
    q.len = time;
    return levo::run_stream(q, reinterpret_cast<cudaStream_t>(stream), "levo_snakebeta_f32");
}

LEVO_OPS_API int levo_channel_bias_add_f32(const float *in, const void *bias, int bias_dtype,
                                           float *out, int64_t channels, int64_t time,
                                           levo_stream_t stream) {
    levo::clear_error();
    levo::StreamRequest q{};
    q.need_bias = true;
    q.u = in;
    q.ldu = time;
    q.bias = bias;
    q.pdtype = bias_dtype;
    q.y_out = out;
    q.ldy = time;
    q.rows = channels;
    q.len = time;
    return levo::run_stream(q, reinterpret_cast<cudaStream_t>(stream), "levo_channel_bias_add_f32");
}

LEVO_OPS_API int levo_vae_fused_unit_f32(const levo_fused_unit *unit, levo_stream_t stream) {
    levo::clear_error();
    if (unit == nullptr)
        return levo::set_error(LEVO_OPS_EINVAL, "levo_vae_fused_unit_f32: descriptor is null");
    return levo::fused_unit(*unit, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
