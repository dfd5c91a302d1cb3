// Decoder elementwise chain driver (a4): the stage loop of the Oobleck decoder
// (reference: src/levo-vae.cpp:172-276) with every elementwise node fused into
// one HBM pass per convolution output.
//
// Per stage (C = stage width, L = stage length), with conv outputs raw (no bias):
//   upsample conv  -> [UPSAMPLE] x = u + b_up;            y = snake_pre0(x)   12 B/elem
//   per residual r:
//     conv.0       -> [POST]     y = snake_post_r(u + b0)                      8 B/elem
//     conv.1       -> [RESIDUAL] x = x + (u + b1);         y = snake_next(x)  16 B/elem
//                                 (the last unit skips storing x: 12 B/elem)
// where snake_next is the next unit's pre activation, the next stage's upsample
// activation, or the output activation.  The input conv is followed by [ENTRY]
// y = snake_up0(u + b_in) (8 B/elem).  Every fused unit writes y in place over
// its conv output, which the next conv then reads.
//
// Convolutions are not part of this layer: a callback performs them.  Without
// one, built-in stand-ins run instead (index-map copies for the input, upsample
// and output convs; identity aliases for the residual convs).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "common.cuh"

namespace levo {
int fused_unit(const levo_fused_unit &unit, cudaStream_t stream);

namespace {

// Row form for any row length: blockIdx.y walks output rows, each thread writes
// 4 consecutive samples of the row (one division by the stride per 4 samples).
__global__ void __launch_bounds__(256) conv_standin_kernel(const float *in, int64_t cin, int64_t lin,
                                                          float *out, int64_t cout, int64_t lout,
                                                          int32_t stride) {
    pdl_wait();
    pdl_trigger();
    for (int64_t c = blockIdx.y; c < cout; c += gridDim.y) {
        const float *src = in + (c % cin) * lin;
        float *dst = out + c * lout;
        for (int64_t t0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; t0 < lout;
             t0 += static_cast<int64_t>(gridDim.x) * blockDim.x * 4) {
            int64_t st = t0 / stride;
            int32_t phase = static_cast<int32_t>(t0 - st * stride);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (t0 + k < lout) dst[t0 + k] = st < lin ? __ldg(src + st) : 0.f;
                if (++phase == stride) {
                    phase = 0;
                    ++st;
                }
            }
        }
    }
}

// Vector form for rows whose length is a multiple of 8 (32-byte aligned rows):
// each thread writes 8 consecutive samples of one row with one 256-bit store;
// the source index advances by one every `stride` samples.
__global__ void __launch_bounds__(256) conv_standin_vec8_kernel(const float *in, int64_t cin,
                                                               int64_t lin, float *out,
                                                               int64_t cout, int64_t lout,
                                                               int32_t stride, double inv_lout) {
    pdl_wait();
    pdl_trigger();
    const int64_t nvec = cout * lout / 8;
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec;
         v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = v * 8;
        const int64_t c = row_of(e, lout, inv_lout);
        const int64_t t0 = e - c * lout;
        const float *src = in + (c % cin) * lin;
        int64_t st = t0 / stride;
        int32_t phase = static_cast<int32_t>(t0 - st * stride);
        f32x8 o;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            o.v[k] = st < lin ? __ldg(src + st) : 0.f;
            if (++phase == stride) {
                phase = 0;
                ++st;
            }
        }
        st8(out + e, o);
    }
}

struct SnakeRef {
    const void *alpha;
    const void *beta;
};

struct StageOffsets {
    int64_t up_alpha, up_beta, up_bias;
    int64_t pre_alpha[LEVO_VAE_MAX_RESIDUALS], pre_beta[LEVO_VAE_MAX_RESIDUALS];
    int64_t bias0[LEVO_VAE_MAX_RESIDUALS];
    int64_t post_alpha[LEVO_VAE_MAX_RESIDUALS], post_beta[LEVO_VAE_MAX_RESIDUALS];
    int64_t bias1[LEVO_VAE_MAX_RESIDUALS];
};

struct Layout {
    int64_t in_bias;
    StageOffsets stage[LEVO_VAE_MAX_STAGES];
    int64_t out_alpha, out_beta;
    int64_t total;
};

bool valid_topology(const levo_vae_topology &t, std::string *why) {
    auto bad = [why](const char *m) {
        *why = m;
        return false;
    };
    if (t.latent_dim <= 0 || t.audio_channels <= 0 || t.entry_width <= 0)
        return bad("latent_dim, audio_channels and entry_width must be positive");
    if (t.n_stages < 1 || t.n_stages > LEVO_VAE_MAX_STAGES) return bad("n_stages must be 1..8");
    if (t.n_residual < 0 || t.n_residual > LEVO_VAE_MAX_RESIDUALS) return bad("n_residual must be 0..4");
    for (int s = 0; s < t.n_stages; ++s)
        if (t.stage_width[s] <= 0 || t.stage_stride[s] <= 0) return bad("stage widths and strides must be positive");
    for (int r = 0; r < t.n_residual; ++r)
        if (t.dilation[r] <= 0) return bad("dilations must be positive");
    return true;
}

Layout make_layout(const levo_vae_topology &t) {
    Layout l{};
    int64_t off = 0;
    l.in_bias = off;
    off += t.entry_width;
    int64_t cin = t.entry_width;
    for (int s = 0; s < t.n_stages; ++s) {
        const int64_t c = t.stage_width[s];
        StageOffsets &so = l.stage[s];
        so.up_alpha = off;
        off += cin;
        so.up_beta = off;
        off += cin;
        so.up_bias = off;
        off += c;
        for (int r = 0; r < t.n_residual; ++r) {
            so.pre_alpha[r] = off;
            off += c;
            so.pre_beta[r] = off;
            off += c;
            so.bias0[r] = off;
            off += c;
            so.post_alpha[r] = off;
            off += c;
            so.post_beta[r] = off;
            off += c;
            so.bias1[r] = off;
            off += c;
        }
        cin = c;
    }
    l.out_alpha = off;
    off += cin;
    l.out_beta = off;
    off += cin;
    l.total = off;
    return l;
}

int64_t total_upsampling(const levo_vae_topology &t) {
    int64_t f = 1;
    for (int s = 0; s < t.n_stages; ++s) f *= t.stage_stride[s];
    return f;
}

class DeviceGuard {
   public:
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&previous_) != cudaSuccess) previous_ = -1;
        if (previous_ != device) cudaSetDevice(device);
    }
    ~DeviceGuard() {
        if (previous_ >= 0) cudaSetDevice(previous_);
    }

   private:
    int previous_ = -1;
};

// NVTX range for profilers (ncu --nvtx, Nsight Systems): one per decoded window
// and per decoder stage.  Header-only NVTX v3: without an attached tool each
// push / pop is a few nanoseconds.
class NvtxRange {
   public:
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};

constexpr const char *kStageRangeNames[LEVO_VAE_MAX_STAGES] = {
    "levo.vae.stage0", "levo.vae.stage1", "levo.vae.stage2", "levo.vae.stage3",
    "levo.vae.stage4", "levo.vae.stage5", "levo.vae.stage6", "levo.vae.stage7"};

struct TimedLaunch {
    int kclass;
    int ev_start, ev_end;
    double bytes, elems;
};

}  // namespace
}  // namespace levo

struct levo_vae_chain {
    int device = 0;
    levo_vae_topology topo{};
    levo::Layout layout{};
    int64_t max_frames = 0;
    int64_t max_elems = 0;
    void *params = nullptr;       // packed parameters, F32 or F16 (pdtype)
    int pdtype = LEVO_DTYPE_F32;
    // dtype the fused units read the parameters with: an F32 chain holds every
    // SnakeBeta layer prepared (alpha, 1/beta) and reads LEVO_DTYPE_SNAKE_PREPARED
    int unit_pdtype = LEVO_DTYPE_F32;
    float *X = nullptr;
    float *A = nullptr;
    float *B = nullptr;
    float *lat[2] = {nullptr, nullptr};
    float *audio[2] = {nullptr, nullptr};
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t computed[2] = {nullptr, nullptr};
    cudaEvent_t copied[2] = {nullptr, nullptr};
    levo_conv_fn conv = nullptr;
    void *conv_user = nullptr;
    // stage capture (levo_vae_chain_set_stage_capture): per-stage destinations, host or device
    float *capture[LEVO_VAE_MAX_STAGES] = {};
    int32_t n_capture = 0;
    // timing
    std::vector<cudaEvent_t> events;
    int next_event = 0;
    std::vector<levo::TimedLaunch> launches;
    levo_kernel_timing totals[LEVO_KCLASS_COUNT] = {};
};

namespace levo {
namespace {

int cuda_fail(cudaError_t err, const std::string &what) {
    return set_error(err == cudaErrorMemoryAllocation ? LEVO_OPS_ENOMEM : LEVO_OPS_ECUDA,
                     what + ": " + cudaGetErrorString(err));
}

void free_chain(levo_vae_chain *c) {
    if (c == nullptr) return;
    DeviceGuard guard(c->device);
    cudaFree(c->params);
    cudaFree(c->X);
    cudaFree(c->A);
    cudaFree(c->B);
    for (int i = 0; i < 2; ++i) {
        cudaFree(c->lat[i]);
        cudaFree(c->audio[i]);
        if (c->computed[i]) cudaEventDestroy(c->computed[i]);
        if (c->copied[i]) cudaEventDestroy(c->copied[i]);
    }
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    for (cudaEvent_t e : c->events) cudaEventDestroy(e);
    delete c;
}

int take_event(levo_vae_chain *c, int *index) {
    if (c->next_event >= static_cast<int>(c->events.size())) {
        cudaEvent_t e = nullptr;
        const cudaError_t err = cudaEventCreate(&e);
        if (err != cudaSuccess) return cuda_fail(err, "levo_vae_chain timing event");
        c->events.push_back(e);
    }
    *index = c->next_event++;
    return LEVO_OPS_OK;
}

// Runs `body` and, when timing, brackets it with a pair of events.
template <class F>
int timed(levo_vae_chain *c, bool timing, int kclass, double bytes, double elems, cudaStream_t s,
          F &&body) {
    int e0 = -1, e1 = -1;
    if (timing) {
        int rc = take_event(c, &e0);
        if (rc == LEVO_OPS_OK) rc = take_event(c, &e1);
        if (rc != LEVO_OPS_OK) return rc;
        cudaEventRecord(c->events[e0], s);
    }
    const int rc = body();
    if (rc != LEVO_OPS_OK) return rc;
    if (timing) {
        cudaEventRecord(c->events[e1], s);
        c->launches.push_back(TimedLaunch{kclass, e0, e1, bytes, elems});
    }
    return LEVO_OPS_OK;
}

int run_unit(levo_vae_chain *c, bool timing, int kclass, const levo_fused_unit &u, cudaStream_t s) {
    const double n = static_cast<double>(u.channels) * static_cast<double>(u.time);
    const double bytes =
        4.0 * n * (1 + (u.residual ? 1 : 0) + (u.x_out ? 1 : 0) + (u.y_out ? 1 : 0));
    return timed(c, timing, kclass, bytes, n, s, [&] { return fused_unit(u, s); });
}

int run_conv(levo_vae_chain *c, bool timing, levo_conv_call &call, cudaStream_t s) {
    call.result = call.output;
    if (c->conv) {
        const int rc = timed(c, timing, LEVO_KCLASS_CONV, 0.0, 0.0, s, [&] {
            const int r = c->conv(c->conv_user, &call, reinterpret_cast<levo_stream_t>(s));
            if (r != 0)
                return set_error(LEVO_OPS_ECUDA, "levo_vae_chain: convolution callback failed (kind " +
                                                     std::to_string(call.kind) + ", code " +
                                                     std::to_string(r) + ")");
            return static_cast<int>(LEVO_OPS_OK);
        });
        if (rc != LEVO_OPS_OK) return rc;
        if (call.result != call.output &&
            (call.result != call.input || call.in_channels != call.out_channels ||
             call.in_length != call.out_length))
            return set_error(LEVO_OPS_EINVAL,
                             "levo_vae_chain: a convolution callback may only alias an "
                             "identically shaped input");
        return LEVO_OPS_OK;
    }
    if (call.kind == LEVO_CONV_RES0 || call.kind == LEVO_CONV_RES1) {
        call.result = const_cast<float *>(call.input);
        return LEVO_OPS_OK;
    }
    const double n_out = static_cast<double>(call.out_channels) * call.out_length;
    const double n_in = static_cast<double>(call.in_channels) * call.in_length;
    return timed(c, timing, LEVO_KCLASS_CONV, 4.0 * (n_in + n_out), n_out, s, [&] {
        return levo_conv_standin_f32(call.input, call.in_channels, call.in_length, call.output,
                                     call.out_channels, call.out_length,
                                     call.kind == LEVO_CONV_UPSAMPLE ? call.stride : 1,
                                     reinterpret_cast<levo_stream_t>(s));
    });
}

float *other_of(levo_vae_chain *c, const float *cur) { return cur == c->A ? c->B : c->A; }

int decode_one(levo_vae_chain *c, const float *latent, int64_t frames, float *audio_out,
               uint32_t flags, cudaStream_t s) {
    const levo_vae_topology &t = c->topo;
    const Layout &l = c->layout;
    const size_t esize = c->pdtype == LEVO_DTYPE_F16 ? 2 : 4;
    const char *base = static_cast<const char *>(c->params);
    auto P = [&](int64_t off) -> const void * { return base + off * esize; };
    NvtxRange window_range("levo.vae.decode");
    const bool timing = (flags & LEVO_CHAIN_TIMING) != 0;
    const bool capturing = c->n_capture > 0;
    auto snake_of = [&](int stage, int unit) -> SnakeRef {
        // Activation applied before conv `unit` of `stage`; unit == n_residual
        // means the next stage's upsample activation (or the output one).
        if (stage < t.n_stages && unit < t.n_residual)
            return {P(l.stage[stage].pre_alpha[unit]), P(l.stage[stage].pre_beta[unit])};
        if (stage + 1 < t.n_stages) return {P(l.stage[stage + 1].up_alpha), P(l.stage[stage + 1].up_beta)};
        return {P(l.out_alpha), P(l.out_beta)};
    };

    // Input conv + ENTRY unit.
    levo_conv_call call{};
    call.kind = LEVO_CONV_INPUT;
    call.stage = -1;
    call.unit = -1;
    call.kernel = 7;
    call.stride = 1;
    call.padding = 3;
    call.dilation = 1;
    call.input = latent;
    call.in_channels = t.latent_dim;
    call.in_length = frames;
    call.output = c->B;
    call.out_channels = t.entry_width;
    call.out_length = frames;
    int rc = run_conv(c, timing, call, s);
    if (rc != LEVO_OPS_OK) return rc;
    float *cur = call.result;
    {
        levo_fused_unit u{};
        u.u = cur;
        u.bias = P(l.in_bias);
        u.alpha_log = P(l.stage[0].up_alpha);
        u.beta_log = P(l.stage[0].up_beta);
        u.y_out = cur;
        u.channels = t.entry_width;
        u.time = frames;
        u.param_dtype = c->unit_pdtype;
        rc = run_unit(c, timing, LEVO_KCLASS_ENTRY, u, s);
        if (rc != LEVO_OPS_OK) return rc;
    }

    int64_t cin = t.entry_width;
    int64_t len = frames;
    for (int st = 0; st < t.n_stages; ++st) {
        NvtxRange stage_range(kStageRangeNames[st]);
        const int64_t cout = t.stage_width[st];
        const int64_t lout = len * t.stage_stride[st];
        const StageOffsets &so = l.stage[st];
        call = levo_conv_call{};
        call.kind = LEVO_CONV_UPSAMPLE;
        call.stage = st;
        call.unit = -1;
        call.kernel = 2 * t.stage_stride[st];
        call.stride = t.stage_stride[st];
        call.padding = (t.stage_stride[st] + 1) / 2;
        call.dilation = 1;
        call.input = cur;
        call.in_channels = cin;
        call.in_length = len;
        call.output = other_of(c, cur);
        call.out_channels = cout;
        call.out_length = lout;
        rc = run_conv(c, timing, call, s);
        if (rc != LEVO_OPS_OK) return rc;
        cur = call.result;
        {
            const SnakeRef sn = snake_of(st, 0);
            levo_fused_unit u{};
            u.u = cur;
            u.bias = P(so.up_bias);
            u.alpha_log = sn.alpha;
            u.beta_log = sn.beta;
            u.x_out = (t.n_residual > 0 || capturing) ? c->X : nullptr;
            u.y_out = cur;
            u.channels = cout;
            u.time = lout;
            u.param_dtype = c->unit_pdtype;
            rc = run_unit(c, timing, LEVO_KCLASS_UPSAMPLE, u, s);
            if (rc != LEVO_OPS_OK) return rc;
        }
        for (int r = 0; r < t.n_residual; ++r) {
            call = levo_conv_call{};
            call.kind = LEVO_CONV_RES0;
            call.stage = st;
            call.unit = r;
            call.kernel = 7;
            call.stride = 1;
            call.padding = 3 * t.dilation[r];
            call.dilation = t.dilation[r];
            call.input = cur;
            call.in_channels = cout;
            call.in_length = lout;
            call.output = other_of(c, cur);
            call.out_channels = cout;
            call.out_length = lout;
            rc = run_conv(c, timing, call, s);
            if (rc != LEVO_OPS_OK) return rc;
            cur = call.result;
            {
                levo_fused_unit u{};
                u.u = cur;
                u.bias = P(so.bias0[r]);
                u.alpha_log = P(so.post_alpha[r]);
                u.beta_log = P(so.post_beta[r]);
                u.y_out = cur;
                u.channels = cout;
                u.time = lout;
                u.param_dtype = c->unit_pdtype;
                rc = run_unit(c, timing, LEVO_KCLASS_POST, u, s);
                if (rc != LEVO_OPS_OK) return rc;
            }
            call = levo_conv_call{};
            call.kind = LEVO_CONV_RES1;
            call.stage = st;
            call.unit = r;
            call.kernel = 1;
            call.stride = 1;
            call.padding = 0;
            call.dilation = 1;
            call.input = cur;
            call.in_channels = cout;
            call.in_length = lout;
            call.output = other_of(c, cur);
            call.out_channels = cout;
            call.out_length = lout;
            rc = run_conv(c, timing, call, s);
            if (rc != LEVO_OPS_OK) return rc;
            cur = call.result;
            {
                const SnakeRef sn = snake_of(st, r + 1);
                levo_fused_unit u{};
                u.u = cur;
                u.bias = P(so.bias1[r]);
                u.residual = c->X;
                u.alpha_log = sn.alpha;
                u.beta_log = sn.beta;
                u.x_out = (r + 1 < t.n_residual || capturing) ? c->X : nullptr;
                u.y_out = cur;
                u.channels = cout;
                u.time = lout;
                u.param_dtype = c->unit_pdtype;
                rc = run_unit(c, timing, LEVO_KCLASS_RESIDUAL, u, s);
                if (rc != LEVO_OPS_OK) return rc;
            }
        }
        if (capturing) {
            // the stage output (src/levo-vae.cpp:230-231) is x, now in X
            const cudaError_t err = cudaMemcpyAsync(c->capture[st], c->X,
                                                    static_cast<size_t>(cout * lout) * sizeof(float),
                                                    cudaMemcpyDefault, s);
            if (err != cudaSuccess) return cuda_fail(err, "levo_vae_chain: stage capture copy");
        }
        cin = cout;
        len = lout;
    }

    // Output conv (no bias) + optional tanh epilogue.
    call = levo_conv_call{};
    call.kind = LEVO_CONV_OUTPUT;
    call.stage = -1;
    call.unit = -1;
    call.kernel = 7;
    call.stride = 1;
    call.padding = 3;
    call.dilation = 1;
    call.input = cur;
    call.in_channels = cin;
    call.in_length = len;
    call.output = audio_out;
    call.out_channels = t.audio_channels;
    call.out_length = len;
    rc = run_conv(c, timing, call, s);
    if (rc != LEVO_OPS_OK) return rc;
    if (call.result != audio_out)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain: the output convolution must write the audio buffer");
    if (flags & LEVO_CHAIN_TANH) {
        levo_fused_unit u{};
        u.u = audio_out;
        u.y_out = audio_out;
        u.channels = t.audio_channels;
        u.time = len;
        u.param_dtype = c->unit_pdtype;
        u.flags = LEVO_FUSED_TANH;
        rc = run_unit(c, timing, LEVO_KCLASS_EPILOGUE, u, s);
        if (rc != LEVO_OPS_OK) return rc;
    }
    return LEVO_OPS_OK;
}

// True when no value of p[0..n) is an infinity or a NaN: a branch-free OR over
// the exponent fields, which the compiler vectorises (a window's latent is
// 192 KB at 750 frames).
bool finite_values(const float *p, int64_t n) {
    uint32_t bad = 0;
    for (int64_t i = 0; i < n; ++i) {
        uint32_t bits;
        std::memcpy(&bits, p + i, sizeof(bits));
        bad |= static_cast<uint32_t>((bits & 0x7f800000u) == 0x7f800000u);
    }
    return bad == 0;
}

int check_decode_args(levo_vae_chain *c, int64_t frames, uint32_t flags, const char *what) {
    if (c == nullptr) return set_error(LEVO_OPS_EINVAL, std::string(what) + ": chain is null");
    if (frames <= 0 || frames > c->max_frames)
        return set_error(LEVO_OPS_EINVAL,
                         std::string(what) + ": latent frame count must be in 1..max_frames");
    if (flags & ~(LEVO_CHAIN_TANH | LEVO_CHAIN_TIMING))
        return set_error(LEVO_OPS_EINVAL, std::string(what) + ": unknown flag bits");
    return LEVO_OPS_OK;
}

}  // namespace
}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_vae_topology_reference(levo_vae_topology *out) {
    levo::clear_error();
    if (out == nullptr) return levo::set_error(LEVO_OPS_EINVAL, "levo_vae_topology_reference: out is null");
    levo_vae_topology t{};
    t.latent_dim = 64;
    t.audio_channels = 2;
    t.entry_width = 2048;
    t.n_stages = 5;
    const int32_t widths[5] = {1024, 512, 256, 128, 128};
    const int32_t strides[5] = {10, 6, 4, 4, 2};
    for (int s = 0; s < 5; ++s) {
        t.stage_width[s] = widths[s];
        t.stage_stride[s] = strides[s];
    }
    t.n_residual = 3;
    t.dilation[0] = 1;
    t.dilation[1] = 3;
    t.dilation[2] = 9;
    *out = t;
    return LEVO_OPS_OK;
}

LEVO_OPS_API int64_t levo_vae_param_count(const levo_vae_topology *topology) {
    levo::clear_error();
    std::string why;
    if (topology == nullptr || !levo::valid_topology(*topology, &why))
        return levo::set_error(LEVO_OPS_EINVAL, "levo_vae_param_count: invalid topology: " + why);
    return levo::make_layout(*topology).total;
}

LEVO_OPS_API int levo_conv_standin_f32(const float *in, int64_t in_channels, int64_t in_length,
                                       float *out, int64_t out_channels, int64_t out_length,
                                       int32_t stride, levo_stream_t stream) {
    using namespace levo;
    if (in == nullptr || out == nullptr)
        return set_error(LEVO_OPS_EINVAL, "levo_conv_standin_f32: required pointer is null");
    if (in_channels <= 0 || in_length <= 0 || out_channels < 0 || out_length < 0 || stride <= 0)
        return set_error(LEVO_OPS_EINVAL, "levo_conv_standin_f32: invalid shape or stride");
    const int64_t n = out_channels * out_length;
    if (n == 0) return LEVO_OPS_OK;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (out_length % 8 == 0 && aligned_to(out, 32)) {
        // one vector per thread, one CTA per 256 vectors (short-lived CTAs stream best)
        const int64_t grid = std::min<int64_t>((n / 8 + 255) / 256, 0x7fffffff);
        const cudaError_t err =
            launch_pdl(conv_standin_vec8_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, s, in,
                       in_channels, in_length, out, out_channels, out_length, stride,
                       1.0 / static_cast<double>(out_length));
        if (err != cudaSuccess)
            return set_error(LEVO_OPS_ELAUNCH, std::string("levo_conv_standin_f32: kernel launch failed: ") +
                                                   cudaGetErrorString(err));
    } else {
        const int64_t gx = std::min<int64_t>((out_length + 1023) / 1024, 64);
        const int64_t gy = std::min<int64_t>(out_channels, 65535);
        const cudaError_t err =
            launch_pdl(conv_standin_kernel, dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), dim3(256), 0,
                       s, in, in_channels, in_length, out, out_channels, out_length, stride);
        if (err != cudaSuccess)
            return set_error(LEVO_OPS_ELAUNCH, std::string("levo_conv_standin_f32: kernel launch failed: ") +
                                                   cudaGetErrorString(err));
    }
    return check_launch("levo_conv_standin_f32");
}

// An F32 chain replaces each SnakeBeta layer's (alpha_log, beta_log) by
// (alpha, 1/beta) once, with the library's own prepare kernel (bit-identical to
// the exponentials every launch would otherwise take, src/levo-audio-ops.cpp:
// 146-151): the fused units then start each chunk with three plain loads.  The
// activation buffer A is the scratch; the work runs and is waited for on the
// legacy default stream, like the parameter upload before it.
static int prepare_snake_layers(levo_vae_chain *c) {
    using namespace levo;
    const levo_vae_topology &t = c->topo;
    const Layout &l = c->layout;
    float *p = static_cast<float *>(c->params);
    struct Pair {
        int64_t alpha, beta, n;
    };
    std::vector<Pair> pairs;
    int64_t cin = t.entry_width;
    for (int s = 0; s < t.n_stages; ++s) {
        pairs.push_back({l.stage[s].up_alpha, l.stage[s].up_beta, cin});
        for (int r = 0; r < t.n_residual; ++r) {
            pairs.push_back({l.stage[s].pre_alpha[r], l.stage[s].pre_beta[r], t.stage_width[s]});
            pairs.push_back({l.stage[s].post_alpha[r], l.stage[s].post_beta[r], t.stage_width[s]});
        }
        cin = t.stage_width[s];
    }
    pairs.push_back({l.out_alpha, l.out_beta, cin});
    for (const Pair &q : pairs) {
        if (2 * q.n > c->max_elems) return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_create: scratch too small");
        const int rc = levo_snake_params_prepare(p + q.alpha, p + q.beta, LEVO_DTYPE_F32, q.n, c->A, c->A + q.n,
                                                 nullptr);
        if (rc != LEVO_OPS_OK) return rc;
        const size_t bytes = static_cast<size_t>(q.n) * sizeof(float);
        cudaError_t err = cudaMemcpyAsync(p + q.alpha, c->A, bytes, cudaMemcpyDeviceToDevice, nullptr);
        if (err == cudaSuccess)
            err = cudaMemcpyAsync(p + q.beta, c->A + q.n, bytes, cudaMemcpyDeviceToDevice, nullptr);
        if (err != cudaSuccess) return cuda_fail(err, "levo_vae_chain_create: parameter preparation");
    }
    const cudaError_t err = cudaStreamSynchronize(nullptr);
    if (err != cudaSuccess) return cuda_fail(err, "levo_vae_chain_create: parameter preparation");
    c->unit_pdtype = LEVO_DTYPE_SNAKE_PREPARED;
    return LEVO_OPS_OK;
}

static int create_chain(levo_vae_chain **out, const levo_vae_topology *topology, const void *params_host,
                        int pdtype, int64_t max_frames, levo_conv_fn conv, void *conv_user, int device) {
    using namespace levo;
    clear_error();
    if (out == nullptr || topology == nullptr || params_host == nullptr)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_create: required pointer is null");
    *out = nullptr;
    std::string why;
    if (!valid_topology(*topology, &why))
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_create: invalid topology: " + why);
    if (max_frames <= 0) return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_create: max_frames must be positive");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_create: no such CUDA device");

    levo_vae_chain *c = new (std::nothrow) levo_vae_chain();
    if (c == nullptr) return set_error(LEVO_OPS_ENOMEM, "levo_vae_chain_create: out of host memory");
    c->device = device;
    c->pdtype = pdtype;
    c->unit_pdtype = pdtype;
    c->topo = *topology;
    c->layout = make_layout(*topology);
    c->max_frames = max_frames;
    c->conv = conv;
    c->conv_user = conv_user;
    const levo_vae_topology &t = c->topo;
    int64_t elems = static_cast<int64_t>(t.entry_width) * max_frames;
    int64_t len = max_frames;
    int64_t cin = t.entry_width;
    for (int s = 0; s < t.n_stages; ++s) {
        if (len > (int64_t(1) << 40) / t.stage_stride[s]) {
            free_chain(c);
            return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_create: decoded length overflows");
        }
        elems = std::max(elems, cin * len);
        len *= t.stage_stride[s];
        elems = std::max(elems, static_cast<int64_t>(t.stage_width[s]) * len);
        cin = t.stage_width[s];
    }
    c->max_elems = elems;
    const size_t act_bytes = static_cast<size_t>(elems) * sizeof(float);
    const size_t lat_bytes = static_cast<size_t>(t.latent_dim) * max_frames * sizeof(float);
    const size_t audio_bytes = static_cast<size_t>(t.audio_channels) * len * sizeof(float);

    DeviceGuard guard(device);
    cudaError_t err = cudaSuccess;
    const size_t param_bytes = static_cast<size_t>(c->layout.total) * (pdtype == LEVO_DTYPE_F16 ? 2 : 4);
    if (err == cudaSuccess) err = cudaMalloc(&c->params, param_bytes);
    if (err == cudaSuccess) err = cudaMalloc(&c->X, act_bytes);
    if (err == cudaSuccess) err = cudaMalloc(&c->A, act_bytes);
    if (err == cudaSuccess) err = cudaMalloc(&c->B, act_bytes);
    for (int i = 0; i < 2 && err == cudaSuccess; ++i) {
        err = cudaMalloc(&c->lat[i], lat_bytes);
        if (err == cudaSuccess) err = cudaMalloc(&c->audio[i], audio_bytes);
        if (err == cudaSuccess) err = cudaEventCreateWithFlags(&c->computed[i], cudaEventDisableTiming);
        if (err == cudaSuccess) err = cudaEventCreateWithFlags(&c->copied[i], cudaEventDisableTiming);
    }
    if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking);
    if (err == cudaSuccess) err = cudaMemcpy(c->params, params_host, param_bytes, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        const int rc = cuda_fail(err, "levo_vae_chain_create");
        free_chain(c);
        return rc;
    }
    if (pdtype == LEVO_DTYPE_F32) {
        const int rc = prepare_snake_layers(c);
        if (rc != LEVO_OPS_OK) {
            free_chain(c);
            return rc;
        }
    }
    *out = c;
    return LEVO_OPS_OK;
}

LEVO_OPS_API int levo_vae_chain_create(levo_vae_chain **out, const levo_vae_topology *topology,
                                       const float *params_host, int64_t max_frames,
                                       levo_conv_fn conv, void *conv_user, int device) {
    return create_chain(out, topology, params_host, LEVO_DTYPE_F32, max_frames, conv, conv_user, device);
}

LEVO_OPS_API int levo_vae_chain_create_f16(levo_vae_chain **out, const levo_vae_topology *topology,
                                           const uint16_t *params_host, int64_t max_frames,
                                           levo_conv_fn conv, void *conv_user, int device) {
    return create_chain(out, topology, params_host, LEVO_DTYPE_F16, max_frames, conv, conv_user, device);
}

LEVO_OPS_API void levo_vae_chain_destroy(levo_vae_chain *chain) {
    if (chain == nullptr) return;
    {
        levo::DeviceGuard guard(chain->device);
        cudaDeviceSynchronize();
    }
    levo::free_chain(chain);
}

LEVO_OPS_API int levo_vae_chain_set_stage_capture(levo_vae_chain *chain, float *const *stage_out,
                                                  int32_t count) {
    using namespace levo;
    clear_error();
    if (chain == nullptr) return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_set_stage_capture: chain is null");
    if (stage_out == nullptr || count == 0) {
        chain->n_capture = 0;
        return LEVO_OPS_OK;
    }
    if (count != chain->topo.n_stages)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_set_stage_capture: one destination per stage is required");
    for (int32_t i = 0; i < count; ++i)
        if (stage_out[i] == nullptr || !aligned_to(stage_out[i], 4))
            return set_error(LEVO_OPS_EINVAL,
                             "levo_vae_chain_set_stage_capture: stage destination is null or not 4-byte aligned");
    for (int32_t i = 0; i < count; ++i) chain->capture[i] = stage_out[i];
    chain->n_capture = count;
    return LEVO_OPS_OK;
}

LEVO_OPS_API int levo_vae_chain_decode(levo_vae_chain *chain, const float *latent, int64_t frames,
                                       float *audio, uint32_t flags, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    int rc = check_decode_args(chain, frames, flags, "levo_vae_chain_decode");
    if (rc != LEVO_OPS_OK) return rc;
    if (latent == nullptr || audio == nullptr)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_decode: required pointer is null");
    if (!aligned_to(latent, 4) || !aligned_to(audio, 4))
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_decode: pointer is not 4-byte aligned");
    DeviceGuard guard(chain->device);
    return decode_one(chain, latent, frames, audio, flags, reinterpret_cast<cudaStream_t>(stream));
}

LEVO_OPS_API int levo_vae_chain_decode_windows(levo_vae_chain *chain, const float *latents_host,
                                               int64_t windows, int64_t frames, float *audio_host,
                                               uint32_t flags, levo_cancel_fn cancel,
                                               void *cancel_user, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    int rc = check_decode_args(chain, frames, flags, "levo_vae_chain_decode_windows");
    if (rc != LEVO_OPS_OK) return rc;
    if (latents_host == nullptr || audio_host == nullptr || windows < 0)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_decode_windows: invalid host buffers or window count");
    if (chain->n_capture > 0 && windows > 1)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_decode_windows: stage capture holds one window");
    DeviceGuard guard(chain->device);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const levo_vae_topology &t = chain->topo;
    const int64_t lat_elems = static_cast<int64_t>(t.latent_dim) * frames;
    const int64_t audio_elems = static_cast<int64_t>(t.audio_channels) * frames * total_upsampling(t);
    bool pending[2] = {false, false};
    cudaError_t err = cudaSuccess;
    auto non_finite = [](int64_t window) {
        return set_error(LEVO_OPS_ENONFINITE, "levo_vae_chain_decode_windows: latent payload contains a non-finite "
                                              "value (window " + std::to_string(window) + ")");
    };
    // Every exit waits for both streams: no copy of this call may still be
    // writing into audio_host once the call has returned.
    auto drained = [&](int rc) {
        cudaStreamSynchronize(s);
        cudaStreamSynchronize(chain->copy_stream);
        return rc;
    };
    for (int64_t w = 0; w < windows; ++w) {
        if (cancel != nullptr && cancel(cancel_user) != 0)
            return drained(set_error(LEVO_OPS_ECANCELLED,
                                     "levo_vae_chain_decode_windows: cancelled before window " + std::to_string(w)));
        // vae_decoder::decode rejects non-finite latents (src/levo-vae.cpp:189-191).  The check runs on
        // the host while the GPU already decodes the window, and before the window's audio copy is
        // enqueued, so a rejected window still writes nothing to audio_host; with stage capture it
        // runs first, as nothing may reach the capture buffers either.
        const float *lat_w = latents_host + w * lat_elems;
        const bool check_first = chain->n_capture > 0;
        if (check_first && !finite_values(lat_w, lat_elems)) return drained(non_finite(w));
        const int slot = static_cast<int>(w & 1);
        // The slot's previous audio must have left the device before reuse.
        if (pending[slot]) err = cudaStreamWaitEvent(s, chain->copied[slot], 0);
        if (err == cudaSuccess)
            err = cudaMemcpyAsync(chain->lat[slot], lat_w,
                                  static_cast<size_t>(lat_elems) * sizeof(float), cudaMemcpyHostToDevice, s);
        if (err != cudaSuccess) return drained(cuda_fail(err, "levo_vae_chain_decode_windows: latent upload"));
        rc = decode_one(chain, chain->lat[slot], frames, chain->audio[slot], flags, s);
        if (rc != LEVO_OPS_OK) return drained(rc);
        if (!check_first && !finite_values(lat_w, lat_elems)) return drained(non_finite(w));
        err = cudaEventRecord(chain->computed[slot], s);
        if (err == cudaSuccess) err = cudaStreamWaitEvent(chain->copy_stream, chain->computed[slot], 0);
        if (err == cudaSuccess)
            err = cudaMemcpyAsync(audio_host + w * audio_elems, chain->audio[slot],
                                  static_cast<size_t>(audio_elems) * sizeof(float), cudaMemcpyDeviceToHost,
                                  chain->copy_stream);
        if (err == cudaSuccess) err = cudaEventRecord(chain->copied[slot], chain->copy_stream);
        if (err != cudaSuccess) return drained(cuda_fail(err, "levo_vae_chain_decode_windows: audio download"));
        pending[slot] = true;
    }
    err = cudaStreamSynchronize(chain->copy_stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return drained(cuda_fail(err, "levo_vae_chain_decode_windows: synchronize"));
    return LEVO_OPS_OK;
}

LEVO_OPS_API int levo_vae_chains_decode_windows(levo_vae_chain *const *chains, int32_t n_chains,
                                                const float *latents_host, int64_t windows, int64_t frames,
                                                float *audio_host, uint32_t flags, levo_cancel_fn cancel,
                                                void *cancel_user) {
    using namespace levo;
    clear_error();
    const char *w = "levo_vae_chains_decode_windows";
    if (chains == nullptr || n_chains <= 0)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": at least one chain is required");
    for (int32_t i = 0; i < n_chains; ++i) {
        if (chains[i] == nullptr) return set_error(LEVO_OPS_EINVAL, std::string(w) + ": chain is null");
        // a chain's workspace, slots, copy stream and events serve one thread at a time
        for (int32_t j = 0; j < i; ++j)
            if (chains[j] == chains[i])
                return set_error(LEVO_OPS_EINVAL, std::string(w) + ": the same chain is passed twice (chains " +
                                                      std::to_string(j) + " and " + std::to_string(i) + ")");
    }
    for (int32_t i = 0; i < n_chains; ++i) {
        if (std::memcmp(&chains[i]->topo, &chains[0]->topo, sizeof(levo_vae_topology)) != 0)
            return set_error(LEVO_OPS_EINVAL, std::string(w) + ": chains must share one topology");
        const int rc = check_decode_args(chains[i], frames, flags, w);
        if (rc != LEVO_OPS_OK) return rc;
    }
    if (latents_host == nullptr || audio_host == nullptr || windows < 0)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": invalid host buffers or window count");
    const levo_vae_topology &t = chains[0]->topo;
    const int64_t lat_elems = static_cast<int64_t>(t.latent_dim) * frames;
    const int64_t audio_elems = static_cast<int64_t>(t.audio_channels) * frames * total_upsampling(t);
    std::vector<int> codes(static_cast<size_t>(n_chains), LEVO_OPS_OK);
    std::vector<std::string> messages(static_cast<size_t>(n_chains));
    auto work = [&](int32_t i) {
        // contiguous block [start, stop) of the windows, sizes differing by at most one
        const int64_t base = windows / n_chains, extra = windows % n_chains;
        const int64_t start = i * base + std::min<int64_t>(i, extra);
        const int64_t count = base + (i < extra ? 1 : 0);
        if (count == 0) return;
        levo_vae_chain *c = chains[i];
        DeviceGuard guard(c->device);
        cudaStream_t stream = nullptr;
        cudaError_t err = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
        int rc = err == cudaSuccess ? LEVO_OPS_OK : cuda_fail(err, std::string(w) + ": stream");
        if (rc == LEVO_OPS_OK)
            rc = levo_vae_chain_decode_windows(c, latents_host + start * lat_elems, count, frames,
                                               audio_host + start * audio_elems, flags, cancel, cancel_user,
                                               reinterpret_cast<levo_stream_t>(stream));
        if (stream != nullptr) cudaStreamDestroy(stream);
        codes[static_cast<size_t>(i)] = rc;
        if (rc != LEVO_OPS_OK) messages[static_cast<size_t>(i)] = levo_ops_last_error();
    };
    std::vector<std::thread> threads;
    threads.reserve(static_cast<size_t>(n_chains));
    for (int32_t i = 1; i < n_chains; ++i) threads.emplace_back(work, i);
    work(0);
    for (std::thread &th : threads) th.join();
    for (int32_t i = 0; i < n_chains; ++i)
        if (codes[static_cast<size_t>(i)] != LEVO_OPS_OK) {
            const int64_t start = i * (windows / n_chains) + std::min<int64_t>(i, windows % n_chains);
            return set_error(codes[static_cast<size_t>(i)],
                             messages[static_cast<size_t>(i)] + " (chain " + std::to_string(i) +
                                 ", whose windows start at " + std::to_string(start) + ")");
        }
    return LEVO_OPS_OK;
}

LEVO_OPS_API int levo_vae_chain_timing(levo_vae_chain *chain, levo_kernel_timing *out, int reset) {
    using namespace levo;
    clear_error();
    if (chain == nullptr || out == nullptr)
        return set_error(LEVO_OPS_EINVAL, "levo_vae_chain_timing: required pointer is null");
    DeviceGuard guard(chain->device);
    for (const TimedLaunch &tl : chain->launches) {
        const cudaError_t err = cudaEventSynchronize(chain->events[tl.ev_end]);
        if (err != cudaSuccess) return cuda_fail(err, "levo_vae_chain_timing");
        float ms = 0.f;
        cudaEventElapsedTime(&ms, chain->events[tl.ev_start], chain->events[tl.ev_end]);
        levo_kernel_timing &k = chain->totals[tl.kclass];
        k.launches += 1;
        k.milliseconds += ms;
        k.algorithmic_bytes += tl.bytes;
        k.elements += tl.elems;
    }
    chain->launches.clear();
    chain->next_event = 0;
    std::memcpy(out, chain->totals, sizeof(chain->totals));
    if (reset) std::memset(chain->totals, 0, sizeof(chain->totals));
    return LEVO_OPS_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode (levo_vae_decode_noalloc_f32)
//
// Some callers cannot let this library call cudaMalloc: a real-time render
// thread (cudaMalloc may synchronise the whole device), or a host engine that
// owns a fixed device-memory budget and hands out only its own buffers (as the
// reference's GGML backend does with its graph allocator).  For them the three
// activation buffers of the decoder chain live in one file-scope device array
// of fixed size instead of a levo_vae_chain workspace.  Every GPU that loads
// this library holds the array (kNoallocFloats floats, 24 MiB) until the
// process exits.
// ---------------------------------------------------------------------------
namespace levo {
namespace {

constexpr int64_t kNoallocBufferFloats = int64_t(1) << 21;           // one activation buffer: 8 MiB
constexpr int64_t kNoallocFloats = 3 * kNoallocBufferFloats;          // X, A and B: 24 MiB

static __device__ __align__(256) float g_noalloc_scratch[kNoallocFloats];

// Device address of g_noalloc_scratch per device, looked up with that device
// current (the symbol's host-side name is not a device address).  It is looked
// up again on every call made outside stream capture, so a device reset (a new
// primary context, where the array may sit elsewhere) never leaves a stale
// address behind; a call under capture uses the last address looked up, so the
// first call on a device comes before any capture.
constexpr int kNoallocMaxDevices = 64;
float *g_noalloc_ptr[kNoallocMaxDevices] = {};
std::mutex g_noalloc_mutex;

int noalloc_scratch(int device, cudaStream_t stream, float **out) {
    if (device < 0 || device >= kNoallocMaxDevices)
        return set_error(LEVO_OPS_EUNSUPPORTED, "levo_vae_decode_noalloc_f32: device index out of range");
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess) {
        cudaGetLastError();
        capture = cudaStreamCaptureStatusNone;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[device] == nullptr || capture == cudaStreamCaptureStatusNone) {
        void *ptr = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (err != cudaSuccess || ptr == nullptr)
            return set_error(LEVO_OPS_ECUDA, std::string("levo_vae_decode_noalloc_f32: cannot resolve the "
                                                         "static scratch array: ") + cudaGetErrorString(err));
        g_noalloc_ptr[device] = static_cast<float *>(ptr);
    }
    *out = g_noalloc_ptr[device];
    return LEVO_OPS_OK;
}

}  // namespace
}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_vae_decode_noalloc_f32(const levo_vae_topology *topology, const float *params,
                                             const float *latent, int64_t frames, float *audio,
                                             levo_conv_fn conv, void *conv_user, uint32_t flags,
                                             levo_stream_t stream) {
    using namespace levo;
    clear_error();
    const char *w = "levo_vae_decode_noalloc_f32";
    std::string why;
    if (topology == nullptr || !valid_topology(*topology, &why))
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": invalid topology: " + why);
    if (params == nullptr || latent == nullptr || audio == nullptr)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": required pointer is null");
    if (!aligned_to(params, 4) || !aligned_to(latent, 4) || !aligned_to(audio, 4))
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": pointer is not 4-byte aligned");
    if (flags & ~LEVO_CHAIN_TANH)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": only LEVO_CHAIN_TANH is accepted");
    if (frames <= 0) return set_error(LEVO_OPS_EINVAL, std::string(w) + ": latent frame count must be positive");
    // Largest activation tensor of the stage loop; each of the three buffers must hold it.
    int64_t elems = static_cast<int64_t>(topology->entry_width) * frames;
    int64_t len = frames;
    int64_t cin = topology->entry_width;
    for (int st = 0; st < topology->n_stages; ++st) {
        if (len > kNoallocBufferFloats) break;
        elems = std::max(elems, cin * len);
        len *= topology->stage_stride[st];
        elems = std::max(elems, static_cast<int64_t>(topology->stage_width[st]) * len);
        cin = topology->stage_width[st];
    }
    if (elems > kNoallocBufferFloats || len > kNoallocBufferFloats)
        return set_error(LEVO_OPS_EINVAL,
                         std::string(w) + ": the largest activation tensor (" + std::to_string(elems) +
                             " floats) exceeds the static scratch limit of " +
                             std::to_string(kNoallocBufferFloats) +
                             " floats per buffer; use levo_vae_chain_create / levo_vae_chain_decode");
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess)
        return set_error(LEVO_OPS_ECUDA, std::string(w) + ": no current CUDA device");
    float *scratch = nullptr;
    const int rc = noalloc_scratch(device, reinterpret_cast<cudaStream_t>(stream), &scratch);
    if (rc != LEVO_OPS_OK) return rc;

    // A chain view over caller memory and the static scratch: no workspace,
    // no events, nothing allocated.
    levo_vae_chain view;
    view.device = device;
    view.topo = *topology;
    view.layout = make_layout(*topology);
    view.max_frames = frames;
    view.max_elems = kNoallocBufferFloats;
    view.params = const_cast<float *>(params);
    view.X = scratch;
    view.A = scratch + kNoallocBufferFloats;
    view.B = scratch + 2 * kNoallocBufferFloats;
    view.conv = conv;
    view.conv_user = conv_user;
    return decode_one(&view, latent, frames, audio, flags, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
