// Window assembly (next item after the decode): linear crossfade of decoded
// windows into one song, crop, and optional L/R interleave.
//
// Reference: assemble_renderer_audio (src/levo-renderer-pattern.cpp:137-203)
// writes window 0, then for every later window k crossfades its first
// `overlap` samples with what is already there,
//   out = out * (1 - alpha) + cur * alpha,  alpha = s / (overlap - 1),
// copies the rest, and finally crops to the target length; the render result
// is then interleaved L,R,L,R (src/levo-render.cpp:476-480).  With
// hop >= overlap and hop + overlap <= window (the reference's 750/250/1000
// frames) every output sample depends on at most two windows, so one pass
// computes each sample directly from the latest window that starts at or
// before it; the F32 expression order is the reference's, so the result is
// bit-identical.  When every length is a multiple of 4 a thread produces four
// consecutive samples from float4 loads (one window index per four samples).
//
// The reference rejects a decoded window holding a non-finite sample
// (require_finite_audio, :159-160; windows in order, left before right).  With
// a status word the kernel checks every sample it loads, and also the samples
// no output reads (past hop + overlap, or past the crop; none for the
// reference's own schedule), and records the first (window, channel) in that
// order with atomicMax on LEVO_ASSEMBLE_STATUS(window * channels + channel).
#include <algorithm>

#include "common.cuh"

namespace levo {
namespace {

struct AsmArgs {
    const float *win;  // [windows][channels][window_samples]
    float *out;        // planar [channels][target] or interleaved [target][channels]
    int64_t windows, channels, window_samples, hop, overlap, target;
    float denom;       // overlap - 1
    int interleaved;
    int32_t *status;   // optional: first non-finite (window, channel)
};

__device__ __forceinline__ void note_sample(const AsmArgs &a, float v, int64_t k, int64_t c) {
    if (a.status != nullptr && !isfinite(v))
        atomicMax(a.status, static_cast<int32_t>(LEVO_ASSEMBLE_STATUS(k * a.channels + c)));
}

// prev * (1 - alpha) + cur * alpha with alpha = s / (overlap - 1), rounded step by step as the
// reference's crossfade does
__device__ __forceinline__ float blend(float prev, float cur, int64_t s, float denom) {
    const float alpha = __fdiv_rn(static_cast<float>(s), denom);
    return __fadd_rn(__fmul_rn(prev, __fsub_rn(1.0f, alpha)), __fmul_rn(cur, alpha));
}

__device__ __forceinline__ float assembled_sample(const AsmArgs &a, int64_t c, int64_t t) {
    int64_t k = t / a.hop;
    if (k > a.windows - 1) k = a.windows - 1;
    const int64_t s = t - k * a.hop;
    const float cur = a.win[(k * a.channels + c) * a.window_samples + s];
    note_sample(a, cur, k, c);
    if (k == 0 || s >= a.overlap) return cur;
    const float prev = a.win[((k - 1) * a.channels + c) * a.window_samples + s + a.hop];
    note_sample(a, prev, k - 1, c);
    return blend(prev, cur, s, a.denom);
}

// Samples no output reads (past hop + overlap in every window but the last, and past the crop) are
// checked by blocks b, b + G, ... of rows r0 + k * rstep: window k < windows - 1 is read up to hop +
// overlap, the last one entirely, and none of them past the crop.
__device__ __forceinline__ void check_unread_rows(const AsmArgs &a, int64_t r0, int64_t rstep, int64_t block,
                                                  int64_t blocks) {
    const int64_t rows = a.windows * a.channels;
    for (int64_t r = r0 + block * rstep; r < rows; r += blocks * rstep) {
        const int64_t k = r / a.channels;
        const int64_t reach = k < a.windows - 1 ? a.hop + a.overlap : a.window_samples;
        const int64_t cropped = a.target - k * a.hop > 0 ? a.target - k * a.hop : 0;
        const int64_t unread = reach < cropped ? reach : cropped;
        for (int64_t s = unread + threadIdx.x; s < a.window_samples; s += blockDim.x)
            note_sample(a, a.win[r * a.window_samples + s], k, r - k * a.channels);
    }
}

__global__ void __launch_bounds__(256) assemble_kernel(const AsmArgs a) {
    const int64_t n = a.channels * a.target;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        // Output-major index: consecutive threads write consecutive output words.
        int64_t c, t;
        if (a.interleaved) {
            t = e / a.channels;
            c = e - t * a.channels;
        } else {
            c = e / a.target;
            t = e - c * a.target;
        }
        a.out[e] = assembled_sample(a, c, t);
    }
    if (a.status != nullptr) check_unread_rows(a, 0, 1, blockIdx.x, gridDim.x);
}

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

__device__ __forceinline__ void note4(const AsmArgs &a, const float4 &v, int64_t k, int64_t c) {
    if (a.status != nullptr && !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w)))
        atomicMax(a.status, static_cast<int32_t>(LEVO_ASSEMBLE_STATUS(k * a.channels + c)));
}

// Outputs t0..t0+3 of channel c (t0 % 4 == 0): with hop and overlap multiples of 4 the four share
// their window k and their side of the overlap edge, so each source is one float4 load.
__device__ __forceinline__ float4 assembled4(const AsmArgs &a, int64_t c, int64_t t0) {
    int64_t k = t0 / a.hop;
    if (k > a.windows - 1) k = a.windows - 1;
    const int64_t s = t0 - k * a.hop;
    const float4 cur = ld4(a.win + (k * a.channels + c) * a.window_samples + s);
    note4(a, cur, k, c);
    if (k == 0 || s >= a.overlap) return cur;
    const float4 prev = ld4(a.win + ((k - 1) * a.channels + c) * a.window_samples + s + a.hop);
    note4(a, prev, k - 1, c);
    return make_float4(blend(prev.x, cur.x, s, a.denom), blend(prev.y, cur.y, s + 1, a.denom),
                       blend(prev.z, cur.z, s + 2, a.denom), blend(prev.w, cur.w, s + 3, a.denom));
}

// Vector form (hop, overlap, window and target lengths multiples of 4, 16-byte aligned tensors).
// Planar: blockIdx.y is the channel, a thread writes one float4 of its row.  STEREO (interleaved,
// 2 channels): a thread writes L,R of four consecutive samples, two float4.  Same arithmetic as
// assembled_sample, so the same bits.
template <bool STEREO>
__global__ void __launch_bounds__(256) assemble_vec4_kernel(const AsmArgs a) {
    const int64_t nvec = a.target / 4;
    const int64_t c = STEREO ? 0 : blockIdx.y;
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec;
         v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t0 = 4 * v;
        if (STEREO) {
            const float4 l = assembled4(a, 0, t0), r = assembled4(a, 1, t0);
            float4 *o = reinterpret_cast<float4 *>(a.out + 2 * t0);
            o[0] = make_float4(l.x, r.x, l.y, r.y);
            o[1] = make_float4(l.z, r.z, l.w, r.w);
        } else {
            *reinterpret_cast<float4 *>(a.out + c * a.target + t0) = assembled4(a, c, t0);
        }
    }
    if (a.status == nullptr) return;
    if (STEREO)
        check_unread_rows(a, 0, 1, blockIdx.x, gridDim.x);
    else
        check_unread_rows(a, c, a.channels, blockIdx.x, gridDim.x);
}

}  // namespace
}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_assemble_windows_f32(const float *windows, int64_t n_windows, int64_t channels,
                                           int64_t window_samples, int64_t hop_samples,
                                           int64_t overlap_samples, int64_t target_samples,
                                           float *out, int32_t interleaved, int32_t *status,
                                           levo_stream_t stream) {
    using namespace levo;
    clear_error();
    const char *w = "levo_assemble_windows_f32";
    if (n_windows <= 0 || channels <= 0 || window_samples <= 0)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": renderer schedule is empty");
    if (hop_samples <= 0 || overlap_samples < 0 || overlap_samples == 1 ||
        overlap_samples >= window_samples || hop_samples < overlap_samples ||
        hop_samples + overlap_samples > window_samples)
        return set_error(LEVO_OPS_EINVAL,
                         std::string(w) + ": renderer overlap descriptor is invalid (need 2 <= overlap <= "
                                          "hop and hop + overlap <= window, or overlap = 0)");
    const int64_t assembled = (n_windows - 1) * hop_samples + window_samples;
    if (target_samples < 0 || target_samples > assembled)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": renderer target crop exceeds assembled output");
    if (target_samples == 0 && status == nullptr) return LEVO_OPS_OK;
    if (windows == nullptr || (out == nullptr && target_samples > 0))
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": required pointer is null");
    if (!aligned_to(windows, 4) || !aligned_to(out, 4) || (status != nullptr && !aligned_to(status, 4)))
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": pointer is not 4-byte aligned");
    if (status != nullptr && n_windows > (LEVO_ASSEMBLE_STATUS_LIMIT - 1) / channels)
        return set_error(LEVO_OPS_EUNSUPPORTED, std::string(w) + ": too many window channels for the status word");
    const AsmArgs a{windows, out, n_windows, channels, window_samples, hop_samples, overlap_samples,
                    target_samples, static_cast<float>(overlap_samples - 1), interleaved ? 1 : 0, status};
    const int64_t n = channels * target_samples;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    // The vector form: every length a multiple of 4 and 16-byte aligned tensors, so four consecutive
    // outputs share their window and overlap side and each source is one float4 (the reference's
    // 750 / 250 / 1000-frame schedule, 1920 samples a frame, always qualifies).
    const bool vec = hop_samples % 4 == 0 && overlap_samples % 4 == 0 && window_samples % 4 == 0 &&
                     target_samples % 4 == 0 && aligned_to(windows, 16) && aligned_to(out, 16) &&
                     (interleaved ? channels == 2 : channels <= 65535);
    if (vec) {
        const int64_t per_row = std::max<int64_t>((target_samples / 4 + 255) / 256, 1);
        if (interleaved) {
            // two rows per window in the unread-sample check
            const int64_t grid = std::min<int64_t>(std::max<int64_t>(per_row, status ? n_windows * 2 : 0), cap);
            assemble_vec4_kernel<true><<<static_cast<unsigned>(grid), 256, 0, s>>>(a);
        } else {
            const int64_t gx = std::min<int64_t>(std::max<int64_t>(per_row, status ? n_windows : 0),
                                                 std::max<int64_t>(cap / channels, 1));
            assemble_vec4_kernel<false><<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(channels)), 256, 0, s>>>(a);
        }
        return check_launch(w);
    }
    // output elements, and with a status word the window rows of the unread-sample check too
    const int64_t grid = std::min<int64_t>(std::max<int64_t>((n + 255) / 256, status ? n_windows * channels : 0), cap);
    assemble_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(a);
    return check_launch(w);
}

}  // extern "C"
