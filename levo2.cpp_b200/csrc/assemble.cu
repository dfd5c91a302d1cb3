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
// bit-identical.
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

__device__ __forceinline__ float assembled_sample(const AsmArgs &a, int64_t c, int64_t t) {
    int64_t k = t / a.hop;
    if (k > a.windows - 1) k = a.windows - 1;
    const int64_t s = t - k * a.hop;
    const float cur = a.win[(k * a.channels + c) * a.window_samples + s];
    note_sample(a, cur, k, c);
    if (k == 0 || s >= a.overlap) return cur;
    const float prev = a.win[((k - 1) * a.channels + c) * a.window_samples + s + a.hop];
    note_sample(a, prev, k - 1, c);
    const float alpha = __fdiv_rn(static_cast<float>(s), a.denom);
    return __fadd_rn(__fmul_rn(prev, __fsub_rn(1.0f, alpha)), __fmul_rn(cur, alpha));
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
    if (a.status == nullptr) return;
    // Samples no output reads: window k < windows - 1 is read up to hop + overlap,
    // the last one entirely, and none of them past the crop.
    const int64_t rows = a.windows * a.channels;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int64_t k = r / a.channels;
        const int64_t reach = k < a.windows - 1 ? a.hop + a.overlap : a.window_samples;
        const int64_t cropped = a.target - k * a.hop > 0 ? a.target - k * a.hop : 0;
        const int64_t unread = reach < cropped ? reach : cropped;
        for (int64_t s = unread + threadIdx.x; s < a.window_samples; s += blockDim.x)
            note_sample(a, a.win[r * a.window_samples + s], k, r - k * a.channels);
    }
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
    // output elements, and with a status word the window rows of the unread-sample check too
    const int64_t grid = std::min<int64_t>(std::max<int64_t>((n + 255) / 256, status ? n_windows * channels : 0), cap);
    assemble_kernel<<<static_cast<unsigned>(grid), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    return check_launch(w);
}

}  // extern "C"
