// Latent normalisation around the Flow renderer and the layout change into the
// VAE (next item f2).
//
// Reference:
//   normalize_latents   out = (raw - mean[c]) / stddev[c]      (src/levo-flow-conditioning.cpp:113-123)
//   denormalize_latents out = x * stddev[c] + mean[c]          (src/levo-flow-conditioning.cpp:125-135)
//   channel_major_latent [frames][dim] -> [dim][frames]         (src/levo-render.cpp:181-193)
// The VAE input path is one kernel: de-normalise while transposing through a
// shared-memory tile (coalesced reads of frame-major rows, coalesced writes of
// channel-major rows).  F32 arithmetic in the reference's order, no FMA:
// results are bit-identical.  Both reference functions first reject a
// non-finite input value ("raw latent" / "normalized latent contains a
// non-finite value", :116,128); with a status word the kernels set its bit 0
// when they load one.
#include <algorithm>

#include "common.cuh"

namespace levo {
namespace {

constexpr int kTile = 32;

__global__ void __launch_bounds__(kTile * 8) denorm_transpose_kernel(const float *in, const float *mean,
                                                                    const float *stddev, int64_t frames,
                                                                    int64_t dim, float *out, int denorm,
                                                                    int32_t *status) {
    __shared__ float tile[kTile][kTile + 1];
    const int64_t f0 = static_cast<int64_t>(blockIdx.x) * kTile;
    const int64_t c0 = static_cast<int64_t>(blockIdx.y) * kTile;
    // read: rows = frames, columns = channels (contiguous)
    for (int r = threadIdx.y; r < kTile; r += blockDim.y) {
        const int64_t f = f0 + r, c = c0 + threadIdx.x;
        if (f < frames && c < dim) {
            float v = in[f * dim + c];
            if (status != nullptr && !isfinite(v)) atomicOr(status, 1);
            if (denorm) v = __fadd_rn(__fmul_rn(v, stddev[c]), mean[c]);
            tile[r][threadIdx.x] = v;
        }
    }
    __syncthreads();
    // write: rows = channels, columns = frames (contiguous)
    for (int r = threadIdx.y; r < kTile; r += blockDim.y) {
        const int64_t c = c0 + r, f = f0 + threadIdx.x;
        if (c < dim && f < frames) out[c * frames + f] = tile[threadIdx.x][r];
    }
}

__global__ void __launch_bounds__(256) normalize_kernel(const float *in, const float *mean, const float *stddev,
                                                        int64_t n, int64_t dim, float *out, int32_t *status) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t c = i % dim;
        const float v = in[i];
        if (status != nullptr && !isfinite(v)) atomicOr(status, 1);
        out[i] = __fdiv_rn(__fsub_rn(v, mean[c]), stddev[c]);
    }
}

int check_common(const char *w, const float *in, const float *mean, const float *stddev, int64_t frames,
                 int64_t dim, const float *out, bool need_stats, const int32_t *status) {
    if (frames <= 0 || dim <= 0)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": latent dimensions must be positive");
    if (in == nullptr || out == nullptr || (need_stats && (mean == nullptr || stddev == nullptr)))
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": required pointer is null");
    const void *ptrs[5] = {in, mean, stddev, out, status};
    for (const void *p : ptrs)
        if (p && !aligned_to(p, 4))
            return set_error(LEVO_OPS_EINVAL, std::string(w) + ": pointer is not 4-byte aligned");
    return LEVO_OPS_OK;
}

}  // namespace
}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_latent_to_vae_f32(const float *frame_major, const float *mean, const float *stddev,
                                        int64_t frames, int64_t dim, float *channel_major,
                                        int32_t *status, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    const char *w = "levo_latent_to_vae_f32";
    const bool denorm = mean != nullptr || stddev != nullptr;
    int rc = check_common(w, frame_major, mean, stddev, frames, dim, channel_major, denorm, status);
    if (rc != LEVO_OPS_OK) return rc;
    if (frame_major == channel_major)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": the transpose cannot run in place");
    if ((dim + kTile - 1) / kTile > 65535 || (frames + kTile - 1) / kTile > 0x7fffffff)
        return set_error(LEVO_OPS_EUNSUPPORTED, std::string(w) + ": latent too large for one launch");
    const dim3 grid(static_cast<unsigned>((frames + kTile - 1) / kTile), static_cast<unsigned>((dim + kTile - 1) / kTile));
    denorm_transpose_kernel<<<grid, dim3(kTile, 8), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        frame_major, mean, stddev, frames, dim, channel_major, denorm ? 1 : 0, status);
    return check_launch(w);
}

LEVO_OPS_API int levo_latent_normalize_f32(const float *raw, const float *mean, const float *stddev,
                                           int64_t frames, int64_t dim, float *normalized, int32_t *status,
                                           levo_stream_t stream) {
    using namespace levo;
    clear_error();
    const char *w = "levo_latent_normalize_f32";
    int rc = check_common(w, raw, mean, stddev, frames, dim, normalized, true, status);
    if (rc != LEVO_OPS_OK) return rc;
    const int64_t n = frames * dim;
    const int64_t grid = std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(sm_count()) * 8);
    normalize_kernel<<<static_cast<unsigned>(grid), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        raw, mean, stddev, n, dim, normalized, status);
    return check_launch(w);
}

}  // extern "C"
