// Greedy next-token selection over LeLM logits (next item f3).
//
// Reference: Sampler::sample_streams with use_sampling = false
// (src/levo-sampling.cpp:129-152 -> sample_top_k_counted, :75-97):
//   1. every distinct recent token id in [0, limit) divides its logit once by
//      the repetition penalty (apply_unique_token_repetition_penalty, :39-48);
//   2. on the first stream only, ignored token ids become -inf (:146-148);
//   3. the result is the index of the FIRST maximum (std::max_element, :93-95);
//      top-k filtering never removes the maximum, so greedy selection does not
//      depend on it.  A NaN logit is an error in the reference (:81); here it
//      sets bit 0 (value 1) of the optional status word.
// One CTA per stream row: the recent / ignored ids are marked in shared-memory
// bitmaps, the row is scanned once (a scalar head up to its 16-byte boundary,
// then float4 groups whose loads go out ahead of the comparisons), and
// (value, index) pairs are reduced with a first-index tie break, a total order,
// so the result is exact whatever the order of the comparisons.
#include <algorithm>

#include "common.cuh"

namespace levo {
namespace {

constexpr int kThreads = 512;
constexpr int64_t kMaxVocab = int64_t(1) << 17;  // two 16 KB bitmaps (within 48 KB of shared memory)

struct GreedyArgs {
    const float *logits;
    int64_t rows, vocab, ld;
    const int64_t *recent;
    int64_t recent_len;
    float penalty;
    int64_t limit;
    const int64_t *ignore;
    int64_t n_ignore;
    int64_t *out;
    int32_t *status;
    int vec;  // float4 scan after a scalar head to each row's 16-byte boundary
};

// a beats b: larger value, or equal value at a smaller index.
__device__ __forceinline__ bool better(float va, int64_t ia, float vb, int64_t ib) {
    return va > vb || (va == vb && ia < ib);
}

__global__ void __launch_bounds__(kThreads, 2) greedy_kernel(const GreedyArgs a) {
    extern __shared__ uint32_t bits[];  // [pen words][ign words]
    __shared__ float red_v[kThreads / 32];
    __shared__ int64_t red_i[kThreads / 32];
    __shared__ int red_nan;
    const int64_t words = (a.vocab + 31) / 32;
    uint32_t *pen = bits;
    uint32_t *ign = bits + words;
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        __syncthreads();  // shared state of the previous row is consumed
        for (int64_t w = threadIdx.x; w < 2 * words; w += blockDim.x) bits[w] = 0u;
        if (threadIdx.x == 0) red_nan = 0;
        __syncthreads();
        if (a.recent) {
            for (int64_t k = threadIdx.x; k < a.recent_len; k += blockDim.x) {
                const int64_t t = a.recent[row * a.recent_len + k];
                if (t >= 0 && t < a.limit) atomicOr(&pen[t >> 5], 1u << (t & 31));
            }
        }
        if (row == 0 && a.ignore) {
            for (int64_t k = threadIdx.x; k < a.n_ignore; k += blockDim.x) {
                const int64_t t = a.ignore[k];
                if (t >= 0 && t < a.vocab) atomicOr(&ign[t >> 5], 1u << (t & 31));
            }
        }
        __syncthreads();
        const float *x = a.logits + row * a.ld;
        float best = -INFINITY;
        int64_t bidx = INT64_MAX;
        bool nan = false;
        // one logit: penalty, ignore list, NaN flag, then the (value, smaller index) order
        auto consider = [&](float v, int64_t i, uint32_t pbit, uint32_t ibit) {
            if (pbit) v = __fdiv_rn(v, a.penalty);
            if (ibit) v = -INFINITY;
            if (isnan(v)) {
                nan = true;
                return;
            }
            if (better(v, i, best, bidx)) {
                best = v;
                bidx = i;
            }
        };
        int64_t i0 = 0;  // first logit of the scalar tail
        if (a.vec) {
            // A scalar head up to the row's first 16-byte boundary, then four logits per float4 whose
            // bitmap bits come from one 64-bit window of two words; the loads of a thread's groups go
            // out before the comparisons.
            const int64_t head = (4 - static_cast<int64_t>((reinterpret_cast<uintptr_t>(x) >> 2) & 3)) & 3;
            if (threadIdx.x < head && threadIdx.x < a.vocab) {
                const int64_t i = threadIdx.x;
                const uint32_t m = 1u << (i & 31);
                consider(x[i], i, pen[i >> 5] & m, ign[i >> 5] & m);
            }
            const int nv = static_cast<int>((a.vocab - head) / 4);
            const float4 *x4 = reinterpret_cast<const float4 *>(x + head);
            constexpr int kAhead = 4;
            for (int g0 = threadIdx.x; g0 < nv; g0 += kAhead * kThreads) {
                float4 q[kAhead];
#pragma unroll
                for (int j = 0; j < kAhead; ++j)
                    if (g0 + j * kThreads < nv) q[j] = x4[g0 + j * kThreads];
#pragma unroll
                for (int j = 0; j < kAhead; ++j) {
                    const int g = g0 + j * kThreads;
                    if (g >= nv) break;
                    const int64_t i = head + 4 * static_cast<int64_t>(g);
                    const int64_t w = i >> 5;
                    const int sh = static_cast<int>(i & 31);
                    const bool two = w + 1 < words;
                    const uint32_t pw = static_cast<uint32_t>(
                        ((static_cast<uint64_t>(two ? pen[w + 1] : 0u) << 32) | pen[w]) >> sh);
                    const uint32_t iw = static_cast<uint32_t>(
                        ((static_cast<uint64_t>(two ? ign[w + 1] : 0u) << 32) | ign[w]) >> sh);
                    consider(q[j].x, i, pw & 1u, iw & 1u);
                    consider(q[j].y, i + 1, pw & 2u, iw & 2u);
                    consider(q[j].z, i + 2, pw & 4u, iw & 4u);
                    consider(q[j].w, i + 3, pw & 8u, iw & 8u);
                }
            }
            i0 = head + 4 * static_cast<int64_t>(nv);
        }
        for (int64_t i = i0 + threadIdx.x; i < a.vocab; i += blockDim.x) {
            const uint32_t m = 1u << (i & 31);
            consider(x[i], i, pen[i >> 5] & m, ign[i >> 5] & m);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, bidx, o);
            if (better(ov, oi, best, bidx)) {
                best = ov;
                bidx = oi;
            }
        }
        if (nan) red_nan = 1;
        if ((threadIdx.x & 31) == 0) {
            red_v[threadIdx.x >> 5] = best;
            red_i[threadIdx.x >> 5] = bidx;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float bv = red_v[0];
            int64_t bi = red_i[0];
            for (int w = 1; w < kThreads / 32; ++w)
                if (better(red_v[w], red_i[w], bv, bi)) {
                    bv = red_v[w];
                    bi = red_i[w];
                }
            a.out[row] = bi == INT64_MAX ? 0 : bi;  // every logit NaN: index 0, status set
            if (red_nan && a.status) atomicOr(a.status, 1);
        }
    }
}

}  // namespace
}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_greedy_tokens_f32(const float *logits, int64_t rows, int64_t vocab, int64_t ld,
                                        const int64_t *recent, int64_t recent_len, float penalty,
                                        int64_t penalty_limit, const int64_t *ignore, int64_t n_ignore,
                                        int64_t *tokens_out, int32_t *status, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    const char *w = "levo_greedy_tokens_f32";
    if (rows < 0 || vocab < 0 || recent_len < 0 || n_ignore < 0)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": negative size");
    if (rows == 0) return LEVO_OPS_OK;
    if (vocab == 0) return set_error(LEVO_OPS_EINVAL, std::string(w) + ": cannot sample an empty vocabulary");
    if (vocab > kMaxVocab) return set_error(LEVO_OPS_EUNSUPPORTED, std::string(w) + ": vocabulary above 131072");
    if (ld < vocab) return set_error(LEVO_OPS_EINVAL, std::string(w) + ": row stride smaller than the vocabulary");
    if (logits == nullptr || tokens_out == nullptr)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": required pointer is null");
    if (recent != nullptr && recent_len > 0 && (!(penalty > 0.0f) || !std::isfinite(penalty)))
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": repetition penalty must be finite and positive");
    if ((n_ignore > 0 && ignore == nullptr))
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": ignore list is null");
    const void *ptrs[5] = {logits, recent, ignore, tokens_out, status};
    const size_t align[5] = {4, 8, 8, 8, 4};
    for (int i = 0; i < 5; ++i)
        if (ptrs[i] && !aligned_to(ptrs[i], align[i]))
            return set_error(LEVO_OPS_EINVAL, std::string(w) + ": pointer is not aligned to its element size");
    const int64_t limit = penalty_limit <= 0 ? vocab : std::min(penalty_limit, vocab);
    const int vec = aligned_to(logits, 4) ? 1 : 0;  // each row finds its own 16-byte boundary
    const GreedyArgs a{logits, rows, vocab, ld, recent_len > 0 ? recent : nullptr, recent_len, penalty, limit,
                       n_ignore > 0 ? ignore : nullptr, n_ignore, tokens_out, status, vec};
    const size_t smem = static_cast<size_t>(2 * ((vocab + 31) / 32)) * sizeof(uint32_t);
    const int64_t grid = std::min<int64_t>(rows, static_cast<int64_t>(sm_count()) * 4);
    greedy_kernel<<<static_cast<unsigned>(grid), kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    return check_launch(w);
}

}  // extern "C"
