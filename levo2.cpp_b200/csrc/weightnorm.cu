// Weight-norm fold (a9): w[o][:] = v[o][:] * (g[o] / ||v[o][:]||).
//
// One CTA per row, one HBM read of v and one write of w (8 B per element):
//  * rows up to kMaxStagedCols values are copied into shared memory with
//    cp.async (a 1024 x 7168 weight: 28 KB per CTA, 7 CTAs per SM, the whole
//    tensor in flight in one wave), reduced from there and scaled out, in
//    passes unrolled over a compile-time chunk count per thread;
//  * longer rows up to 16384 values stay in registers, longer still are
//    streamed twice (the second read mostly hits L2).  The arithmetic follows the reference's numpy
// expression (convert/convert_vae.py:196-199): norm = sqrt(sum(v*v)) in F32,
// scale = g / norm, w = v * scale.
#include <algorithm>

#include "common.cuh"

namespace levo {
namespace {

struct WnArgs {
    const float *v;
    const float *g;
    float *w;
    float *norms;
    int64_t rows;
    int64_t cols;
};

__device__ __forceinline__ float block_sum(float s, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncthreads();  // red is reused across rows
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float t = 0.f;
    const int warps = blockDim.x >> 5;
    for (int w = 0; w < warps; ++w) t += red[w];
    return t;
}

// gain = g[row], loaded by the caller before the row's reduction: a load after
// block_sum's barrier could not be moved above it and would add one memory
// round trip between the reduction and the stores of every row.
__device__ __forceinline__ float row_scale(const WnArgs &a, int64_t row, float gain, float sumsq) {
    const float norm = __fsqrt_rn(sumsq);
    if (a.norms && threadIdx.x == 0) a.norms[row] = norm;
    return __fdiv_rn(gain, norm);
}

// VPT > 0: the row is register resident (VPT 8-float vectors per thread).
// VPT == 0: the row is streamed twice.
template <int VPT>
__global__ void __launch_bounds__(256) weightnorm_vec_kernel(const WnArgs a) {
    __shared__ float red[32];
    const int64_t nvec = a.cols / 8;
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const float gain = a.g[row];
        const float *vr = a.v + row * a.cols;
        float *wr = a.w + row * a.cols;
        if constexpr (VPT > 0) {
            f32x8 buf[VPT];
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int64_t vi = k * static_cast<int64_t>(blockDim.x) + threadIdx.x;
                if (vi < nvec) buf[k] = ld8(vr + vi * 8);
            }
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int64_t vi = k * static_cast<int64_t>(blockDim.x) + threadIdx.x;
                if (vi < nvec) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) s = fmaf(buf[k].v[j], buf[k].v[j], s);
                }
            }
            const float scale = row_scale(a, row, gain, block_sum(s, red));
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
                const int64_t vi = k * static_cast<int64_t>(blockDim.x) + threadIdx.x;
                if (vi < nvec) {
                    f32x8 o;
#pragma unroll
                    for (int j = 0; j < 8; ++j) o.v[j] = __fmul_rn(buf[k].v[j], scale);
                    st8(wr + vi * 8, o);
                }
            }
        } else {
            float s = 0.f;
            for (int64_t vi = threadIdx.x; vi < nvec; vi += blockDim.x) {
                const f32x8 b = ld8(vr + vi * 8);
#pragma unroll
                for (int j = 0; j < 8; ++j) s = fmaf(b.v[j], b.v[j], s);
            }
            const float scale = row_scale(a, row, gain, block_sum(s, red));
            for (int64_t vi = threadIdx.x; vi < nvec; vi += blockDim.x) {
                f32x8 b = ld8(vr + vi * 8);
#pragma unroll
                for (int j = 0; j < 8; ++j) b.v[j] = __fmul_rn(b.v[j], scale);
                st8(wr + vi * 8, b);
            }
        }
    }
}

constexpr int64_t kMaxStagedCols = 12032;  // <= 48 KB of shared memory per CTA with red[]
constexpr int kStagedThreads = 128;
constexpr int kStagedMaxCpt = (kMaxStagedCols / 4 + kStagedThreads - 1) / kStagedThreads;  // 24

constexpr int kStagedRowsPerCta = 2;  // rows per CTA a launch aims for (the next row's copy overlaps)

// CPT: 16-byte chunks per thread (compile time).  The row is copied into shared
// memory with cp.async, then read into registers in one unrolled burst; as
// soon as every thread holds its chunks the buffer takes the CTA's next row's
// copies, which overlap this row's reduction and output.  The grid aims at
// about kStagedRowsPerCta rows per CTA in whole CTAs per SM.
template <int CPT>
__global__ void __launch_bounds__(kStagedThreads, 4) weightnorm_staged_kernel(const WnArgs a) {
    extern __shared__ float4 row_buf[];
    __shared__ float red[32];
    const int nchunk = static_cast<int>(a.cols / 4);
    const int t = threadIdx.x;
    auto issue = [&](int64_t row) {
        const float4 *vr = reinterpret_cast<const float4 *>(a.v + row * a.cols);
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int i = t + kStagedThreads * k;
            if (i < nchunk) cp_async16(row_buf + i, vr + i);
        }
    };
    int64_t row = blockIdx.x;
    if (row < a.rows) issue(row);
    cp_async_commit();
    for (; row < a.rows; row += gridDim.x) {
        const float gain = a.g[row];
        cp_async_wait_group<0>();
        __syncthreads();  // the row is in shared memory
        float4 b[CPT];
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int i = t + kStagedThreads * k;
            if (i < nchunk) b[k] = row_buf[i];
        }
        __syncthreads();  // every thread holds its chunks: the buffer takes the next row
        const int64_t next = row + gridDim.x;
        if (next < a.rows) issue(next);
        cp_async_commit();
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            if (t + kStagedThreads * k < nchunk) {
                s = fmaf(b[k].x, b[k].x, s);
                s = fmaf(b[k].y, b[k].y, s);
                s = fmaf(b[k].z, b[k].z, s);
                s = fmaf(b[k].w, b[k].w, s);
            }
        }
        const float scale = row_scale(a, row, gain, block_sum(s, red));
        float4 *wr = reinterpret_cast<float4 *>(a.w + row * a.cols);
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int i = t + kStagedThreads * k;
            if (i < nchunk)
                wr[i] = make_float4(__fmul_rn(b[k].x, scale), __fmul_rn(b[k].y, scale), __fmul_rn(b[k].z, scale),
                                    __fmul_rn(b[k].w, scale));
        }
    }
    cp_async_wait_group<0>();  // nothing of this thread's is left in flight at exit
}

template <int CPT>
void run_staged(const WnArgs &a, cudaStream_t stream) {
    auto kernel = weightnorm_staged_kernel<CPT>;
    const size_t smem = static_cast<size_t>(a.cols) * sizeof(float);
    int resident = 0;
    if (resident_ctas(reinterpret_cast<const void *>(kernel), kStagedThreads, smem, &resident) != cudaSuccess ||
        resident <= 0) {
        cudaGetLastError();
        resident = 1;
    }
    const int64_t sms = sm_count();
    int64_t per_sm = (a.rows + sms * kStagedRowsPerCta - 1) / (sms * kStagedRowsPerCta);
    per_sm = std::min<int64_t>(std::max<int64_t>(per_sm, 1), resident);
    const int64_t grid = std::min<int64_t>(a.rows, sms * per_sm);
    kernel<<<static_cast<unsigned>(grid), kStagedThreads, smem, stream>>>(a);
}

// The smallest instantiated chunk count that covers the row (cpt <= kStagedMaxCpt).
void launch_staged(const WnArgs &a, int cpt, cudaStream_t stream) {
    if (cpt <= 1) return run_staged<1>(a, stream);
    if (cpt <= 2) return run_staged<2>(a, stream);
    if (cpt <= 4) return run_staged<4>(a, stream);
    if (cpt <= 6) return run_staged<6>(a, stream);
    if (cpt <= 8) return run_staged<8>(a, stream);
    if (cpt <= 12) return run_staged<12>(a, stream);
    if (cpt <= 14) return run_staged<14>(a, stream);
    if (cpt <= 16) return run_staged<16>(a, stream);
    return run_staged<kStagedMaxCpt>(a, stream);
}

// Any row length / alignment.
__global__ void __launch_bounds__(256) weightnorm_scalar_kernel(const WnArgs a) {
    __shared__ float red[32];
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const float gain = a.g[row];
        const float *vr = a.v + row * a.cols;
        float *wr = a.w + row * a.cols;
        float s = 0.f;
        for (int64_t j = threadIdx.x; j < a.cols; j += blockDim.x) s = fmaf(vr[j], vr[j], s);
        const float scale = row_scale(a, row, gain, block_sum(s, red));
        for (int64_t j = threadIdx.x; j < a.cols; j += blockDim.x) wr[j] = __fmul_rn(vr[j], scale);
    }
}

template <int VPT>
void launch_wn(const WnArgs &a, int threads, cudaStream_t stream) {
    const int64_t grid = std::min<int64_t>(a.rows, static_cast<int64_t>(sm_count()) * 64);
    weightnorm_vec_kernel<VPT><<<static_cast<unsigned>(grid), threads, 0, stream>>>(a);
}

}  // namespace
}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_weightnorm_f32(const float *v, const float *g, float *w, float *norms_out,
                                     int64_t rows, int64_t cols, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    if (rows < 0 || cols < 0) return set_error(LEVO_OPS_EINVAL, "levo_weightnorm_f32: negative shape");
    if (rows == 0 || cols == 0) return LEVO_OPS_OK;  // empty: nothing to read or write
    if (v == nullptr || g == nullptr || w == nullptr)
        return set_error(LEVO_OPS_EINVAL, "levo_weightnorm_f32: required pointer is null");
    const void *ptrs[4] = {v, g, w, norms_out};
    for (const void *p : ptrs)
        if (p && !aligned_to(p, 4))
            return set_error(LEVO_OPS_EINVAL, "levo_weightnorm_f32: pointer is not 4-byte aligned");
    const WnArgs a{v, g, w, norms_out, rows, cols};
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const bool vec = cols % 8 == 0 && aligned_to(v, 32) && aligned_to(w, 32);
    const bool staged = cols <= kMaxStagedCols && cols % 4 == 0 && aligned_to(v, 16) && aligned_to(w, 16);
    if (!vec && !staged) {
        const int64_t grid = std::min<int64_t>(rows, static_cast<int64_t>(sm_count()) * 64);
        weightnorm_scalar_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(a);
        return check_launch("levo_weightnorm_f32");
    }
    if (staged) {
        launch_staged(a, static_cast<int>((cols / 4 + kStagedThreads - 1) / kStagedThreads), s);
        return check_launch("levo_weightnorm_f32");
    }
    const int64_t nvec = cols / 8;
    // Register-resident rows: 128 threads while the row fits in 8 vectors per
    // thread, then 256 threads, then the streamed form.
    const int threads = nvec <= 128 * 8 ? 128 : 256;
    const int64_t vpt = (nvec + threads - 1) / threads;
    switch (vpt) {
        case 1: launch_wn<1>(a, threads, s); break;
        case 2: launch_wn<2>(a, threads, s); break;
        case 3: launch_wn<3>(a, threads, s); break;
        case 4: launch_wn<4>(a, threads, s); break;
        case 5: launch_wn<5>(a, threads, s); break;
        case 6: launch_wn<6>(a, threads, s); break;
        case 7: launch_wn<7>(a, threads, s); break;
        case 8: launch_wn<8>(a, threads, s); break;
        default: launch_wn<0>(a, 256, s); break;
    }
    return check_launch("levo_weightnorm_f32");
}

}  // extern "C"
