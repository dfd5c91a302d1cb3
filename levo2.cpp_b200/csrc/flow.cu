// Flow renderer CFG combine and Euler update (a7, a8).
//
// All arithmetic uses the _rn intrinsics in the reference's expression order,
// so results are bit-identical to the reference's host loops compiled without
// FMA contraction:
//   CFG:     u + g * (c - u)                  (src/levo-renderer-pattern.cpp:133,
//                                              src/levo-flow-renderer.cpp:307)
//   Euler:   x + dt * v, dt = 1 / steps       (src/levo-flow-renderer.cpp:90,105)
//   prefix:  ns * noise + t * context,
//            t = step * dt, ns = 1 - (1 - sigma_min) * t
//                                             (src/levo-flow-renderer.cpp:93-101)
// The reference's finiteness checks (src/levo-flow-renderer.cpp:104,106) become
// bits in an optional device status word.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace levo {
namespace {

constexpr int kThreads = 256;
constexpr int kStepChunk = 16;  // velocity steps prefetched per round (multi-step kernel)

__device__ __forceinline__ float cfg_mix(float u, float c, float g) {
    return __fadd_rn(u, __fmul_rn(g, __fsub_rn(c, u)));
}

__device__ __forceinline__ float step_dt(int64_t steps) {
    return __fdiv_rn(1.0f, static_cast<float>(steps));
}

__device__ __forceinline__ void prefix_times(int64_t step, float dt, float sigma_min, float &t,
                                             float &ns) {
    t = __fmul_rn(static_cast<float>(step), dt);
    ns = __fsub_rn(1.0f, __fmul_rn(__fsub_rn(1.0f, sigma_min), t));
}

__device__ __forceinline__ void flag_status(int32_t *status, int bits) {
    if (status && bits) atomicOr(status, bits);
}

struct CfgArgs {
    const float *u;
    const float *c;
    float *out;
    int64_t n;
    float g;
};

__global__ void __launch_bounds__(kThreads) cfg_combine_kernel(const CfgArgs a, int vec) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (vec) {
        const int64_t nvec = a.n / 8;
        for (int64_t i = tid; i < nvec; i += stride) {
            const f32x8 u = ld8(a.u + i * 8), c = ld8(a.c + i * 8);
            f32x8 o;
#pragma unroll
            for (int k = 0; k < 8; ++k) o.v[k] = cfg_mix(u.v[k], c.v[k], a.g);
            st8(a.out + i * 8, o);
        }
        done = nvec * 8;
    }
    for (int64_t i = done + tid; i < a.n; i += stride) a.out[i] = cfg_mix(a.u[i], a.c[i], a.g);
}

struct StepArgs {
    float *x;
    const float *u;
    const float *c;
    int64_t n;
    int cfg;
    float g;
    int64_t steps;
    int32_t *status;
};

__device__ __forceinline__ float euler_one(const StepArgs &a, float x, float u, float c, float dt,
                                           int &bits) {
    const float v = a.cfg ? cfg_mix(u, c, a.g) : u;
    if (!isfinite(v)) bits |= 1;
    const float nx = __fadd_rn(x, __fmul_rn(dt, v));
    if (!isfinite(nx)) bits |= 2;
    return nx;
}

__global__ void __launch_bounds__(kThreads) euler_step_kernel(const StepArgs a, int vec) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const float dt = step_dt(a.steps);
    int bits = 0;
    int64_t done = 0;
    if (vec) {
        const int64_t nvec = a.n / 8;
        for (int64_t i = tid; i < nvec; i += stride) {
            f32x8 x = ld8(a.x + i * 8);
            const f32x8 u = ld8(a.u + i * 8);
            f32x8 c{};
            if (a.cfg) c = ld8(a.c + i * 8);
#pragma unroll
            for (int k = 0; k < 8; ++k) x.v[k] = euler_one(a, x.v[k], u.v[k], c.v[k], dt, bits);
            st8(a.x + i * 8, x);
        }
        done = nvec * 8;
    }
    for (int64_t i = done + tid; i < a.n; i += stride)
        a.x[i] = euler_one(a, a.x[i], a.u[i], a.cfg ? a.c[i] : 0.f, dt, bits);
    flag_status(a.status, bits);
}

struct PrefixArgs {
    float *state;
    const float *noise;
    const float *ctx;
    int64_t batch, row, prefix;
    int64_t step, steps;
    float sigma_min;
};

__global__ void __launch_bounds__(kThreads) incontext_kernel(const PrefixArgs a) {
    const float dt = step_dt(a.steps);
    float t, ns;
    prefix_times(a.step, dt, a.sigma_min, t, ns);
    const int64_t total = a.batch * a.prefix;
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < total;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = k / a.prefix;
        const int64_t i = b * a.row + (k - b * a.prefix);
        a.state[i] = __fadd_rn(__fmul_rn(ns, a.noise[i]), __fmul_rn(t, a.ctx[i]));
    }
}

struct MultiArgs {
    float *state;
    const float *noise;
    const float *ctx;
    const float *u;  // [count][batch*row]
    const float *c;
    int64_t batch, row, prefix;
    int64_t first, count, steps;
    int cfg;
    float g, sigma_min;
    int32_t *status;
};

// One thread per state element; the steps run in order in registers while the
// velocities of the next kStepChunk steps are prefetched together.
__global__ void __launch_bounds__(kThreads) euler_multi_kernel(const MultiArgs a) {
    const int64_t n = a.batch * a.row;
    const float dt = step_dt(a.steps);
    int bits = 0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const bool in_prefix = (i % a.row) < a.prefix;
        float x = a.state[i];
        const float nz = in_prefix ? a.noise[i] : 0.f;
        const float cx = in_prefix ? a.ctx[i] : 0.f;
        for (int64_t k0 = 0; k0 < a.count; k0 += kStepChunk) {
            float uu[kStepChunk], cc[kStepChunk];
#pragma unroll
            for (int j = 0; j < kStepChunk; ++j) {
                if (k0 + j < a.count) {
                    uu[j] = a.u[(k0 + j) * n + i];
                    cc[j] = a.cfg ? a.c[(k0 + j) * n + i] : 0.f;
                }
            }
#pragma unroll
            for (int j = 0; j < kStepChunk; ++j) {
                if (k0 + j >= a.count) break;
                if (in_prefix) {
                    float t, ns;
                    prefix_times(a.first + k0 + j, dt, a.sigma_min, t, ns);
                    x = __fadd_rn(__fmul_rn(ns, nz), __fmul_rn(t, cx));
                }
                const float v = a.cfg ? cfg_mix(uu[j], cc[j], a.g) : uu[j];
                if (!isfinite(v)) bits |= 1;
                x = __fadd_rn(x, __fmul_rn(dt, v));
                if (!isfinite(x)) bits |= 2;
            }
        }
        if (in_prefix && a.first + a.count == a.steps) x = cx;
        a.state[i] = x;
    }
    flag_status(a.status, bits);
}

// Staged form: a CTA of kStagedThreads threads owns kStagedThreads consecutive
// elements; the velocities of up to kStagedSteps steps for them are copied into
// shared memory with cp.async in one burst (all of config 2's 13 MB is in
// flight at once), then each thread runs its steps from shared memory.
constexpr int kStagedThreads = 64;
constexpr int kStagedSteps = 64;

__global__ void __launch_bounds__(kStagedThreads) euler_multi_staged_kernel(const MultiArgs a) {
    extern __shared__ float4 stage[];  // [2][steps][kStagedThreads/4] float4
    const int64_t n = a.batch * a.row;
    const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kStagedThreads;
    const int64_t i = i0 + threadIdx.x;
    const bool active = i < n;
    const int per_step = kStagedThreads / 4;  // float4 chunks per step and array
    const float dt = step_dt(a.steps);
    int bits = 0;
    const bool in_prefix = active && (i % a.row) < a.prefix;
    float x = active ? a.state[i] : 0.f;
    const float nz = in_prefix ? a.noise[i] : 0.f;
    const float cx = in_prefix ? a.ctx[i] : 0.f;
    const int64_t full = (n - i0) >= kStagedThreads ? per_step : (n - i0 + 3) / 4;
    for (int64_t k0 = 0; k0 < a.count; k0 += kStagedSteps) {
        const int cnt = static_cast<int>(a.count - k0 < kStagedSteps ? a.count - k0 : kStagedSteps);
        __syncthreads();  // the previous chunk has been consumed
        // Thread t copies chunk (t % per_step) of steps t / per_step, + kGroups, ...
        // for both arrays: no division inside the loop.
        {
            constexpr int kGroups = kStagedThreads / (kStagedThreads / 4);  // step rows copied per pass
            const int ch = threadIdx.x % per_step;
            const int st0 = threadIdx.x / per_step;
            if (ch < full) {
                const float *ub = a.u + (k0 + st0) * n + i0 + ch * 4;
                const float *cb = a.cfg ? a.c + (k0 + st0) * n + i0 + ch * 4 : nullptr;
                for (int st = st0; st < cnt; st += kGroups) {
                    cp_async16(stage + st * per_step + ch, ub);
                    if (a.cfg) cp_async16(stage + (kStagedSteps + st) * per_step + ch, cb);
                    ub += kGroups * n;
                    if (a.cfg) cb += kGroups * n;
                }
            }
        }
        cp_async_wait_all();
        __syncthreads();
        if (active) {
            const float *su = reinterpret_cast<const float *>(stage);
            const float *sc = su + kStagedSteps * kStagedThreads;
#pragma unroll 10
            for (int j = 0; j < cnt; ++j) {
                if (in_prefix) {
                    float t, ns;
                    prefix_times(a.first + k0 + j, dt, a.sigma_min, t, ns);
                    x = __fadd_rn(__fmul_rn(ns, nz), __fmul_rn(t, cx));
                }
                const float u = su[j * kStagedThreads + threadIdx.x];
                const float v = a.cfg ? cfg_mix(u, sc[j * kStagedThreads + threadIdx.x], a.g) : u;
                if (!isfinite(v)) bits |= 1;
                x = __fadd_rn(x, __fmul_rn(dt, v));
                if (!isfinite(x)) bits |= 2;
            }
        }
    }
    if (active) {
        if (in_prefix && a.first + a.count == a.steps) x = cx;
        a.state[i] = x;
    }
    flag_status(a.status, bits);
}

int64_t grid_for(int64_t items) {
    return std::max<int64_t>(
        1, std::min<int64_t>((items + kThreads - 1) / kThreads, static_cast<int64_t>(sm_count()) * 16));
}

}  // namespace
}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_cfg_combine_f32(const float *uncond, const float *cond, float *out, int64_t n,
                                      float guidance, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    if (uncond == nullptr || cond == nullptr || out == nullptr)
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_combine_f32: required pointer is null");
    if (n <= 0)
        return set_error(LEVO_OPS_EINVAL,
                         "levo_cfg_combine_f32: CFG vectors must have equal non-empty lengths");
    if (!std::isfinite(guidance))
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_combine_f32: CFG guidance scale must be finite");
    if (!aligned_to(uncond, 4) || !aligned_to(cond, 4) || !aligned_to(out, 4))
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_combine_f32: pointer is not 4-byte aligned");
    const int vec = aligned_to(uncond, 32) && aligned_to(cond, 32) && aligned_to(out, 32);
    const CfgArgs a{uncond, cond, out, n, guidance};
    cfg_combine_kernel<<<static_cast<unsigned>(grid_for(vec ? n / 8 + 8 : n)), kThreads, 0,
                         reinterpret_cast<cudaStream_t>(stream)>>>(a, vec);
    return check_launch("levo_cfg_combine_f32");
}

LEVO_OPS_API int levo_flow_incontext_f32(float *state, const float *noise, const float *context,
                                         int64_t batch, int64_t row, int64_t prefix, int64_t step,
                                         int64_t steps, float sigma_min, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    if (state == nullptr || noise == nullptr || context == nullptr)
        return set_error(LEVO_OPS_EINVAL, "levo_flow_incontext_f32: required pointer is null");
    if (batch <= 0 || row <= 0)
        return set_error(LEVO_OPS_EINVAL, "levo_flow_incontext_f32: Euler state dimensions must be positive");
    if (prefix < 0 || prefix > row)
        return set_error(LEVO_OPS_EINVAL,
                         "levo_flow_incontext_f32: Euler in-context length exceeds frame count");
    if (steps <= 0 || step < 0 || step >= steps)
        return set_error(LEVO_OPS_EINVAL, "levo_flow_incontext_f32: step outside [0, steps)");
    if (!std::isfinite(sigma_min) || sigma_min <= 0.f)
        return set_error(LEVO_OPS_EINVAL,
                         "levo_flow_incontext_f32: Euler sigma_min must be finite and positive");
    if (prefix == 0) return LEVO_OPS_OK;
    const PrefixArgs a{state, noise, context, batch, row, prefix, step, steps, sigma_min};
    incontext_kernel<<<static_cast<unsigned>(grid_for(batch * prefix)), kThreads, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(a);
    return check_launch("levo_flow_incontext_f32");
}

LEVO_OPS_API int levo_euler_cfg_step_f32(float *state, const float *uncond, const float *cond,
                                         int64_t n, int32_t cfg, float guidance, int64_t steps,
                                         int32_t *status, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    if (state == nullptr || uncond == nullptr || (cfg && cond == nullptr))
        return set_error(LEVO_OPS_EINVAL, "levo_euler_cfg_step_f32: required pointer is null");
    if (n <= 0)
        return set_error(LEVO_OPS_EINVAL, "levo_euler_cfg_step_f32: Euler state dimensions must be positive");
    if (steps <= 0)
        return set_error(LEVO_OPS_EINVAL, "levo_euler_cfg_step_f32: Euler step count must be positive");
    if (cfg && !std::isfinite(guidance))
        return set_error(LEVO_OPS_EINVAL, "levo_euler_cfg_step_f32: CFG guidance scale must be finite");
    const void *ptrs[4] = {state, uncond, cond, status};
    for (const void *p : ptrs)
        if (p && !aligned_to(p, 4))
            return set_error(LEVO_OPS_EINVAL, "levo_euler_cfg_step_f32: pointer is not 4-byte aligned");
    const int vec = aligned_to(state, 32) && aligned_to(uncond, 32) && (!cfg || aligned_to(cond, 32));
    const StepArgs a{state, uncond, cond, n, cfg ? 1 : 0, guidance, steps, status};
    euler_step_kernel<<<static_cast<unsigned>(grid_for(vec ? n / 8 + 8 : n)), kThreads, 0,
                        reinterpret_cast<cudaStream_t>(stream)>>>(a, vec);
    return check_launch("levo_euler_cfg_step_f32");
}

LEVO_OPS_API int levo_cfg_euler_multi_f32(float *state, const float *noise, const float *context,
                                          const float *uncond, const float *cond, int64_t batch,
                                          int64_t row, int64_t prefix, int64_t first_step,
                                          int64_t count, int64_t steps, int32_t cfg,
                                          float guidance, float sigma_min, int32_t *status,
                                          levo_stream_t stream) {
    using namespace levo;
    clear_error();
    if (state == nullptr || (count > 0 && (uncond == nullptr || (cfg && cond == nullptr))))
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_euler_multi_f32: required pointer is null");
    if (prefix > 0 && (noise == nullptr || context == nullptr))
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_euler_multi_f32: in-context tensors are null");
    if (batch <= 0 || row <= 0)
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_euler_multi_f32: Euler state dimensions must be positive");
    if (steps <= 0)
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_euler_multi_f32: Euler step count must be positive");
    if (prefix < 0 || prefix > row)
        return set_error(LEVO_OPS_EINVAL,
                         "levo_cfg_euler_multi_f32: Euler in-context length exceeds frame count");
    if (first_step < 0 || count < 0 || first_step > steps || count > steps - first_step)
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_euler_multi_f32: Euler resume step exceeds total steps");
    if (!std::isfinite(sigma_min) || sigma_min <= 0.f)
        return set_error(LEVO_OPS_EINVAL,
                         "levo_cfg_euler_multi_f32: Euler sigma_min must be finite and positive");
    if (cfg && !std::isfinite(guidance))
        return set_error(LEVO_OPS_EINVAL, "levo_cfg_euler_multi_f32: CFG guidance scale must be finite");
    const void *ptrs[6] = {state, noise, context, uncond, cond, status};
    for (const void *p : ptrs)
        if (p && !aligned_to(p, 4))
            return set_error(LEVO_OPS_EINVAL, "levo_cfg_euler_multi_f32: pointer is not 4-byte aligned");
    const MultiArgs a{state, noise, context, uncond, cond, batch, row, prefix, first_step,
                      count, steps, cfg ? 1 : 0, guidance, sigma_min, status};
    const int64_t n = batch * row;
    // one staged CTA per kStagedThreads elements: the grid must fit in 2^31 - 1 blocks
    const bool staged = count > 0 && n % 4 == 0 && aligned_to(uncond, 16) && (!cfg || aligned_to(cond, 16)) &&
                        (n + kStagedThreads - 1) / kStagedThreads <= 0x7fffffff;
    if (staged) {
        // [2][kStagedSteps][kStagedThreads] F32 = 32 KB of shared memory
        const size_t smem = 2 * kStagedSteps * kStagedThreads * sizeof(float);
        euler_multi_staged_kernel<<<static_cast<unsigned>((n + kStagedThreads - 1) / kStagedThreads),
                                    kStagedThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    } else {
        euler_multi_kernel<<<static_cast<unsigned>(grid_for(n)), kThreads, 0,
                             reinterpret_cast<cudaStream_t>(stream)>>>(a);
    }
    return check_launch("levo_cfg_euler_multi_f32");
}

}  // extern "C"
