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
// an optional device status word.  The per-step kernel ORs the failure kinds
// into it; the multi-step kernels record the first failing step (the one the
// reference throws at) with atomicMax on LEVO_EULER_STATUS(step, kind), and an
// element stops updating at its first failure, keeping its state after the
// last step it completed.
#include <algorithm>
#include <cmath>
#include <string>

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

// Whether element i of a [batch][row] state lies in its row's in-context prefix.  No
// division at all without a prefix, a 32-bit one when the indices fit (a 64-bit
// remainder is a long instruction sequence).
__device__ __forceinline__ bool in_context_prefix(int64_t i, int64_t row, int64_t prefix) {
    if (prefix <= 0) return false;
    if (i <= INT32_MAX && row <= INT32_MAX)
        return static_cast<int64_t>(static_cast<uint32_t>(i) % static_cast<uint32_t>(row)) < prefix;
    return (i % row) < prefix;
}

__device__ __forceinline__ void flag_status(int32_t *status, int bits) {
    if (status && bits) atomicOr(status, bits);
}

// The earliest failing step wins; on a tie the velocity kind (3 > 2), which the
// reference checks before the state.
__device__ __forceinline__ void record_failure(int32_t *status, int64_t step, int kind) {
    if (status) atomicMax(status, static_cast<int32_t>(LEVO_EULER_STATUS(step, kind)));
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
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const bool in_prefix = in_context_prefix(i, a.row, a.prefix);
        float x = a.state[i];
        const float nz = in_prefix ? a.noise[i] : 0.f;
        const float cx = in_prefix ? a.ctx[i] : 0.f;
        bool failed = false;
        for (int64_t k0 = 0; k0 < a.count && !failed; k0 += kStepChunk) {
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
                const int64_t step = a.first + k0 + j;
                float xs = x;
                if (in_prefix) {
                    float t, ns;
                    prefix_times(step, dt, a.sigma_min, t, ns);
                    xs = __fadd_rn(__fmul_rn(ns, nz), __fmul_rn(t, cx));
                }
                const float v = a.cfg ? cfg_mix(uu[j], cc[j], a.g) : uu[j];
                if (!isfinite(v)) {
                    record_failure(a.status, step, 3);
                    failed = true;
                    break;
                }
                const float nx = __fadd_rn(xs, __fmul_rn(dt, v));
                if (!isfinite(nx)) {
                    record_failure(a.status, step, 2);
                    failed = true;
                    break;
                }
                x = nx;
            }
        }
        if (!failed && in_prefix && a.first + a.count == a.steps) x = cx;
        a.state[i] = x;
    }
}

// Staged form.  A CTA owns kStagedElems consecutive elements; its 256 threads
// copy the velocities of up to kStagedSteps steps for them into shared memory
// with cp.async in one burst (all of config 2's 13 MB is in flight at once).
// Then, per round:
//   velocity phase: four threads per element (steps q, q + 4, ...) form the CFG
//     combine and replace u by dt * v in place (the reference rounds dt * v
//     before adding it, so x + w is its x + dt * v bit for bit);
//   chain phase: one thread per element runs the dependent x = x + w (after
//     the in-context interpolation for prefix elements).
// No step is checked on the way.  dt = 1 / steps lies in (0, 1], so w is
// non-finite exactly when v is, and outside the prefix a state that turned
// non-finite (through w or an overflow) stays so: the chain checks x once at
// the end of the round and, only when it failed, replays the round from its
// start with the reference's per-step checks, velocity first, to find the
// step and the kind.  Prefix elements, re-interpolated every step, always
// take the checked replay.
constexpr int kStagedElems = 64;
constexpr int kStagedLanes = 4;
constexpr int kStagedThreads = kStagedElems * kStagedLanes;
constexpr int kStagedSteps = 64;

__global__ void __launch_bounds__(kStagedThreads) euler_multi_staged_kernel(const MultiArgs a) {
    extern __shared__ float4 stage[];  // [2][kStagedSteps][kStagedElems] F32: u (then dt * v), c
    float *su = reinterpret_cast<float *>(stage);
    float *sc = su + kStagedSteps * kStagedElems;
    const int64_t n = a.batch * a.row;
    const int64_t i0 = static_cast<int64_t>(blockIdx.x) * kStagedElems;
    const int tid = threadIdx.x;
    const int e = tid % kStagedElems;  // element of the velocity phase
    const int q = tid / kStagedElems;  // its step lane
    const int64_t i = i0 + tid;        // element of the chain phase (threads < kStagedElems)
    const bool active = tid < kStagedElems && i < n;
    // n % 4 == 0 (launcher), so this CTA's elements are whole 16-byte chunks
    const int valid = static_cast<int>(n - i0 < kStagedElems ? n - i0 : kStagedElems);
    const int chunks_valid = valid / 4;
    constexpr int kChunksPerStep = kStagedElems / 4;
    const float dt = step_dt(a.steps);
    const bool in_prefix = active && in_context_prefix(i, a.row, a.prefix);
    float x = 0.f, nz = 0.f, cx = 0.f;
    bool failed = false;
    for (int64_t k0 = 0; k0 < a.count; k0 += kStagedSteps) {
        const int cnt = static_cast<int>(a.count - k0 < kStagedSteps ? a.count - k0 : kStagedSteps);
        if (k0 > 0) __syncthreads();  // the previous round has been consumed
        // the copies go out first: nothing else stands between the launch and the DRAM requests.
        // Thread t copies chunk t % 16 of step rows t / 16, + 16, ... of both arrays (no division
        // inside the loop).
        {
            constexpr int kRowsPerPass = kStagedThreads / kChunksPerStep;
            const int ch = tid % kChunksPerStep;
            if (ch < chunks_valid) {
                const int64_t col = i0 + ch * 4;
                const float *bu = a.u + k0 * n + col;
                const float *bc = a.cfg ? a.c + k0 * n + col : nullptr;
                for (int st = tid / kChunksPerStep; st < cnt; st += kRowsPerPass) {
                    cp_async16(su + st * kStagedElems + ch * 4, bu + st * n);
                    if (a.cfg) cp_async16(sc + st * kStagedElems + ch * 4, bc + st * n);
                }
            }
        }
        if (k0 == 0 && active) {
            x = a.state[i];
            if (in_prefix) {
                nz = a.noise[i];
                cx = a.ctx[i];
            }
        }
        cp_async_wait_all();
        __syncthreads();
        if (e < valid) {
            for (int st = q; st < cnt; st += kStagedLanes) {
                const float u = su[st * kStagedElems + e];
                const float v = a.cfg ? cfg_mix(u, sc[st * kStagedElems + e], a.g) : u;
                su[st * kStagedElems + e] = __fmul_rn(dt, v);
            }
        }
        __syncthreads();
        if (active && !failed) {
            const float x0 = x;
            if (!in_prefix) {
#pragma unroll 8
                for (int st = 0; st < cnt; ++st) x = __fadd_rn(x, su[st * kStagedElems + tid]);
            }
            // Rare path: the round replayed from x0 with the reference's per-step checks.  With
            // 0 < dt <= 1, w = dt * v is non-finite exactly when v is, so a non-finite velocity
            // leaves x non-finite too, and outside the prefix (no re-interpolation) a non-finite
            // x stays so: one check after the plain chain finds every failing round.
            if (in_prefix || !isfinite(x)) {
                x = x0;
                for (int st = 0; st < cnt; ++st) {
                    const float w = su[st * kStagedElems + tid];
                    int kind = 0;
                    float nx = x;
                    if (!isfinite(w)) {
                        kind = LEVO_EULER_FAIL_VELOCITY;
                    } else {
                        float xs = x;
                        if (in_prefix) {
                            float t, ns;
                            prefix_times(a.first + k0 + st, dt, a.sigma_min, t, ns);
                            xs = __fadd_rn(__fmul_rn(ns, nz), __fmul_rn(t, cx));
                        }
                        nx = __fadd_rn(xs, w);
                        if (!isfinite(nx)) kind = LEVO_EULER_FAIL_STATE;
                    }
                    if (kind != 0) {
                        failed = true;
                        record_failure(a.status, a.first + k0 + st, kind);
                        break;
                    }
                    x = nx;
                }
            }
        }
    }
    if (active) {
        if (!failed && in_prefix && a.first + a.count == a.steps) x = cx;
        a.state[i] = x;
    }
}

int64_t grid_for(int64_t items) {
    return std::max<int64_t>(
        1, std::min<int64_t>((items + kThreads - 1) / kThreads, static_cast<int64_t>(sm_count()) * 16));
}

// Argument checks of the multi-step form, in the reference's order
// (src/levo-flow-renderer.cpp:63-70), shared by the multi-step call and the solve.
int multi_args_error(const std::string &w, const float *state, const float *noise, const float *context,
                     const float *uncond, const float *cond, int64_t batch, int64_t row, int64_t prefix,
                     int64_t first_step, int64_t count, int64_t steps, int32_t cfg, float guidance,
                     float sigma_min, const int32_t *status) {
    if (state == nullptr || (count > 0 && (uncond == nullptr || (cfg && cond == nullptr))))
        return set_error(LEVO_OPS_EINVAL, w + ": required pointer is null");
    if (prefix > 0 && (noise == nullptr || context == nullptr))
        return set_error(LEVO_OPS_EINVAL, w + ": in-context tensors are null");
    if (batch <= 0 || row <= 0)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler state dimensions must be positive");
    if (steps <= 0)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler step count must be positive");
    if (prefix < 0 || prefix > row)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler in-context length exceeds frame count");
    if (first_step < 0 || count < 0 || first_step > steps || count > steps - first_step)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler resume step exceeds total steps");
    if (steps >= LEVO_EULER_STEP_LIMIT)
        return set_error(LEVO_OPS_EUNSUPPORTED, w + ": Euler step count above the status limit");
    if (!std::isfinite(sigma_min) || sigma_min <= 0.f)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler sigma_min must be finite and positive");
    if (cfg && !std::isfinite(guidance))
        return set_error(LEVO_OPS_EINVAL, w + ": CFG guidance scale must be finite");
    const void *ptrs[6] = {state, noise, context, uncond, cond, status};
    for (const void *p : ptrs)
        if (p && !aligned_to(p, 4))
            return set_error(LEVO_OPS_EINVAL, w + ": pointer is not 4-byte aligned");
    return LEVO_OPS_OK;
}

// solve_flow_euler's finiteness checks of its inputs before the first step
// (src/levo-flow-renderer.cpp:71-72,81): bit 0 the noise, bit 1 the in-context
// latent, bit 2 the resume state (any of them may be null).  One warp-wide OR,
// one atomic per warp.
__global__ void euler_inputs_kernel(const float *noise, const float *ctx, const float *resume, int64_t n,
                                    int32_t *bits_out) {
    int bits = 0;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        if (noise != nullptr && !isfinite(noise[i])) bits |= 1;
        if (ctx != nullptr && !isfinite(ctx[i])) bits |= 2;
        if (resume != nullptr && !isfinite(resume[i])) bits |= 4;
    }
    bits = static_cast<int>(__reduce_or_sync(0xffffffffu, static_cast<unsigned>(bits)));
    if ((threadIdx.x & 31) == 0 && bits != 0) atomicOr(bits_out, bits);
}

// Runs those checks on `stream` with `scratch` (one device int32) and returns
// the reference's error for the first input it names, or LEVO_OPS_OK.
int euler_inputs_error(const std::string &w, const float *noise, const float *ctx, const float *resume, int64_t n,
                       int32_t *scratch, cudaStream_t stream) {
    cudaError_t err = cudaMemsetAsync(scratch, 0, sizeof(int32_t), stream);
    if (err == cudaSuccess) {
        euler_inputs_kernel<<<static_cast<unsigned>(grid_for(n)), kThreads, 0, stream>>>(noise, ctx, resume, n,
                                                                                          scratch);
        err = cudaGetLastError();
    }
    int32_t bits = 0;
    if (err == cudaSuccess) err = cudaMemcpyAsync(&bits, scratch, sizeof(int32_t), cudaMemcpyDeviceToHost, stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
    if (err != cudaSuccess) return set_error(LEVO_OPS_ECUDA, w + ": " + cudaGetErrorString(err));
    if (bits & 1) return set_error(LEVO_OPS_ENONFINITE, w + ": Euler noise contains a non-finite value");
    if (bits & 2) return set_error(LEVO_OPS_ENONFINITE, w + ": Euler in-context latent contains a non-finite value");
    if (bits & 4) return set_error(LEVO_OPS_ENONFINITE, w + ": Euler resume state contains a non-finite value");
    return LEVO_OPS_OK;
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
    const int rc = multi_args_error("levo_cfg_euler_multi_f32", state, noise, context, uncond, cond, batch, row,
                                    prefix, first_step, count, steps, cfg, guidance, sigma_min, status);
    if (rc != LEVO_OPS_OK) return rc;
    const MultiArgs a{state, noise, context, uncond, cond, batch, row, prefix, first_step,
                      count, steps, cfg ? 1 : 0, guidance, sigma_min, status};
    const int64_t n = batch * row;
    // one staged CTA per kStagedElems elements: the grid must fit in 2^31 - 1 blocks
    const bool staged = count > 0 && n % 4 == 0 && aligned_to(uncond, 16) && (!cfg || aligned_to(cond, 16)) &&
                        (n + kStagedElems - 1) / kStagedElems <= 0x7fffffff;
    if (staged) {
        // [2][kStagedSteps][kStagedElems] F32 = 32 KB of shared memory
        const size_t smem = 2 * kStagedSteps * kStagedElems * sizeof(float);
        euler_multi_staged_kernel<<<static_cast<unsigned>((n + kStagedElems - 1) / kStagedElems),
                                    kStagedThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    } else {
        euler_multi_kernel<<<static_cast<unsigned>(grid_for(n)), kThreads, 0,
                             reinterpret_cast<cudaStream_t>(stream)>>>(a);
    }
    return check_launch("levo_cfg_euler_multi_f32");
}

LEVO_OPS_API int levo_cfg_euler_solve_f32(float *state, const float *noise, const float *context,
                                          const float *uncond, const float *cond, int64_t batch,
                                          int64_t row, int64_t prefix, int64_t first_step,
                                          int64_t count, int64_t steps, int32_t cfg,
                                          float guidance, float sigma_min, float *checkpoint,
                                          int32_t *status, int64_t *completed_steps,
                                          levo_stream_t stream) {
    using namespace levo;
    clear_error();
    const char *w = "levo_cfg_euler_solve_f32";
    if (checkpoint == nullptr || status == nullptr || completed_steps == nullptr)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": checkpoint, status and completed_steps are required");
    if (!aligned_to(checkpoint, 4) || !aligned_to(status, 4))
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": pointer is not 4-byte aligned");
    if (state == nullptr || batch <= 0 || row <= 0)
        return set_error(LEVO_OPS_EINVAL, std::string(w) + ": Euler state dimensions must be positive");
    *completed_steps = first_step;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int rc = multi_args_error(w, state, noise, context, uncond, cond, batch, row, prefix, first_step, count, steps,
                              cfg, guidance, sigma_min, status);
    if (rc != LEVO_OPS_OK) return rc;
    // The reference checks its noise, in-context latent and resume state before any step
    // (src/levo-flow-renderer.cpp:71-72,81).  Without a noise tensor (no in-context prefix) the
    // state the solve starts from is the noise.
    rc = euler_inputs_error(w, noise != nullptr ? noise : (first_step == 0 ? state : nullptr), context,
                            first_step > 0 ? state : nullptr, batch * row, status, s);
    if (rc != LEVO_OPS_OK) return rc;
    const size_t bytes = static_cast<size_t>(batch * row) * sizeof(float);
    // the checkpoint of the call's start, then the fused steps
    cudaError_t err = cudaMemcpyAsync(checkpoint, state, bytes, cudaMemcpyDeviceToDevice, s);
    if (err == cudaSuccess) err = cudaMemsetAsync(status, 0, sizeof(int32_t), s);
    if (err != cudaSuccess) return set_error(LEVO_OPS_ECUDA, std::string(w) + ": " + cudaGetErrorString(err));
    rc = levo_cfg_euler_multi_f32(state, noise, context, uncond, cond, batch, row, prefix, first_step, count,
                                  steps, cfg, guidance, sigma_min, status, stream);
    if (rc != LEVO_OPS_OK) {
        cudaStreamSynchronize(s);
        return rc;
    }
    int32_t word = 0;
    err = cudaMemcpyAsync(&word, status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return set_error(LEVO_OPS_ECUDA, std::string(w) + ": " + cudaGetErrorString(err));
    if (word == 0) {
        *completed_steps = first_step + count;
        return LEVO_OPS_OK;
    }
    // Some element failed at step `fail`: every element goes back to the call's
    // start and replays the steps before it (they were finite for all), which
    // is the reference's checkpoint of the last completed step.
    const int64_t fail = LEVO_EULER_STATUS_STEP(word);
    const int kind = LEVO_EULER_STATUS_KIND(word);
    if (fail < first_step || fail >= first_step + count)
        return set_error(LEVO_OPS_ECUDA, std::string(w) + ": inconsistent status word");
    err = cudaMemcpyAsync(state, checkpoint, bytes, cudaMemcpyDeviceToDevice, s);
    if (err != cudaSuccess) return set_error(LEVO_OPS_ECUDA, std::string(w) + ": " + cudaGetErrorString(err));
    if (fail > first_step) {
        rc = levo_cfg_euler_multi_f32(state, noise, context, uncond, cond, batch, row, prefix, first_step,
                                      fail - first_step, steps, cfg, guidance, sigma_min, nullptr, stream);
        if (rc != LEVO_OPS_OK) {
            cudaStreamSynchronize(s);
            return rc;
        }
    }
    err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return set_error(LEVO_OPS_ECUDA, std::string(w) + ": " + cudaGetErrorString(err));
    *completed_steps = fail;
    return set_error(LEVO_OPS_ENONFINITE,
                     std::string(w) + (kind == LEVO_EULER_FAIL_VELOCITY ? ": Euler velocity" : ": Euler state") +
                         " contains a non-finite value (step " + std::to_string(fail) + ")");
}

LEVO_OPS_API int levo_flow_euler_solve_f32(float *state, const float *noise, const float *context,
                                           int64_t frames, int64_t latent_dim, int64_t incontext_frames,
                                           float sigma_min, int64_t steps, int64_t first_step, int32_t cfg,
                                           float guidance, levo_velocity_fn velocity, void *velocity_user,
                                           levo_cancel_fn cancel, void *cancel_user, float *checkpoint,
                                           int32_t *status, int64_t *completed_steps, levo_stream_t stream) {
    using namespace levo;
    clear_error();
    const std::string w = "levo_flow_euler_solve_f32";
    if (completed_steps == nullptr || status == nullptr || velocity == nullptr)
        return set_error(LEVO_OPS_EINVAL, w + ": velocity, status and completed_steps are required");
    *completed_steps = first_step;
    // the reference's input checks (src/levo-flow-renderer.cpp:63-70)
    if (steps <= 0) return set_error(LEVO_OPS_EINVAL, w + ": Euler step count must be positive");
    if (frames <= 0 || latent_dim <= 0)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler state dimensions must be positive");
    if (incontext_frames < 0 || incontext_frames > frames)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler in-context length exceeds frame count");
    if (!std::isfinite(sigma_min) || sigma_min <= 0.f)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler sigma_min must be finite and positive");
    if (first_step < 0 || first_step > steps)
        return set_error(LEVO_OPS_EINVAL, w + ": Euler resume step exceeds total steps");
    if (state == nullptr || noise == nullptr || context == nullptr)
        return set_error(LEVO_OPS_EINVAL, w + ": required pointer is null");
    if (cfg && !std::isfinite(guidance)) return set_error(LEVO_OPS_EINVAL, w + ": CFG guidance scale must be finite");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t n = frames * latent_dim;
    const int64_t prefix = incontext_frames * latent_dim;
    const size_t bytes = static_cast<size_t>(n) * sizeof(float);
    if (!aligned_to(state, 4) || !aligned_to(noise, 4) || !aligned_to(context, 4) || !aligned_to(status, 4) ||
        (checkpoint != nullptr && !aligned_to(checkpoint, 4)))
        return set_error(LEVO_OPS_EINVAL, w + ": pointer is not 4-byte aligned");
    // the reference's finiteness checks of its inputs before any step (:71-72,81)
    int rc = euler_inputs_error(w, noise, context, first_step > 0 ? state : nullptr, n, status, s);
    if (rc != LEVO_OPS_OK) return rc;
    const float dt = 1.0f / static_cast<float>(steps);
    auto cuda_error = [&](cudaError_t err) {
        return set_error(LEVO_OPS_ECUDA, w + ": " + cudaGetErrorString(err));
    };
    for (int64_t step = first_step; step < steps; ++step) {
        if (cancel != nullptr && cancel(cancel_user) != 0) {
            cudaStreamSynchronize(s);
            return set_error(LEVO_OPS_ECANCELLED, w + ": cancelled before step " + std::to_string(step));
        }
        cudaError_t err = cudaSuccess;
        if (checkpoint != nullptr) err = cudaMemcpyAsync(checkpoint, state, bytes, cudaMemcpyDeviceToDevice, s);
        if (err == cudaSuccess) err = cudaMemsetAsync(status, 0, sizeof(int32_t), s);
        if (err != cudaSuccess) return cuda_error(err);
        rc = LEVO_OPS_OK;
        if (prefix > 0)
            rc = levo_flow_incontext_f32(state, noise, context, 1, n, prefix, step, steps, sigma_min, stream);
        if (rc != LEVO_OPS_OK) return rc;
        const float time = static_cast<float>(step) * dt;
        const float *v = velocity(velocity_user, state, step, time, stream);
        if (v == nullptr) {
            if (checkpoint != nullptr) cudaMemcpyAsync(state, checkpoint, bytes, cudaMemcpyDeviceToDevice, s);
            cudaStreamSynchronize(s);
            return set_error(LEVO_OPS_ECUDA, w + ": velocity callback failed at step " + std::to_string(step));
        }
        rc = levo_euler_cfg_step_f32(state, v, cfg ? v + n : nullptr, n, cfg, guidance, steps, status, stream);
        if (rc != LEVO_OPS_OK) return rc;
        int32_t word = 0;
        err = cudaMemcpyAsync(&word, status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
        if (err == cudaSuccess) err = cudaStreamSynchronize(s);
        if (err != cudaSuccess) return cuda_error(err);
        if (word != 0) {
            if (checkpoint != nullptr) {
                err = cudaMemcpyAsync(state, checkpoint, bytes, cudaMemcpyDeviceToDevice, s);
                if (err == cudaSuccess) err = cudaStreamSynchronize(s);
                if (err != cudaSuccess) return cuda_error(err);
            }
            return set_error(LEVO_OPS_ENONFINITE, w + ((word & 1) ? ": Euler velocity" : ": Euler state") +
                                                      " contains a non-finite value (step " +
                                                      std::to_string(step) + ")");
        }
        *completed_steps = step + 1;
    }
    // final context restore (src/levo-flow-renderer.cpp:113-114): a zero-step multi-step call
    rc = levo_cfg_euler_multi_f32(state, noise, context, nullptr, nullptr, 1, n, prefix, steps, 0, steps, 0,
                                      1.0f, sigma_min, nullptr, stream);
    if (rc != LEVO_OPS_OK) return rc;
    const cudaError_t err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return cuda_error(err);
    *completed_steps = steps;
    return LEVO_OPS_OK;
}

}  // extern "C"
