// Shared device helpers for the sm_100a kernels of this library:
// 256-bit global loads/stores, per-channel parameter promotion, the SnakeBeta
// arithmetic in the reference's operator order, and the host-side status
// plumbing behind levo_ops_last_error().
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "levo_ops.h"

namespace levo {

// ---------------------------------------------------------------------------
// Host-side status handling
// ---------------------------------------------------------------------------
int set_error(int code, const std::string &message);
void clear_error();
// Records a launch failure (cudaGetLastError) for `what`; returns LEVO_OPS_OK
// when the launch went through.
int check_launch(const char *what);
// Number of SMs of the current device (cached per device).
int sm_count();
// Resident CTAs per SM of `kernel` at this block size and dynamic shared
// memory on the current device, opting the kernel in to more than 48 KB of
// shared memory when needed.  Both are done once per (kernel, device, size) and
// cached, not on every launch.
cudaError_t resident_ctas(const void *kernel, int threads, size_t smem_bytes, int *per_sm);

inline bool aligned_to(const void *p, uintptr_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

// Programmatic dependent launch (sm_90+): the next kernel in the stream may be
// scheduled while this one drains.  Every kernel launched this way calls
// pdl_wait() before it reads anything an earlier kernel wrote (a hardware
// wait for the preceding grid's completion and memory flush; a no-op for a
// normal launch), then pdl_trigger() to let its own successor be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// 256-bit vector memory access (sm_100 supports .v8.b32 global ld/st).
// Loads bypass L1 allocation: every byte of a streaming operand is read once.
// ---------------------------------------------------------------------------
struct f32x8 {
    float v[8];
};

__device__ __forceinline__ f32x8 ld8(const float *p) {
    f32x8 r;
    asm volatile(
        "ld.global.L1::no_allocate.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3]), "=f"(r.v[4]), "=f"(r.v[5]),
          "=f"(r.v[6]), "=f"(r.v[7])
        : "l"(p));
    return r;
}

__device__ __forceinline__ void st8(float *p, const f32x8 &r) {
    asm volatile("st.global.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(r.v[0]),
                 "f"(r.v[1]), "f"(r.v[2]), "f"(r.v[3]), "f"(r.v[4]), "f"(r.v[5]), "f"(r.v[6]),
                 "f"(r.v[7])
                 : "memory");
}

// Read-only operand reused by many CTAs (per-column gamma/beta): cached path.
__device__ __forceinline__ f32x8 ld8_ro(const float *p) {
    f32x8 r;
    asm volatile("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3]), "=f"(r.v[4]),
                   "=f"(r.v[5]), "=f"(r.v[6]), "=f"(r.v[7])
                 : "l"(p));
    return r;
}

// 32 bytes of 16-bit values as eight 32-bit words.
struct u32x8 {
    uint32_t v[8];
};

__device__ __forceinline__ u32x8 ld8u(const void *p) {
    u32x8 r;
    asm volatile(
        "ld.global.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]), "=r"(r.v[5]),
          "=r"(r.v[6]), "=r"(r.v[7])
        : "l"(p));
    return r;
}

__device__ __forceinline__ void st8u(void *p, const u32x8 &r) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(r.v[0]),
                 "r"(r.v[1]), "r"(r.v[2]), "r"(r.v[3]), "r"(r.v[4]), "r"(r.v[5]), "r"(r.v[6]),
                 "r"(r.v[7])
                 : "memory");
}

// ---------------------------------------------------------------------------
// Asynchronous global -> shared copies (cp.async, 16 bytes, L2 only).  The
// wait is the hardware's cp.async.wait_all: no software spin loop.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(gmem_src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// Groups: copies issued since the last commit form one group; wait_group<N>
// returns once at most N of this thread's groups are still in flight.
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// Parameters
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_param(const void *p, int64_t i, int dtype) {
    if (dtype == LEVO_DTYPE_F16) return __half2float(static_cast<const __half *>(p)[i]);
    return static_cast<const float *>(p)[i];
}

// SnakeBeta of the reference graph (src/levo-audio-ops.cpp:146-151):
//   alpha = exp(alpha_log), beta = exp(beta_log)*1 + 1e-9, y = x + sin(x*alpha)^2 / beta.
// Per channel the kernels stage alpha and 1/beta (IEEE reciprocal of the
// reference's beta); per element they evaluate y = fma(sin^2(x*alpha), 1/beta, x).
// Against the reference's node-by-node rounding (mul, sin, sqr, div, add) this
// differs by a few F32 ulp of the sin^2 term, inside the 1e-5 tolerance.
__device__ __forceinline__ float snake_alpha(float alpha_log) { return expf(alpha_log); }
__device__ __forceinline__ float snake_inv_beta(float beta_log) {
    return __frcp_rn(__fadd_rn(expf(beta_log), 1.0e-9f));
}

// A channel's alpha and 1/beta from its stored parameter: log form (F32 / F16)
// or already prepared by levo_snake_params_prepare (LEVO_DTYPE_SNAKE_PREPARED).
__device__ __forceinline__ float snake_alpha_param(const void *p, int64_t c, int dtype) {
    const float v = load_param(p, c, dtype);
    return dtype == LEVO_DTYPE_SNAKE_PREPARED ? v : snake_alpha(v);
}
__device__ __forceinline__ float snake_inv_beta_param(const void *p, int64_t c, int dtype) {
    const float v = load_param(p, c, dtype);
    return dtype == LEVO_DTYPE_SNAKE_PREPARED ? v : snake_inv_beta(v);
}

// sin(t)^2, written for this library (no sinf call on the common path):
//  1. Cody-Waite argument reduction (W. J. Cody, W. Waite, "Software Manual for
//     the Elementary Functions", 1980): k = rint(t * 2/pi), r = t - k*pi/2 with
//     pi/2 split into two F32 parts applied by FMA; |r| <= pi/4.  (The third
//     part, -1.78e-15, would move r by at most |k| * 1.8e-15 <= 7.5e-11 for
//     |t| <= 65536: below 0.01 ulp of sin^2 in absolute terms.)  k is rounded
//     by adding 1.5*2^23 (the sum's ulp is 1, so the FMA rounds t*2/pi to the
//     nearest integer) and its parity is the sum's lowest mantissa bit.
//  2. sin(t)^2 = sin(r)^2 for even k and 1 - sin(r)^2 for odd k.
//  3. sin(r)^2 = z * Q(z), z = r^2, with Q a degree-5 polynomial fitted here by
//     weighted least squares to sin(r)^2 / r^2 on [0, (pi/4)^2]
//     (F32 relative error of z*Q(z) <= 1e-7; |error of sin^2| <= 1.2e-7 up to |t| = 1e5).
// Valid for |t| <= kSin2FastLimit; callers route larger (or infinite) arguments
// to sin_squared_any(), which uses CUDA's sinf and its large-argument reduction.
constexpr float kSin2FastLimit = 65536.0f;

// The constants of the three steps above (shared by the scalar and paired forms).
constexpr float kSin2Big = 12582912.0f;                 // 1.5 * 2^23
constexpr float kSin2TwoOverPi = 0.636619747f;
constexpr float kSin2PiOver2A = 1.57079637f;  // pi/2 = A + B (+ 1.8e-15)
constexpr float kSin2PiOver2B = -4.37113883e-08f;
constexpr float kSin2Q0 = -4.103582341e-06f;  // Q(z) = ((((Q0 z + Q1) z + Q2) z + Q3) z + Q4) z + Q5
constexpr float kSin2Q1 = 1.409736724e-04f;
constexpr float kSin2Q2 = -3.174564568e-03f;
constexpr float kSin2Q3 = 4.444443807e-02f;
constexpr float kSin2Q4 = -3.333333433e-01f;
constexpr float kSin2Q5 = 1.0f;

// Every step rounds on its own (explicit _rn operations, no contraction), so the
// paired form below gives the same bits.
__device__ __forceinline__ float sin_squared_fast(float t) {
    const float ks = __fmaf_rn(t, kSin2TwoOverPi, kSin2Big);
    const int odd = __float_as_int(ks) & 1;
    const float k = __fadd_rn(ks, -kSin2Big);
    float r = __fmaf_rn(k, -kSin2PiOver2A, t);
    r = __fmaf_rn(k, -kSin2PiOver2B, r);
    const float z = __fmul_rn(r, r);
    float q = __fmaf_rn(z, kSin2Q0, kSin2Q1);
    q = __fmaf_rn(q, z, kSin2Q2);
    q = __fmaf_rn(q, z, kSin2Q3);
    q = __fmaf_rn(q, z, kSin2Q4);
    q = __fmaf_rn(q, z, kSin2Q5);
    const float p = __fmul_rn(z, q);
    return odd ? __fadd_rn(1.0f, -p) : p;
}

// Two arguments at once with sm_100's paired F32 instructions (__ffma2_rn,
// __fmul2_rn, __fadd2_rn: each lane one IEEE round-to-nearest operation), so the
// result is bit-identical to two sin_squared_fast calls in half the arithmetic
// instructions.
__device__ __forceinline__ float2 pair(float v) { return make_float2(v, v); }

__device__ __forceinline__ float2 sin_squared_fast2(float2 t) {
    const float2 ks = __ffma2_rn(t, pair(kSin2TwoOverPi), pair(kSin2Big));
    const int odd_x = __float_as_int(ks.x) & 1;
    const int odd_y = __float_as_int(ks.y) & 1;
    const float2 k = __fadd2_rn(ks, pair(-kSin2Big));
    float2 r = __ffma2_rn(k, pair(-kSin2PiOver2A), t);
    r = __ffma2_rn(k, pair(-kSin2PiOver2B), r);
    const float2 z = __fmul2_rn(r, r);
    float2 q = __ffma2_rn(z, pair(kSin2Q0), pair(kSin2Q1));
    q = __ffma2_rn(q, z, pair(kSin2Q2));
    q = __ffma2_rn(q, z, pair(kSin2Q3));
    q = __ffma2_rn(q, z, pair(kSin2Q4));
    q = __ffma2_rn(q, z, pair(kSin2Q5));
    const float2 p = __fmul2_rn(z, q);
    const float2 om = __fadd2_rn(pair(1.0f), make_float2(-p.x, -p.y));
    return make_float2(odd_x ? om.x : p.x, odd_y ? om.y : p.y);
}

__device__ __forceinline__ float sin_squared_any(float t) {
    if (fabsf(t) > kSin2FastLimit) {
        const float s = sinf(t);
        return s * s;
    }
    return sin_squared_fast(t);
}

__device__ __forceinline__ float snake_eval(float x, float alpha, float inv_beta) {
    return __fmaf_rn(sin_squared_any(__fmul_rn(x, alpha)), inv_beta, x);
}

// SnakeBeta of 8 values of one channel: one range check per vector, then the
// branch-free fast path (the common case) or the general one.
__device__ __forceinline__ void snake_eval8(float (&v)[8], float alpha, float inv_beta) {
    float2 t[4];
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        t[k] = __fmul2_rn(make_float2(v[2 * k], v[2 * k + 1]), pair(alpha));
        m = fmaxf(m, fmaxf(fabsf(t[k].x), fabsf(t[k].y)));
    }
    if (m <= kSin2FastLimit) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 y = __ffma2_rn(sin_squared_fast2(t[k]), pair(inv_beta), make_float2(v[2 * k], v[2 * k + 1]));
            v[2 * k] = y.x;
            v[2 * k + 1] = y.y;
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[2 * k] = __fmaf_rn(sin_squared_any(t[k].x), inv_beta, v[2 * k]);
            v[2 * k + 1] = __fmaf_rn(sin_squared_any(t[k].y), inv_beta, v[2 * k + 1]);
        }
    }
}

// Block b's share [begin, end) of `items` split over the grid in contiguous
// ranges whose sizes differ by at most one (quotient and remainder: no
// items * blockIdx product that could overflow for huge tensors).
__device__ __forceinline__ void block_range(int64_t items, int64_t &begin, int64_t &end) {
    const int64_t per = items / gridDim.x, extra = items % gridDim.x, b = blockIdx.x;
    begin = per * b + (b < extra ? b : extra);
    end = begin + per + (b < extra ? 1 : 0);
}

// ---------------------------------------------------------------------------
// Flat index -> row (channel) of a dense [rows][len] tensor.  The quotient is
// estimated in double (exact for e < 2^53) and corrected by one step.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t row_of(int64_t e, int64_t len, double inv_len) {
    int64_t c = static_cast<int64_t>(static_cast<double>(e) * inv_len);
    const int64_t base = c * len;
    if (base > e) {
        --c;
    } else if (base + len <= e) {
        ++c;
    }
    return c;
}

}  // namespace levo
