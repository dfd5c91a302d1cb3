// Shared device helpers for the sm_100a kernels of this library:
// 256-bit global loads/stores, per-channel parameter promotion, the SnakeBeta
// arithmetic in the reference's operator order, and the host-side status
// plumbing behind levo_ops_last_error().
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

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

inline bool aligned_to(const void *p, uintptr_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
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
// Parameters
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_param(const void *p, int64_t i, int dtype) {
    if (dtype == LEVO_DTYPE_F16) return __half2float(static_cast<const __half *>(p)[i]);
    return static_cast<const float *>(p)[i];
}

// SnakeBeta of the reference graph (src/levo-audio-ops.cpp:181-186), one GGML
// node per operation: alpha = exp(alpha_log), beta = exp(beta_log)*1 + 1e-9,
// t = x*alpha, s = sin(t), p = s*s, q = p/beta, y = x + q.  The _rn intrinsics
// keep each node's own rounding (no FMA contraction across nodes).
__device__ __forceinline__ float snake_alpha(float alpha_log) { return expf(alpha_log); }
__device__ __forceinline__ float snake_beta_den(float beta_log) {
    return __fadd_rn(expf(beta_log), 1.0e-9f);
}

__device__ __forceinline__ float snake_eval(float x, float alpha, float beta) {
    const float s = sinf(__fmul_rn(x, alpha));
    const float p = __fmul_rn(s, s);
    const float q = __fdiv_rn(p, beta);
    return __fadd_rn(x, q);
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
