// Residual add + RMSNorm / LayerNorm row reductions (a5, a6).
//
// Every form reads x and r from HBM once and writes h and y once: 8 B per
// element for F16 activations.
// Register path (the common case: 16-byte aligned rows of at most 4 KB, i.e.
// F16 dim <= 2048 / F32 dim <= 1024, without the Flow modulation): one warp per
// row, 8 rows per CTA, x and r copied into shared memory with cp.async, then
// held packed in registers while the statistics and y are computed; gamma and
// beta staged once per CTA; about two rows per warp so the next row's copies
// overlap the current row's arithmetic (4096 x 1536 F16: 296 CTAs).
// Staged path (longer rows of <= 12.5 KB, and the Flow adaLN form): one warp
// per row, 8 rows per CTA.  x and r are copied into shared memory with cp.async
// so the whole input is in flight at once without holding it in registers;
// h = x + r is written back over x, the row statistics are reduced with warp
// shuffles (LayerNorm two-pass over shared memory), and y leaves in 16-byte
// stores.
// Vector path (longer rows): a row group of 32*wpr threads keeps the row in
// registers (<= 64 F32 values per thread) and reduces across warps in shared
// memory.  Scalar path (rows whose byte length is not a multiple of 16, or
// unaligned pointers): one CTA per row, re-reading the row from L2.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace levo {
namespace {

constexpr int kThreads = 256;

struct NormArgs {
    const void *x;
    const void *r;
    const float *gamma;
    const float *beta;
    void *h_out;
    void *y_out;
    int64_t rows;
    int dim;
    int wpr;  // warps per row (vector path)
    float eps;
    int f16_boundary;
    // Flow adaLN form (MOD kernels only): per-batch [rows / batch_rows][dim] F32 vectors.
    const float *gate;   // h = r + x * gate       (src/levo-flow-estimator.cpp:221-227)
    const float *scale;  // y = y * (1 + scale) + shift (src/levo-flow-estimator.cpp:89-93)
    const float *shift;
    int64_t batch_rows;
};

template <typename T>
struct Act;
template <>
struct Act<__half> {
    static constexpr int kVec = 16;  // elements per 32-byte vector
    __device__ static float round(float v) { return __half2float(__float2half_rn(v)); }
    __device__ static void unpack(const u32x8 &w, float *out) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const __half2 h2 = *reinterpret_cast<const __half2 *>(&w.v[i]);
            const float2 f = __half22float2(h2);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    }
    __device__ static u32x8 pack(const float *in) {
        u32x8 w;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const __half2 h2 = __floats2half2_rn(in[2 * i], in[2 * i + 1]);
            w.v[i] = *reinterpret_cast<const uint32_t *>(&h2);
        }
        return w;
    }
    // One 32-bit word = two values.
    __device__ static float2 word(uint32_t w) {
        return __half22float2(*reinterpret_cast<const __half2 *>(&w));
    }
    __device__ static uint32_t make_word(float a, float b) {
        const __half2 h2 = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h2);
    }
    static constexpr int kPerWord = 2;
    __device__ static float load1(const void *p, int64_t i) {
        return __half2float(static_cast<const __half *>(p)[i]);
    }
    __device__ static void store1(void *p, int64_t i, float v) {
        static_cast<__half *>(p)[i] = __float2half_rn(v);
    }
};
template <>
struct Act<float> {
    static constexpr int kVec = 8;
    __device__ static float round(float v) { return v; }
    __device__ static void unpack(const u32x8 &w, float *out) {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = __uint_as_float(w.v[i]);
    }
    __device__ static u32x8 pack(const float *in) {
        u32x8 w;
#pragma unroll
        for (int i = 0; i < 8; ++i) w.v[i] = __float_as_uint(in[i]);
        return w;
    }
    __device__ static float2 word(uint32_t w) { return make_float2(__uint_as_float(w), 0.f); }
    __device__ static uint32_t make_word(float a, float) { return __float_as_uint(a); }
    static constexpr int kPerWord = 1;
    __device__ static float load1(const void *p, int64_t i) {
        return static_cast<const float *>(p)[i];
    }
    __device__ static void store1(void *p, int64_t i, float v) {
        static_cast<float *>(p)[i] = v;
    }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over the `wpr` warps of a row group.  Every thread of the CTA calls it
// (the __syncthreads are CTA-wide); `slot` is the group's first warp.
__device__ __forceinline__ float group_sum(float v, int wpr, float *red) {
    v = warp_sum(v);
    if (wpr == 1) return v;
    const int warp = threadIdx.x >> 5;
    const int first = (warp / wpr) * wpr;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
    for (int w = 0; w < wpr; ++w) s += red[first + w];
    return s;
}

// Final y value from the normalised value n for column j.
template <typename T, bool LAYER>
__device__ __forceinline__ float norm_output(const NormArgs &a, float n, float g, float b) {
    if (a.f16_boundary) n = Act<T>::round(n);
    float y = __fmul_rn(n, g);
    if (LAYER) y = __fadd_rn(y, b);
    return y;
}

// add_scale_shift (src/levo-flow-estimator.cpp:89-93): y * (scale*1 + 1) + shift.
__device__ __forceinline__ float modulate(const NormArgs &a, float y, float s, float sh) {
    if (a.scale) y = __fmul_rn(y, __fadd_rn(s, 1.0f));
    if (a.shift) y = __fadd_rn(y, sh);
    return y;
}

// Word-wise helpers: a 32-byte vector is 8 words of kPerWord values each; the
// math touches one word (<= 2 values) at a time so only the packed row stays live.
template <typename T>
__device__ __forceinline__ float word_sum(uint32_t w, bool layer, float mean) {
    const float2 f = Act<T>::word(w);
    if (layer) {
        const float d0 = __fsub_rn(f.x, mean);
        float s = d0 * d0;
        if (Act<T>::kPerWord == 2) {
            const float d1 = __fsub_rn(f.y, mean);
            s = fmaf(d1, d1, s);
        }
        return s;
    }
    float s = f.x * f.x;
    if (Act<T>::kPerWord == 2) s = fmaf(f.y, f.y, s);
    return s;
}

template <typename T>
__device__ __forceinline__ float word_plain_sum(uint32_t w) {
    const float2 f = Act<T>::word(w);
    return Act<T>::kPerWord == 2 ? f.x + f.y : f.x;
}

template <typename T, int VPL, bool LAYER, bool MOD>
// RMSNorm rows of up to 96 bytes per thread are held to 64 registers (4 CTAs =
// 32 warps per SM, one wave of 4096 rows on 148 SMs).  LayerNorm keeps its
// registers: the same cap spills its two-pass variance.
__global__ void __launch_bounds__(kThreads, (!LAYER && !MOD && VPL * Act<T>::kVec * sizeof(T) <= 96) ? 4 : 1)
    add_norm_vec_kernel(const NormArgs a) {
    constexpr int VE = Act<T>::kVec;
    constexpr int PW = Act<T>::kPerWord;
    __shared__ float red[kThreads / 32];
    const int group_threads = 32 * a.wpr;
    const int groups = kThreads / group_threads;
    const int group = threadIdx.x / group_threads;
    const int gl = threadIdx.x % group_threads;
    const int nvec = a.dim / VE;
    const float inv_dim = 1.0f / static_cast<float>(a.dim);

    for (int64_t row0 = static_cast<int64_t>(blockIdx.x) * groups; row0 < a.rows;
         row0 += static_cast<int64_t>(gridDim.x) * groups) {
        const int64_t row = row0 + group;
        const bool active = row < a.rows;
        const size_t row_off = static_cast<size_t>(row) * a.dim * sizeof(T);
        const int64_t mod_off = MOD ? (row / a.batch_rows) * a.dim : 0;
        // hw holds the row packed in the activation type: h = x + r is exactly
        // representable there, so the row costs 8 registers per vector.
        u32x8 hw[VPL], rw[VPL];
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int vi = k * group_threads + gl;
            if (active && vi < nvec) {
                hw[k] = ld8u(static_cast<const char *>(a.x) + row_off + vi * 32);
                if (a.r) rw[k] = ld8u(static_cast<const char *>(a.r) + row_off + vi * 32);
            }
        }
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int vi = k * group_threads + gl;
            if (active && vi < nvec) {
                if (MOD && a.gate) {
                    // h = r + x * gate, one gate value per column of this row's batch
                    const float *gp = a.gate + mod_off + vi * VE;
#pragma unroll
                    for (int i8 = 0; i8 < VE; i8 += 8) {
                        const f32x8 g = ld8_ro(gp + i8);
#pragma unroll
                        for (int j = 0; j < 8 / PW; ++j) {
                            const int wi = i8 / PW + j;
                            const float2 x = Act<T>::word(hw[k].v[wi]);
                            const float2 r = a.r ? Act<T>::word(rw[k].v[wi]) : make_float2(0.f, 0.f);
                            const float h0 = __fmul_rn(x.x, g.v[j * PW]);
                            const float h1 = PW == 2 ? __fmul_rn(x.y, g.v[j * PW + 1]) : 0.f;
                            hw[k].v[wi] = a.r ? Act<T>::make_word(__fadd_rn(h0, r.x), __fadd_rn(h1, r.y))
                                              : Act<T>::make_word(h0, h1);
                        }
                    }
                } else if (a.r) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float2 x = Act<T>::word(hw[k].v[i]);
                        const float2 r = Act<T>::word(rw[k].v[i]);
                        hw[k].v[i] = Act<T>::make_word(__fadd_rn(x.x, r.x), __fadd_rn(x.y, r.y));
                    }
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    sum += LAYER ? word_plain_sum<T>(hw[k].v[i]) : word_sum<T>(hw[k].v[i], false, 0.f);
            }
        }
        sum = group_sum(sum, a.wpr, red);
        float mean = 0.f, scale;
        if (LAYER) {
            mean = sum * inv_dim;
            float sq = 0.f;
#pragma unroll
            for (int k = 0; k < VPL; ++k) {
                const int vi = k * group_threads + gl;
                if (active && vi < nvec) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) sq += word_sum<T>(hw[k].v[i], true, mean);
                }
            }
            sq = group_sum(sq, a.wpr, red);
            scale = 1.0f / sqrtf(sq * inv_dim + a.eps);
        } else {
            scale = 1.0f / sqrtf(sum * inv_dim + a.eps);
        }
        if (!active) continue;
#pragma unroll
        for (int k = 0; k < VPL; ++k) {
            const int vi = k * group_threads + gl;
            if (vi >= nvec) continue;
            const int col = vi * VE;
            if (a.h_out && (a.r || (MOD && a.gate)))
                st8u(static_cast<char *>(a.h_out) + row_off + vi * 32, hw[k]);
            u32x8 yw;
#pragma unroll
            for (int i8 = 0; i8 < VE; i8 += 8) {
                const f32x8 g = ld8_ro(a.gamma + col + i8);
                f32x8 b{}, ms{}, mh{};
                if (LAYER) b = ld8_ro(a.beta + col + i8);
                if (MOD && a.scale) ms = ld8_ro(a.scale + mod_off + col + i8);
                if (MOD && a.shift) mh = ld8_ro(a.shift + mod_off + col + i8);
#pragma unroll
                for (int j = 0; j < 8 / PW; ++j) {
                    const int wi = i8 / PW + j;
                    const float2 h = Act<T>::word(hw[k].v[wi]);
                    const float n0 = LAYER ? __fmul_rn(__fsub_rn(h.x, mean), scale) : __fmul_rn(h.x, scale);
                    float y0 = norm_output<T, LAYER>(a, n0, g.v[j * PW], b.v[j * PW]);
                    if (MOD) y0 = modulate(a, y0, ms.v[j * PW], mh.v[j * PW]);
                    float y1 = 0.f;
                    if (PW == 2) {
                        const float n1 = LAYER ? __fmul_rn(__fsub_rn(h.y, mean), scale) : __fmul_rn(h.y, scale);
                        y1 = norm_output<T, LAYER>(a, n1, g.v[j * PW + 1], b.v[j * PW + 1]);
                        if (MOD) y1 = modulate(a, y1, ms.v[j * PW + 1], mh.v[j * PW + 1]);
                    }
                    yw.v[wi] = Act<T>::make_word(y0, y1);
                }
            }
            st8u(static_cast<char *>(a.y_out) + row_off + vi * 32, yw);
        }
    }
}

constexpr int kStagedRows = 8;                   // warps = rows per CTA
constexpr size_t kStagedMaxSmem = 200 * 1024;    // opt-in dynamic shared memory cap

template <typename T>
struct Chunk;  // 16 bytes of activations
template <>
struct Chunk<__half> {
    static constexpr int kN = 8;
    __device__ static void unpack(const uint4 &c, float *v) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    __device__ static uint4 pack(const float *v) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t *>(&h2);
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
    __device__ static float first(const uint4 &c) {
        return __half2float(__ushort_as_half(static_cast<unsigned short>(c.x & 0xffffu)));
    }
    // sm_100 mixed-precision forms: the F16 halves of a word enter the F32 arithmetic directly
    // (the product of two F16 values is exact in F32, so fma.f32.f16 rounds once, like an F32 FMA
    // of the converted values; add.f32.f16 likewise equals the F32 add of the converted value).
    __device__ static void halves(uint32_t w, unsigned short &lo, unsigned short &hi) {
        asm("mov.b32 {%0, %1}, %2;" : "=h"(lo), "=h"(hi) : "r"(w));
    }
    __device__ static float sq_add(unsigned short h, float c) {
        float d;
        asm("fma.rn.f32.f16 %0, %1, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
        return d;
    }
    __device__ static float add_f32(unsigned short h, float c) {
        float d;
        asm("add.rn.f32.f16 %0, %1, %2;" : "=f"(d) : "h"(h), "f"(c));
        return d;
    }
    // sum of squares of the chunk, even and odd columns in two accumulators (as a paired FFMA2)
    __device__ static float sq_sum(const uint4 &c) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
        float ax = 0.f, ay = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            unsigned short lo, hi;
            halves(w[i], lo, hi);
            ax = sq_add(lo, ax);
            ay = sq_add(hi, ay);
        }
        return ax + ay;
    }
    // (h - k) for the chunk's values, in column pairs
    __device__ static void minus(const uint4 &c, float k, float2 *d) {
        const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            unsigned short lo, hi;
            halves(w[i], lo, hi);
            d[i] = make_float2(add_f32(lo, -k), add_f32(hi, -k));
        }
    }
    // x + r rounded to F16 in one HADD2 per pair.  The F32 sum of two F16
    // values rounded to F16 is the same number: F32 carries 24 >= 2*11 + 1
    // significand bits, so the double rounding is innocuous (S. A. Figueroa,
    // "When is double rounding innocuous?", SIGNUM Newsletter 30(3), 1995).
    __device__ static uint4 add(const uint4 &a, const uint4 &b) {
        const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2 s = __hadd2(*reinterpret_cast<const __half2 *>(&wa[i]),
                                      *reinterpret_cast<const __half2 *>(&wb[i]));
            w[i] = *reinterpret_cast<const uint32_t *>(&s);
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
};
template <>
struct Chunk<float> {
    static constexpr int kN = 4;
    __device__ static float first(const uint4 &c) { return __uint_as_float(c.x); }
    __device__ static float sq_sum(const uint4 &c) {
        const float2 v0 = make_float2(__uint_as_float(c.x), __uint_as_float(c.y));
        const float2 v1 = make_float2(__uint_as_float(c.z), __uint_as_float(c.w));
        float2 acc = __ffma2_rn(v0, v0, make_float2(0.f, 0.f));
        acc = __ffma2_rn(v1, v1, acc);
        return acc.x + acc.y;
    }
    __device__ static void minus(const uint4 &c, float k, float2 *d) {
        d[0] = __fadd2_rn(make_float2(__uint_as_float(c.x), __uint_as_float(c.y)), pair(-k));
        d[1] = __fadd2_rn(make_float2(__uint_as_float(c.z), __uint_as_float(c.w)), pair(-k));
    }
    __device__ static void unpack(const uint4 &c, float *v) {
        v[0] = __uint_as_float(c.x);
        v[1] = __uint_as_float(c.y);
        v[2] = __uint_as_float(c.z);
        v[3] = __uint_as_float(c.w);
    }
    __device__ static uint4 pack(const float *v) {
        return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                          __float_as_uint(v[3]));
    }
    __device__ static uint4 add(const uint4 &a, const uint4 &b) {
        return make_uint4(__float_as_uint(__fadd_rn(__uint_as_float(a.x), __uint_as_float(b.x))),
                          __float_as_uint(__fadd_rn(__uint_as_float(a.y), __uint_as_float(b.y))),
                          __float_as_uint(__fadd_rn(__uint_as_float(a.z), __uint_as_float(b.z))),
                          __float_as_uint(__fadd_rn(__uint_as_float(a.w), __uint_as_float(b.w))));
    }
};

// kN consecutive F32 column parameters starting at p (16-byte aligned).
template <int N>
__device__ __forceinline__ void load_cols(const float *p, float *out) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
        const float4 f = __ldg(reinterpret_cast<const float4 *>(p + i));
        out[i] = f.x;
        out[i + 1] = f.y;
        out[i + 2] = f.z;
        out[i + 3] = f.w;
    }
}

// One row whose x (and r) are in shared memory (xs, rs: dim / Chunk<T>::kN
// chunks each), processed by one warp: h = [x * gate] + r is written back over
// xs, then the row statistics, then h and y leave in 16-byte stores.
template <typename T, bool LAYER, bool MOD>
__device__ __forceinline__ void norm_row_from_smem(const NormArgs &a, int64_t row, uint4 *xs, const uint4 *rs,
                                                   int lane, int chunks, float inv_dim) {
    constexpr int N = Chunk<T>::kN;
    const bool has_r = a.r != nullptr;
    const int64_t mod_off = MOD ? (row / a.batch_rows) * a.dim : 0;
    // pass 1: h = [x * gate] + r (rounded to T) back into xs; row sum / sum of squares
    float sum = 0.f;
    for (int i = lane; i < chunks; i += 32) {
        float h[N];
        const bool gated = MOD && a.gate;
        if (!gated && has_r) {
            // plain residual add, in the activation type; sums on paired F32 lanes
            const uint4 hc = Chunk<T>::add(xs[i], rs[i]);
            xs[i] = hc;
            Chunk<T>::unpack(hc, h);
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int j = 0; j < N; j += 2) {
                const float2 v = make_float2(h[j], h[j + 1]);
                acc = LAYER ? __fadd2_rn(acc, v) : __ffma2_rn(v, v, acc);
            }
            sum += acc.x + acc.y;
            continue;
        }
        Chunk<T>::unpack(xs[i], h);
        if (gated) {
            float g[N];
            load_cols<N>(a.gate + mod_off + i * N, g);
#pragma unroll
            for (int j = 0; j < N; ++j) h[j] = __fmul_rn(h[j], g[j]);
        }
        if (has_r) {
            float r[N];
            Chunk<T>::unpack(rs[i], r);
#pragma unroll
            for (int j = 0; j < N; ++j) h[j] = __fadd_rn(h[j], r[j]);
        }
        if (gated || has_r) {
#pragma unroll
            for (int j = 0; j < N; ++j) h[j] = Act<T>::round(h[j]);
            xs[i] = Chunk<T>::pack(h);
        }
#pragma unroll
        for (int j = 0; j < N; ++j) sum += LAYER ? h[j] : h[j] * h[j];
    }
    sum = warp_sum(sum);
    float mean = 0.f, scale;
    if (LAYER) {
        mean = sum * inv_dim;
        float sq = 0.f;
        for (int i = lane; i < chunks; i += 32) {
            float h[N];
            Chunk<T>::unpack(xs[i], h);
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int j = 0; j < N; j += 2) {
                const float2 d = __fadd2_rn(make_float2(h[j], h[j + 1]), pair(-mean));
                acc = __ffma2_rn(d, d, acc);
            }
            sq += acc.x + acc.y;
        }
        sq = warp_sum(sq);
        scale = 1.0f / sqrtf(sq * inv_dim + a.eps);
    } else {
        scale = 1.0f / sqrtf(sum * inv_dim + a.eps);
    }
    uint4 *hg = (a.h_out && (has_r || (MOD && a.gate)))
                    ? reinterpret_cast<uint4 *>(static_cast<char *>(a.h_out) + row * a.dim * sizeof(T))
                    : nullptr;
    uint4 *yg = reinterpret_cast<uint4 *>(static_cast<char *>(a.y_out) + row * a.dim * sizeof(T));
    for (int i = lane; i < chunks; i += 32) {
        const uint4 hc = xs[i];
        if (hg) hg[i] = hc;
        float h[N], g[N], b[N];
        Chunk<T>::unpack(hc, h);
        load_cols<N>(a.gamma + i * N, g);
        if (LAYER) load_cols<N>(a.beta + i * N, b);
        float ms[N], mh[N];
        if (MOD && a.scale) load_cols<N>(a.scale + mod_off + i * N, ms);
        if (MOD && a.shift) load_cols<N>(a.shift + mod_off + i * N, mh);
        // n = (h [- mean]) * scale, y = n * gamma [+ beta] [* (1 + s) + shift]: the same
        // rounded steps as norm_output / modulate, two columns per instruction
#pragma unroll
        for (int j = 0; j < N; j += 2) {
            float2 v = make_float2(h[j], h[j + 1]);
            if (LAYER) v = __fadd2_rn(v, pair(-mean));
            v = __fmul2_rn(v, pair(scale));
            if (a.f16_boundary) v = make_float2(Act<T>::round(v.x), Act<T>::round(v.y));
            v = __fmul2_rn(v, make_float2(g[j], g[j + 1]));
            if (LAYER) v = __fadd2_rn(v, make_float2(b[j], b[j + 1]));
            if (MOD && a.scale) v = __fmul2_rn(v, __fadd2_rn(make_float2(ms[j], ms[j + 1]), pair(1.0f)));
            if (MOD && a.shift) v = __fadd2_rn(v, make_float2(mh[j], mh[j + 1]));
            h[j] = v.x;
            h[j + 1] = v.y;
        }
        yg[i] = Chunk<T>::pack(h);
    }
}

// Single-wave form: one warp per row, 8 rows per CTA; every row's bytes are in
// flight at once (cp.async into shared memory).
template <typename T, bool LAYER, bool MOD>
__global__ void __launch_bounds__(kStagedRows * 32) add_norm_staged_kernel(const NormArgs a) {
    extern __shared__ uint4 sbuf[];
    constexpr int N = Chunk<T>::kN;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int chunks = a.dim / N;
    uint4 *xs = sbuf + static_cast<size_t>(warp) * 2 * chunks;
    uint4 *rs = xs + chunks;
    const float inv_dim = 1.0f / static_cast<float>(a.dim);
    for (int64_t row0 = static_cast<int64_t>(blockIdx.x) * kStagedRows; row0 < a.rows;
         row0 += static_cast<int64_t>(gridDim.x) * kStagedRows) {
        const int64_t row = row0 + warp;
        if (row >= a.rows) continue;  // warp-uniform; no CTA-wide barrier in this loop
        const uint4 *xg = reinterpret_cast<const uint4 *>(static_cast<const char *>(a.x) + row * a.dim * sizeof(T));
        const uint4 *rg = a.r ? reinterpret_cast<const uint4 *>(static_cast<const char *>(a.r) + row * a.dim * sizeof(T))
                              : nullptr;
        __syncwarp();  // the previous row's shared-memory reads are done
        for (int i = lane; i < chunks; i += 32) {
            cp_async16(xs + i, xg + i);
            if (rg) cp_async16(rs + i, rg + i);
        }
        cp_async_wait_all();
        __syncwarp();
        norm_row_from_smem<T, LAYER, MOD>(a, row, xs, rs, lane, chunks, inv_dim);
    }
}

// Register form (rows of at most 32 * kRegsMaxCpl 16-byte chunks; add+norm
// without the Flow modulation).  Like the staged form, a warp's row is copied
// into shared memory with cp.async, one warp per row.  Once it lands the row
// is read out of shared memory in one unrolled burst and held packed in the
// activation type (h = x + r, CPL 16-byte chunks per lane), so the reductions
// and the output pass are straight-line code on registers.  gamma (and beta)
// are copied into shared memory once per CTA, ahead of the rows, so the output
// pass never waits on L2.  A warp with a further row issues that row's copies
// as soon as the current row is in registers, overlapping them with its
// arithmetic.
//
// Rows of one wave land at nearly the same time, so the SM's issue slots, not
// the memory system, set the tail of a launch: the per-row instruction count is
// kept low by making the F16-boundary rounding a template parameter and by
// branching on the residual / h_out pointers once per row, not per chunk, and
// LayerNorm takes its mean and variance in one pass over the registers
// (shifted sums, below) instead of two.  RMSNorm keeps the rounded steps of
// norm_row_from_smem (same per-lane order of the paired partial sums, same
// butterfly): both forms give the same bits.  For LayerNorm the two forms
// differ only in the rounding of the statistics (a few F32 ulp).
constexpr int kRegsMaxCpl = 8;
constexpr int kRegsWarps = 8;        // warps (= rows in flight) per CTA
constexpr int kRegsRowsPerWarp = 2;  // rows per warp a launch aims for (copies of the next row overlap)

template <typename T, bool LAYER, bool BOUND>
__device__ __forceinline__ uint4 norm_chunk_out(uint4 hc, const float4 *gs, const float4 *bs, int i, float mean,
                                                float scale) {
    constexpr int N = Chunk<T>::kN;
    float h[N];
    float2 dm[N / 2];
    if (LAYER) {
        Chunk<T>::minus(hc, mean, dm);  // h - mean, the reference's first rounded step
    } else {
        Chunk<T>::unpack(hc, h);
    }
#pragma unroll
    for (int q = 0; q < N / 4; ++q) {
        const float4 g = gs[i * (N / 4) + q];
        float2 v0 = LAYER ? dm[2 * q] : make_float2(h[4 * q], h[4 * q + 1]);
        float2 v1 = LAYER ? dm[2 * q + 1] : make_float2(h[4 * q + 2], h[4 * q + 3]);
        v0 = __fmul2_rn(v0, pair(scale));
        v1 = __fmul2_rn(v1, pair(scale));
        if (BOUND) {
            v0 = make_float2(Act<T>::round(v0.x), Act<T>::round(v0.y));
            v1 = make_float2(Act<T>::round(v1.x), Act<T>::round(v1.y));
        }
        v0 = __fmul2_rn(v0, make_float2(g.x, g.y));
        v1 = __fmul2_rn(v1, make_float2(g.z, g.w));
        if (LAYER) {
            const float4 b = bs[i * (N / 4) + q];
            v0 = __fadd2_rn(v0, make_float2(b.x, b.y));
            v1 = __fadd2_rn(v1, make_float2(b.z, b.w));
        }
        h[4 * q] = v0.x;
        h[4 * q + 1] = v0.y;
        h[4 * q + 2] = v1.x;
        h[4 * q + 3] = v1.y;
    }
    return Chunk<T>::pack(h);
}

// Shared memory of a CTA whose rows fill its CPL chunks per lane: two rows (x, r)
// per warp plus gamma (and beta) in F32.  When 4 such CTAs do not fit an SM
// (228 KB, 1 KB reserved per CTA), the register cap is that of 3 CTAs (~85)
// instead of 64: at dim 1536 F16 LayerNorm (60 KB) the 64-register schedule
// cost ~0.25 us at config 1, and RMSNorm / LayerNorm with 8 chunks spilled.
template <typename T, bool LAYER, int CPL>
constexpr int regs_min_ctas() {
    constexpr int smem = kRegsWarps * 2 * CPL * 32 * 16 + (LAYER ? 2 : 1) * CPL * 32 * Chunk<T>::kN * 4;
    return 4 * (smem + 1024) <= 228 * 1024 ? 4 : 3;
}

template <typename T, bool LAYER, bool BOUND, int CPL>
__global__ void __launch_bounds__(kRegsWarps * 32, regs_min_ctas<T, LAYER, CPL>()) add_norm_regs_kernel(const NormArgs a) {
    extern __shared__ uint4 sbuf[];
    constexpr int N = Chunk<T>::kN;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int chunks = a.dim / N;   // 16-byte chunks of a row
    const int pchunks = a.dim / 4;  // 16-byte chunks of gamma / beta
    float4 *gs = reinterpret_cast<float4 *>(sbuf);
    float4 *bs = gs + pchunks;
    uint4 *xs = reinterpret_cast<uint4 *>(gs + (LAYER ? 2 : 1) * pchunks) + static_cast<size_t>(warp) * 2 * chunks;
    uint4 *rs = xs + chunks;
    const bool has_r = a.r != nullptr;
    const bool has_h = has_r && a.h_out != nullptr;
    const float inv_dim = 1.0f / static_cast<float>(a.dim);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * warps;
    const size_t row_bytes = static_cast<size_t>(a.dim) * sizeof(T);
    // number of this lane's chunks inside the row (chunks lane, lane + 32, ...)
    const int mine = chunks > lane ? (chunks - lane + 31) / 32 : 0;

    auto issue_row = [&](int64_t row) {
        const char *xg = static_cast<const char *>(a.x) + row * row_bytes;
        const char *rg = static_cast<const char *>(a.r) + row * row_bytes;
#pragma unroll
        for (int k = 0; k < CPL; ++k)
            if (k < mine) cp_async16(xs + lane + 32 * k, xg + 16 * (lane + 32 * k));
        if (has_r) {
#pragma unroll
            for (int k = 0; k < CPL; ++k)
                if (k < mine) cp_async16(rs + lane + 32 * k, rg + 16 * (lane + 32 * k));
        }
    };

    // group 0: the CTA's gamma / beta; group 1: this warp's first row
    for (int i = threadIdx.x; i < pchunks; i += blockDim.x) {
        cp_async16(gs + i, a.gamma + 4 * i);
        if (LAYER) cp_async16(bs + i, a.beta + 4 * i);
    }
    cp_async_commit();
    int64_t row = static_cast<int64_t>(blockIdx.x) * warps + warp;
    if (row < a.rows) issue_row(row);
    cp_async_commit();
    cp_async_wait_group<1>();
    __syncthreads();  // every thread's share of gamma / beta has landed

    for (; row < a.rows; row += stride) {
        cp_async_wait_group<0>();
        __syncwarp();
        // h = x + r (rounded to T), held packed; paired partial sums per chunk
        uint4 hreg[CPL];
        float sum = 0.f;
        if (has_r) {
#pragma unroll
            for (int k = 0; k < CPL; ++k)
                if (k < mine) hreg[k] = Chunk<T>::add(xs[lane + 32 * k], rs[lane + 32 * k]);
        } else {
#pragma unroll
            for (int k = 0; k < CPL; ++k)
                if (k < mine) hreg[k] = xs[lane + 32 * k];
        }
        // the row is in registers: the next row's copies go out now, and h
        // leaves before the reductions so its stores drain under their latency
        __syncwarp();
        const int64_t next = row + stride;
        if (next < a.rows) issue_row(next);
        cp_async_commit();
        if (has_h) {
            uint4 *hg = reinterpret_cast<uint4 *>(static_cast<char *>(a.h_out) + row * row_bytes);
#pragma unroll
            for (int k = 0; k < CPL; ++k)
                if (k < mine) hg[lane + 32 * k] = hreg[k];
        }

        float mean = 0.f, scale;
        if (LAYER) {
            // One pass over the registers: sums of d = h - K and of d^2 around
            // the row's first value K (shifted data: no cancellation between
            // E[d^2] and E[d]^2 when |mean| >> stddev), then
            // mean = K + E[d], var = E[d^2] - E[d]^2.
            const float K = __shfl_sync(0xffffffffu, Chunk<T>::first(hreg[0]), 0);
            float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < CPL; ++k) {
                if (k < mine) {
                    float2 d[N / 2];
                    Chunk<T>::minus(hreg[k], K, d);
#pragma unroll
                    for (int j = 0; j < N / 2; ++j) {
                        s1 = __fadd2_rn(s1, d[j]);
                        s2 = __ffma2_rn(d[j], d[j], s2);
                    }
                }
            }
            float sd = s1.x + s1.y, sq = s2.x + s2.y;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                sd += __shfl_xor_sync(0xffffffffu, sd, o);
                sq += __shfl_xor_sync(0xffffffffu, sq, o);
            }
            const float md = sd * inv_dim;
            const float var = fmaxf(__fsub_rn(sq * inv_dim, md * md), 0.f);
            mean = __fadd_rn(K, md);
            scale = 1.0f / sqrtf(var + a.eps);
        } else {
#pragma unroll
            for (int k = 0; k < CPL; ++k)
                if (k < mine) sum += Chunk<T>::sq_sum(hreg[k]);
            sum = warp_sum(sum);
            scale = 1.0f / sqrtf(sum * inv_dim + a.eps);
        }
        uint4 *yg = reinterpret_cast<uint4 *>(static_cast<char *>(a.y_out) + row * row_bytes);
#pragma unroll
        for (int k = 0; k < CPL; ++k)
            if (k < mine)
                yg[lane + 32 * k] = norm_chunk_out<T, LAYER, BOUND>(hreg[k], gs, bs, lane + 32 * k, mean, scale);
    }
    cp_async_wait_group<0>();  // nothing of this thread's is left in flight at exit
}

// Launches the register form when the row fits it; returns false (nothing
// launched) otherwise.  CTAs of kRegsWarps warps; grid: a whole number of CTAs
// per SM, enough for about kRegsRowsPerWarp rows per warp, at most the
// resident capacity.  (Measured at [4096, 1536] F16: 8-warp CTAs with about
// two rows per warp beat one wave of 8- or 16-warp CTAs and three rows per
// warp, for both norms.)
template <typename T, bool LAYER, bool BOUND, int CPL>
bool launch_regs_cpl(const NormArgs &a, cudaStream_t stream) {
    auto kernel = add_norm_regs_kernel<T, LAYER, BOUND, CPL>;
    const size_t param_bytes = static_cast<size_t>(LAYER ? 2 : 1) * a.dim * sizeof(float);
    const size_t smem = param_bytes + static_cast<size_t>(kRegsWarps) * 2 * a.dim * sizeof(T);
    if (smem > kStagedMaxSmem) return false;
    int resident = 0;
    if (resident_ctas(reinterpret_cast<const void *>(kernel), kRegsWarps * 32, smem, &resident) != cudaSuccess) {
        cudaGetLastError();  // clear the failed opt-in; the caller falls back
        return false;
    }
    if (resident <= 0) return false;
    const int64_t sms = sm_count();
    const int64_t ctas_needed = (a.rows + kRegsWarps - 1) / kRegsWarps;
    int64_t per_sm = (a.rows + sms * kRegsWarps * kRegsRowsPerWarp - 1) / (sms * kRegsWarps * kRegsRowsPerWarp);
    per_sm = std::min<int64_t>(std::max<int64_t>(per_sm, 1), resident);
    const int64_t grid = std::min<int64_t>(ctas_needed, sms * per_sm);
    kernel<<<static_cast<unsigned>(grid), kRegsWarps * 32, smem, stream>>>(a);
    return true;
}

template <typename T, bool LAYER, bool BOUND>
bool launch_regs_b(const NormArgs &a, int cpl, cudaStream_t stream) {
    switch (cpl) {
        case 1: return launch_regs_cpl<T, LAYER, BOUND, 1>(a, stream);
        case 2: return launch_regs_cpl<T, LAYER, BOUND, 2>(a, stream);
        case 3: return launch_regs_cpl<T, LAYER, BOUND, 3>(a, stream);
        case 4: return launch_regs_cpl<T, LAYER, BOUND, 4>(a, stream);
        case 5:
        case 6: return launch_regs_cpl<T, LAYER, BOUND, 6>(a, stream);
        case 7:
        case 8: return launch_regs_cpl<T, LAYER, BOUND, 8>(a, stream);
        default: return false;
    }
}

template <typename T, bool LAYER>
bool launch_regs(const NormArgs &a, int cpl, cudaStream_t stream) {
    if constexpr (sizeof(T) == 2) {
        if (a.f16_boundary) return launch_regs_b<T, LAYER, true>(a, cpl, stream);
    }
    return launch_regs_b<T, LAYER, false>(a, cpl, stream);
}

// Fallback: one CTA per row, any dim and alignment.
template <typename T, bool LAYER>
__global__ void __launch_bounds__(kThreads) add_norm_scalar_kernel(const NormArgs a) {
    __shared__ float red[kThreads / 32];
    const float inv_dim = 1.0f / static_cast<float>(a.dim);
    for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const int64_t base = row * a.dim;
        const int64_t mod_off = a.batch_rows > 0 ? (row / a.batch_rows) * a.dim : 0;
        auto hval = [&](int j) {
            float v = Act<T>::load1(a.x, base + j);
            if (a.gate) {
                v = __fmul_rn(v, a.gate[mod_off + j]);
                if (a.r) v = __fadd_rn(v, Act<T>::load1(a.r, base + j));
                v = Act<T>::round(v);
            } else if (a.r) {
                v = Act<T>::round(__fadd_rn(v, Act<T>::load1(a.r, base + j)));
            }
            return v;
        };
        float sum = 0.f;
        for (int j = threadIdx.x; j < a.dim; j += kThreads) {
            const float v = hval(j);
            sum += LAYER ? v : v * v;
        }
        __syncthreads();
        sum = warp_sum(sum);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
        __syncthreads();
        sum = 0.f;
        for (int w = 0; w < kThreads / 32; ++w) sum += red[w];
        float mean = 0.f, scale;
        if (LAYER) {
            mean = sum * inv_dim;
            float sq = 0.f;
            for (int j = threadIdx.x; j < a.dim; j += kThreads) {
                const float d = __fsub_rn(hval(j), mean);
                sq += d * d;
            }
            __syncthreads();
            sq = warp_sum(sq);
            if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
            __syncthreads();
            sq = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) sq += red[w];
            scale = 1.0f / sqrtf(sq * inv_dim + a.eps);
        } else {
            scale = 1.0f / sqrtf(sum * inv_dim + a.eps);
        }
        for (int j = threadIdx.x; j < a.dim; j += kThreads) {
            const float v = hval(j);
            if (a.h_out && (a.r || a.gate)) Act<T>::store1(a.h_out, base + j, v);
            const float n = LAYER ? __fmul_rn(__fsub_rn(v, mean), scale) : __fmul_rn(v, scale);
            float y = norm_output<T, LAYER>(a, n, a.gamma[j], LAYER ? a.beta[j] : 0.f);
            y = modulate(a, y, a.scale ? a.scale[mod_off + j] : 0.f, a.shift ? a.shift[mod_off + j] : 0.f);
            Act<T>::store1(a.y_out, base + j, y);
        }
    }
}

template <typename T, int VPL, bool LAYER, bool MOD>
void launch_vec(const NormArgs &a, cudaStream_t stream) {
    const int groups = kThreads / (32 * a.wpr);
    const int64_t grid = std::min<int64_t>((a.rows + groups - 1) / groups,
                                           static_cast<int64_t>(sm_count()) * 64);
    add_norm_vec_kernel<T, VPL, LAYER, MOD><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(a);
}

template <typename T, bool LAYER, bool MOD = false>
int run_norm(const char *what, const void *x, const void *r, const float *gamma, const float *beta,
             void *h_out, void *y_out, int64_t rows, int64_t dim, float eps, uint32_t flags,
             cudaStream_t stream, const float *gate = nullptr, const float *mscale = nullptr,
             const float *mshift = nullptr, int64_t batch_rows = 0) {
    clear_error();
    const std::string w(what);
    if (rows < 0 || dim < 0) return set_error(LEVO_OPS_EINVAL, w + ": negative shape");
    if (!(eps >= 0.f) || !std::isfinite(eps))
        return set_error(LEVO_OPS_EINVAL, w + ": eps must be finite and non-negative");
    if (flags & ~LEVO_NORM_F16_BOUNDARY) return set_error(LEVO_OPS_EINVAL, w + ": unknown flag bits");
    if ((flags & LEVO_NORM_F16_BOUNDARY) && sizeof(T) != 2)
        return set_error(LEVO_OPS_EINVAL, w + ": the F16 boundary flag needs F16 activations");
    if (rows == 0 || dim == 0) return LEVO_OPS_OK;  // empty: nothing to read or write
    if (x == nullptr || y_out == nullptr || gamma == nullptr || (LAYER && beta == nullptr))
        return set_error(LEVO_OPS_EINVAL, w + ": required pointer is null");
    const void *ptrs[6] = {x, r, h_out, y_out, gamma, beta};
    for (int i = 0; i < 6; ++i)
        if (ptrs[i] && !aligned_to(ptrs[i], i < 4 ? sizeof(T) : 4))
            return set_error(LEVO_OPS_EINVAL, w + ": pointer is not aligned to its element size");
    if (dim > (1 << 20)) return set_error(LEVO_OPS_EUNSUPPORTED, w + ": dim above 1048576");

    if (MOD && (batch_rows <= 0 || rows % batch_rows != 0))
        return set_error(LEVO_OPS_EINVAL, w + ": batch_rows must be positive and divide rows");
    const void *mods[3] = {gate, mscale, mshift};
    for (const void *m : mods)
        if (m && !aligned_to(m, 4))
            return set_error(LEVO_OPS_EINVAL, w + ": pointer is not aligned to its element size");
    NormArgs a{x, r, gamma, beta, h_out, y_out, rows, static_cast<int>(dim), 1, eps,
               (flags & LEVO_NORM_F16_BOUNDARY) ? 1 : 0, gate, mscale, mshift, MOD ? batch_rows : 0};
    {
        const size_t smem = static_cast<size_t>(kStagedRows) * 2 * dim * sizeof(T);
        bool staged = (dim * sizeof(T)) % 16 == 0 && dim % 4 == 0 && smem <= kStagedMaxSmem;
        for (int i = 0; i < 6 && staged; ++i)
            if (ptrs[i] && !aligned_to(ptrs[i], 16)) staged = false;
        for (const void *m : mods)
            if (m && !aligned_to(m, 16)) staged = false;
        if constexpr (!MOD) {
            const int64_t chunks = dim * static_cast<int64_t>(sizeof(T)) / 16;
            const int cpl = static_cast<int>((chunks + 31) / 32);
            if (staged && cpl <= kRegsMaxCpl && launch_regs<T, LAYER>(a, cpl, stream)) return check_launch(what);
        }
        if (staged) {
            auto kernel = add_norm_staged_kernel<T, LAYER, MOD>;
            int per_sm = 0;
            if (resident_ctas(reinterpret_cast<const void *>(kernel), kStagedRows * 32, smem, &per_sm) !=
                cudaSuccess) {
                cudaGetLastError();  // clear the failed opt-in; fall back to the register form
                staged = false;
            }
            if (staged) {
                const int64_t grid = std::min<int64_t>((rows + kStagedRows - 1) / kStagedRows,
                                                       static_cast<int64_t>(sm_count()) * per_sm);
                kernel<<<static_cast<unsigned>(grid), kStagedRows * 32, smem, stream>>>(a);
                return check_launch(what);
            }
        }
    }
    constexpr int VE = Act<T>::kVec;
    constexpr int kMaxVpl = sizeof(T) == 2 ? 4 : 8;  // <= 64 F32 values per thread
    bool vec = (dim * sizeof(T)) % 32 == 0 && (dim % 8 == 0);
    for (int i = 0; i < 6 && vec; ++i)
        if (ptrs[i] && !aligned_to(ptrs[i], 32)) vec = false;
    for (const void *m : mods)
        if (m && !aligned_to(m, 32)) vec = false;
    int vpl = 0;
    if (vec) {
        const int nvec = static_cast<int>(dim / VE);
        // Fewest warps per row whose share fits the register budget; prefer
        // <= 3 vectors per thread (lean registers) when a wider group allows it.
        for (int pass = 0; pass < 2 && vpl == 0; ++pass) {
            const int limit = pass == 0 ? 3 : kMaxVpl;
            for (int wpr = 1; wpr <= 8; wpr *= 2) {
                const int need = (nvec + 32 * wpr - 1) / (32 * wpr);
                if (need <= limit) {
                    a.wpr = wpr;
                    vpl = need;
                    break;
                }
            }
        }
        if (vpl == 0) vec = false;
    }
    if (vec) {
        // Instantiated vectors-per-thread: 1,2,3,4 (+6,8 for F32); a larger
        // count than needed is masked per vector.
        if (vpl == 1) {
            launch_vec<T, 1, LAYER, MOD>(a, stream);
        } else if (vpl == 2) {
            launch_vec<T, 2, LAYER, MOD>(a, stream);
        } else if (vpl == 3) {
            launch_vec<T, 3, LAYER, MOD>(a, stream);
        } else if (vpl == 4) {
            launch_vec<T, 4, LAYER, MOD>(a, stream);
        } else if constexpr (sizeof(T) == 4) {
            if (vpl <= 6) launch_vec<T, 6, LAYER, MOD>(a, stream);
            else launch_vec<T, 8, LAYER, MOD>(a, stream);
        }
    } else {
        const int64_t grid = std::min<int64_t>(rows, static_cast<int64_t>(sm_count()) * 8);
        add_norm_scalar_kernel<T, LAYER><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(a);
    }
    return check_launch(what);
}

}  // namespace
}  // namespace levo

extern "C" {

LEVO_OPS_API int levo_add_rmsnorm_f16(const void *x, const void *r, const float *gamma, void *h_out,
                                      void *y_out, int64_t rows, int64_t dim, float eps,
                                      uint32_t flags, levo_stream_t stream) {
    return levo::run_norm<__half, false>("levo_add_rmsnorm_f16", x, r, gamma, nullptr, h_out, y_out,
                                         rows, dim, eps, flags,
                                         reinterpret_cast<cudaStream_t>(stream));
}

LEVO_OPS_API int levo_add_rmsnorm_f32(const float *x, const float *r, const float *gamma,
                                      float *h_out, float *y_out, int64_t rows, int64_t dim,
                                      float eps, uint32_t flags, levo_stream_t stream) {
    return levo::run_norm<float, false>("levo_add_rmsnorm_f32", x, r, gamma, nullptr, h_out, y_out,
                                        rows, dim, eps, flags,
                                        reinterpret_cast<cudaStream_t>(stream));
}

LEVO_OPS_API int levo_add_layernorm_f16(const void *x, const void *r, const float *gamma,
                                        const float *beta, void *h_out, void *y_out, int64_t rows,
                                        int64_t dim, float eps, uint32_t flags,
                                        levo_stream_t stream) {
    return levo::run_norm<__half, true>("levo_add_layernorm_f16", x, r, gamma, beta, h_out, y_out,
                                        rows, dim, eps, flags,
                                        reinterpret_cast<cudaStream_t>(stream));
}

LEVO_OPS_API int levo_gated_layernorm_modulate_f32(const float *x, const float *gate, const float *r,
                                                   const float *gamma, const float *beta,
                                                   const float *scale, const float *shift,
                                                   int64_t batch_rows, float *h_out, float *y_out,
                                                   int64_t rows, int64_t dim, float eps,
                                                   levo_stream_t stream) {
    return levo::run_norm<float, true, true>("levo_gated_layernorm_modulate_f32", x, r, gamma, beta, h_out,
                                             y_out, rows, dim, eps, 0,
                                             reinterpret_cast<cudaStream_t>(stream), gate, scale, shift,
                                             batch_rows);
}

LEVO_OPS_API int levo_add_layernorm_f32(const float *x, const float *r, const float *gamma,
                                        const float *beta, float *h_out, float *y_out,
                                        int64_t rows, int64_t dim, float eps, uint32_t flags,
                                        levo_stream_t stream) {
    return levo::run_norm<float, true>("levo_add_layernorm_f32", x, r, gamma, beta, h_out, y_out,
                                       rows, dim, eps, flags,
                                       reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
