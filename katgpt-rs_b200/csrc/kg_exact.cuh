// kg_exact.cuh — device arithmetic in the reference's x86-64 AVX2 operation order.
//
// Files that include this header are compiled with -fmad=false so that a*b+c is
// never contracted; an FMA appears only where the reference issues one
// (_mm256_fmadd_ps), written here as fmaf(). Division and sqrtf are IEEE
// round-to-nearest (nvcc defaults -prec-div=true -prec-sqrt=true), denormals are
// kept (no -ftz), matching x86 SSE/AVX without flush-to-zero.
//
// Lane model: an AVX2 accumulator is 8 lanes; the reference's dot product
// (crates/katgpt-types/src/simd/dot.rs:157-229) keeps 4 accumulators over 32-wide
// chunks, so element k of a 32-chunk feeds lane-chain L = k mod 32 = 8*j + l.
// The chains are combined as ((acc0+acc1)+(acc2+acc3)) lane-wise and then
// reduced by horizontal_sum_256 (simd/horizontal.rs:31-51):
// ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)).
//
// The header also compiles as plain C++ (g++ -ffp-contract=off), so that the
// CPU tests can hold these helpers against the oracle bit for bit.
#pragma once
#include <cstdint>
#ifdef __CUDACC__
#include <cuda_runtime.h>
#else
#include <algorithm>
#include <cmath>
#include <cstring>
#define __device__
#define __forceinline__ inline
inline float __uint_as_float(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
inline float __int_as_float(int32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
using std::isnan;
using std::max;
using std::min;
#endif

namespace kgx {

__device__ __forceinline__ float hsum8(const float *v) {
    float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    return (s0 + s1) + (s2 + s3);
}

// simd_dot_f32, compile-time length. a/b may live in registers or memory.
template <int LEN, typename A, typename B>
__device__ __forceinline__ float dot(const A &a, const B &b) {
    constexpr int C4 = LEN / 32;
    constexpr int REM = (LEN - C4 * 32) / 8;
    constexpr int T0 = C4 * 32 + REM * 8;
    float sum;
    if constexpr (C4 > 0) {
        float acc[32];
#pragma unroll
        for (int l = 0; l < 32; ++l) acc[l] = 0.0f;
#pragma unroll
        for (int c = 0; c < C4; ++c)
#pragma unroll
            for (int l = 0; l < 32; ++l) acc[l] = fmaf(a[32 * c + l], b[32 * c + l], acc[l]);
        float t[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) t[l] = (acc[l] + acc[8 + l]) + (acc[16 + l] + acc[24 + l]);
        sum = hsum8(t);
    } else {
        sum = 0.0f;
    }
    float r[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) r[l] = 0.0f;
#pragma unroll
    for (int c = 0; c < REM; ++c)
#pragma unroll
        for (int l = 0; l < 8; ++l) r[l] = fmaf(a[C4 * 32 + 8 * c + l], b[C4 * 32 + 8 * c + l], r[l]);
    sum = sum + hsum8(r);
#pragma unroll
    for (int i = T0; i < LEN; ++i) sum = sum + a[i] * b[i];
    return sum;
}

// simd_dot_f32 for a run-time length len <= 16 (no 32-element chunks): the
// 8-lane FMA chunks, +0 + hsum, then the scalar tail. Unrolled with
// predicates so register arrays stay in registers; reads a[i], b[i] for i < len only.
template <typename A, typename B>
__device__ __forceinline__ float dot_rt16(const A &a, const B &b, int len) {
    const int chunks = len >> 3;
    float r[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) r[l] = 0.0f;
#pragma unroll
    for (int c = 0; c < 2; ++c)
        if (c < chunks) {
#pragma unroll
            for (int l = 0; l < 8; ++l) r[l] = fmaf(a[8 * c + l], b[8 * c + l], r[l]);
        }
    float sum = 0.0f;
    sum = sum + hsum8(r);
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (i >= chunks * 8 && i < len) sum = sum + a[i] * b[i];
    return sum;
}

// lora_apply (crates/katgpt-types/src/lora.rs:452-467) for an adapter of at
// most 16 x 16 x rank 16: buf = A @ in (matmul: row dots over in_dim), then
// out[r] += scale * dot(B_r, buf) for r < out_dim, the product rounded before
// the add; scale = alpha / rank. A [rank][in_dim], B [out_dim][rank].
template <typename O, typename I>
__device__ __forceinline__ void lora_apply16(O &out, const I &in, const float *A, const float *B, int rank, int in_dim,
                                             int out_dim, float scale) {
    float buf[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) buf[j] = j < rank ? dot_rt16(A + j * in_dim, in, in_dim) : 0.0f;
#pragma unroll
    for (int r = 0; r < 16; ++r)
        if (r < out_dim) out[r] = out[r] + scale * dot_rt16(B + r * rank, buf, rank);
}

// simd_sum_sq (simd/research.rs:298-338): 2 accumulators over 16-chunks.
template <int LEN, typename A>
__device__ __forceinline__ float sum_sq(const A &x) {
    constexpr int C2 = LEN / 16;
    constexpr int REM = (LEN - C2 * 16) / 8;
    constexpr int T0 = C2 * 16 + REM * 8;
    float a0[8], a1[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) a0[l] = a1[l] = 0.0f;
#pragma unroll
    for (int c = 0; c < C2; ++c)
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            a0[l] = fmaf(x[16 * c + l], x[16 * c + l], a0[l]);
            a1[l] = fmaf(x[16 * c + 8 + l], x[16 * c + 8 + l], a1[l]);
        }
    float t[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) t[l] = a0[l] + a1[l];
    float sum = hsum8(t);
    float r[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) r[l] = 0.0f;
#pragma unroll
    for (int c = 0; c < REM; ++c)
#pragma unroll
        for (int l = 0; l < 8; ++l) r[l] = fmaf(x[C2 * 16 + 8 * c + l], x[C2 * 16 + 8 * c + l], r[l]);
    sum = sum + hsum8(r);
#pragma unroll
    for (int i = T0; i < LEN; ++i) sum = sum + x[i] * x[i];
    return sum;
}

// simd_sum_f32 (simd/elementwise.rs:1004-1050) over a runtime length n <= MAXN
// (entries at index >= n are ignored). 4 accumulators over 32-chunks.
template <int MAXN>
__device__ __forceinline__ float sum_rt(const float (&x)[MAXN], int n) {
    static_assert(MAXN % 8 == 0, "MAXN must be a multiple of 8");
    const int c4 = n / 32;
    const int rem = (n - c4 * 32) / 8;
    float acc[32];
#pragma unroll
    for (int l = 0; l < 32; ++l) acc[l] = 0.0f;
    // 8-chunk k belongs to accumulator (k mod 4) while k < 4*c4.
#pragma unroll
    for (int k = 0; k < MAXN / 8; ++k)
        if (k < c4 * 4)
#pragma unroll
            for (int l = 0; l < 8; ++l) acc[(k & 3) * 8 + l] = acc[(k & 3) * 8 + l] + x[8 * k + l];
    float t[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) t[l] = (acc[l] + acc[8 + l]) + (acc[16 + l] + acc[24 + l]);
    float sum = hsum8(t);
    float r[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) r[l] = 0.0f;
#pragma unroll
    for (int k = 0; k < MAXN / 8; ++k)
        if (k >= c4 * 4 && k < c4 * 4 + rem)
#pragma unroll
            for (int l = 0; l < 8; ++l) r[l] = r[l] + x[8 * k + l];
    sum = sum + hsum8(r);
    const int t0 = c4 * 32 + rem * 8;
#pragma unroll
    for (int i = 0; i < MAXN; ++i)
        if (i >= t0 && i < n) sum = sum + x[i];
    return sum;
}

// simd_sum_f32 over x[0..n) for n < 32 (no 32-wide chunk): sum = hsum(0),
// then one accumulator over 8-chunks, then the scalar tail.
template <int MAXN>
__device__ __forceinline__ float sum_small(const float *x, int n) {
    static_assert(MAXN < 32, "sum_small handles n < 32");
    float r[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) r[l] = 0.0f;
    const int rem = n / 8;
#pragma unroll 1
    for (int c = 0; c < rem; ++c)
#pragma unroll
        for (int l = 0; l < 8; ++l) r[l] = r[l] + x[8 * c + l];
    float z[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    float sum = hsum8(z);
    sum = sum + hsum8(r);
#pragma unroll 1
    for (int i = rem * 8; i < n; ++i) sum = sum + x[i];
    return sum;
}

// ---- Cephes exp (crates/katgpt-types/src/simd/activations.rs:18-20,189-221,405-480,660-748)
__device__ __forceinline__ float cephes_poly(float g) {
    float p6 = 1.0f + g * (1.0f / 6.0f);
    float p5 = 1.0f + (g * 0.2f) * p6;
    float p4 = 1.0f + (g * 0.25f) * p5;
    float p3 = 1.0f + (g * (1.0f / 3.0f)) * p4;
    float p2 = 1.0f + (g * 0.5f) * p3;
    return 1.0f + g * p2;
}
constexpr float kLn2Hi = 6.9314575e-1f;
constexpr float kLn2Lo = 1.4286068e-6f;
constexpr float kInvLn2 = 1.44269504088896340736f;

// One AVX2 lane: n = round-half-even(x*log2e); `clamp` selects the
// exp_inplace form (n clamped to [-126,127]) vs the exp_sum_inplace form.
__device__ __forceinline__ float cephes_lane(float x, bool clamp) {
    float nf = rintf(x * kInvLn2);
    int32_t ni;
    if (isnan(nf) || nf >= 2147483648.0f || nf < -2147483648.0f) ni = INT32_MIN;
    else ni = (int32_t)nf;
    float g = (x - nf * kLn2Hi) - nf * kLn2Lo;
    float q = cephes_poly(g);
    int32_t e = ni;
    if (clamp) e = max(min(e, 127), -126);
    uint32_t bits = ((uint32_t)e + 127u) << 23;
    return __uint_as_float(bits) * q;
}
// Scalar tail (cephes_exp_scalar): round half away from zero, early exits.
__device__ __forceinline__ float cephes_scalar(float x) {
    float rf = roundf(x * kInvLn2);
    int32_t n;
    if (isnan(rf)) n = 0;
    else if (rf >= 2147483648.0f) n = INT32_MAX;
    else if (rf <= -2147483648.0f) n = INT32_MIN;
    else n = (int32_t)rf;
    if (n < -126) return 0.0f;
    if (n > 127) return __int_as_float(0x7f800000);
    float nf = (float)n;
    float g = (x - nf * kLn2Hi) - nf * kLn2Lo;
    return __uint_as_float((uint32_t)(n + 127) << 23) * cephes_poly(g);
}

// libm expf as the sp_kv path calls it (f32::exp -> glibc expf, which is
// within 0.502 ulp): evaluated in double and rounded once, so the result is
// the correctly rounded value.
__device__ __forceinline__ float expf_libm(float x) { return (float)exp((double)x); }

// f32::max (NaN operand ignored)
__device__ __forceinline__ float fmax_rs(float a, float b) {
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

}  // namespace kgx
