// kg_oracle.cpp — CPU oracle (test infrastructure only; see kg_oracle.h).
//
// Restates the reference's x86-64 AVX2 path operation for operation. Build with
// -O2 -mavx2 -mfma -ffp-contract=off and WITHOUT -ffast-math: Rust never
// contracts a*b+c, so FMAs appear only where the reference uses an FMA
// intrinsic. libm calls (logf, cosf, powf, expf, log, exp, sin) are the glibc
// ones that Rust's f32/f64 methods lower to on x86-64 Linux.
//
// Every function cites the reference file:line it follows (paths relative to
// the katgpt-rs repository root).

#include "kg_oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// ------------------------------------------------------------------------
// Rng — crates/katgpt-types/src/rng.rs:26-72
// ------------------------------------------------------------------------
struct Rng {
    uint64_t state;
    explicit Rng(uint64_t seed) {
        // SplitMix64 finaliser (rng.rs:26-38)
        uint64_t z = seed + 0x9E3779B97F4A7C15ULL;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
        uint64_t s = z ^ (z >> 31);
        state = s == 0 ? 1 : s;
    }
    uint64_t next() {  // rng.rs:42-47
        state ^= state << 13;
        state ^= state >> 7;
        state ^= state << 17;
        return state;
    }
    float uniform() {  // rng.rs:56-62
        uint32_t bits = ((uint32_t)(next() >> 40) & 0x007fffffu) | 0x3f800000u;
        float f;
        std::memcpy(&f, &bits, 4);
        return f - 1.0f;
    }
    float normal() {  // rng.rs:66-71 (Box-Muller, glibc logf/cosf)
        float u1 = uniform();
        if (!(u1 > 1e-10f)) u1 = 1e-10f;  // f32::max(u1, 1e-10)
        float u2 = uniform();
        const float two_pi = 2.0f * 3.14159265358979323846f;   // 2.0 * PI (exact doubling)
        return sqrtf(-2.0f * logf(u1)) * cosf(two_pi * u2);
    }
};

// ------------------------------------------------------------------------
// Horizontal reducers — crates/katgpt-types/src/simd/horizontal.rs:10-51
// ------------------------------------------------------------------------
static inline float hsum128(__m128 v) {
    __m128 sh = _mm_shuffle_ps(v, v, 0xB1);
    __m128 s = _mm_add_ps(v, sh);
    __m128 sh2 = _mm_shuffle_ps(s, s, 0x2A);
    return _mm_cvtss_f32(_mm_add_ss(s, sh2));
}
static inline float hsum256(__m256 v) {
    return hsum128(_mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1)));
}
static inline float hmax256(__m256 v) {
    __m128 m = _mm_max_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    __m128 m2 = _mm_max_ps(m, _mm_shuffle_ps(m, m, 0xB1));
    __m128 m3 = _mm_max_ps(m2, _mm_shuffle_ps(m2, m2, 0x4E));
    return _mm_cvtss_f32(m3);
}

// f32::max (IEEE maxNum: NaN operand ignored)
static inline float fmax_rs(float a, float b) {
    if (std::isnan(a)) return b;
    if (std::isnan(b)) return a;
    return a > b ? a : b;
}

// ------------------------------------------------------------------------
// Dot product — simd/dot.rs:157-229 (avx2_dot_f32)
// ------------------------------------------------------------------------
static float dot(const float *a, const float *b, int64_t len) {
    __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
    int64_t i = 0;
    for (int64_t c = 0, n4 = len / 32; c < n4; ++c, i += 32) {
        a0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), a0);
        a1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), a1);
        a2 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 16), _mm256_loadu_ps(b + i + 16), a2);
        a3 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 24), _mm256_loadu_ps(b + i + 24), a3);
    }
    float sum = hsum256(_mm256_add_ps(_mm256_add_ps(a0, a1), _mm256_add_ps(a2, a3)));
    __m256 acc = _mm256_setzero_ps();
    for (int64_t c = 0, r = (len - i) / 8; c < r; ++c, i += 8)
        acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc);
    sum += hsum256(acc);
    for (; i < len; ++i) sum += a[i] * b[i];
    return sum;
}

// simd/research.rs:298-338 (avx2_sum_sq)
static float sum_sq(const float *x, int64_t len) {
    __m256 a0 = _mm256_setzero_ps(), a1 = a0;
    int64_t i = 0;
    for (int64_t c = 0, n2 = len / 16; c < n2; ++c, i += 16) {
        __m256 v0 = _mm256_loadu_ps(x + i);
        a0 = _mm256_fmadd_ps(v0, v0, a0);
        __m256 v1 = _mm256_loadu_ps(x + i + 8);
        a1 = _mm256_fmadd_ps(v1, v1, a1);
    }
    float sum = hsum256(_mm256_add_ps(a0, a1));
    __m256 acc = _mm256_setzero_ps();
    for (int64_t c = 0, r = (len - i) / 8; c < r; ++c, i += 8) {
        __m256 v = _mm256_loadu_ps(x + i);
        acc = _mm256_fmadd_ps(v, v, acc);
    }
    sum += hsum256(acc);
    for (; i < len; ++i) sum += x[i] * x[i];
    return sum;
}

// simd/elementwise.rs:1004-1050 (avx2_sum_f32)
static float sum_f32(const float *x, int64_t len) {
    __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
    int64_t i = 0;
    for (int64_t c = 0, n4 = len / 32; c < n4; ++c, i += 32) {
        a0 = _mm256_add_ps(a0, _mm256_loadu_ps(x + i));
        a1 = _mm256_add_ps(a1, _mm256_loadu_ps(x + i + 8));
        a2 = _mm256_add_ps(a2, _mm256_loadu_ps(x + i + 16));
        a3 = _mm256_add_ps(a3, _mm256_loadu_ps(x + i + 24));
    }
    float sum = hsum256(_mm256_add_ps(_mm256_add_ps(a0, a1), _mm256_add_ps(a2, a3)));
    __m256 acc = _mm256_setzero_ps();
    for (int64_t c = 0, r = (len - i) / 8; c < r; ++c, i += 8)
        acc = _mm256_add_ps(acc, _mm256_loadu_ps(x + i));
    sum += hsum256(acc);
    for (; i < len; ++i) sum += x[i];
    return sum;
}

// simd/elementwise.rs:348-380, 1163-1215 (simd_max_f32 / avx2_max_f32)
static float max_f32(const float *x, int64_t len) {
    if (len == 0) return -INFINITY;
    if (len < 8) {
        float m = x[0];
        for (int64_t j = 1; j < len; ++j)
            if (x[j] > m) m = x[j];
        return m;
    }
    __m256 v0 = _mm256_loadu_ps(x), v1 = v0, v2 = v0, v3 = v0;
    int64_t i = 0;
    for (int64_t c = 0, n4 = len / 32; c < n4; ++c, i += 32) {
        v0 = _mm256_max_ps(v0, _mm256_loadu_ps(x + i));
        v1 = _mm256_max_ps(v1, _mm256_loadu_ps(x + i + 8));
        v2 = _mm256_max_ps(v2, _mm256_loadu_ps(x + i + 16));
        v3 = _mm256_max_ps(v3, _mm256_loadu_ps(x + i + 24));
    }
    __m256 v = _mm256_max_ps(_mm256_max_ps(v0, v1), _mm256_max_ps(v2, v3));
    for (; i + 8 <= len; i += 8) v = _mm256_max_ps(v, _mm256_loadu_ps(x + i));
    float m = hmax256(v);
    for (; i < len; ++i)
        if (x[i] > m) m = x[i];
    return m;
}

// Elementwise kernels — simd/elementwise.rs (AVX2 bodies are one lane-wise op;
// tails restate the scalar expression as written).
static void scale_inplace(float *x, int64_t len, float s) {  // :88-113
    for (int64_t i = 0; i < len; ++i) x[i] *= s;
}
static void add_scalar_inplace(float *x, int64_t len, float v) {  // :945-965
    for (int64_t i = 0; i < len; ++i) x[i] += v;
}
static void fused_sub_scale_inplace(float *x, int64_t len, float sub, float s) {  // :967-1000
    for (int64_t i = 0; i < len; ++i) x[i] = (x[i] - sub) * s;
}
static void add_into(float *d, const float *a, const float *b, int64_t len) {  // :1141-1160
    for (int64_t i = 0; i < len; ++i) d[i] = a[i] + b[i];
}
static void add_inplace(float *d, const float *s, int64_t len) {  // :923-943
    for (int64_t i = 0; i < len; ++i) d[i] += s[i];
}
static void scale_mul_inplace(float *x, const float *g, int64_t len, float s) {  // :1249-1270
    int64_t body = len / 8 * 8;
    for (int64_t i = 0; i < body; ++i) x[i] = g[i] * (x[i] * s);   // vector: g*(x*s)
    for (int64_t i = body; i < len; ++i) x[i] = g[i] * x[i] * s;   // tail: (g*x)*s
}
// simd/research.rs:1054-1075 (avx2_fused_scale_acc): dst += s*src
static void fused_scale_acc(float *d, const float *src, float s, int64_t len) {
    int64_t body = len / 8 * 8;
    for (int64_t i = 0; i < body; ++i) d[i] = fmaf(s, src[i], d[i]);
    for (int64_t i = body; i < len; ++i) d[i] += s * src[i];
}
// simd/research.rs:967-990 (avx2_fused_sub_acc): dst += a - b
static void fused_sub_acc(float *d, const float *a, const float *b, int64_t len) {
    for (int64_t i = 0; i < len; ++i) d[i] += a[i] - b[i];
}

// ------------------------------------------------------------------------
// Cephes exp — simd/activations.rs:18-20, 189-221, 405-480, 660-748
// ------------------------------------------------------------------------
static const float kLn2Hi = 6.9314575e-1f;
static const float kLn2Lo = 1.4286068e-6f;
static const float kInvLn2 = 1.44269504088896340736f;  // std::f32::consts::LOG2_E

static inline float f32_from_bits(uint32_t b) {
    float f;
    std::memcpy(&f, &b, 4);
    return f;
}
// Rust `f as i32`: saturating, NaN -> 0
static inline int32_t sat_i32(float f) {
    if (std::isnan(f)) return 0;
    if (f >= 2147483648.0f) return INT32_MAX;
    if (f <= -2147483648.0f) return INT32_MIN;
    return (int32_t)f;
}
static inline float cephes_poly(float g) {
    const float one = 1.0f;
    float p6 = one + g * (1.0f / 6.0f);
    float p5 = one + (g * 0.2f) * p6;
    float p4 = one + (g * 0.25f) * p5;
    float p3 = one + (g * (1.0f / 3.0f)) * p4;
    float p2 = one + (g * 0.5f) * p3;
    return one + g * p2;
}
// activations.rs:189-221 (scalar tail: round half away from zero, early exits)
static float cephes_exp_scalar(float x) {
    int32_t n = sat_i32(roundf(x * kInvLn2));
    if (n < -126) return 0.0f;
    if (n > 127) return INFINITY;
    float nf = (float)n;
    float g = (x - nf * kLn2Hi) - nf * kLn2Lo;
    float q = cephes_poly(g);
    return f32_from_bits((uint32_t)(n + 127) << 23) * q;
}
// One AVX2 lane of avx2_exp_inplace (clamped) / avx2_exp_sum_inplace (unclamped).
static inline float cephes_exp_lane(float x, bool clamp) {
    float nf = nearbyintf(x * kInvLn2);  // _mm256_round_ps(.., nearest-even)
    // _mm256_cvtps_epi32 of an integral value: exact; out-of-range/NaN -> INT_MIN
    int32_t ni = (std::isnan(nf) || nf >= 2147483648.0f || nf < -2147483648.0f) ? INT32_MIN
                                                                                : (int32_t)nf;
    float g = (x - nf * kLn2Hi) - nf * kLn2Lo;
    float q = cephes_poly(g);
    int32_t e = ni;
    if (clamp) e = std::max(std::min(e, 127), -126);
    uint32_t bits = (uint32_t)((uint32_t)e + 127u) << 23;  // wrapping add, then shift
    return f32_from_bits(bits) * q;
}
static void exp_inplace(float *x, int64_t len) {  // activations.rs:405-480
    int64_t body = len / 8 * 8;
    for (int64_t i = 0; i < body; ++i) x[i] = cephes_exp_lane(x[i], true);
    for (int64_t i = body; i < len; ++i) x[i] = cephes_exp_scalar(x[i]);
}
static float exp_sum_inplace(float *x, int64_t len) {  // activations.rs:660-748
    float acc[4][8] = {};
    int64_t i = 0;
    for (int64_t c = 0, n4 = len / 32; c < n4; ++c, i += 32)
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 8; ++l) {
                float r = cephes_exp_lane(x[i + 8 * j + l], false);
                x[i + 8 * j + l] = r;
                acc[j][l] = acc[j][l] + r;
            }
    __m256 A0 = _mm256_loadu_ps(acc[0]), A1 = _mm256_loadu_ps(acc[1]);
    __m256 A2 = _mm256_loadu_ps(acc[2]), A3 = _mm256_loadu_ps(acc[3]);
    float sum = hsum256(_mm256_add_ps(_mm256_add_ps(A0, A1), _mm256_add_ps(A2, A3)));
    float rem[8] = {};
    for (int64_t c = 0, r = (len - i) / 8; c < r; ++c, i += 8)
        for (int l = 0; l < 8; ++l) {
            float e = cephes_exp_lane(x[i + l], false);
            x[i + l] = e;
            rem[l] = rem[l] + e;
        }
    sum += hsum256(_mm256_loadu_ps(rem));
    for (; i < len; ++i) {
        float e = cephes_exp_scalar(x[i]);
        x[i] = e;
        sum += e;
    }
    return sum;
}

// ------------------------------------------------------------------------
// Sparse dot — simd/sparse.rs:22-75, 159-218
// ------------------------------------------------------------------------
static float sparse_dot(const float *w, const int64_t *idx, const float *val, int64_t alive) {
    if (alive <= 4) {
        float s = 0.0f;
        for (int64_t i = 0; i < alive; ++i) s += w[idx[i]] * val[i];
        return s;
    }
    __m256 acc = _mm256_setzero_ps();
    int64_t i = 0;
    for (int64_t c = 0, n = alive / 8; c < n; ++c, i += 8) {
        __m256i vi = _mm256_set_epi32((int)idx[i + 7], (int)idx[i + 6], (int)idx[i + 5],
                                      (int)idx[i + 4], (int)idx[i + 3], (int)idx[i + 2],
                                      (int)idx[i + 1], (int)idx[i]);
        __m256 ww = _mm256_i32gather_ps(w, vi, 4);
        acc = _mm256_fmadd_ps(ww, _mm256_loadu_ps(val + i), acc);
    }
    float s = hsum256(acc);
    for (; i < alive; ++i) s += w[idx[i]] * val[i];
    return s;
}

// ------------------------------------------------------------------------
// Math — crates/katgpt-types/src/math.rs
// ------------------------------------------------------------------------
static void matmul(float *out, const float *w, const float *x, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) out[r] = dot(w + r * cols, x, cols);  // math.rs:238-240
}
static void matmul_relu(float *out, const float *w, const float *x, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {  // dot.rs:699-713
        float s = dot(w + r * cols, x, cols);
        out[r] = s > 0.0f ? s : 0.0f;
    }
}
// LoraAdapter (crates/katgpt-types/src/lora.rs:5-12): A [rank][in_dim],
// B [out_dim][rank]; lora_apply (:452-467): buf = A @ in (matmul, row dots),
// then out[r] += (alpha / rank) * dot(B_r, buf), the product rounded before the add.
struct Lora {
    int64_t rank = 0, in_dim = 0, out_dim = 0;
    float alpha = 0.0f;
    std::vector<float> a, b;
};
static void lora_apply(float *out, const Lora &lo, const float *in, float *buf) {
    const float scale = lo.alpha / (float)lo.rank;
    matmul(buf, lo.a.data(), in, lo.rank, lo.in_dim);
    for (int64_t r = 0; r < lo.out_dim; ++r) {
        const float sum = dot(&lo.b[r * lo.rank], buf, lo.rank);
        out[r] += scale * sum;
    }
}
// LoraPair (lora.rs:470-490): [0] reader (forward_prefill), [1] writer
// (forward_base); rank 0 = None
static Lora g_lora[2];

static void rmsnorm(float *x, int64_t n) {  // math.rs:56-69
    float ss = sum_sq(x, n);
    float inv = 1.0f / sqrtf(ss / (float)n + 1e-5f);
    scale_inplace(x, n, inv);
}
static void rmsnorm_gamma(float *x, const float *g, int64_t n) {  // math.rs:218-233
    float ss = sum_sq(x, n);
    float inv = 1.0f / sqrtf(ss / (float)n + (float)1e-5);
    scale_mul_inplace(x, g, n, inv);
}
// math.rs:315-355 + dot.rs/sparse.rs:300-316: returns alive count
static int64_t sparse_matmul(float *out, const float *w, const float *in, int64_t rows,
                             int64_t cols, int64_t *aidx, float *aval) {
    int64_t alive = 0;
    for (int64_t c = 0; c < cols; ++c)
        if (in[c] > 0.0f) {
            aidx[alive] = c;
            aval[alive] = in[c];
            ++alive;
        }
    for (int64_t r = 0; r < rows; ++r) out[r] = sparse_dot(w + r * cols, aidx, aval, alive);
    return alive;
}
// math.rs:36-50
static void softmax_scaled(float *x, int64_t len, float inv_temp) {
    if (len == 0) return;
    float m = max_f32(x, len);
    fused_sub_scale_inplace(x, len, m, inv_temp);
    float s = exp_sum_inplace(x, len);
    scale_inplace(x, len, 1.0f / s);
}

// ------------------------------------------------------------------------
// Model
// ------------------------------------------------------------------------
struct Dims {
    int64_t V, B, n, nh, hd, nkv, kvd, m, L, nblocks;
};
static Dims dims_of(const or_config *c) {
    Dims d;
    d.V = c->vocab_size;
    d.B = c->block_size;
    d.n = c->n_embd;
    d.nh = c->n_head;
    d.hd = c->head_dim;
    d.nkv = c->n_kv_head;
    d.kvd = (int64_t)c->n_kv_head * c->head_dim;  // config.rs:1581 kv_dim
    d.m = c->mlp_hidden;
    d.L = c->n_layer;
    d.nblocks = (d.L + 3) / 4;  // delta routing B=4 (transformer.rs:166-170)
    return d;
}
struct LayerW {
    const float *wq, *wk, *wv, *wo, *w1, *w2;
};
struct Weights {
    const float *wte, *wpe, *lm_head, *dq, *dn;
    const float *ag, *mg;  // attn_norm_gamma / mlp_norm_gamma [L][n] (weights.rs:20-25, 142-145)
    std::vector<LayerW> layers;
};
static int64_t weights_count(const Dims &d) {
    int64_t per_layer = 2 * d.n * d.n + 2 * d.kvd * d.n + 2 * d.m * d.n;
    return d.V * d.n + d.B * d.n + d.L * per_layer + d.V * d.n + 4 * d.L * d.n;
}
static Weights view_weights(const Dims &d, const float *w) {
    Weights W;
    const float *p = w;
    W.wte = p; p += d.V * d.n;
    W.wpe = p; p += d.B * d.n;
    for (int64_t l = 0; l < d.L; ++l) {
        LayerW lw;
        lw.wq = p; p += d.n * d.n;
        lw.wk = p; p += d.kvd * d.n;
        lw.wv = p; p += d.kvd * d.n;
        lw.wo = p; p += d.n * d.n;
        lw.w1 = p; p += d.m * d.n;
        lw.w2 = p; p += d.n * d.m;
        W.layers.push_back(lw);
    }
    W.lm_head = p; p += d.V * d.n;
    W.dq = p; p += d.L * d.n;
    W.dn = p; p += d.L * d.n;
    W.ag = p; p += d.L * d.n;
    W.mg = p;
    return W;
}

// transformer.rs:333-389 (attention_head, Cephes exp, AVX2 helpers)
static void attention_head(const float *q, const float *K, const float *Vc, float *out,
                           float *scores, int64_t qoff, int64_t kvoff, int64_t kvd, int64_t hd,
                           int64_t tn, float scale) {
    for (int64_t t = 0; t < tn; ++t) scores[t] = dot(q + qoff, K + t * kvd + kvoff, hd);
    scale_inplace(scores, tn, scale);
    float mx = max_f32(scores, tn);
    add_scalar_inplace(scores, tn, -mx);
    exp_inplace(scores, tn);
    float sum = sum_f32(scores, tn);
    float inv = 1.0f / sum;
    scale_inplace(scores, tn, inv);
    for (int64_t d = 0; d < hd; ++d) out[qoff + d] = 0.0f;
    for (int64_t t = 0; t < tn; ++t) fused_scale_acc(out + qoff, Vc + t * kvd + kvoff, scores[t], hd);
}

// src/sp_kv/forward.rs:166-245 (attention_head_core<GateBias>, libm expf, d-outer PV)
static void attention_head_gated(const float *q, const float *K, const float *Vc, float *out,
                                 float *scores, int64_t qoff, int64_t kvoff, int64_t kvd,
                                 int64_t hd, int64_t tn, float scale, const float *bias) {
    float mx = -INFINITY;
    for (int64_t t = 0; t < tn; ++t) {
        float b = bias[t];
        if (b == -INFINITY) {
            scores[t] = -INFINITY;
            continue;
        }
        float s = dot(q + qoff, K + t * kvd + kvoff, hd) * scale + b;
        scores[t] = s;
        mx = fmax_rs(mx, s);
    }
    float sum = 0.0f;
    for (int64_t t = 0; t < tn; ++t) {
        float e = expf(scores[t] - mx);
        scores[t] = e;
        sum += e;
    }
    float inv = 1.0f / sum;
    for (int64_t d = 0; d < hd; ++d) {
        float v = 0.0f;
        for (int64_t t = 0; t < tn; ++t) v += scores[t] * inv * Vc[t * kvd + kvoff + d];
        out[qoff + d] = v;
    }
}

// transformer.rs:1707-1765 (depth_route_with_indices) + :287-320 (depth_route_blocks)
static void depth_route(float *x, std::vector<std::vector<float>> &deltas, int64_t bidx,
                        const float *query, const float *normw, int64_t n,
                        std::vector<float> &scaled) {
    int64_t limit = std::min<int64_t>(bidx + 1, (int64_t)deltas.size());
    float logits[64];
    float mx = -INFINITY;
    for (int64_t i = 0; i < limit; ++i) {
        const float *src = deltas[i].data();
        float ss = sum_sq(src, n);
        float rms = sqrtf(ss / (float)n + 1e-5f);
        float inv = 1.0f / rms;
        std::memcpy(scaled.data(), src, n * sizeof(float));
        scale_mul_inplace(scaled.data(), normw, n, inv);
        float lg = dot(scaled.data(), query, n);
        logits[i] = lg;
        mx = fmax_rs(mx, lg);
    }
    add_scalar_inplace(logits, limit, -mx);
    exp_inplace(logits, limit);
    float se = sum_f32(logits, limit);
    float inv_sum = 1.0f / se;
    for (int64_t i = 0; i < limit; ++i)
        fused_scale_acc(x, deltas[i].data(), logits[i] * inv_sum, n);
    std::fill(deltas[bidx].begin(), deltas[bidx].end(), 0.0f);
}

// ------------------------------------------------------------------------
// TurboQuant — src/turboquant/*
// ------------------------------------------------------------------------
static int64_t packed_len(int64_t n, int bits) {  // kv_cache.rs:499-509
    switch (bits) {
        case 2: return (n + 3) / 4;
        case 3:
        case 4: return (n + 1) / 2;
        case 8: return n;
        default: return (n * bits + 7) / 8;
    }
}
static void pack_into(const uint8_t *idx, int64_t n, int bits, uint8_t *out) {  // :560-632
    int64_t pl = packed_len(n, bits);
    if (bits == 8) {
        std::memcpy(out, idx, n);
        return;
    }
    std::memset(out, 0, pl);
    if (bits == 2) {
        for (int64_t i = 0; i < n; ++i) out[i / 4] |= (uint8_t)((idx[i] & 0x3) << ((i % 4) * 2));
    } else if (bits == 3 || bits == 4) {
        for (int64_t i = 0; i < n; ++i) out[i / 2] |= (uint8_t)((idx[i] & 0xF) << ((i % 2) * 4));
    } else {
        int64_t bp = 0;
        for (int64_t i = 0; i < n; ++i, bp += bits) {
            int64_t byte = bp / 8, sh = bp % 8;
            out[byte] |= (uint8_t)(idx[i] << sh);
            if (sh + bits > 8) out[byte + 1] |= (uint8_t)(idx[i] >> (8 - sh));
        }
    }
}
static void unpack_into(const uint8_t *p, int64_t n, int bits, uint8_t *out) {  // :688-757
    if (bits == 2) {
        for (int64_t i = 0; i < n; ++i) out[i] = (p[i / 4] >> ((i % 4) * 2)) & 0x3;
    } else if (bits == 3 || bits == 4) {
        for (int64_t i = 0; i < n; ++i) out[i] = (p[i / 2] >> ((i % 2) * 4)) & 0xF;
    } else if (bits == 8) {
        std::memcpy(out, p, n);
    } else {
        uint8_t mask = (uint8_t)((1u << bits) - 1);
        int64_t bp = 0;
        for (int64_t i = 0; i < n; ++i, bp += bits) {
            int64_t byte = bp / 8, sh = bp % 8;
            uint8_t v = (p[byte] >> sh) & mask;
            if (sh + bits > 8) v |= (uint8_t)(p[byte + 1] << (8 - sh)) & mask;
            out[i] = v;
        }
    }
}

// codebook.rs:84-117 (Lanczos ln_gamma)
static double ln_gamma(double x) {
    const double g = 7.0;
    static const double coef[9] = {0.99999999999980993,  676.5203681218851,
                                   -1259.1392167224028,  771.32342877765313,
                                   -176.61502916214059,  12.507343278686905,
                                   -0.13857109526572012, 9.9843695780195716e-6,
                                   1.5056327351493116e-7};
    const double PI = 3.14159265358979323846;
    if (x < 0.5) return PI / log(sin(PI * x)) - ln_gamma(1.0 - x);
    double z = x - 1.0;
    double acc = coef[0];
    double t = z + g + 0.5;
    for (int i = 0; i < 8; ++i) acc = acc + coef[i + 1] / (z + (double)i + 1.0);
    return ((log(sqrt(2.0 * PI)) + log(t + 0.5) * (z + 0.5)) - t) + log(acc);
}
// codebook.rs:79-82
static float gamma_ratio(int64_t d) {
    double df = (double)d;
    const double PI = 3.14159265358979323846;
    double lr = ln_gamma(df / 2.0) - ln_gamma((df - 1.0) / 2.0) - log(PI / 2.0);
    return (float)exp(lr);
}
// codebook.rs:67-73
static float beta_pdf(float x, int64_t d) {
    if (fabsf(x) >= 1.0f) return 0.0f;
    float expo = (float)(d - 3) / 2.0f;
    float c = gamma_ratio(d);
    return c * powf(1.0f - x * x, expo);
}
// codebook.rs:124-158
static void compute_centroids(const std::vector<float> &bnd, int64_t dim, std::vector<float> &cent) {
    size_t n = bnd.size() + 1;
    cent.assign(n, 0.0f);
    const int ns = 1000;
    std::vector<float> edges(n + 1);
    edges[0] = -1.0f;
    for (size_t i = 0; i + 1 < n; ++i) edges[i + 1] = bnd[i];
    edges[n] = 1.0f;
    for (size_t i = 0; i < n; ++i) {
        float lo = edges[i], hi = edges[i + 1];
        float dx = (hi - lo) / (float)ns;
        double sfx = 0.0, sxfx = 0.0;
        for (int j = 0; j <= ns; ++j) {
            float x = lo + dx * (float)j;
            float pdf = beta_pdf(x, dim);
            double w = (j == 0 || j == ns) ? 0.5 : 1.0;
            sfx += (double)pdf * w;
            sxfx += (double)x * (double)pdf * w;
        }
        cent[i] = sfx > 1e-12 ? (float)(sxfx / sfx) : (lo + hi) / 2.0f;
    }
}
// codebook.rs:175-198
static float compute_mse(const std::vector<float> &bnd, const std::vector<float> &cent, int64_t dim) {
    size_t n = cent.size();
    std::vector<float> edges(n + 1);
    edges[0] = -1.0f;
    for (size_t i = 0; i + 1 < n; ++i) edges[i + 1] = bnd[i];
    edges[n] = 1.0f;
    const int ns = 500;
    double total = 0.0;
    for (size_t i = 0; i < n; ++i) {
        float lo = edges[i], hi = edges[i + 1];
        float dx = (hi - lo) / (float)ns;
        double im = 0.0;
        for (int j = 0; j <= ns; ++j) {
            float x = lo + dx * (float)j;
            float pdf = beta_pdf(x, dim);
            double w = (j == 0 || j == ns) ? 0.5 : 1.0;
            double diff = (double)x - (double)cent[i];
            im += diff * diff * (double)pdf * w;
        }
        total += im * (double)dx;
    }
    return (float)total;
}
// codebook.rs:20-60
static void codebook(int64_t dim, int bits, std::vector<float> &cent, std::vector<float> &bnd,
                     float *mse) {
    int64_t nl = (int64_t)1 << bits;
    int64_t nb = nl - 1;
    bnd.resize(nb);
    for (int64_t i = 0; i < nb; ++i) bnd[i] = -1.0f + 2.0f * (float)(i + 1) / (float)nl;
    std::vector<float> c, nbd(nb);
    for (int it = 0; it < 50; ++it) {
        compute_centroids(bnd, dim, c);
        for (int64_t i = 0; i < nb; ++i) nbd[i] = (c[i] + c[i + 1]) / 2.0f;
        bool conv = true;
        for (int64_t i = 0; i < nb; ++i)
            if (!(fabsf(bnd[i] - nbd[i]) < 1e-6f)) conv = false;
        bnd = nbd;
        if (conv) break;
    }
    compute_centroids(bnd, dim, cent);
    if (mse) *mse = compute_mse(bnd, cent, dim);
}
// rotation.rs:11-52 (modified Gram-Schmidt, scalar sequential sums)
static void rotation_from(int64_t dim, const float *mat, float *q);
static void rotation(int64_t dim, uint64_t seed, float *q) {
    Rng rng(seed);
    std::vector<float> mat(dim * dim);
    for (auto &e : mat) e = rng.normal();
    rotation_from(dim, mat.data(), q);
}
static void rotation_from(int64_t dim, const float *mat, float *q) {
    std::vector<float> v(dim * dim);
    for (int64_t col = 0; col < dim; ++col)
        for (int64_t row = 0; row < dim; ++row) v[col * dim + row] = mat[row * dim + col];
    std::fill(q, q + dim * dim, 0.0f);
    // Right-looking order: column i receives the projections of q_0, q_1, ...
    // in the same sequence (and with the same operands) as the reference's
    // left-looking loop, so every value is bit-identical; it only lets the
    // columns be updated in parallel.
    unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    std::vector<float> qj(dim);  // column j of q, contiguous (same values, same order of use)
    for (int64_t j = 0; j < dim; ++j) {
        float *vj = &v[j * dim];
        float nrm = sqrtf(sum_sq(vj, dim));
        std::fill(qj.begin(), qj.end(), 0.0f);
        if (nrm > 1e-8f)
            for (int64_t k = 0; k < dim; ++k) q[k * dim + j] = qj[k] = vj[k] / nrm;
        auto work = [&](int64_t i0, int64_t i1) {
            for (int64_t i = i0; i < i1; ++i) {
                float *vi = &v[i * dim];
                float d = -0.0f;  // Iterator::<f32>::sum starts at -0.0
                for (int64_t k = 0; k < dim; ++k) d = d + qj[k] * vi[k];
                for (int64_t k = 0; k < dim; ++k) vi[k] -= d * qj[k];
            }
        };
        int64_t rem = dim - (j + 1);
        if (rem <= 0) continue;
        if (rem < 64 || nt == 1) {
            work(j + 1, dim);
        } else {
            std::vector<std::thread> th;
            int64_t per = (rem + nt - 1) / nt;
            for (unsigned t = 0; t < nt; ++t) {
                int64_t a = j + 1 + t * per, b = std::min<int64_t>(dim, a + per);
                if (a < b) th.emplace_back(work, a, b);
            }
            for (auto &t : th) t.join();
        }
    }
}
static inline uint8_t quantize(const float *bnd, int64_t nb, float v) {  // codebook.rs:202-204
    int64_t c = 0;
    while (c < nb && v >= bnd[c]) ++c;  // partition_point(|b| v >= b) on monotone boundaries
    return (uint8_t)c;
}

struct TQ {
    int64_t dim;
    int kbits, vbits;
    std::vector<float> rot, rot_t, kc, kb, vc, vb;
};
// `timing`: tables for the CPU-baseline timing harness only, whose rotation is
// a scaled Gaussian matrix of the same size instead of the O(dim^3) MGS
// orthogonalisation (the encode / dequant work per vector is the same dim^2
// dot products either way).
static const TQ &tq_tables(int64_t dim, int kbits, int vbits, bool timing = false) {
    // small process-wide cache (tables are deterministic in (dim, bits))
    static std::vector<std::pair<bool, TQ *>> cache;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : cache)
        if (e.first == timing && e.second->dim == dim && e.second->kbits == kbits && e.second->vbits == vbits)
            return *e.second;
    TQ *t = new TQ;
    t->dim = dim;
    t->kbits = kbits;
    t->vbits = vbits;
    t->rot.resize(dim * dim);
    if (timing) {
        Rng g(42);
        const float sc = 1.0f / sqrtf((float)dim);
        for (auto &v : t->rot) v = g.uniform() * 2.0f * sc - sc;
    } else {
        rotation(dim, 42, t->rot.data());  // kv_cache.rs:63-77: seed 42, shared by layers
    }
    t->rot_t.resize(dim * dim);
    for (int64_t i = 0; i < dim; ++i)
        for (int64_t j = 0; j < dim; ++j) t->rot_t[i * dim + j] = t->rot[j * dim + i];
    codebook(dim, kbits, t->kc, t->kb, nullptr);
    codebook(dim, vbits, t->vc, t->vb, nullptr);
    cache.push_back({timing, t});
    return *t;
}

// kv_cache.rs:156-195 (store_key / store_value)
static void tq_store(const float *rot, const float *bnd, int bits, int64_t dim, const float *x,
                     uint8_t *packed, float *norm_out, float *scratch_n, float *scratch_r,
                     uint8_t *scratch_i) {
    float norm = sqrtf(sum_sq(x, dim));
    *norm_out = norm;
    if (norm < 1e-8f) return;  // indices left untouched (reference quirk)
    float inv = 1.0f / norm;
    std::memcpy(scratch_n, x, dim * sizeof(float));
    scale_inplace(scratch_n, dim, inv);
    matmul(scratch_r, rot, scratch_n, dim, dim);
    int64_t nb = ((int64_t)1 << bits) - 1;
    for (int64_t i = 0; i < dim; ++i) scratch_i[i] = quantize(bnd, nb, scratch_r[i]);
    pack_into(scratch_i, dim, bits, packed);
}
// kv_cache.rs:279-317 (dequantize_*_into)
static void tq_dequant(const float *rot_t, const float *cent, int bits, int64_t dim,
                       const uint8_t *packed, float norm, float *out, float *scratch_r,
                       uint8_t *scratch_i) {
    if (norm < 1e-8f) {
        std::fill(out, out + dim, 0.0f);
        return;
    }
    unpack_into(packed, dim, bits, scratch_i);
    int64_t nl = (int64_t)1 << bits;
    for (int64_t i = 0; i < dim; ++i) scratch_r[i] = scratch_i[i] < nl ? cent[scratch_i[i]] : 0.0f;
    matmul(out, rot_t, scratch_r, dim, dim);
    scale_inplace(out, dim, norm);
}

// ---- SpectralQuant (src/spectralquant/spectral.rs, spectral_kv_cache.rs) ----
// Calibration (Jacobi eigenbasis of the sample covariance, participation
// ratio), the per-layer build of SpectralQuantKVCache::from_calibration (bit
// allocation, optional water-fill, identity -> random rotation, Lloyd-Max
// codebooks fitted on synthetic rotated unit vectors) and the codec
// (store_vector / dequantize_*_into). Tables use a fixed [kvd][64] centroid
// layout: dimension j's codebook is cent[j*64 .. j*64 + nlev[j]).
constexpr int kSqLevels = 64;

// jacobi_eigendecompose (spectral.rs:73-158): at most 50 single rotations of
// the largest off-diagonal element, f64, then a stable descending sort.
static void sq_jacobi(const std::vector<double> &m, int64_t d, std::vector<float> &evals, std::vector<float> &evecs) {
    std::vector<double> a = m, v(d * d, 0.0);
    for (int64_t i = 0; i < d; ++i) v[i * d + i] = 1.0;
    for (int sweep = 0; sweep < 50; ++sweep) {
        double max_val = 0.0;
        int64_t p = 0, q = 1;
        for (int64_t i = 0; i < d; ++i)
            for (int64_t j = i + 1; j < d; ++j) {
                const double val = std::fabs(a[i * d + j]);
                if (val > max_val) max_val = val, p = i, q = j;
            }
        if (max_val < 1e-10) break;
        const double app = a[p * d + p], aqq = a[q * d + q], apq = a[p * d + q];
        const double theta = 0.5 * std::atan2(2.0 * apq, app - aqq);
        const double c = std::cos(theta), s = std::sin(theta);
        for (int64_t i = 0; i < d; ++i) {
            if (i == p || i == q) continue;
            const double aip = a[i * d + p], aiq = a[i * d + q];
            a[i * d + p] = c * aip + s * aiq;
            a[p * d + i] = a[i * d + p];
            a[i * d + q] = -s * aip + c * aiq;
            a[q * d + i] = a[i * d + q];
        }
        const double npp = c * c * app + 2.0 * s * c * apq + s * s * aqq;
        const double nqq = s * s * app - 2.0 * s * c * apq + c * c * aqq;
        a[p * d + p] = npp;
        a[q * d + q] = nqq;
        a[p * d + q] = 0.0;
        a[q * d + p] = 0.0;
        for (int64_t i = 0; i < d; ++i) {
            const double vip = v[i * d + p], viq = v[i * d + q];
            v[i * d + p] = c * vip + s * viq;
            v[i * d + q] = -s * vip + c * viq;
        }
    }
    std::vector<float> ev(d), vec(d * d);
    for (int64_t i = 0; i < d; ++i) ev[i] = (float)a[i * d + i];
    for (int64_t i = 0; i < d * d; ++i) vec[i] = (float)v[i];
    std::vector<int64_t> order(d);
    for (int64_t i = 0; i < d; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int64_t x, int64_t y) { return ev[x] > ev[y]; });
    evals.resize(d);
    evecs.assign(d * d, 0.0f);
    for (int64_t nc = 0; nc < d; ++nc) {
        evals[nc] = ev[order[nc]];
        for (int64_t r = 0; r < d; ++r) evecs[r * d + nc] = vec[r * d + order[nc]];
    }
}

// participation_ratio (spectral.rs:11-24): (sum)^2 / sum of squares, f64 with mul_add.
static float sq_participation_ratio(const float *ev, int64_t n) {
    double sum = 0.0, sq = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const double x = (double)ev[i];
        sum += x;
        sq = std::fma(x, x, sq);
    }
    if (sq < 1e-12) return 0.0f;
    return (float)((sum * sum) / sq);
}

// slice::partition_point(|c| c < x), the binary search of Rust >= 1.82
// (identical to any search when the centroids are sorted)
static size_t sq_partition_point(const float *c, size_t n, float x) {
    if (n == 0) return 0;
    size_t base = 0, size = n;
    while (size > 1) {
        const size_t half = size / 2, mid = base + half;
        if (c[mid] < x) base = mid;
        size -= half;
    }
    return base + (c[base] < x ? 1 : 0);
}

// LloydMaxQuantizer::nearest_centroid (spectral.rs:711-733)
static size_t sq_nearest(float x, const std::vector<float> &c) {
    if (c.size() <= 1) return 0;
    const size_t idx = sq_partition_point(c.data(), c.size(), x);
    if (idx == 0) return 0;
    if (idx >= c.size()) return c.size() - 1;
    const float dl = std::fabs(x - c[idx - 1]), dr = std::fabs(c[idx] - x);
    return dl <= dr ? idx - 1 : idx;
}

// LloydMaxQuantizer::fit (spectral.rs:523-589): quantile start, mean updates
// in f64, empty cells reseeded from the data with Rng(seed), stop below 1e-6.
static std::vector<float> sq_lloyd_fit(const std::vector<float> &data, int bits, int max_iter, uint64_t seed) {
    const size_t nl = (size_t)1 << bits;
    if (data.empty()) return std::vector<float>(nl, 0.0f);
    std::vector<float> sorted = data;
    std::stable_sort(sorted.begin(), sorted.end(), [](float x, float y) { return x < y; });
    std::vector<float> c(nl);
    for (size_t i = 0; i < nl; ++i) {
        const float f = ((float)i + 0.5f) / (float)nl * (float)sorted.size();
        size_t idx = f >= 1.8446744e19f ? SIZE_MAX : (f > 0.0f ? (size_t)f : 0);
        c[i] = sorted[std::min(idx, sorted.size() - 1)];
    }
    Rng rng(seed);
    for (int it = 0; it < max_iter; ++it) {
        std::vector<double> sums(nl, 0.0);
        std::vector<size_t> counts(nl, 0);
        for (float x : data) {
            const size_t k = sq_nearest(x, c);
            sums[k] += (double)x;
            counts[k] += 1;
        }
        std::vector<float> nc(nl);
        for (size_t i = 0; i < nl; ++i)
            nc[i] = counts[i] ? (float)(sums[i] / (double)counts[i]) : data[(size_t)(rng.next() % data.size())];
        float md = 0.0f;
        for (size_t i = 0; i < nl; ++i) md = fmax_rs(md, std::fabs(c[i] - nc[i]));
        c = nc;
        if (md < 1e-6f) break;
    }
    return c;
}

// waterfill_bits (spectral.rs:443-478): +1 bit at a time to the highest
// lambda / 4^(b+1), lowest index on ties, capped at max_bits.
static std::vector<uint8_t> sq_waterfill(const std::vector<double> &ev, size_t total, int min_bits, int max_bits) {
    const size_t d = ev.size();
    std::vector<uint8_t> bits(d, (uint8_t)min_bits);
    size_t allocated = d * (size_t)min_bits;
    while (allocated < total) {
        size_t best = 0;
        double best_gain = 0.0;
        for (size_t i = 0; i < d; ++i) {
            if (bits[i] >= max_bits) continue;
            double p4 = 1.0;
            for (int e = 0; e < bits[i] + 1; ++e) p4 *= 4.0;
            const double gain = ev[i] / p4;
            if (gain > best_gain || (gain == best_gain && i < best)) best_gain = gain, best = i;
        }
        if (best_gain <= 0.0) break;
        bits[best] += 1;
        allocated += 1;
    }
    return bits;
}

// generate_random_rotation (spectral_kv_cache.rs:1034-1077): Gram-Schmidt on
// Rng(seed) normals, sequential f32 sums.
static std::vector<float> sq_random_rotation(int64_t d, uint64_t seed) {
    Rng rng(seed);
    std::vector<float> m(d * d);
    for (auto &x : m) x = rng.normal();
    for (int64_t col = 0; col < d; ++col) {
        for (int64_t prev = 0; prev < col; ++prev) {
            float dot = 0.0f;
            for (int64_t r = 0; r < d; ++r) dot += m[r * d + col] * m[r * d + prev];
            for (int64_t r = 0; r < d; ++r) m[r * d + col] -= dot * m[r * d + prev];
        }
        float ns = 0.0f;
        for (int64_t r = 0; r < d; ++r) ns += m[r * d + col] * m[r * d + col];
        const float nrm = sqrtf(ns);
        if (nrm > 1e-8f) {
            const float inv = 1.0f / nrm;
            for (int64_t r = 0; r < d; ++r) m[r * d + col] *= inv;
        } else {
            m[col * d + col] = 1.0f;
        }
    }
    return m;
}

// rotate_into (spectral_kv_cache.rs:993-1005): out[j] = sum over i in order of V[i][j] * x[i]
static void sq_rotate(const float *V, int64_t d, const float *x, float *out) {
    for (int64_t j = 0; j < d; ++j) out[j] = 0.0f;
    for (int64_t i = 0; i < d; ++i)
        for (int64_t j = 0; j < d; ++j) out[j] += V[i * d + j] * x[i];
}

struct SqTab {
    std::vector<float> eig;    // [kvd*kvd]
    std::vector<uint8_t> bits;  // [kvd]
    std::vector<int32_t> nlev;  // [kvd]
    std::vector<float> cent;    // [kvd][stride]
    int32_t d_eff = 0;
    int stride = kSqLevels;     // centroid slots per dimension
};

// One layer of SpectralQuantKVCache::from_calibration (spectral_kv_cache.rs:99-347).
static int sq_build_layer(const or_sq_params &P, int64_t kvd, int64_t layer, const float *eig_in, const float *eval_in,
                          float d_eff_f, SqTab &T, int max_levels = kSqLevels) {
    auto ceil_to_size = [](float f) -> size_t {  // `f.ceil() as usize` (saturating)
        const float c = ceilf(f);
        if (!(c > 0.0f)) return 0;
        return c >= 1.8446744e19f ? SIZE_MAX : (size_t)c;
    };
    const size_t d_eff = std::min<size_t>(std::max<size_t>(ceil_to_size(d_eff_f), 1), (size_t)kvd);
    // BitAllocator::allocate (spectral.rs:420-436)
    float bl = roundf(P.avg_bits - (float)d_eff / (float)kvd);
    bl = fmax_rs(bl, 1.0f);
    bl = bl < (float)P.max_bits ? bl : (float)P.max_bits;
    const int b_low = (int)bl;
    const int b_high = std::min(b_low + 1, P.max_bits);
    std::vector<uint8_t> sem_bits;
    const bool wf = P.use_water_fill && b_high > 0;
    if (wf) {
        std::vector<double> ev(d_eff);
        for (size_t i = 0; i < d_eff; ++i) ev[i] = (double)eval_in[i];
        sem_bits = sq_waterfill(ev, (size_t)b_high * d_eff, P.wf_min_bits, P.wf_max_bits);
    }
    const int tail_bits = std::max(b_low, 1);
    T.bits.assign(kvd, (uint8_t)tail_bits);
    for (size_t i = 0; i < d_eff; ++i) T.bits[i] = wf ? sem_bits[i] : (uint8_t)b_high;
    T.d_eff = (int32_t)d_eff;
    T.eig.assign(eig_in, eig_in + kvd * kvd);
    bool ident = true;
    for (int64_t i = 0; i < kvd && ident; ++i)
        for (int64_t j = 0; j < kvd; ++j)
            if (std::fabs(T.eig[i * kvd + j] - (i == j ? 1.0f : 0.0f)) > 1e-4f) {
                ident = false;
                break;
            }
    if (ident) T.eig = sq_random_rotation(kvd, P.seed + (uint64_t)layer * 7919);
    // synthetic unit vectors rotated by V^T
    const size_t nsyn = std::max<size_t>((size_t)std::max(P.calibration_samples, 0), 256);
    Rng rng(P.seed + (uint64_t)layer * 31);
    std::vector<float> syn(nsyn * kvd), x(kvd);
    for (size_t s = 0; s < nsyn; ++s) {
        for (auto &v : x) v = rng.normal();
        const float nrm = fmax_rs(sqrtf(sum_sq(x.data(), kvd)), 1e-8f);
        scale_inplace(x.data(), kvd, 1.0f / nrm);
        sq_rotate(T.eig.data(), kvd, x.data(), &syn[s * kvd]);
    }
    auto column_block = [&](size_t j0, size_t j1) {
        std::vector<float> out;
        out.reserve(nsyn * (j1 - j0));
        for (size_t s = 0; s < nsyn; ++s)
            for (size_t j = j0; j < j1; ++j) out.push_back(syn[s * kvd + j]);
        return out;
    };
    T.stride = max_levels;
    T.nlev.assign(kvd, 0);
    T.cent.assign(kvd * max_levels, 0.0f);
    auto put = [&](size_t j, const std::vector<float> &c) {
        if (c.size() > (size_t)max_levels) return false;
        T.nlev[j] = (int32_t)c.size();
        std::copy(c.begin(), c.end(), &T.cent[j * max_levels]);
        return true;
    };
    const std::vector<float> tail = sq_lloyd_fit(column_block(d_eff, kvd), tail_bits, P.lloyd_max_iter,
                                                 P.seed + (uint64_t)layer * 51 + 1);
    for (size_t j = d_eff; j < (size_t)kvd; ++j)
        if (!put(j, tail)) return -3;
    if (!wf) {
        const std::vector<float> sem = sq_lloyd_fit(column_block(0, d_eff), std::max(b_high, 1), P.lloyd_max_iter,
                                                    P.seed + (uint64_t)layer * 51 + 2);
        for (size_t j = 0; j < d_eff; ++j)
            if (!put(j, sem)) return -3;
    } else {
        for (size_t j = 0; j < d_eff; ++j) {
            const std::vector<float> cj = sq_lloyd_fit(column_block(j, j + 1), std::max<int>(sem_bits[j], 1),
                                                       P.lloyd_max_iter, P.seed + (uint64_t)(j + 10));
            if (!put(j, cj)) return -3;
        }
    }
    return 0;
}

// quantize_to_idx (spectral_kv_cache.rs:1079-1111): nearest centroid by
// bisection, ties to the lower index.
static uint8_t sq_quantize(float v, const float *c, int n) {
    if (n <= 1) return 0;
    int lo = 0, hi = n - 1;
    if (v <= c[lo]) return (uint8_t)lo;
    if (v >= c[hi]) return (uint8_t)hi;
    while (lo + 1 < hi) {
        const int mid = lo + (hi - lo) / 2;
        if (c[mid] <= v) lo = mid;
        else hi = mid;
    }
    return std::fabs(v - c[lo]) <= std::fabs(c[hi] - v) ? (uint8_t)lo : (uint8_t)hi;
}

// pack_variable_bits (:1125-1164), LSB first; returns the byte count
static int64_t sq_pack(const uint8_t *idx, const uint8_t *bits, int64_t n, uint8_t *out) {
    uint64_t buf = 0;
    uint32_t have = 0;
    int64_t w = 0;
    for (int64_t i = 0; i < n; ++i) {
        buf |= (uint64_t)idx[i] << have;
        have += bits[i];
        while (have >= 8) {
            out[w++] = (uint8_t)(buf & 0xFF);
            buf >>= 8;
            have -= 8;
        }
    }
    if (have > 0) out[w++] = (uint8_t)(buf & 0xFF);
    return w;
}

// unpack_variable_bits (:1167-1187)
static void sq_unpack(const uint8_t *p, int64_t plen, const uint8_t *bits, int64_t n, uint8_t *out) {
    uint64_t buf = 0;
    uint32_t have = 0;
    int64_t b = 0;
    for (int64_t i = 0; i < n; ++i) {
        while (have < bits[i] && b < plen) {
            buf |= (uint64_t)p[b++] << have;
            have += 8;
        }
        out[i] = (uint8_t)(buf & ((1ULL << bits[i]) - 1));
        buf >>= bits[i];
        have -= bits[i];
    }
}

// store_vector (spectral_kv_cache.rs:399-470): zero-norm vectors store norm 0
// and leave their codes as they were.
static void sq_store(const SqTab &T, int64_t kvd, const float *x, uint8_t *packed, float *norm_out,
                     std::vector<float> &xn, std::vector<float> &r, std::vector<uint8_t> &idx) {
    const float nrm = sqrtf(sum_sq(x, kvd));
    if (nrm < 1e-8f) {
        *norm_out = 0.0f;
        return;
    }
    *norm_out = nrm;
    std::copy(x, x + kvd, xn.begin());
    scale_inplace(xn.data(), kvd, 1.0f / nrm);
    sq_rotate(T.eig.data(), kvd, xn.data(), r.data());
    for (int64_t j = 0; j < kvd; ++j) idx[j] = sq_quantize(r[j], &T.cent[j * T.stride], T.nlev[j]);
    sq_pack(idx.data(), T.bits.data(), kvd, packed);
}

// dequantize_*_into (:567-672): unpack, centroid lookup, V x (simd_matmul_rows), * norm
static void sq_dequant(const SqTab &T, int64_t kvd, const uint8_t *packed, float nrm, float *out,
                       std::vector<float> &r, std::vector<uint8_t> &idx) {
    if (nrm < 1e-8f) {
        std::fill(out, out + kvd, 0.0f);
        return;
    }
    sq_unpack(packed, kvd, T.bits.data(), kvd, idx.data());
    for (int64_t j = 0; j < kvd; ++j) r[j] = idx[j] < T.nlev[j] ? T.cent[j * T.stride + idx[j]] : 0.0f;
    matmul(out, T.eig.data(), r.data(), kvd, kvd);
    scale_inplace(out, kvd, nrm);
}

// utility predictor — src/sp_kv/utility_predictor.rs:16-87, weights types.rs:224-258
struct Predictor {
    int64_t hidden;
    std::vector<float> w1, b1, w2, b2;
};
static Predictor make_predictor(int64_t d_model, int64_t hidden, int64_t nkv, float init_bias) {
    Predictor p;
    p.hidden = hidden;
    float s1 = sqrtf(2.0f / (float)d_model), s2 = sqrtf(2.0f / (float)hidden);
    Rng rng(42);
    p.w1.resize(hidden * d_model);
    for (auto &e : p.w1) e = rng.normal() * s1;
    p.b1.assign(hidden, 0.0f);
    p.w2.resize(nkv * hidden);
    for (auto &e : p.w2) e = rng.normal() * s2;
    p.b2.assign(nkv, init_bias);
    return p;
}
static float silu(float x) { return x * (1.0f / (1.0f + expf(-x))); }
static float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

// ------------------------------------------------------------------------
// Per-sequence forward state
// ------------------------------------------------------------------------
struct Seq {
    Dims d;
    const Weights *W;
    int mode;
    bool quant_shared_flat;  // forward_quantized as written (one flat buffer for all layers)
    // scratch (ForwardContext, transformer.rs:59-176)
    std::vector<float> x, xr, xr2, q, k, v, att, scores, hidden, aval, scaled, logits;
    std::vector<int64_t> aidx;
    std::vector<std::vector<float>> deltas;
    // f32 KV (MultiLayerKVCache)
    std::vector<float> Kc, Vc;
    // TurboQuant cache
    const TQ *tq = nullptr;
    int kbits = 4, vbits = 4;
    int64_t kpl = 0, vpl = 0;
    std::vector<uint8_t> kcodes, vcodes;
    std::vector<float> knorm, vnorm;
    std::vector<float> flatK, flatV;  // [L][B][kvd] (or [B][kvd] when shared)
    std::vector<int64_t> dequant_pos;
    std::vector<float> sn, sr;
    std::vector<uint8_t> si;
    // SpectralQuant codec (tables per layer); null = TurboQuant
    const std::vector<SqTab> *sqt = nullptr;
    std::vector<uint8_t> sq_idx;
    // LoRA of forward_base (the pair's writer) and forward_prefill (its reader)
    const Lora *lora_w = nullptr, *lora_r = nullptr;
    std::vector<float> lbuf;
    // SP-KV
    const Predictor *pred = nullptr;
    std::vector<float> pbuf, hu, util, bias;
    std::vector<uint8_t> retained;

    void init(const Dims &dd, const Weights *w, int md, int kb, int vb) {
        d = dd;
        W = w;
        mode = md;
        quant_shared_flat = false;
        x.assign(d.n, 0.f); xr = x; xr2 = x; q = x; att = x; scaled = x;
        k.assign(d.kvd, 0.f); v = k;
        scores.assign(d.B, 0.f);
        hidden.assign(d.m, 0.f); aval = hidden; aidx.assign(d.m, 0);
        logits.assign(d.V, 0.f);
        deltas.assign(d.nblocks, std::vector<float>(d.n, 0.f));
        lora_r = g_lora[0].rank ? &g_lora[0] : nullptr;
        lora_w = g_lora[1].rank ? &g_lora[1] : nullptr;
        lbuf.assign(std::max<int64_t>(std::max(g_lora[0].rank, g_lora[1].rank), 1), 0.f);
        if (mode == OR_MODE_BASE) {
            Kc.assign(d.L * d.B * d.kvd, 0.f);
            Vc = Kc;
        } else {
            kbits = kb;
            vbits = vb;
            kpl = packed_len(d.kvd, kb);
            vpl = packed_len(d.kvd, vb);
            kcodes.assign(d.L * d.B * kpl, 0);
            vcodes.assign(d.L * d.B * vpl, 0);
            knorm.assign(d.L * d.B, 0.f);
            vnorm = knorm;
            flatK.assign(d.L * d.B * d.kvd, 0.f);
            flatV = flatK;
            dequant_pos.assign(d.L, 0);
            sn.assign(d.kvd, 0.f); sr = sn; si.assign(d.kvd, 0);
            util.assign(d.L * d.B, 0.f);
            retained.assign(d.L * d.B, 0);
            bias.assign(d.B, 0.f);
        }
    }

    // optional copy of the rotated unit coordinates each store quantizes
    // ([L][rot_T][2][kvd]; untouched for zero-norm vectors), for parity tests
    float *rot_out = nullptr;
    int64_t rot_T = 0;
    // codes imposed on every store ([L][force_T][kpl + vpl], K then V): the
    // quantization decisions of another implementation, replayed
    const uint8_t *force = nullptr;
    int64_t force_T = 0;
    void store_kv(int64_t l, int64_t pos) {
        int64_t at = l * d.B + pos;
        if (sqt) {  // SpectralQuantKVCache::store_key / store_value: one table for K and V
            sq_store((*sqt)[l], d.kvd, k.data(), &kcodes[at * kpl], &knorm[at], sn, sr, sq_idx);
            sq_store((*sqt)[l], d.kvd, v.data(), &vcodes[at * vpl], &vnorm[at], sn, sr, sq_idx);
            return;
        }
        tq_store(tq->rot.data(), tq->kb.data(), kbits, d.kvd, k.data(), &kcodes[at * kpl],
                 &knorm[at], sn.data(), sr.data(), si.data());
        if (rot_out) std::memcpy(rot_out + ((l * rot_T + pos) * 2 + 0) * d.kvd, sr.data(), d.kvd * 4);
        tq_store(tq->rot.data(), tq->vb.data(), vbits, d.kvd, v.data(), &vcodes[at * vpl],
                 &vnorm[at], sn.data(), sr.data(), si.data());
        if (rot_out) std::memcpy(rot_out + ((l * rot_T + pos) * 2 + 1) * d.kvd, sr.data(), d.kvd * 4);
        if (force) {  // the norms stay this store's own
            const uint8_t *f = force + (l * force_T + pos) * (kpl + vpl);
            std::memcpy(&kcodes[at * kpl], f, kpl);
            std::memcpy(&vcodes[at * vpl], f + kpl, vpl);
        }
    }
    void deq_key(int64_t l, int64_t t, float *out) {
        int64_t at = l * d.B + t;
        if (sqt) return sq_dequant((*sqt)[l], d.kvd, &kcodes[at * kpl], knorm[at], out, sr, sq_idx);
        tq_dequant(tq->rot_t.data(), tq->kc.data(), kbits, d.kvd, &kcodes[at * kpl], knorm[at], out,
                   sr.data(), si.data());
    }
    void deq_val(int64_t l, int64_t t, float *out) {
        int64_t at = l * d.B + t;
        if (sqt) return sq_dequant((*sqt)[l], d.kvd, &vcodes[at * vpl], vnorm[at], out, sr, sq_idx);
        tq_dequant(tq->rot_t.data(), tq->vc.data(), vbits, d.kvd, &vcodes[at * vpl], vnorm[at], out,
                   sr.data(), si.data());
    }

    // MLP block shared by all three forwards: xr2=x; norm; relu(W1); sparse/dense W2; += xr2
    // with a LoRA: onto the post-ReLU hidden (before the alive count) and onto
    // W2's output (transformer.rs:2036-2038, 2110-2112)
    void mlp(const LayerW &lw, bool gamma_norm, const float *gamma, const Lora *lo = nullptr) {
        xr2 = x;
        if (gamma_norm) rmsnorm_gamma(x.data(), gamma, d.n);
        else rmsnorm(x.data(), d.n);
        matmul_relu(hidden.data(), lw.w1, x.data(), d.m, d.n);
        if (lo) lora_apply(hidden.data(), *lo, x.data(), lbuf.data());
        int64_t alive = sparse_matmul(x.data(), lw.w2, hidden.data(), d.n, d.m, aidx.data(), aval.data());
        // transformer.rs:2080-2101: dense recompute when alive fraction > 1 - threshold
        if ((float)alive / (float)d.m > (1.0f - sparse_threshold))
            matmul(x.data(), lw.w2, hidden.data(), d.n, d.m);
        if (lo) lora_apply(x.data(), *lo, hidden.data(), lbuf.data());
        add_inplace(x.data(), xr2.data(), d.n);
    }
    float sparse_threshold = 0.8f;

    void delta_route(int64_t l) {  // transformer.rs:2129-2158
        int64_t bidx = l / 4, pib = l % 4;
        if (bidx < (int64_t)deltas.size()) fused_sub_acc(deltas[bidx].data(), x.data(), xr.data(), d.n);
        if (pib == 3 && bidx < (int64_t)deltas.size())
            depth_route(x.data(), deltas, bidx, W->dq + l * d.n, W->dn + l * d.n, d.n, scaled);
    }

    // transformer.rs:1821-2200 (forward_base, default features);
    // kog_cpu_fusion applies attn_norm_gamma (:1893-1895) and mlp_norm_gamma
    // (:2023-2026) at run time through rmsnorm_with_gamma. With a LoRA
    // (lora_w) it is added after each of the six projections (:1904-1941,
    // 2018-2020, 2036-2038, 2110-2112).
    void forward_base(int64_t tok, int64_t pos) {
        add_into(x.data(), W->wte + tok * d.n, W->wpe + pos * d.n, d.n);
        float scale = 1.0f / sqrtf((float)d.hd);
        for (int64_t l = 0; l < d.L; ++l) {
            const LayerW &lw = W->layers[l];
            rmsnorm_gamma(x.data(), W->ag + l * d.n, d.n);
            xr = x;
            matmul(q.data(), lw.wq, x.data(), d.n, d.n);
            if (lora_w) lora_apply(q.data(), *lora_w, x.data(), lbuf.data());
            matmul(k.data(), lw.wk, x.data(), d.kvd, d.n);
            if (lora_w) lora_apply(k.data(), *lora_w, x.data(), lbuf.data());
            matmul(v.data(), lw.wv, x.data(), d.kvd, d.n);
            if (lora_w) lora_apply(v.data(), *lora_w, x.data(), lbuf.data());
            float *K = &Kc[l * d.B * d.kvd], *Vv = &Vc[l * d.B * d.kvd];
            std::memcpy(K + pos * d.kvd, k.data(), d.kvd * 4);
            std::memcpy(Vv + pos * d.kvd, v.data(), d.kvd * 4);
            for (int64_t h = 0; h < d.nh; ++h) {
                int64_t g = h * d.nkv / d.nh;
                attention_head(q.data(), K, Vv, att.data(), scores.data(), h * d.hd, g * d.hd,
                               d.kvd, d.hd, pos + 1, scale);
            }
            matmul(x.data(), lw.wo, att.data(), d.n, d.n);
            if (lora_w) lora_apply(x.data(), *lora_w, att.data(), lbuf.data());
            add_inplace(x.data(), xr.data(), d.n);
            mlp(lw, true, W->mg + l * d.n, lora_w);
            delta_route(l);
        }
        matmul(logits.data(), W->lm_head, x.data(), d.V, d.n);
    }

    // transformer.rs:2606-3004 (forward_prefill, default features; the LoRA
    // is the pair's reader, lora_r):
    // per layer, phase A over every prompt position (double rmsnorm, K/V into
    // the f32 cache, Q and the residual kept), then phase B over every
    // position: attention over ALL prompt positions (bidirectional), Wo +
    // residual, MLP with the TwELL switch, delta routing with the context's
    // block deltas accumulating across positions. Returns the last position's
    // hidden state in x; the caller computes lm_head.
    void forward_prefill(const int32_t *toks, int64_t P) {
        std::vector<float> hidden(P * d.n), queries(P * d.n), residuals(P * d.n);
        if (d.L > 1)
            for (int64_t p = 0; p < P; ++p)
                add_into(&hidden[p * d.n], W->wte + (int64_t)toks[p] * d.n, W->wpe + p * d.n, d.n);
        const float scale = 1.0f / sqrtf((float)d.hd);
        for (int64_t l = 0; l < d.L; ++l) {
            const LayerW &lw = W->layers[l];
            float *K = &Kc[l * d.B * d.kvd], *Vv = &Vc[l * d.B * d.kvd];
            for (int64_t p = 0; p < P; ++p) {  // phase A (:2657-2757)
                if (d.L > 1) std::memcpy(x.data(), &hidden[p * d.n], d.n * 4);
                else add_into(x.data(), W->wte + (int64_t)toks[p] * d.n, W->wpe + p * d.n, d.n);
                rmsnorm(x.data(), d.n);
                xr = x;
                rmsnorm(x.data(), d.n);
                matmul(k.data(), lw.wk, x.data(), d.kvd, d.n);
                if (lora_r) lora_apply(k.data(), *lora_r, x.data(), lbuf.data());  // :2681-2687
                matmul(v.data(), lw.wv, x.data(), d.kvd, d.n);
                if (lora_r) lora_apply(v.data(), *lora_r, x.data(), lbuf.data());
                std::memcpy(K + p * d.kvd, k.data(), d.kvd * 4);
                std::memcpy(Vv + p * d.kvd, v.data(), d.kvd * 4);
                matmul(q.data(), lw.wq, x.data(), d.n, d.n);
                if (lora_r) lora_apply(q.data(), *lora_r, x.data(), lbuf.data());  // :2738-2740
                std::memcpy(&queries[p * d.n], q.data(), d.n * 4);
                std::memcpy(&residuals[p * d.n], xr.data(), d.n * 4);
            }
            for (int64_t p = 0; p < P; ++p) {  // phase B (:2797-2987)
                std::memcpy(xr.data(), &residuals[p * d.n], d.n * 4);
                std::fill(att.begin(), att.end(), 0.0f);
                std::memcpy(q.data(), &queries[p * d.n], d.n * 4);
                for (int64_t h = 0; h < d.nh; ++h) {
                    int64_t g = h * d.nkv / d.nh;
                    attention_head(q.data(), K, Vv, att.data(), scores.data(), h * d.hd, g * d.hd, d.kvd, d.hd, P,
                                   scale);
                }
                matmul(x.data(), lw.wo, att.data(), d.n, d.n);
                if (lora_r) lora_apply(x.data(), *lora_r, att.data(), lbuf.data());  // :2901-2903
                add_inplace(x.data(), xr.data(), d.n);
                mlp(lw, false, nullptr, lora_r);
                delta_route(l);
                if (d.L > 1) std::memcpy(&hidden[p * d.n], x.data(), d.n * 4);
            }
        }
    }

    // transformer.rs:3305-3504 (forward_paged, default features): forward
    // with K/V in PagedKVCache pages (crates/katgpt-transformer/src/kv_cache.rs:
    // 187-420). Per layer: rmsnorm, save the residual, rmsnorm again (no
    // gammas), separate Q/K/V matmuls, write_kv into the page that holds pos,
    // read_kv of positions 0..pos into a flat buffer, attention_head per head,
    // Wo + residual, the MLP with the TwELL switch, delta routing; lm_head.
    // pool: pages of [K: 16 x kvd | V: 16 x kvd] floats; table: this
    // sequence's page list per layer, [L][maxp] page indices.
    void forward_paged(int64_t tok, int64_t pos, float *pool, const int64_t *table, int64_t maxp) {
        const int64_t PS = 16;  // PAGE_SIZE (kv_cache.rs:189)
        add_into(x.data(), W->wte + tok * d.n, W->wpe + pos * d.n, d.n);
        const float scale = 1.0f / sqrtf((float)d.hd);
        const int64_t tn = pos + 1;
        std::vector<float> fk(tn * d.kvd), fv(tn * d.kvd);
        auto page_row = [&](int64_t l, int64_t t, int which) {
            const int64_t pg = table[l * maxp + t / PS];
            return pool + ((pg * 2 + which) * PS + t % PS) * d.kvd;
        };
        for (int64_t l = 0; l < d.L; ++l) {
            const LayerW &lw = W->layers[l];
            rmsnorm(x.data(), d.n);
            xr = x;
            rmsnorm(x.data(), d.n);
            matmul(q.data(), lw.wq, x.data(), d.n, d.n);
            matmul(k.data(), lw.wk, x.data(), d.kvd, d.n);
            matmul(v.data(), lw.wv, x.data(), d.kvd, d.n);
            std::memcpy(page_row(l, pos, 0), k.data(), d.kvd * 4);  // write_kv (:298-309)
            std::memcpy(page_row(l, pos, 1), v.data(), d.kvd * 4);
            for (int64_t t = 0; t < tn; ++t) {  // read_kv into the flat buffers (:3390-3398)
                std::memcpy(&fk[t * d.kvd], page_row(l, t, 0), d.kvd * 4);
                std::memcpy(&fv[t * d.kvd], page_row(l, t, 1), d.kvd * 4);
            }
            for (int64_t h = 0; h < d.nh; ++h) {
                int64_t g = h * d.nkv / d.nh;
                attention_head(q.data(), fk.data(), fv.data(), att.data(), scores.data(), h * d.hd, g * d.hd,
                               d.kvd, d.hd, tn, scale);
            }
            matmul(x.data(), lw.wo, att.data(), d.n, d.n);
            add_inplace(x.data(), xr.data(), d.n);
            mlp(lw, false, nullptr);
            delta_route(l);
        }
        matmul(logits.data(), W->lm_head, x.data(), d.V, d.n);
    }

    // transformer.rs:4042-4233 (forward_quantized<TurboQuantKVCache>)
    void forward_quant(int64_t tok, int64_t pos) {
        add_into(x.data(), W->wte + tok * d.n, W->wpe + pos * d.n, d.n);
        float scale = 1.0f / sqrtf((float)d.hd);
        int64_t tn = pos + 1;
        for (int64_t l = 0; l < d.L; ++l) {
            const LayerW &lw = W->layers[l];
            rmsnorm(x.data(), d.n);
            xr = x;
            matmul(q.data(), lw.wq, x.data(), d.n, d.n);
            matmul(k.data(), lw.wk, x.data(), d.kvd, d.n);
            matmul(v.data(), lw.wv, x.data(), d.kvd, d.n);
            store_kv(l, pos);
            // Per-layer flat buffers (the intended semantics). With
            // quant_shared_flat the single ForwardContext buffer of the
            // reference is reproduced as written.
            int64_t fo = quant_shared_flat ? 0 : l * d.B * d.kvd;
            float *FK = &flatK[fo], *FV = &flatV[fo];
            int64_t last = dequant_pos[l];
            if (last + 1 == pos && pos > 0) {
                deq_key(l, pos, FK + pos * d.kvd);
                deq_val(l, pos, FV + pos * d.kvd);
            } else {
                for (int64_t t = 0; t < tn; ++t) {
                    deq_key(l, t, FK + t * d.kvd);
                    deq_val(l, t, FV + t * d.kvd);
                }
            }
            dequant_pos[l] = pos;
            for (int64_t h = 0; h < d.nh; ++h) {
                int64_t g = h * d.nkv / d.nh;
                attention_head(q.data(), FK, FV, att.data(), scores.data(), h * d.hd, g * d.hd,
                               d.kvd, d.hd, tn, scale);
            }
            matmul(x.data(), lw.wo, att.data(), d.n, d.n);
            add_inplace(x.data(), xr.data(), d.n);
            mlp(lw, false, nullptr);
            delta_route(l);
        }
        matmul(logits.data(), W->lm_head, x.data(), d.V, d.n);
    }

    // src/sp_kv/forward.rs:610-822 (forward_sp_kv_quant, Hard gate, default
    // SpKvConfig; its `lora` is the pair's writer, lora_w)
    void forward_spkv(int64_t tok, int64_t pos) {
        const int64_t window = 128;
        const float threshold = 0.5f;
        add_into(x.data(), W->wte + tok * d.n, W->wpe + pos * d.n, d.n);
        int64_t tn = pos + 1;
        for (int64_t l = 0; l < d.L; ++l) {
            const LayerW &lw = W->layers[l];
            rmsnorm(x.data(), d.n);
            xr = x;
            rmsnorm(x.data(), d.n);
            // utility predictor (utility_predictor.rs:51-87), Max aggregation
            for (int64_t i = 0; i < pred->hidden; ++i)
                pbuf[i] = silu(dot(&pred->w1[i * d.n], x.data(), d.n) + pred->b1[i]);
            for (int64_t kh = 0; kh < d.nkv; ++kh)
                hu[kh] = sigmoid(dot(&pred->w2[kh * pred->hidden], pbuf.data(), pred->hidden) + pred->b2[kh]);
            float u = hu[0];
            for (int64_t kh = 1; kh < d.nkv; ++kh) u = fmax_rs(u, hu[kh]);
            matmul(q.data(), lw.wq, x.data(), d.n, d.n);
            if (lora_w) lora_apply(q.data(), *lora_w, x.data(), lbuf.data());  // forward.rs:673-684
            matmul(k.data(), lw.wk, x.data(), d.kvd, d.n);
            if (lora_w) lora_apply(k.data(), *lora_w, x.data(), lbuf.data());
            matmul(v.data(), lw.wv, x.data(), d.kvd, d.n);
            if (lora_w) lora_apply(v.data(), *lora_w, x.data(), lbuf.data());
            // write_gated(pos_is_in_window = true) — types.rs:505-527
            util[l * d.B + pos] = u;
            store_kv(l, pos);
            retained[l * d.B + pos] = 1;
            // build_hard — types.rs:343-356
            for (int64_t s = 0; s <= pos; ++s) {
                bool inw = (pos - s) < window;
                bool keep = inw || util[l * d.B + s] >= threshold || retained[l * d.B + s];
                bias[s] = keep ? 0.0f : -INFINITY;
            }
            // dequantize_retained_*_into — full rebuild 0..=pos (types.rs:534-575)
            float *FK = &flatK[0], *FV = &flatV[0];
            for (int64_t t = 0; t < tn; ++t) {
                if (retained[l * d.B + t]) {
                    deq_key(l, t, FK + t * d.kvd);
                    deq_val(l, t, FV + t * d.kvd);
                } else {
                    std::fill(FK + t * d.kvd, FK + (t + 1) * d.kvd, 0.f);
                    std::fill(FV + t * d.kvd, FV + (t + 1) * d.kvd, 0.f);
                }
            }
            float scale = 1.0f / sqrtf((float)d.hd);
            std::fill(att.begin(), att.end(), 0.f);
            for (int64_t h = 0; h < d.nh; ++h) {
                int64_t g = h * d.nkv / d.nh;
                attention_head_gated(q.data(), FK, FV, att.data(), scores.data(), h * d.hd,
                                     g * d.hd, d.kvd, d.hd, tn, scale, bias.data());
            }
            matmul(x.data(), lw.wo, att.data(), d.n, d.n);
            if (lora_w) lora_apply(x.data(), *lora_w, att.data(), lbuf.data());  // forward.rs:753-756
            add_inplace(x.data(), xr.data(), d.n);
            mlp(lw, false, nullptr, lora_w);  // :769-771, 805-807
        }
        matmul(logits.data(), W->lm_head, x.data(), d.V, d.n);
    }
};

static const Predictor &predictor_for(int64_t n, int64_t nkv) {
    static std::vector<std::pair<std::pair<int64_t, int64_t>, Predictor *>> cache;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : cache)
        if (e.first.first == n && e.first.second == nkv) return *e.second;
    int64_t hidden = std::max<int64_t>(n / 4, 16);  // SpKvConfig::resolve_hidden (types.rs:58-65)
    Predictor *p = new Predictor(make_predictor(n, hidden, nkv, 5.0f));
    cache.push_back({{n, nkv}, p});
    return *p;
}

static int run_one(const or_config *c, int mode, int kb, int vb, const Weights &W, const Dims &d,
                   const int32_t *tokens, int32_t T, float *logits, int32_t t0, uint8_t *codes,
                   float *norms, float *utilities, bool shared_flat, Seq &s, float *rot_out = nullptr) {
    s.init(d, &W, mode == 3 ? OR_MODE_QUANT : mode, kb, vb);
    s.rot_out = rot_out;
    s.rot_T = T;
    s.sparse_threshold = c->sparse_threshold;
    s.quant_shared_flat = shared_flat;
    if (mode != OR_MODE_BASE) s.tq = &tq_tables(d.kvd, kb, vb);
    if (mode == OR_MODE_SPKV_QUANT) {
        s.pred = &predictor_for(d.n, d.nkv);
        s.pbuf.assign(s.pred->hidden, 0.f);
        s.hu.assign(d.nkv, 0.f);
    }
    for (int32_t p = 0; p < T; ++p) {
        int64_t tok = tokens[p];
        if (tok < 0 || tok >= d.V) return -2;
        if (mode == OR_MODE_BASE) s.forward_base(tok, p);
        else if (mode == OR_MODE_SPKV_QUANT) s.forward_spkv(tok, p);
        else s.forward_quant(tok, p);
        if (logits && p >= t0) std::memcpy(logits + (int64_t)(p - t0) * d.V, s.logits.data(), d.V * 4);
    }
    if (mode != OR_MODE_BASE) {
        for (int64_t l = 0; l < d.L; ++l)
            for (int64_t p = 0; p < T; ++p) {
                int64_t at = l * d.B + p;
                int64_t o = (l * T + p);
                if (codes) {
                    std::memcpy(codes + o * (s.kpl + s.vpl), &s.kcodes[at * s.kpl], s.kpl);
                    std::memcpy(codes + o * (s.kpl + s.vpl) + s.kpl, &s.vcodes[at * s.vpl], s.vpl);
                }
                if (norms) {
                    norms[o * 2] = s.knorm[at];
                    norms[o * 2 + 1] = s.vnorm[at];
                }
                if (utilities) utilities[o] = s.util[at];
            }
    }
    return 0;
}

static int check_cfg(const or_config *c, int32_t T) {
    if (!c || c->n_embd <= 0 || c->n_head <= 0 || c->head_dim <= 0 || c->n_kv_head <= 0 ||
        c->n_layer <= 0 || c->vocab_size <= 0 || c->mlp_hidden <= 0)
        return -1;
    if (T < 0 || T > c->block_size) return -1;
    if ((int64_t)c->n_head * c->head_dim != c->n_embd) return -1;
    if (c->n_head % c->n_kv_head != 0) return -1;
    return 0;
}

}  // namespace

extern "C" {

void or_rng_uniforms(uint64_t seed, int64_t n, float *out) {
    Rng r(seed);
    for (int64_t i = 0; i < n; ++i) out[i] = r.uniform();
}
void or_rng_normals(uint64_t seed, int64_t n, float *out) {
    Rng r(seed);
    for (int64_t i = 0; i < n; ++i) out[i] = r.normal();
}

int64_t or_weights_count(const or_config *c) { return weights_count(dims_of(c)); }

void or_weights_init(const or_config *c, uint64_t seed, int scale_mode, float std_, float *out) {
    Dims d = dims_of(c);
    Rng rng(seed);
    float es = sqrtf(2.0f / (float)d.n);                       // weights.rs:79
    float ls = sqrtf(2.0f / ((float)d.n * (float)d.L));        // weights.rs:80
    if (scale_mode == 1) es = ls = std_;
    float *p = out;
    for (int64_t i = 0; i < d.V * d.n; ++i) *p++ = rng.normal() * es;
    for (int64_t i = 0; i < d.B * d.n; ++i) *p++ = rng.normal() * es;
    for (int64_t l = 0; l < d.L; ++l) {
        int64_t cnt = 2 * d.n * d.n + 2 * d.kvd * d.n + 2 * d.m * d.n;
        for (int64_t i = 0; i < cnt; ++i) *p++ = rng.normal() * ls;
    }
    for (int64_t i = 0; i < d.V * d.n; ++i) *p++ = rng.normal() * es;
    for (int64_t i = 0; i < d.L * d.n; ++i) *p++ = 0.0f;  // delta query: zeros (weights.rs:161-168)
    for (int64_t i = 0; i < d.L * d.n; ++i) *p++ = 1.0f;  // delta norm gamma: ones (:169-176)
    for (int64_t i = 0; i < d.L * d.n; ++i) *p++ = 1.0f;  // attn_norm_gamma: ones (:142-143)
    for (int64_t i = 0; i < d.L * d.n; ++i) *p++ = 1.0f;  // mlp_norm_gamma: ones (:144-145)
}

float or_dot(const float *a, const float *b, int64_t len) { return dot(a, b, len); }
float or_sum_sq(const float *x, int64_t len) { return sum_sq(x, len); }
float or_sum(const float *x, int64_t len) { return sum_f32(x, len); }
float or_max(const float *x, int64_t len) { return max_f32(x, len); }
void or_exp_inplace(float *x, int64_t len) { exp_inplace(x, len); }
float or_exp_sum_inplace(float *x, int64_t len) { return exp_sum_inplace(x, len); }
float or_sparse_dot(const float *w, const int64_t *idx, const float *val, int64_t alive) {
    return sparse_dot(w, idx, val, alive);
}
void or_softmax_scaled(float *x, int64_t len, float inv_temp) { softmax_scaled(x, len, inv_temp); }
float or_scalar_exp(float x) { return cephes_exp_scalar(x); }

// math.rs:398-422 (sample_token_into)
int64_t or_sample_token(const float *probs, int64_t n, uint64_t seed) {
    Rng rng(seed);
    float r = rng.uniform();
    while (r == 0.0f) r = rng.uniform();
    if (n == 0) return 0;
    std::vector<float> cdf(n);
    float s = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        s += probs[i];
        cdf[i] = s;
    }
    int64_t idx = std::partition_point(cdf.begin(), cdf.end(), [&](float c) { return c <= r; }) -
                  cdf.begin();
    return std::min(idx, n - 1);
}

// sample_token_into called k times with one generator (math.rs:398-422):
// row j of probs [k][n] gets the j-th draw of Rng::new(seed)
void or_sample_tokens(const float *probs, int64_t n, int64_t k, uint64_t seed, int64_t *out) {
    Rng rng(seed);
    std::vector<float> cdf(n);
    for (int64_t j = 0; j < k; ++j) {
        float r = rng.uniform();
        while (r == 0.0f) r = rng.uniform();
        const float *p = probs + j * n;
        float s = 0.0f;
        for (int64_t i = 0; i < n; ++i) {
            s += p[i];
            cdf[i] = s;
        }
        int64_t idx = std::partition_point(cdf.begin(), cdf.end(), [&](float c) { return c <= r; }) - cdf.begin();
        out[j] = n == 0 ? 0 : std::min(idx, n - 1);
    }
}

// crates/katgpt-core/src/speculative/sampling.rs:26-40 (sample_from_distribution)
static int64_t sample_dist(const float *probs, int64_t n, Rng &rng) {
    float r = rng.uniform();
    while (r == 0.0f) r = rng.uniform();
    float cdf = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        cdf += probs[i];
        if (r < cdf) return i;
    }
    return n > 0 ? n - 1 : 0;
}
// sampling.rs:50-116 (sample_residual_distribution_into)
static int64_t sample_residual(const float *p, const float *q, int64_t n, Rng &rng) {
    std::vector<float> scratch(n);
    const int64_t chunks = n / 4;
    float sum = 0.0f;
    for (int64_t c = 0; c < chunks; ++c) {
        const int64_t i = c * 4;
        const float r0 = fmax_rs(p[i] - q[i], 0.0f), r1 = fmax_rs(p[i + 1] - q[i + 1], 0.0f);
        const float r2 = fmax_rs(p[i + 2] - q[i + 2], 0.0f), r3 = fmax_rs(p[i + 3] - q[i + 3], 0.0f);
        scratch[i] = r0; scratch[i + 1] = r1; scratch[i + 2] = r2; scratch[i + 3] = r3;
        sum += (r0 + r1) + (r2 + r3);
    }
    for (int64_t i = chunks * 4; i < n; ++i) {
        const float r = fmax_rs(p[i] - q[i], 0.0f);
        scratch[i] = r;
        sum += r;
    }
    if (sum > 0.0f) {
        const float inv = 1.0f / sum;
        for (int64_t i = 0; i < n; ++i) scratch[i] *= inv;
        return sample_dist(scratch.data(), n, rng);
    }
    return sample_dist(p, n, rng);
}

// speculative_step_rollback's acceptance loop for one path (src/speculative/step.rs:150-222):
// p [k][n] = the target's softmax_scaled distributions at the path's positions,
// q [k][n] = the draft marginals, drafts [k]; out [k+1], returns the count
int32_t or_verify_path(const float *p, const float *q, const int32_t *drafts, int32_t k, int64_t n, uint64_t seed,
                       int32_t *out) {
    Rng rng(seed);
    int32_t count = 0;
    int64_t cur = 0;
    bool all = true;
    for (int32_t i = 0; i < k; ++i) {
        const int64_t d = drafts[i];
        const bool inr = d >= 0 && d < n;
        const float qi = inr ? q[i * n + d] : 0.0f;
        const float pi = inr ? p[cur * n + d] : 0.0f;
        const float acc = qi > 0.0f ? std::min(pi / qi, 1.0f) : 1.0f;
        if (rng.uniform() <= acc) {
            out[count++] = (int32_t)d;
            if (i + 1 < k) cur = i + 1;
        } else {
            out[count++] = (int32_t)sample_residual(p + cur * n, q + i * n, n, rng);
            all = false;
            break;
        }
    }
    if (all && k > 0) out[count++] = (int32_t)sample_dist(p + cur * n, n, rng);
    return count;
}

int64_t or_tq_packed_len(int64_t dim, int bits) { return packed_len(dim, bits); }

void or_tq_codebook(int64_t dim, int bits, float *centroids, float *boundaries, float *mse) {
    std::vector<float> c, b;
    codebook(dim, bits, c, b, mse);
    std::memcpy(centroids, c.data(), c.size() * 4);
    std::memcpy(boundaries, b.data(), b.size() * 4);
}
void or_tq_rotation(int64_t dim, uint64_t seed, float *rot) { rotation(dim, seed, rot); }
void or_tq_rotation_from(int64_t dim, const float *gauss, float *rot) { rotation_from(dim, gauss, rot); }
void or_rng_normals_rawstate(uint64_t state, int64_t n, float *out) {
    // Rng before the SplitMix64 seed expansion (katgpt-core CHANGELOG, issue 296):
    // the seed itself is the XorShift64 state.
    Rng r(0);
    r.state = state == 0 ? 1 : state;
    for (int64_t i = 0; i < n; ++i) out[i] = r.normal();
}

void or_tq_store(const float *rot, const float *bnd, int bits, int64_t dim, const float *x,
                 uint8_t *packed, float *norm) {
    std::vector<float> sn(dim), sr(dim);
    std::vector<uint8_t> si(dim);
    tq_store(rot, bnd, bits, dim, x, packed, norm, sn.data(), sr.data(), si.data());
}
void or_tq_dequant(const float *rot_t, const float *cent, int bits, int64_t dim,
                   const uint8_t *packed, float norm, float *out) {
    std::vector<float> sr(dim);
    std::vector<uint8_t> si(dim);
    tq_dequant(rot_t, cent, bits, dim, packed, norm, out, sr.data(), si.data());
}
// kv_cache.rs:243-258 + :471-495 (dequantize_key: scalar column loop over R)
void or_tq_dequant_scalar(const float *rot, const float *cent, int bits, int64_t dim,
                          const uint8_t *packed, float norm, float *out) {
    if (norm < 1e-8f) {
        std::fill(out, out + dim, 0.0f);
        return;
    }
    std::vector<uint8_t> idx(dim);
    unpack_into(packed, dim, bits, idx.data());
    std::vector<float> r(dim);
    int64_t nl = (int64_t)1 << bits;
    for (int64_t i = 0; i < dim; ++i) r[i] = idx[i] < nl ? cent[idx[i]] : 0.0f;
    for (int64_t i = 0; i < dim; ++i) {
        float s = 0.0f;
        for (int64_t j = 0; j < dim; ++j) s += rot[j * dim + i] * r[j];
        out[i] = s * norm;
    }
}
void or_tq_pack(const uint8_t *idx, int64_t n, int bits, uint8_t *out) { pack_into(idx, n, bits, out); }
void or_tq_unpack(const uint8_t *p, int64_t n, int bits, uint8_t *out) { unpack_into(p, n, bits, out); }

// src/turboquant/forward.rs:171-180
float or_cosine(const float *a, const float *b, int64_t len) {
    float dd = dot(a, b, len);
    float na = sqrtf(dot(a, a, len)), nb = sqrtf(dot(b, b, len));
    if (na < 1e-8f || nb < 1e-8f) return 0.0f;
    return dd / (na * nb);
}

int or_run_sequence(const or_config *c, int mode, int kb, int vb, const float *weights,
                    const int32_t *tokens, int32_t T, float *logits, uint8_t *codes, float *norms,
                    float *utilities) {
    if (check_cfg(c, T)) return -1;
    if (mode < 0 || mode > 3) return -1;
    Dims d = dims_of(c);
    Weights W = view_weights(d, weights);
    Seq s;
    // mode 3: forward_quantized with the reference's single shared flat buffer
    return run_one(c, mode, kb, vb, W, d, tokens, T, logits, 0, codes, norms, utilities, mode == 3,
                   s);
}

// forward_prefill over prompt[0..P) (src/transformer.rs:2606-3004), then
// forward_base of cont[0..n_cont) at positions P.. over the prefill's cache
// (the decode half of generate_with_prefill, :3010-3106). logits_out rows:
// the prefill's last position, then one per continuation token.
int or_run_sequence_forced(const or_config *c, int key_bits, int val_bits, const float *weights,
                           const int32_t *tokens, int32_t T, const uint8_t *codes_in, float *logits) {
    if (check_cfg(c, T) || !codes_in) return -1;
    Dims d = dims_of(c);
    Weights W = view_weights(d, weights);
    Seq s;
    s.force = codes_in;
    s.force_T = T;
    return run_one(c, OR_MODE_QUANT, key_bits, val_bits, W, d, tokens, T, logits, 0, nullptr, nullptr, nullptr, false,
                   s);
}

int or_prefill_then_decode(const or_config *c, const float *weights, const int32_t *prompt, int32_t P,
                           const int32_t *cont, int32_t n_cont, float *logits_out) {
    if (check_cfg(c, P + n_cont) || P < 1 || n_cont < 0) return -1;
    Dims d = dims_of(c);
    Weights W = view_weights(d, weights);
    for (int32_t i = 0; i < P; ++i)
        if (prompt[i] < 0 || prompt[i] >= d.V) return -2;
    for (int32_t i = 0; i < n_cont; ++i)
        if (cont[i] < 0 || cont[i] >= d.V) return -2;
    Seq s;
    s.init(d, &W, OR_MODE_BASE, 4, 4);
    s.sparse_threshold = c->sparse_threshold;
    s.forward_prefill(prompt, P);
    matmul(logits_out, W.lm_head, s.x.data(), d.V, d.n);  // matmul_parallel: the same row dots
    for (int32_t i = 0; i < n_cont; ++i) {
        s.forward_base(cont[i], P + i);
        std::memcpy(logits_out + (int64_t)(i + 1) * d.V, s.logits.data(), d.V * 4);
    }
    return 0;
}

// One forward_paged token (src/transformer.rs:3305-3504) of a sequence whose
// pages the caller has ensured (PagedKVCache::ensure_pages): writes K/V of
// `pos` into `pool` and vocab_size logits. table [L][maxp] is the sequence's
// page list per layer (entries past its length unused).
int or_forward_paged(const or_config *c, const float *weights, float *pool, const int64_t *table, int64_t maxp,
                     int32_t token, int32_t pos, float *logits) {
    if (check_cfg(c, 0) || !pool || !table || maxp < 1 || pos < 0 || pos >= c->block_size || pos / 16 >= maxp)
        return -1;
    Dims d = dims_of(c);
    if (token < 0 || token >= d.V) return -2;
    Weights W = view_weights(d, weights);
    Seq s;
    s.init(d, &W, OR_MODE_BASE, 4, 4);
    s.sparse_threshold = c->sparse_threshold;
    s.forward_paged(token, pos, pool, table, maxp);
    std::memcpy(logits, s.logits.data(), d.V * 4);
    return 0;
}

// ---- SpectralQuant ----
static int sq_tables_from(int64_t kvd, int32_t L, const float *eig, const uint8_t *bits, const float *cent,
                          const int32_t *nlev, std::vector<SqTab> &T) {
    T.assign(L, SqTab());
    for (int32_t l = 0; l < L; ++l) {
        T[l].eig.assign(eig + l * kvd * kvd, eig + (l + 1) * kvd * kvd);
        T[l].bits.assign(bits + l * kvd, bits + (l + 1) * kvd);
        T[l].cent.assign(cent + l * kvd * kSqLevels, cent + (l + 1) * kvd * kSqLevels);
        T[l].nlev.assign(nlev + l * kvd, nlev + (l + 1) * kvd);
        for (int64_t j = 0; j < kvd; ++j)
            if (T[l].bits[j] < 1 || T[l].bits[j] > 8 || T[l].nlev[j] > kSqLevels) return -1;
    }
    return 0;
}

// Pieces of the SpectralQuant build, exposed for the reference's own unit
// tests (spectral.rs:845-1183, spectral_kv_cache.rs:1243-1274).
int or_sq_jacobi(const double *m, int64_t dim, float *evals, float *evecs) {
    if (!m || dim < 1) return -1;
    std::vector<float> ev, vec;
    sq_jacobi(std::vector<double>(m, m + dim * dim), dim, ev, vec);
    std::memcpy(evals, ev.data(), dim * 4);
    std::memcpy(evecs, vec.data(), dim * dim * 4);
    return 0;
}
// BitAllocator::new(_, max_bits).allocate(d_eff, avg_bits, head_dim) (spectral.rs:420-436)
void or_sq_allocate(float d_eff, float avg_bits, int64_t head_dim, int max_bits, int32_t *b_high, int32_t *b_low) {
    const float c = ceilf(d_eff);
    int64_t d = c > 0.0f ? (int64_t)c : 0;
    d = std::min<int64_t>(std::max<int64_t>(d, 1), head_dim);
    float bl = roundf(avg_bits - (float)d / (float)head_dim);
    bl = fmax_rs(bl, 1.0f);
    bl = bl < (float)max_bits ? bl : (float)max_bits;
    *b_low = (int32_t)bl;
    *b_high = std::min(*b_low + 1, max_bits);
}
// waterfill_bits (spectral.rs:443-478); max_bits < 0 means None
void or_sq_waterfill(const double *ev, int64_t d, int64_t total, int min_bits, int max_bits, uint8_t *out) {
    const std::vector<uint8_t> b =
        sq_waterfill(std::vector<double>(ev, ev + d), (size_t)total, min_bits, max_bits < 0 ? 1 << 30 : max_bits);
    std::memcpy(out, b.data(), d);
}
// LloydMaxQuantizer::new(bits, max_iter, seed).fit(data) centroids (spectral.rs:523-589)
void or_sq_lloyd_fit(const float *data, int64_t n, int bits, int max_iter, uint64_t seed, float *centroids) {
    const std::vector<float> c = sq_lloyd_fit(std::vector<float>(data, data + n), bits, max_iter, seed);
    std::memcpy(centroids, c.data(), c.size() * 4);
}
// LloydMaxQuantizer::quantize's nearest_centroid (spectral.rs:711-733)
int64_t or_sq_nearest(float x, const float *centroids, int64_t n) {
    return (int64_t)sq_nearest(x, std::vector<float>(centroids, centroids + n));
}
// pack_variable_bits / unpack_variable_bits (spectral_kv_cache.rs:1125-1187)
int64_t or_sq_pack(const uint8_t *idx, const uint8_t *bits, int64_t n, uint8_t *out) { return sq_pack(idx, bits, n, out); }
void or_sq_unpack(const uint8_t *p, int64_t plen, const uint8_t *bits, int64_t n, uint8_t *out) {
    sq_unpack(p, plen, bits, n, out);
}

// LoraPair for the forwards that take one: which 0 = reader (forward_prefill),
// 1 = writer (forward_base); rank 0 clears. The adapter must stay inside
// every projection it is applied to (in_dim <= n_embd, out_dim <= n_embd and
// <= kv_dim): the reference indexes past the output otherwise.
int or_set_lora(int which, int64_t rank, int64_t in_dim, int64_t out_dim, float alpha, const float *a,
                const float *b) {
    if (which < 0 || which > 1 || rank < 0) return -1;
    Lora &lo = g_lora[which];
    if (rank == 0) {
        lo = Lora();
        return 0;
    }
    if (in_dim < 1 || out_dim < 1 || !a || !b) return -1;
    lo.rank = rank;
    lo.in_dim = in_dim;
    lo.out_dim = out_dim;
    lo.alpha = alpha;
    lo.a.assign(a, a + rank * in_dim);
    lo.b.assign(b, b + out_dim * rank);
    return 0;
}
void or_lora_apply(int64_t rank, int64_t in_dim, int64_t out_dim, float alpha, const float *a, const float *b,
                   const float *in, float *out) {
    Lora lo;
    lo.rank = rank;
    lo.in_dim = in_dim;
    lo.out_dim = out_dim;
    lo.alpha = alpha;
    lo.a.assign(a, a + rank * in_dim);
    lo.b.assign(b, b + out_dim * rank);
    std::vector<float> buf(rank);
    lora_apply(out, lo, in, buf.data());
}

// SP-KV pieces for the reference's own unit tests: the utility predictor
// (utility_predictor.rs:51-87 with the weights of types.rs:224-258) and
// attention_head_gated (sp_kv/forward.rs:166-245); bias NULL = no gate.
void or_spkv_predict(int64_t d_model, int64_t hidden, int64_t nkv, float init_bias, const float *h, float *util) {
    const Predictor p = make_predictor(d_model, hidden, nkv, init_bias);
    std::vector<float> buf(hidden);
    for (int64_t i = 0; i < hidden; ++i) buf[i] = silu(dot(&p.w1[i * d_model], h, d_model) + p.b1[i]);
    for (int64_t k = 0; k < nkv; ++k) util[k] = sigmoid(dot(&p.w2[k * hidden], buf.data(), hidden) + p.b2[k]);
}
// The predictor's seeded weights (types.rs:224-258), w1 [hidden][d_model],
// b1 [hidden], w2 [nkv][hidden], b2 [nkv], one after the other.
void or_spkv_predictor_weights(int64_t d_model, int64_t hidden, int64_t nkv, float init_bias, float *out) {
    const Predictor p = make_predictor(d_model, hidden, nkv, init_bias);
    for (const std::vector<float> *v : {&p.w1, &p.b1, &p.w2, &p.b2}) {
        std::memcpy(out, v->data(), v->size() * 4);
        out += v->size();
    }
}
void or_attention_head_gated(const float *q, const float *K, const float *V, float *out, float *scores, int64_t qoff,
                             int64_t kvoff, int64_t kvd, int64_t hd, int64_t tn, float scale, const float *bias) {
    std::vector<float> zero(tn, 0.0f);
    attention_head_gated(q, K, V, out, scores, qoff, kvoff, kvd, hd, tn, scale, bias ? bias : zero.data());
}

// calibrate_eigenbasis (spectral.rs:226-278): covariance (1/N) sum x x^T in f64,
// Jacobi, participation ratio. samples [n][dim].
int or_sq_calibrate_eigenbasis(const float *samples, int64_t n, int64_t dim, float *eigvecs, float *eigvals,
                               float *d_eff) {
    if (!samples || n < 1 || dim < 2) return -1;
    std::vector<double> cov(dim * dim, 0.0);
    for (int64_t s = 0; s < n; ++s) {
        const float *x = samples + s * dim;
        for (int64_t i = 0; i < dim; ++i)
            for (int64_t j = 0; j < dim; ++j) cov[i * dim + j] += (double)x[i] * (double)x[j];
    }
    const double scale = 1.0 / (double)n;
    for (auto &v : cov) v *= scale;
    std::vector<float> ev, vec;
    sq_jacobi(cov, dim, ev, vec);
    std::memcpy(eigvecs, vec.data(), dim * dim * 4);
    std::memcpy(eigvals, ev.data(), dim * 4);
    *d_eff = sq_participation_ratio(ev.data(), dim);
    return 0;
}

// SpectralQuantKVCache::from_calibration per layer: tables as [L][kvd*kvd]
// eigenvectors, [L][kvd] bits, [L][kvd][64] centroids, [L][kvd] level counts,
// [L] d_eff. Returns -3 if a codebook exceeds 64 levels.
int or_sq_build(const or_sq_params *P, int64_t kvd, int32_t L, const float *eig_in, const float *eval_in,
                const float *deff_in, float *eig_out, uint8_t *bits_out, float *cent_out, int32_t *nlev_out,
                int32_t *deff_out) {
    if (!P || kvd < 2 || L < 1 || P->max_bits < 1) return -1;
    for (int32_t l = 0; l < L; ++l) {
        SqTab T;
        int rc = sq_build_layer(*P, kvd, l, eig_in + l * kvd * kvd, eval_in + l * kvd, deff_in[l], T);
        if (rc) return rc;
        std::memcpy(eig_out + l * kvd * kvd, T.eig.data(), kvd * kvd * 4);
        std::memcpy(bits_out + l * kvd, T.bits.data(), kvd);
        std::memcpy(cent_out + l * kvd * kSqLevels, T.cent.data(), kvd * kSqLevels * 4);
        std::memcpy(nlev_out + l * kvd, T.nlev.data(), kvd * 4);
        deff_out[l] = T.d_eff;
    }
    return 0;
}

// store_vector then dequantize_*_into of one vector with one layer's tables
// (packed gets the pack's byte count, returned; -1 on bad tables).
int64_t or_sq_roundtrip(int64_t kvd, const float *eig, const uint8_t *bits, const float *cent, const int32_t *nlev,
                        const float *x, uint8_t *packed, float *norm, float *deq) {
    std::vector<SqTab> T;
    if (sq_tables_from(kvd, 1, eig, bits, cent, nlev, T)) return -1;
    std::vector<float> xn(kvd), r(kvd);
    std::vector<uint8_t> idx(kvd);
    sq_store(T[0], kvd, x, packed, norm, xn, r, idx);
    if (deq) sq_dequant(T[0], kvd, packed, *norm, deq, r, idx);
    int64_t tb = 0;
    for (int64_t j = 0; j < kvd; ++j) tb += bits[j];
    return (tb + 7) / 8;
}

// SpectralQuantKVCache::from_keys on keys[0..n_calib) (one layer, codebooks
// of any width up to 8 bits), then store_key + dequantize_key_into of every
// key: recon [n_keys][dim]. The configuration of the reference's quality
// benchmark (tests/bench_octopus_goat.rs:346-440).
int or_sq_quality_keys(const or_sq_params *P, int64_t dim, const float *keys, int64_t n_keys, int64_t n_calib,
                       float *recon) {
    if (!P || dim < 2 || n_keys < 1 || n_calib < 1 || n_calib > n_keys) return -1;
    std::vector<double> cov(dim * dim, 0.0);
    for (int64_t s = 0; s < n_calib; ++s)
        for (int64_t i = 0; i < dim; ++i)
            for (int64_t j = 0; j < dim; ++j) cov[i * dim + j] += (double)keys[s * dim + i] * (double)keys[s * dim + j];
    const double scale = 1.0 / (double)n_calib;
    for (auto &v : cov) v *= scale;
    std::vector<float> ev, vec;
    sq_jacobi(cov, dim, ev, vec);
    SqTab T;
    if (sq_build_layer(*P, dim, 0, vec.data(), ev.data(), sq_participation_ratio(ev.data(), dim), T, 256)) return -3;
    std::vector<float> xn(dim), r(dim);
    std::vector<uint8_t> idx(dim), packed(dim);
    for (int64_t k = 0; k < n_keys; ++k) {
        float nrm = 0.0f;
        std::fill(packed.begin(), packed.end(), 0);
        sq_store(T, dim, keys + k * dim, packed.data(), &nrm, xn, r, idx);
        sq_dequant(T, dim, packed.data(), nrm, recon + k * dim, r, idx);
    }
    return 0;
}

// forward_quantized<SpectralQuantKVCache> (src/transformer.rs:4042-4233 with
// the codec of src/spectralquant/spectral_kv_cache.rs) of one sequence:
// logits [T][V], codes [L][T][2*kvd] (K row then V row, kvd bytes each, the
// pack in front), norms [L][T][2].
int or_run_sequence_sq(const or_config *c, const float *weights, const float *eig, const uint8_t *bits,
                       const float *cent, const int32_t *nlev, const int32_t *tokens, int32_t T, float *logits,
                       uint8_t *codes, float *norms) {
    if (check_cfg(c, T)) return -1;
    Dims d = dims_of(c);
    Weights W = view_weights(d, weights);
    std::vector<SqTab> tabs;
    if (sq_tables_from(d.kvd, (int32_t)d.L, eig, bits, cent, nlev, tabs)) return -1;
    Seq s;
    s.init(d, &W, OR_MODE_QUANT, 8, 8);  // 8-bit packed rows: kvd bytes per vector
    s.sparse_threshold = c->sparse_threshold;
    s.sqt = &tabs;
    s.sq_idx.assign(d.kvd, 0);
    for (int32_t p = 0; p < T; ++p) {
        if (tokens[p] < 0 || tokens[p] >= d.V) return -2;
        s.forward_quant(tokens[p], p);
        if (logits) std::memcpy(logits + (int64_t)p * d.V, s.logits.data(), d.V * 4);
    }
    for (int64_t l = 0; l < d.L; ++l)
        for (int64_t p = 0; p < T; ++p) {
            const int64_t at = l * d.B + p, o = l * T + p;
            if (codes) {
                std::memcpy(codes + o * 2 * d.kvd, &s.kcodes[at * s.kpl], d.kvd);
                std::memcpy(codes + o * 2 * d.kvd + d.kvd, &s.vcodes[at * s.vpl], d.kvd);
            }
            if (norms) norms[o * 2] = s.knorm[at], norms[o * 2 + 1] = s.vnorm[at];
        }
    return 0;
}

int or_run_sequence_rot(const or_config *c, int mode, int kb, int vb, const float *weights, const int32_t *tokens,
                        int32_t T, float *logits, uint8_t *codes, float *norms, float *rot_out) {
    if (check_cfg(c, T)) return -1;
    if (mode != OR_MODE_QUANT && mode != OR_MODE_SPKV_QUANT) return -1;
    Dims d = dims_of(c);
    Weights W = view_weights(d, weights);
    Seq s;
    return run_one(c, mode, kb, vb, W, d, tokens, T, logits, 0, codes, norms, nullptr, false, s, rot_out);
}

int or_run_batch_tail(const or_config *c, int mode, int kb, int vb, const float *weights,
                      const int32_t *tokens, int32_t n_seq, int32_t T, int32_t t0, float *logits,
                      int n_threads) {
    if (check_cfg(c, T)) return -1;
    if (mode < 0 || mode > 3 || t0 < 0 || t0 > T) return -1;
    Dims d = dims_of(c);
    Weights W = view_weights(d, weights);
    if (mode != OR_MODE_BASE) tq_tables(d.kvd, kb, vb);
    if (mode == OR_MODE_SPKV_QUANT) predictor_for(d.n, d.nkv);
    if (n_threads < 1) n_threads = 1;
    std::vector<int> rc(n_threads, 0);
    auto worker = [&](int tid) {
        Seq s;  // per-worker context (generate_batch map_init, transformer.rs:3588-3606)
        for (int32_t i = tid; i < n_seq; i += n_threads) {
            float *lo = logits ? logits + (int64_t)i * (T - t0) * d.V : nullptr;
            int r = run_one(c, mode, kb, vb, W, d, tokens + (int64_t)i * T, T, lo, t0, nullptr,
                            nullptr, nullptr, mode == 3, s);
            if (r) rc[tid] = r;
        }
    };
    std::vector<std::thread> th;
    for (int t = 1; t < n_threads; ++t) th.emplace_back(worker, t);
    worker(0);
    for (auto &t : th) t.join();
    for (int r : rc)
        if (r) return r;
    return 0;
}

// CPU-baseline timing of forward_quantized (mode 1) or forward_base (mode 0)
// decode at a long context, without running the prompt. Each worker thread owns one sequence (the reference's
// generate_batch, src/transformer.rs:3588-3606). Positions [0, ctx) of its
// cache hold synthetic codes and norms and are marked as already dequantized
// (dequant_pos = ctx - 1, the reference's single shared flat buffer), so the
// timed positions ctx .. ctx + n_pos - 1 run the reference's per-token work at
// that context: QKV/Wo/W1/W2/lm_head matvecs, TurboQuant store of the new K
// and V, incremental dequant of the new position, attention over ctx + 1
// positions, delta routing. `w_one_layer` is the flat layout of the same
// model with n_layer = 1; every layer reads that one layer's matrices (each
// layer's matrices stream from DRAM either way, so the work per token is
// unchanged). Returns tokens/s of the timed positions (all threads), or < 0.
double or_time_decode(const or_config *c, int mode, int kb, int vb, const float *w_one_layer, int32_t ctx,
                      int32_t n_pos, int n_threads) {
    if (check_cfg(c, ctx + n_pos) || ctx < 1 || n_pos < 1) return -1.0;
    if (mode != OR_MODE_BASE && mode != OR_MODE_QUANT) return -1.0;
    Dims d = dims_of(c);
    or_config c1 = *c;
    c1.n_layer = 1;
    Dims d1 = dims_of(&c1);
    Weights W1 = view_weights(d1, w_one_layer);
    Weights W = W1;
    W.layers.assign(d.L, W1.layers[0]);
    std::vector<float> dq(d.L * d.n, 0.0f), dn(d.L * d.n, 1.0f);  // weights.rs:142-145, 161-176 init
    W.dq = dq.data();
    W.dn = dn.data();
    W.ag = dn.data();
    W.mg = dn.data();
    if (mode == OR_MODE_QUANT) tq_tables(d.kvd, kb, vb, true);
    if (n_threads < 1) n_threads = 1;
    std::vector<double> secs(n_threads, 0.0);
    auto worker = [&](int tid) {
        Seq s;
        s.init(d, &W, mode, kb, vb);
        s.sparse_threshold = c->sparse_threshold;
        Rng rng(1000 + tid);
        // synthetic cache contents: a cheap 64-bit counter hash per 8 bytes / value
        uint64_t z = 0x9E3779B97F4A7C15ULL * (uint64_t)(tid + 1);
        auto fill_bytes = [&](std::vector<uint8_t> &v) {
            for (size_t i = 0; i + 8 <= v.size(); i += 8) {
                z = z * 6364136223846793005ULL + 1442695040888963407ULL;
                std::memcpy(&v[i], &z, 8);
            }
        };
        auto fill_vals = [&](float *p, int64_t cnt) {
            for (int64_t i = 0; i < cnt; ++i) {
                z = z * 6364136223846793005ULL + 1442695040888963407ULL;
                p[i] = (float)(int32_t)(z >> 40) * (0.01f / 8388608.0f);
            }
        };
        if (mode == OR_MODE_QUANT) {
            s.quant_shared_flat = true;
            s.tq = &tq_tables(d.kvd, kb, vb, true);
            fill_bytes(s.kcodes);
            fill_bytes(s.vcodes);
            std::fill(s.knorm.begin(), s.knorm.end(), 1.0f);
            std::fill(s.vnorm.begin(), s.vnorm.end(), 1.0f);
            fill_vals(s.flatK.data(), ctx * d.kvd);
            fill_vals(s.flatV.data(), ctx * d.kvd);
            std::fill(s.dequant_pos.begin(), s.dequant_pos.end(), (int64_t)ctx - 1);
        } else {
            for (int64_t l = 0; l < d.L; ++l) {
                fill_vals(&s.Kc[l * d.B * d.kvd], ctx * d.kvd);
                fill_vals(&s.Vc[l * d.B * d.kvd], ctx * d.kvd);
            }
        }
        const auto t0 = std::chrono::steady_clock::now();
        for (int32_t p = ctx; p < ctx + n_pos; ++p) {
            const int64_t tok = (int64_t)(rng.next() % (uint64_t)d.V);
            if (mode == OR_MODE_QUANT) s.forward_quant(tok, p);
            else s.forward_base(tok, p);
        }
        secs[tid] = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    };
    std::vector<std::thread> th;
    for (int t = 1; t < n_threads; ++t) th.emplace_back(worker, t);
    worker(0);
    for (auto &t : th) t.join();
    double mx = 0.0;
    for (double v : secs) mx = std::max(mx, v);
    return mx > 0.0 ? (double)n_threads * n_pos / mx : -1.0;
}

int or_run_batch(const or_config *c, int mode, int kb, int vb, const float *weights,
                 const int32_t *tokens, int32_t n_seq, int32_t T, float *logits, int n_threads) {
    return or_run_batch_tail(c, mode, kb, vb, weights, tokens, n_seq, T, 0, logits, n_threads);
}

}  // extern "C"
