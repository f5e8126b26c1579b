// kg_sq.cpp — host construction of the SpectralQuant codec tables, bit for bit
// as SpectralQuantKVCache::from_keys / from_calibration build them
// (src/spectralquant/spectral.rs, src/spectralquant/spectral_kv_cache.rs).
//
// This is one-time set-up work (a Jacobi eigendecomposition of a kv_dim x
// kv_dim covariance and Lloyd-Max fits on a few thousand scalars), so it runs
// on the host; the device only reads the resulting per-layer tables:
// eigenvectors [kvd*kvd] row-major (columns = eigenvectors), per-dimension bit
// widths, and per-dimension codebooks of at most kSqMaxLevels centroids.
//
// Built with g++ -O2 -ffp-contract=off (no fast-math); glibc atan2/cos/sin/
// logf/cosf are the functions the reference's f64/f32 methods call.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/kg_abi.h"

namespace kg {

// the reference Rng (kg_tables.cpp) over an explicit XorShift64 state
uint64_t host_rng_next_state(uint64_t &state);
uint64_t host_rng_seed_state(uint64_t seed);
float host_rng_normal(uint64_t &state);

namespace sq {

constexpr int kMaxLevels = 64;

// f32::max: a NaN operand is ignored
inline float fmax_nan(float a, float b) { return std::isnan(a) ? b : (std::isnan(b) ? a : (a > b ? a : b)); }

// hsum of one 8-lane AVX2 register (crates/katgpt-types/src/simd/horizontal.rs:31-51):
// lanes i and i+4 first, then (s0 + s1) + (s2 + s3)
inline float hsum8(const float *v) {
    const float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    return (s0 + s1) + (s2 + s3);
}

// simd_sum_sq (crates/katgpt-types/src/simd/research.rs:298-338): two 8-lane
// FMA accumulators over 16-element chunks, one over the 8-element rest, scalar tail
float sum_sq(const float *x, int64_t n) {
    float a[8] = {}, b[8] = {};
    int64_t i = 0;
    for (; i + 16 <= n; i += 16)
        for (int l = 0; l < 8; ++l) {
            a[l] = std::fma(x[i + l], x[i + l], a[l]);
            b[l] = std::fma(x[i + 8 + l], x[i + 8 + l], b[l]);
        }
    float t[8];
    for (int l = 0; l < 8; ++l) t[l] = a[l] + b[l];
    float s = hsum8(t);
    float r[8] = {};
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) r[l] = std::fma(x[i + l], x[i + l], r[l]);
    s = s + hsum8(r);
    for (; i < n; ++i) s = s + x[i] * x[i];
    return s;
}

// Rust's slice::partition_point (the bisection of Rust >= 1.82) for `c < x`
size_t partition_lt(const std::vector<float> &c, float x) {
    size_t base = 0, size = c.size();
    if (!size) return 0;
    while (size > 1) {
        const size_t half = size / 2;
        if (c[base + half] < x) base += half;
        size -= half;
    }
    return base + (c[base] < x);
}

// LloydMaxQuantizer (spectral.rs:504-733)
struct Lloyd {
    static size_t nearest(float x, const std::vector<float> &c) {
        if (c.size() < 2) return 0;
        const size_t k = partition_lt(c, x);
        if (k == 0) return 0;
        if (k >= c.size()) return c.size() - 1;
        return std::fabs(x - c[k - 1]) <= std::fabs(c[k] - x) ? k - 1 : k;
    }
    static std::vector<float> fit(const std::vector<float> &data, int bits, int max_iter, uint64_t seed) {
        const size_t levels = (size_t)1 << bits;
        std::vector<float> c(levels, 0.0f);
        if (data.empty()) return c;
        std::vector<float> sorted(data);
        std::stable_sort(sorted.begin(), sorted.end(), [](float a, float b) { return a < b; });
        for (size_t i = 0; i < levels; ++i) {  // uniform quantile placement, f32 arithmetic
            const float pos = ((float)i + 0.5f) / (float)levels * (float)sorted.size();
            const size_t k = pos > 0.0f ? (size_t)pos : 0;
            c[i] = sorted[std::min(k, sorted.size() - 1)];
        }
        uint64_t rs = host_rng_seed_state(seed);
        std::vector<double> acc(levels);
        std::vector<size_t> cnt(levels);
        for (int it = 0; it < max_iter; ++it) {
            std::fill(acc.begin(), acc.end(), 0.0);
            std::fill(cnt.begin(), cnt.end(), 0);
            for (float x : data) {
                const size_t k = nearest(x, c);
                acc[k] += (double)x;
                ++cnt[k];
            }
            float delta = 0.0f;
            std::vector<float> nc(levels);
            for (size_t i = 0; i < levels; ++i) {
                nc[i] = cnt[i] ? (float)(acc[i] / (double)cnt[i])
                               : data[(size_t)(host_rng_next_state(rs) % (uint64_t)data.size())];
            }
            for (size_t i = 0; i < levels; ++i) delta = fmax_nan(delta, std::fabs(c[i] - nc[i]));
            c.swap(nc);
            if (delta < 1e-6f) break;
        }
        return c;
    }
};

// jacobi_eigendecompose (spectral.rs:73-158)
void jacobi(std::vector<double> a, int64_t n, std::vector<float> &vals, std::vector<float> &vecs) {
    std::vector<double> v(n * n, 0.0);
    for (int64_t i = 0; i < n; ++i) v[i * n + i] = 1.0;
    auto A = [&](int64_t r, int64_t c) -> double & { return a[r * n + c]; };
    for (int rot = 0; rot < 50; ++rot) {
        double big = 0.0;
        int64_t p = 0, q = 1;
        for (int64_t r = 0; r < n; ++r)
            for (int64_t c = r + 1; c < n; ++c)
                if (std::fabs(A(r, c)) > big) {
                    big = std::fabs(A(r, c));
                    p = r;
                    q = c;
                }
        if (big < 1e-10) break;
        const double app = A(p, p), aqq = A(q, q), apq = A(p, q);
        const double th = 0.5 * std::atan2(2.0 * apq, app - aqq);
        const double c = std::cos(th), s = std::sin(th);
        for (int64_t i = 0; i < n; ++i) {
            if (i == p || i == q) continue;
            const double ip = A(i, p), iq = A(i, q);
            A(i, p) = c * ip + s * iq;
            A(p, i) = A(i, p);
            A(i, q) = -s * ip + c * iq;
            A(q, i) = A(i, q);
        }
        A(p, p) = c * c * app + 2.0 * s * c * apq + s * s * aqq;
        A(q, q) = s * s * app - 2.0 * s * c * apq + c * c * aqq;
        A(p, q) = 0.0;
        A(q, p) = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            const double ip = v[i * n + p], iq = v[i * n + q];
            v[i * n + p] = c * ip + s * iq;
            v[i * n + q] = -s * ip + c * iq;
        }
    }
    std::vector<int64_t> order(n);
    for (int64_t i = 0; i < n; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int64_t x, int64_t y) { return (float)A(x, x) > (float)A(y, y); });
    vals.resize(n);
    vecs.resize(n * n);
    for (int64_t k = 0; k < n; ++k) {
        vals[k] = (float)A(order[k], order[k]);
        for (int64_t r = 0; r < n; ++r) vecs[r * n + k] = (float)v[r * n + order[k]];
    }
}

}  // namespace sq

// calibrate_eigenbasis (spectral.rs:226-278): covariance (1/N) sum x x^T in
// f64 without centring, Jacobi, d_eff = participation ratio (spectral.rs:11-24).
void sq_calibrate(const float *samples, int64_t n, int64_t dim, std::vector<float> &vecs, std::vector<float> &vals,
                  float &d_eff) {
    std::vector<double> cov(dim * dim, 0.0);
    for (int64_t s = 0; s < n; ++s)
        for (int64_t i = 0; i < dim; ++i)
            for (int64_t j = 0; j < dim; ++j) cov[i * dim + j] += (double)samples[s * dim + i] * (double)samples[s * dim + j];
    const double inv_n = 1.0 / (double)n;
    for (double &c : cov) c *= inv_n;
    sq::jacobi(cov, dim, vals, vecs);
    double sum = 0.0, sumsq = 0.0;
    for (float ev : vals) {
        sum += (double)ev;
        sumsq = std::fma((double)ev, (double)ev, sumsq);
    }
    d_eff = sumsq < 1e-12 ? 0.0f : (float)((sum * sum) / sumsq);
}

// One layer of SpectralQuantKVCache::from_calibration (spectral_kv_cache.rs:99-347)
// for a calibration (eigenvectors, eigenvalues, d_eff) of dimension kvd. Outputs
// eigenvectors (a seeded random rotation when the calibration's are the
// identity), bits [kvd], centroids [kvd][kMaxLevels], levels [kvd], d_eff.
// Returns false when a codebook has more than kMaxLevels centroids.
bool sq_build_layer(const kg_sq_params &P, int64_t kvd, int64_t layer, const float *eig, const float *eval,
                    float d_eff_in, float *eig_out, uint8_t *bits_out, float *cent_out, int32_t *lev_out,
                    int32_t *d_eff_out) {
    const float dc = std::ceil(d_eff_in);
    const int64_t d = std::min<int64_t>(std::max<int64_t>(dc > 0.0f ? (int64_t)std::min(dc, 1e18f) : 0, 1), kvd);
    // BitAllocator::allocate (spectral.rs:420-436): b_low = round(avg - d/kvd) in [1, max_bits], b_high = b_low + 1
    float lowf = std::round(P.avg_bits - (float)d / (float)kvd);
    lowf = sq::fmax_nan(lowf, 1.0f);
    if (lowf > (float)P.max_bits) lowf = (float)P.max_bits;
    const int b_low = (int)lowf, b_high = std::min(b_low + 1, (int)P.max_bits), b_tail = std::max(b_low, 1);
    std::vector<int> width(kvd, b_tail);
    const bool waterfill = P.use_water_fill && b_high > 0;
    if (waterfill) {
        // waterfill_bits (spectral.rs:443-478) over the first d eigenvalues
        std::vector<int> w(d, P.wf_min_bits);
        size_t have = (size_t)d * P.wf_min_bits;
        const size_t want = (size_t)b_high * d;
        while (have < want) {
            int64_t best = 0;
            double gain_best = 0.0;
            for (int64_t i = 0; i < d; ++i) {
                if (w[i] >= P.wf_max_bits) continue;
                const double g = (double)eval[i] / std::ldexp(1.0, 2 * (w[i] + 1));  // lambda / 4^(b+1)
                if (g > gain_best || (g == gain_best && i < best)) {
                    gain_best = g;
                    best = i;
                }
            }
            if (gain_best <= 0.0) break;
            ++w[best];
            ++have;
        }
        for (int64_t i = 0; i < d; ++i) width[i] = w[i];
    } else {
        for (int64_t i = 0; i < d; ++i) width[i] = b_high;
    }
    // identity eigenvectors -> generate_random_rotation (spectral_kv_cache.rs:1034-1077)
    std::vector<float> V(eig, eig + kvd * kvd);
    bool identity = true;
    for (int64_t i = 0; i < kvd * kvd && identity; ++i)
        identity = std::fabs(V[i] - ((i / kvd == i % kvd) ? 1.0f : 0.0f)) <= 1e-4f;
    if (identity) {
        uint64_t rs = host_rng_seed_state(P.seed + (uint64_t)layer * 7919);
        for (float &x : V) x = host_rng_normal(rs);
        for (int64_t col = 0; col < kvd; ++col) {
            for (int64_t prev = 0; prev < col; ++prev) {
                float dp = 0.0f;
                for (int64_t r = 0; r < kvd; ++r) dp += V[r * kvd + col] * V[r * kvd + prev];
                for (int64_t r = 0; r < kvd; ++r) V[r * kvd + col] -= dp * V[r * kvd + prev];
            }
            float ss = 0.0f;
            for (int64_t r = 0; r < kvd; ++r) ss += V[r * kvd + col] * V[r * kvd + col];
            const float nr = std::sqrt(ss);
            if (nr > 1e-8f) {
                const float inv = 1.0f / nr;
                for (int64_t r = 0; r < kvd; ++r) V[r * kvd + col] *= inv;
            } else {
                V[col * kvd + col] = 1.0f;
            }
        }
    }
    // synthetic unit vectors rotated by V^T; dimension-major copies for the fits
    const int64_t nsyn = std::max<int64_t>(P.calibration_samples, 256);
    uint64_t rs = host_rng_seed_state(P.seed + (uint64_t)layer * 31);
    std::vector<float> by_dim(kvd * nsyn), x(kvd), y(kvd);
    for (int64_t s = 0; s < nsyn; ++s) {
        for (float &e : x) e = host_rng_normal(rs);
        const float inv = 1.0f / sq::fmax_nan(std::sqrt(sq::sum_sq(x.data(), kvd)), 1e-8f);
        for (float &e : x) e = e * inv;
        std::fill(y.begin(), y.end(), 0.0f);
        for (int64_t i = 0; i < kvd; ++i)
            for (int64_t j = 0; j < kvd; ++j) y[j] = y[j] + V[i * kvd + j] * x[i];
        for (int64_t j = 0; j < kvd; ++j) by_dim[j * nsyn + s] = y[j];
    }
    auto gather = [&](int64_t j0, int64_t j1) {  // samples in order, dimensions j0..j1 within each
        std::vector<float> out;
        out.reserve((j1 - j0) * nsyn);
        for (int64_t s = 0; s < nsyn; ++s)
            for (int64_t j = j0; j < j1; ++j) out.push_back(by_dim[j * nsyn + s]);
        return out;
    };
    std::vector<std::vector<float>> book(kvd);
    const std::vector<float> tail = sq::Lloyd::fit(gather(d, kvd), b_tail, P.lloyd_max_iter, P.seed + (uint64_t)layer * 51 + 1);
    for (int64_t j = d; j < kvd; ++j) book[j] = tail;
    if (!waterfill) {
        const std::vector<float> sem =
            sq::Lloyd::fit(gather(0, d), std::max(b_high, 1), P.lloyd_max_iter, P.seed + (uint64_t)layer * 51 + 2);
        for (int64_t j = 0; j < d; ++j) book[j] = sem;
    } else {
        for (int64_t j = 0; j < d; ++j)
            book[j] = sq::Lloyd::fit(gather(j, j + 1), std::max(width[j], 1), P.lloyd_max_iter, P.seed + (uint64_t)(j + 10));
    }
    std::memcpy(eig_out, V.data(), kvd * kvd * sizeof(float));
    std::fill(cent_out, cent_out + kvd * sq::kMaxLevels, 0.0f);
    for (int64_t j = 0; j < kvd; ++j) {
        if (book[j].size() > (size_t)sq::kMaxLevels || width[j] > 8) return false;
        bits_out[j] = (uint8_t)width[j];
        lev_out[j] = (int32_t)book[j].size();
        std::copy(book[j].begin(), book[j].end(), cent_out + j * sq::kMaxLevels);
    }
    *d_eff_out = (int32_t)d;
    return true;
}

}  // namespace kg
