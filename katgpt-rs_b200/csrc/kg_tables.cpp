// kg_tables.cpp — host-side construction of everything the device path needs
// bit-identically to the reference: the XorShift64 Rng and its Box-Muller
// normals, TransformerWeights::new, the TurboQuant Lloyd-Max codebook and the
// Gaussian matrix the rotation is built from, and the SP-KV predictor weights.
//
// Built with g++ -O2 -ffp-contract=off (no fast-math): the reference never
// fuses multiply-adds in these routines, and it calls the glibc libm
// functions (logf, cosf, powf, log, exp, sin) that this file calls.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/kg_abi.h"

namespace kg {

// crates/katgpt-types/src/rng.rs:26-72
struct HostRng {
    uint64_t s;
    explicit HostRng(uint64_t seed) {
        uint64_t z = seed + 0x9E3779B97F4A7C15ULL;  // SplitMix64 finaliser
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
        z ^= z >> 31;
        s = z ? z : 1;
    }
    uint64_t next() {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        return s;
    }
    float uniform() {
        uint32_t b = ((uint32_t)(next() >> 40) & 0x7fffffu) | 0x3f800000u;
        float f;
        std::memcpy(&f, &b, 4);
        return f - 1.0f;
    }
    float normal() {
        float u1 = uniform();
        if (!(u1 > 1e-10f)) u1 = 1e-10f;
        float u2 = uniform();
        return sqrtf(-2.0f * logf(u1)) * cosf((2.0f * 3.14159265358979323846f) * u2);
    }
};

uint64_t host_rng_seed_state(uint64_t seed) { return HostRng(seed).s; }
uint64_t host_rng_next_state(uint64_t &state) {
    HostRng r(0);
    r.s = state;
    const uint64_t v = r.next();
    state = r.s;
    return v;
}
float host_rng_normal(uint64_t &state) {
    HostRng r(0);
    r.s = state;
    const float v = r.normal();
    state = r.s;
    return v;
}

void host_normals(uint64_t seed, int64_t n, float *out) {
    HostRng r(seed);
    for (int64_t i = 0; i < n; ++i) out[i] = r.normal();
}

int64_t weights_count(const kg_config &c) {
    int64_t n = c.n_embd, kvd = (int64_t)c.n_kv_head * c.head_dim, m = c.mlp_hidden;
    int64_t per_layer = 2 * n * n + 2 * kvd * n + 2 * m * n;
    return (int64_t)c.vocab_size * n * 2 + (int64_t)c.block_size * n + c.n_layer * per_layer +
           4 * (int64_t)c.n_layer * n;
}

// crates/katgpt-transformer/src/weights.rs:76-177
void reference_weights(const kg_config &c, uint64_t seed, int scale_mode, float std_, float *out) {
    HostRng rng(seed);
    const int64_t n = c.n_embd, kvd = (int64_t)c.n_kv_head * c.head_dim, m = c.mlp_hidden;
    float es = sqrtf(2.0f / (float)n);
    float ls = sqrtf(2.0f / ((float)n * (float)c.n_layer));
    if (scale_mode == 1) es = ls = std_;
    float *p = out;
    for (int64_t i = 0; i < (int64_t)c.vocab_size * n; ++i) *p++ = rng.normal() * es;
    for (int64_t i = 0; i < (int64_t)c.block_size * n; ++i) *p++ = rng.normal() * es;
    for (int64_t l = 0; l < c.n_layer; ++l) {
        int64_t cnt = 2 * n * n + 2 * kvd * n + 2 * m * n;
        for (int64_t i = 0; i < cnt; ++i) *p++ = rng.normal() * ls;
    }
    for (int64_t i = 0; i < (int64_t)c.vocab_size * n; ++i) *p++ = rng.normal() * es;
    for (int64_t i = 0; i < (int64_t)c.n_layer * n; ++i) *p++ = 0.0f;  // delta_routing_query
    for (int64_t i = 0; i < (int64_t)c.n_layer * n; ++i) *p++ = 1.0f;  // delta_routing_norm
    for (int64_t i = 0; i < (int64_t)c.n_layer * n; ++i) *p++ = 1.0f;  // attn_norm_gamma (weights.rs:142-143)
    for (int64_t i = 0; i < (int64_t)c.n_layer * n; ++i) *p++ = 1.0f;  // mlp_norm_gamma (weights.rs:144-145)
}

// ---- Lloyd-Max codebook, src/turboquant/codebook.rs:20-198 ----
static double lanczos_ln_gamma(double x) {
    static const double cf[9] = {0.99999999999980993,  676.5203681218851,   -1259.1392167224028,
                                 771.32342877765313,   -176.61502916214059, 12.507343278686905,
                                 -0.13857109526572012, 9.9843695780195716e-6, 1.5056327351493116e-7};
    const double pi = 3.14159265358979323846;
    if (x < 0.5) return pi / log(sin(pi * x)) - lanczos_ln_gamma(1.0 - x);
    double z = x - 1.0, t = z + 7.0 + 0.5, a = cf[0];
    for (int i = 1; i < 9; ++i) a = a + cf[i] / (z + (double)(i - 1) + 1.0);
    return ((log(sqrt(2.0 * pi)) + log(t + 0.5) * (z + 0.5)) - t) + log(a);
}
static float marginal_pdf(float x, int64_t d) {
    if (fabsf(x) >= 1.0f) return 0.0f;
    const double pi = 3.14159265358979323846;
    double df = (double)d;
    float c = (float)exp(lanczos_ln_gamma(df / 2.0) - lanczos_ln_gamma((df - 1.0) / 2.0) - log(pi / 2.0));
    return c * powf(1.0f - x * x, (float)(d - 3) / 2.0f);
}
static void centroids_of(const std::vector<float> &bnd, int64_t dim, std::vector<float> &out) {
    const size_t nl = bnd.size() + 1;
    std::vector<float> e(nl + 1);
    e[0] = -1.0f;
    for (size_t i = 0; i < bnd.size(); ++i) e[i + 1] = bnd[i];
    e[nl] = 1.0f;
    out.assign(nl, 0.0f);
    for (size_t i = 0; i < nl; ++i) {
        const float lo = e[i], hi = e[i + 1], dx = (hi - lo) / 1000.0f;
        double m0 = 0.0, m1 = 0.0;
        for (int j = 0; j <= 1000; ++j) {
            float xx = lo + dx * (float)j;
            float f = marginal_pdf(xx, dim);
            double w = (j == 0 || j == 1000) ? 0.5 : 1.0;
            m0 += (double)f * w;
            m1 += (double)xx * (double)f * w;
        }
        out[i] = m0 > 1e-12 ? (float)(m1 / m0) : (lo + hi) / 2.0f;
    }
}
void lloyd_max(int64_t dim, int bits, std::vector<float> &cent, std::vector<float> &bnd) {
    const int64_t nl = (int64_t)1 << bits;
    bnd.assign(nl - 1, 0.0f);
    for (int64_t i = 0; i < nl - 1; ++i) bnd[i] = -1.0f + 2.0f * (float)(i + 1) / (float)nl;
    std::vector<float> c, nb(nl - 1);
    for (int it = 0; it < 50; ++it) {
        centroids_of(bnd, dim, c);
        bool done = true;
        for (int64_t i = 0; i < nl - 1; ++i) {
            nb[i] = (c[i] + c[i + 1]) / 2.0f;
            if (!(fabsf(bnd[i] - nb[i]) < 1e-6f)) done = false;
        }
        bnd = nb;
        if (done) break;
    }
    centroids_of(bnd, dim, cent);
}

// SP-KV utility predictor weights (src/sp_kv/types.rs:224-258): every layer
// draws from a fresh Rng::new(42). Layout per layer: w1[h*n], b1[h], w2[nkv*h], b2[nkv].
void predictor_weights(int64_t n, int64_t hidden, int64_t nkv, float init_bias, std::vector<float> &out) {
    HostRng rng(42);
    float s1 = sqrtf(2.0f / (float)n), s2 = sqrtf(2.0f / (float)hidden);
    out.clear();
    for (int64_t i = 0; i < hidden * n; ++i) out.push_back(rng.normal() * s1);
    for (int64_t i = 0; i < hidden; ++i) out.push_back(0.0f);
    for (int64_t i = 0; i < nkv * hidden; ++i) out.push_back(rng.normal() * s2);
    for (int64_t i = 0; i < nkv; ++i) out.push_back(init_bias);
}

}  // namespace kg
