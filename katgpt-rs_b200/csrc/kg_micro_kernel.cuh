// kg_micro_kernel.cuh — the exact-order micro forward kernel (micro_forward)
// and its per-thread helpers; kg_micro.cu launches it. The source also
// compiles for the host (the CPU tests run it on host threads, with a barrier
// standing for __syncthreads, and compare it with the oracle), hence the
// dynamic shared-memory declaration through KG_MICRO_SMEM.
#pragma once
#include <cstdint>

#include "kg_exact.cuh"
#include "kg_micro_args.h"

#ifdef __CUDACC__
#define KG_MICRO_SMEM(name) extern __shared__ float4 name[]
#endif

namespace kg {
namespace {

constexpr int MODE_BASE = 0, MODE_QUANT = 1, MODE_SPKV = 2, MODE_PREFILL = 3, MODE_PAGED = 4, MODE_SQ = 5;

template <int KVD>
__device__ __forceinline__ uint8_t quantize(float r, const float *bnd, int nb) {
    int c = 0;
    for (int j = 0; j < nb; ++j) c += (r >= bnd[j]) ? 1 : 0;  // partition_point on monotone boundaries
    return (uint8_t)c;
}

// TurboQuantKVCache::store_* followed by dequantize_*_into for one vector.
// Writes packed codes (unless norm < 1e-8: indices untouched, as the reference)
// and the norm; returns the dequantized vector in `deq`.
template <int KVD>
__device__ __forceinline__ void tq_roundtrip(const float (&vec)[KVD], const float *rot,
                                             const float *rot_t, const float *cent,
                                             const float *bnd, int bits, int pl, uint8_t *codes,
                                             float *norm_out, float (&deq)[KVD]) {
    float ss = kgx::sum_sq<KVD>(vec);
    float norm = sqrtf(ss);
    *norm_out = norm;
    if (norm < 1e-8f) {
#pragma unroll
        for (int i = 0; i < KVD; ++i) deq[i] = 0.0f;
        return;
    }
    float inv = 1.0f / norm;
    float xn[KVD];
#pragma unroll
    for (int i = 0; i < KVD; ++i) xn[i] = vec[i] * inv;
    const int nb = (1 << bits) - 1;
    uint8_t cd[KVD];
#pragma unroll
    for (int i = 0; i < KVD; ++i) cd[i] = quantize<KVD>(kgx::dot<KVD>(rot + i * KVD, xn), bnd, nb);
    // pack (kv_cache.rs:560-632)
    if (bits == 2) {
#pragma unroll
        for (int b = 0; b < (KVD + 3) / 4; ++b) {
            uint8_t v = 0;
#pragma unroll
            for (int s = 0; s < 4; ++s)
                if (4 * b + s < KVD) v |= (uint8_t)((cd[4 * b + s] & 3) << (2 * s));
            codes[b] = v;
        }
    } else if (bits == 3 || bits == 4) {
#pragma unroll
        for (int b = 0; b < (KVD + 1) / 2; ++b) {
            uint8_t v = cd[2 * b] & 15;
            if (2 * b + 1 < KVD) v |= (uint8_t)((cd[2 * b + 1] & 15) << 4);
            codes[b] = v;
        }
    } else {
#pragma unroll
        for (int b = 0; b < KVD; ++b) codes[b] = cd[b];
    }
    (void)pl;
    // dequantize: centroid lookup, R^T * c, * norm
    float c[KVD];
#pragma unroll
    for (int i = 0; i < KVD; ++i) c[i] = cent[cd[i]];
#pragma unroll
    for (int i = 0; i < KVD; ++i) deq[i] = kgx::dot<KVD>(rot_t + i * KVD, c) * norm;
}

// SpectralQuantKVCache store_vector then dequantize_*_into for one vector
// (src/spectralquant/spectral_kv_cache.rs:399-470, 567-672): norm, x / norm,
// rotation y_j = sum_i V[i][j] x_i accumulated in i order (rotate_into), per
// dimension the nearest centroid by bisection (quantize_to_idx), LSB-first
// packing at the dimension's width; then centroids, V c (row dots) and * norm.
// A vector with norm < 1e-8 stores norm 0 and keeps its old codes.
// meta[j] = bits | levels << 8; cent: 64 centroids per dimension.
template <int KVD>
__device__ __forceinline__ void sq_roundtrip(const float (&vec)[KVD], const float *eig, const float *cent,
                                             const float *meta, uint8_t *codes, float *norm_out, float (&deq)[KVD]) {
    const float norm = sqrtf(kgx::sum_sq<KVD>(vec));
    if (norm < 1e-8f) {
        *norm_out = 0.0f;
#pragma unroll
        for (int i = 0; i < KVD; ++i) deq[i] = 0.0f;
        return;
    }
    *norm_out = norm;
    const float inv = 1.0f / norm;
    float xn[KVD], y[KVD];
#pragma unroll
    for (int i = 0; i < KVD; ++i) xn[i] = vec[i] * inv;
#pragma unroll
    for (int j = 0; j < KVD; ++j) y[j] = 0.0f;
#pragma unroll
    for (int i = 0; i < KVD; ++i)
#pragma unroll
        for (int j = 0; j < KVD; ++j) y[j] = y[j] + eig[i * KVD + j] * xn[i];
    uint8_t idx[KVD];
    uint64_t buf = 0;
    uint32_t have = 0;
    int w = 0;
#pragma unroll
    for (int j = 0; j < KVD; ++j) {
        const int m = __float_as_int(meta[j]);
        const int bits = m & 255, n = m >> 8;
        const float *c = cent + j * kSqLevels;
        int q = 0;
        if (n > 1) {
            int lo = 0, hi = n - 1;
            const float v = y[j];
            if (v <= c[lo]) q = lo;
            else if (v >= c[hi]) q = hi;
            else {
                while (lo + 1 < hi) {
                    const int mid = lo + (hi - lo) / 2;
                    if (c[mid] <= v) lo = mid;
                    else hi = mid;
                }
                q = fabsf(v - c[lo]) <= fabsf(c[hi] - v) ? lo : hi;
            }
        }
        idx[j] = (uint8_t)q;
        buf |= (uint64_t)q << have;  // pack_variable_bits (:1125-1164)
        have += bits;
        while (have >= 8) {
            codes[w++] = (uint8_t)(buf & 0xFF);
            buf >>= 8;
            have -= 8;
        }
    }
    if (have > 0) codes[w++] = (uint8_t)(buf & 0xFF);
    float cv[KVD];
#pragma unroll
    for (int j = 0; j < KVD; ++j) cv[j] = idx[j] < (__float_as_int(meta[j]) >> 8) ? cent[j * kSqLevels + idx[j]] : 0.0f;
#pragma unroll
    for (int i = 0; i < KVD; ++i) deq[i] = kgx::dot<KVD>(eig + i * KVD, cv) * norm;
}

// rmsnorm (math.rs:56-69): x * (1 / sqrt(sum_sq/n + 1e-5))
template <int N>
__device__ __forceinline__ void rmsnorm(float (&x)[N]) {
    float ss = kgx::sum_sq<N>(x);
    float inv = 1.0f / sqrtf(ss / (float)N + 1e-5f);
#pragma unroll
    for (int i = 0; i < N; ++i) x[i] = x[i] * inv;
}
// rmsnorm_with_gamma (math.rs:218-233 -> simd_scale_mul_inplace, elementwise.rs:1249-1270):
// g * (x * inv) over whole 8-lane chunks, (g * x) * inv in the scalar tail
template <int N>
__device__ __forceinline__ void rmsnorm_gamma(float (&x)[N], const float *g) {
    float ss = kgx::sum_sq<N>(x);
    float inv = 1.0f / sqrtf(ss / (float)N + 1e-5f);
    constexpr int BODY = N / 8 * 8;
#pragma unroll
    for (int i = 0; i < N; ++i) x[i] = i < BODY ? g[i] * (x[i] * inv) : (g[i] * x[i]) * inv;
}

// Delta routing at a routing layer l (l % 4 == 3; transformer.rs:1707-1765,
// :287-320): sources are blocks 0..b-1 (already zeroed) and block b = `delta`;
// softmax over the logits dot(gamma * rmsnorm(source), query) with the Cephes
// exp, then x += w_s * source.
template <int N>
__device__ __forceinline__ void route_block(float (&x)[N], const float (&delta)[N], int l, const float *qw,
                                            const float *nw) {
    const int b = l >> 2;
    float lg[16];
    float zero_logit;
    {
        float z[N];
#pragma unroll
        for (int j = 0; j < N; ++j) z[j] = 0.0f;
        float rms = sqrtf(kgx::sum_sq<N>(z) / (float)N + 1e-5f);
        float inv = 1.0f / rms;
#pragma unroll
        for (int j = 0; j < N; ++j) z[j] = (j < N / 8 * 8) ? nw[j] * (z[j] * inv) : nw[j] * z[j] * inv;
        zero_logit = kgx::dot<N>(z, qw);
    }
    float own_logit;
    {
        float sd[N];
        float rms = sqrtf(kgx::sum_sq<N>(delta) / (float)N + 1e-5f);
        float inv = 1.0f / rms;
#pragma unroll
        for (int j = 0; j < N; ++j) sd[j] = (j < N / 8 * 8) ? nw[j] * (delta[j] * inv) : nw[j] * delta[j] * inv;
        own_logit = kgx::dot<N>(sd, qw);
    }
    const int ns = b + 1;
    float mx = -INFINITY;
#pragma unroll
    for (int s = 0; s < 16; ++s) {
        lg[s] = s < b ? zero_logit : own_logit;
        if (s < ns) mx = kgx::fmax_rs(mx, lg[s]);
    }
    const int body = ns / 8 * 8;
#pragma unroll
    for (int s = 0; s < 16; ++s) {
        float e = lg[s] + (-mx);
        lg[s] = s < body ? kgx::cephes_lane(e, true) : kgx::cephes_scalar(e);
    }
    float se = kgx::sum_rt<16>(lg, ns);
    float inv_sum = 1.0f / se;
#pragma unroll
    for (int s = 0; s < 16; ++s)
        if (s < ns) {
            float w = lg[s] * inv_sum;
#pragma unroll
            for (int j = 0; j < N; ++j) {
                float src = s < b ? 0.0f : delta[j];
                x[j] = (j < N / 8 * 8) ? fmaf(w, src, x[j]) : x[j] + w * src;
            }
        }
}

// lora_apply (crates/katgpt-types/src/lora.rs:452-467) with adapter `w` of the
// pack (kgx::lora_apply16: rank, in_dim, out_dim <= kLoraMax).
template <int OUTN, int INN>
__device__ __forceinline__ void lora_apply(float (&out)[OUTN], const float (&in)[INN], const MicroArgs &p, int w,
                                           const float *sm) {
    static_assert(OUTN >= kLoraMax && INN >= kLoraMax && kLoraMax == 16, "adapter wider than the arrays");
    kgx::lora_apply16(out, in, sm + p.off_lora_a[w], sm + p.off_lora_b[w], p.lora_rank[w], p.lora_in[w],
                      p.lora_out[w], p.lora_scale[w]);
}

// LORA: the pair's reader (MODE_PREFILL) or writer (MODE_BASE, MODE_SPKV) is
// applied after each of the six projections (src/transformer.rs:1904-1941,
// 2018-2020, 2036-2038, 2110-2112; forward_prefill :2681-2687, 2738-2740,
// 2901-2903, 2916-2918, 2949-2951; src/sp_kv/forward.rs:673-684, 753-756,
// 769-771, 805-807).
template <int N, int NH, int NKV, int HD, int M, int VOC, int BLK, int MODE, bool LORA = false>
__global__ void __launch_bounds__(128, 3) micro_forward(const MicroArgs p) {
    constexpr int KVD = NKV * HD;
    constexpr int PH = (N / 4 > 16) ? N / 4 : 16;
    KG_MICRO_SMEM(sm4);
    float *sm = reinterpret_cast<float *>(sm4);
    {
        const float4 *src = reinterpret_cast<const float4 *>(p.pack);
        for (int e = threadIdx.x; e < p.pack_floats / 4; e += blockDim.x) sm4[e] = src[e];
    }
    __syncthreads();

    const int T = p.T;
    const int SB = blockDim.x / T;
    const int sl = threadIdx.x / T, tl = threadIdx.x - sl * T;
    const int n_groups = (p.n_seq + SB - 1) / SB;
    float *scs = sm + p.pack_floats + threadIdx.x * (BLK + 1);  // per-thread score row
    // forward_prefill: this sequence's block-delta accumulator
    float *dacc = sm + p.pack_floats + blockDim.x * (BLK + 1) + (threadIdx.x / p.T) * N;
    for (int grp = blockIdx.x; grp < n_groups; grp += gridDim.x) {
    __syncthreads();  // previous group's attention reads are done
    const int i = grp * SB + sl;
    bool active = (sl < SB) && (i < p.n_seq);
    int slot = 0, pos = 0, tok = 0;
    if (active) {
        slot = p.seq_ids[i];
        pos = (p.start_pos ? p.start_pos[i] : 0) + tl;
        tok = p.tokens[(int64_t)i * T + tl];
        if (slot < 0 || slot >= p.n_slots || pos < 0 || pos >= BLK || tok < 0 || tok >= VOC) {
            atomicExch(p.err, 1);
            active = false;
        }
    }
    if constexpr (MODE == MODE_PAGED) {
        // every page this position reads or writes must exist (ensure_pages ran)
        for (int l = 0; active && l < p.L; ++l) {
            const int32_t *tab = p.ptab + ((int64_t)l * p.n_slots + slot) * p.maxp;
            for (int q = 0; q <= pos / 16; ++q) {
                const int pg = q < p.maxp ? tab[q] : -1;
                if (pg < 0 || pg >= p.n_pages) {
                    atomicExch(p.err, 1);
                    active = false;
                    break;
                }
            }
        }
    }
    if constexpr (MODE == MODE_PREFILL) {
        if (tl == 0)
#pragma unroll
            for (int j = 0; j < N; ++j) dacc[j] = 0.0f;
    }
    const float *wte = sm + p.off_wte, *wpe = sm + p.off_wpe;
    float x[N];
#pragma unroll
    for (int j = 0; j < N; ++j) x[j] = active ? wte[tok * N + j] + wpe[pos * N + j] : 0.0f;
    float delta[N];
#pragma unroll
    for (int j = 0; j < N; ++j) delta[j] = 0.0f;
    const float scale = 1.0f / sqrtf((float)HD);

    for (int l = 0; l < p.L; ++l) {
        const float *wl = sm + p.off_layers + l * p.layer_stride;
        const float *wq = wl, *wk = wq + N * N, *wv = wk + KVD * N, *wo = wv + KVD * N;
        const float *w1 = wo + N * N, *w2 = w1 + M * N;
        const int64_t row = ((int64_t)slot * p.L + l) * BLK;  // [slot][layer] base (positions)

        // forward_base (kog_cpu_fusion) applies attn_norm_gamma at run time
        // (src/transformer.rs:1893-1895); the quantized forwards use plain rmsnorm
        if constexpr (MODE == MODE_BASE)
            rmsnorm_gamma<N>(x, sm + p.off_ag + l * N);
        else
            rmsnorm<N>(x);
        float xr[N];
#pragma unroll
        for (int j = 0; j < N; ++j) xr[j] = x[j];
        // forward_prefill's double norm (:2674-2677), forward_paged's (:3361-3364)
        if constexpr (MODE == MODE_PREFILL || MODE == MODE_PAGED) rmsnorm<N>(x);
        float util = 0.0f;
        if constexpr (MODE == MODE_SPKV) {
            rmsnorm<N>(x);  // double norm (sp_kv/forward.rs:648-651)
            const float *pw1 = sm + p.off_pw1, *pb1 = sm + p.off_pb1;
            const float *pw2 = sm + p.off_pw2, *pb2 = sm + p.off_pb2;
            float hbuf[PH];
#pragma unroll
            for (int h = 0; h < PH; ++h) {
                float v = kgx::dot<N>(pw1 + h * N, x) + pb1[h];
                hbuf[h] = v * (1.0f / (1.0f + kgx::expf_libm(-v)));  // silu
            }
#pragma unroll
            for (int kh = 0; kh < NKV; ++kh) {
                float u = 1.0f / (1.0f + kgx::expf_libm(-(kgx::dot<PH>(pw2 + kh * PH, hbuf) + pb2[kh])));
                util = kh == 0 ? u : kgx::fmax_rs(util, u);
            }
        }
        float q[N], k[KVD], v[KVD];
#pragma unroll
        for (int r = 0; r < N; ++r) q[r] = kgx::dot<N>(wq + r * N, x);
#pragma unroll
        for (int r = 0; r < KVD; ++r) k[r] = kgx::dot<N>(wk + r * N, x);
#pragma unroll
        for (int r = 0; r < KVD; ++r) v[r] = kgx::dot<N>(wv + r * N, x);
        [[maybe_unused]] constexpr int LW = MODE == MODE_PREFILL ? 0 : 1;  // LoraPair: reader in prefill, writer in decode
        if constexpr (LORA) {
            lora_apply(q, x, p, LW, sm);
            lora_apply(k, x, p, LW, sm);
            lora_apply(v, x, p, LW, sm);
        }

        // forward_paged: this layer's page list of the sequence; a position's K
        // row sits at page * 32 + pos % 16 rows of the pool, its V row 16 rows on
        const int32_t *ptab_l = MODE == MODE_PAGED ? p.ptab + ((int64_t)l * p.n_slots + slot) * p.maxp : nullptr;
        if (active) {
            float *kd, *vd;
            if constexpr (MODE == MODE_PAGED) {
                kd = p.pool + ((int64_t)ptab_l[pos >> 4] * 32 + (pos & 15)) * KVD;  // write_kv (:298-309)
                vd = kd + 16 * KVD;
            } else {
                kd = p.Kf + (row + pos) * KVD;
                vd = p.Vf + (row + pos) * KVD;
            }
            if constexpr (MODE == MODE_BASE || MODE == MODE_PREFILL || MODE == MODE_PAGED) {
#pragma unroll
                for (int j = 0; j < KVD; ++j) {
                    kd[j] = k[j];
                    vd[j] = v[j];
                }
            } else if constexpr (MODE == MODE_SQ) {
                uint8_t *cb = p.codes + (row + pos) * (p.kpl + p.vpl);
                float *nb = p.norms + (row + pos) * 2;
                const float *eig = sm + p.off_sq_eig + l * KVD * KVD, *cent = sm + p.off_sq_cent + l * KVD * kSqLevels;
                const float *meta = sm + p.off_sq_meta + l * KVD;
                float dk[KVD], dv[KVD];
                sq_roundtrip<KVD>(k, eig, cent, meta, cb, nb, dk);  // keys and values share the layer's tables
                sq_roundtrip<KVD>(v, eig, cent, meta, cb + p.kpl, nb + 1, dv);
#pragma unroll
                for (int j = 0; j < KVD; ++j) {
                    kd[j] = dk[j];
                    vd[j] = dv[j];
                }
            } else {
                uint8_t *cb = p.codes + (row + pos) * (p.kpl + p.vpl);
                float *nb = p.norms + (row + pos) * 2;
                float dk[KVD], dv[KVD];
                tq_roundtrip<KVD>(k, sm + p.off_rot, sm + p.off_rot_t, sm + p.off_kc, sm + p.off_kb,
                                  p.kbits, p.kpl, cb, nb, dk);
                tq_roundtrip<KVD>(v, sm + p.off_rot, sm + p.off_rot_t, sm + p.off_vc, sm + p.off_vb,
                                  p.vbits, p.vpl, cb + p.kpl, nb + 1, dv);
#pragma unroll
                for (int j = 0; j < KVD; ++j) {
                    kd[j] = dk[j];
                    vd[j] = dv[j];
                }
                if constexpr (MODE == MODE_SPKV) p.util[row + pos] = util;
            }
        }
        __syncthreads();  // every position of this layer is written

        // ---- attention over positions 0..pos
        float att[N];
        // forward_prefill attends every prompt position (bidirectional, :2863)
        const int tn = MODE == MODE_PREFILL ? T : pos + 1;
        const float *Kb = p.Kf + row * KVD, *Vb = p.Vf + row * KVD;
        auto krow = [&](int t) -> const float * {
            if constexpr (MODE == MODE_PAGED) return p.pool + ((int64_t)ptab_l[t >> 4] * 32 + (t & 15)) * KVD;
            else return Kb + t * KVD;
        };
        auto vrow = [&](int t) -> const float * {
            if constexpr (MODE == MODE_PAGED) return p.pool + ((int64_t)ptab_l[t >> 4] * 32 + 16 + (t & 15)) * KVD;
            else return Vb + t * KVD;
        };
#pragma unroll 1
        for (int h = 0; h < NH; ++h) {
            const int g = h * NKV / NH;
            float qh[HD];
#pragma unroll
            for (int d = 0; d < HD; ++d) qh[d] = q[h * HD + d];
            float o[HD];
#pragma unroll
            for (int d = 0; d < HD; ++d) o[d] = 0.0f;
            if (active) {
                if constexpr (MODE != MODE_SPKV) {
                    // attention_head: dot, scale, max, shift, Cephes exp, sum, normalise, P.V
                    float mx = 0.0f;
#pragma unroll 1
                    for (int t = 0; t < tn; ++t) {
                        float sv = kgx::dot<HD>(qh, krow(t) + g * HD) * scale;
                        scs[t] = sv;
                        mx = (t == 0 || sv > mx) ? sv : mx;
                    }
                    const int body = tn / 8 * 8;
#pragma unroll 1
                    for (int t = 0; t < tn; ++t) {
                        float e = scs[t] + (-mx);
                        scs[t] = t < body ? kgx::cephes_lane(e, true) : kgx::cephes_scalar(e);
                    }
                    float ssum;
                    if constexpr (BLK < 32) ssum = kgx::sum_small<BLK>(scs, tn);
                    else ssum = kgx::sum_rt<BLK>(*reinterpret_cast<const float(*)[BLK]>(scs), tn);
                    float inv = 1.0f / ssum;
#pragma unroll 1
                    for (int t = 0; t < tn; ++t) {
                        const float pt = scs[t] * inv;
                        const float *vr = vrow(t) + g * HD;
#pragma unroll
                        for (int d = 0; d < HD; ++d)  // fused_scale_acc: fma body, mul+add tail
                            o[d] = (d < HD / 8 * 8) ? fmaf(pt, vr[d], o[d]) : o[d] + pt * vr[d];
                    }
                } else {
                    // attention_head_core<GateBias>: bias 0 for every position (each
                    // written position is retained; block_size <= window)
                    float mx = -INFINITY;
#pragma unroll 1
                    for (int t = 0; t < tn; ++t) {
                        float sv = kgx::dot<HD>(qh, Kb + t * KVD + g * HD) * scale + 0.0f;
                        scs[t] = sv;
                        mx = kgx::fmax_rs(mx, sv);
                    }
                    float sum = 0.0f;
#pragma unroll 1
                    for (int t = 0; t < tn; ++t) {
                        float e = kgx::expf_libm(scs[t] - mx);
                        scs[t] = e;
                        sum = sum + e;
                    }
                    const float inv = 1.0f / sum;
#pragma unroll 1
                    for (int t = 0; t < tn; ++t) {
                        const float pt = scs[t] * inv;
                        const float *vr = Vb + t * KVD + g * HD;
#pragma unroll
                        for (int d = 0; d < HD; ++d) o[d] = o[d] + pt * vr[d];
                    }
                }
            }
#pragma unroll
            for (int d = 0; d < HD; ++d) att[h * HD + d] = o[d];
        }

        // ---- output projection + residual
        float xo[N];
#pragma unroll
        for (int r = 0; r < N; ++r) xo[r] = kgx::dot<N>(wo + r * N, att);
        if constexpr (LORA) lora_apply(xo, att, p, LW, sm);
#pragma unroll
        for (int j = 0; j < N; ++j) x[j] = xo[j] + xr[j];

        // ---- MLP: xr2 = x; norm; relu(W1 x); TwELL sparse / dense W2; += xr2
        float xr2[N];
#pragma unroll
        for (int j = 0; j < N; ++j) xr2[j] = x[j];
        if constexpr (MODE == MODE_BASE)
            rmsnorm_gamma<N>(x, sm + p.off_mg + l * N);  // mlp_norm_gamma (src/transformer.rs:2023-2026)
        else
            rmsnorm<N>(x);
        float hid[M];
        int alive = 0;
#pragma unroll
        for (int r = 0; r < M; ++r) {
            float s = kgx::dot<N>(w1 + r * N, x);
            hid[r] = s > 0.0f ? s : 0.0f;
            alive += hid[r] > 0.0f ? 1 : 0;
        }
        if constexpr (LORA) {  // onto the post-ReLU activations; sparse_matmul counts after it
            lora_apply(hid, x, p, LW, sm);
            alive = 0;
#pragma unroll
            for (int r = 0; r < M; ++r) alive += hid[r] > 0.0f ? 1 : 0;
        }
        if ((float)alive / (float)M > (1.0f - p.sparse_threshold)) {
#pragma unroll
            for (int r = 0; r < N; ++r) x[r] = kgx::dot<M>(w2 + r * M, hid);
        } else {
            // sparse_matmul: ascending alive list, gathered dot (sparse.rs:22-75,159-218)
            int aidx[M];
            float aval[M];
            int na = 0;
            for (int c = 0; c < M; ++c)
                if (hid[c] > 0.0f) {
                    aidx[na] = c;
                    aval[na] = hid[c];
                    ++na;
                }
            for (int r = 0; r < N; ++r) {
                const float *wr = w2 + r * M;
                float s;
                if (na <= 4) {
                    s = 0.0f;
                    for (int a = 0; a < na; ++a) s = s + wr[aidx[a]] * aval[a];
                } else {
                    float acc[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) acc[u] = 0.0f;
                    int a = 0;
                    for (; a + 8 <= na; a += 8)
#pragma unroll
                        for (int u = 0; u < 8; ++u) acc[u] = fmaf(wr[aidx[a + u]], aval[a + u], acc[u]);
                    s = kgx::hsum8(acc);
                    for (; a < na; ++a) s = s + wr[aidx[a]] * aval[a];
                }
                x[r] = s;
            }
        }
        if constexpr (LORA) lora_apply(x, hid, p, LW, sm);
#pragma unroll
        for (int j = 0; j < N; ++j) x[j] = x[j] + xr2[j];

        // ---- delta routing (not in the sp_kv path)
        if constexpr (MODE == MODE_PREFILL) {
            // forward_prefill keeps one set of block deltas for the whole
            // prompt (src/transformer.rs:2954-2982): positions add their delta
            // in order, and at a routing layer each position routes with the
            // accumulator as it stands and zeroes it. One barrier round per
            // position, the sequence's accumulator in shared memory.
            const float *qw = sm + p.off_dq + l * N, *nw = sm + p.off_dn + l * N;
            for (int rnd = 0; rnd < T; ++rnd) {
                if (active && tl == rnd) {
#pragma unroll
                    for (int j = 0; j < N; ++j) dacc[j] = dacc[j] + (x[j] - xr[j]);
                    if ((l & 3) == 3) {
                        float dl[N];
#pragma unroll
                        for (int j = 0; j < N; ++j) dl[j] = dacc[j];
                        route_block<N>(x, dl, l, qw, nw);
#pragma unroll
                        for (int j = 0; j < N; ++j) dacc[j] = 0.0f;
                    }
                }
                __syncthreads();
            }
        } else if constexpr (MODE != MODE_SPKV) {
#pragma unroll
            for (int j = 0; j < N; ++j) delta[j] = delta[j] + (x[j] - xr[j]);
            if ((l & 3) == 3) {
                route_block<N>(x, delta, l, sm + p.off_dq + l * N, sm + p.off_dn + l * N);
#pragma unroll
                for (int j = 0; j < N; ++j) delta[j] = 0.0f;
            }
        }
    }

    // ---- lm_head (+ softmax_scaled); forward_prefill returns the last position's
    if (!active) continue;
    if constexpr (MODE == MODE_PREFILL) {
        if (tl != T - 1) continue;
    }
    const float *lm = sm + p.off_lm;
    float lg[VOC];
#pragma unroll
    for (int r = 0; r < VOC; ++r) lg[r] = kgx::dot<N>(lm + r * N, x);
    const int64_t orow = (MODE == MODE_PREFILL ? (int64_t)i : (int64_t)i * T + tl) * VOC;
    if (p.logits) {
#pragma unroll
        for (int r = 0; r < VOC; ++r) p.logits[orow + r] = lg[r];
    }
    if (p.probs) {
        float mx = lg[0];
#pragma unroll
        for (int r = 1; r < VOC; ++r) mx = lg[r] > mx ? lg[r] : mx;
#pragma unroll
        for (int r = 0; r < VOC; ++r) lg[r] = (lg[r] - mx) * p.inv_temp;
        // simd_exp_sum_inplace: unclamped lanes over 8-chunks, scalar tail
        constexpr int C4 = VOC / 32, REM = (VOC - C4 * 32) / 8, T0 = C4 * 32 + REM * 8;
        float acc[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) acc[u] = 0.0f;
#pragma unroll
        for (int r = 0; r < C4 * 32; ++r) {
            lg[r] = kgx::cephes_lane(lg[r], false);
            acc[r & 31] = acc[r & 31] + lg[r];
        }
        float t8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) t8[u] = (acc[u] + acc[8 + u]) + (acc[16 + u] + acc[24 + u]);
        float sum = kgx::hsum8(t8);
        float rr[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) rr[u] = 0.0f;
#pragma unroll
        for (int r = C4 * 32; r < T0; ++r) {
            lg[r] = kgx::cephes_lane(lg[r], false);
            rr[(r - C4 * 32) & 7] = rr[(r - C4 * 32) & 7] + lg[r];
        }
        sum = sum + kgx::hsum8(rr);
#pragma unroll
        for (int r = T0; r < VOC; ++r) {
            lg[r] = kgx::cephes_scalar(lg[r]);
            sum = sum + lg[r];
        }
        float inv = 1.0f / sum;
#pragma unroll
        for (int r = 0; r < VOC; ++r) p.probs[orow + r] = lg[r] * inv;
    }
    }  // sequence groups
}

}  // namespace
}  // namespace kg
