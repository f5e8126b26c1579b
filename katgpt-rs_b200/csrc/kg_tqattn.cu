// kg_tqattn.cu — decode attention over the 4-bit / 3-bit TurboQuant KV cache
// as two streaming kernels.
//
// Math, in the rotated domain (forward_quantized attention,
// src/transformer.rs:4123-4141; softmax src/transformer.rs:333-389; a stored
// vector is norm * R^T centroid(code), src/turboquant/kv_cache.rs:279-317):
//   s[t,h] = norm_k[t] * scale * <centroid(code_k[t]), q~_h>
//   u~_h   = sum_t softmax_t(s[., h])[t] * norm_v[t] * centroid(code_v[t])
//
// Scores (per token, positions in 32-row units): code bytes become f16
// centroid pairs through a 32-replica shared-memory table (entry (b, r) is
// word 32 b + r and lane l reads replica l, so a lookup never conflicts), and
// mma.sync m16n8k16 runs with positions as M, heads as N and dims as K. Per
// 16-position chunk c the kernel writes the head maxima c_h, the sums
// l_h = sum_t exp(s - c_h) and e[h,t] = exp(s - c_h) * norm_v[t] (f16).
//   tq_scores_kernel: CTA = (segment of a token's units, token); two groups of
//     G warps, each group owning two shared-memory unit buffers filled by
//     bulk copies (one row per lane) on an mbarrier; the warps of a group split
//     the 64-dim blocks and keep their q~ fragments in registers, exchange the
//     partial sums through shared memory and each finalises its share of the
//     (m-tile, head-tile) pieces.
//   tq_scores_stream_kernel (shapes whose q~ does not fit in registers): CTA =
//     (128-position chunk, token), every warp streams its 32 rows' code bytes
//     into registers, q~ through L1.
// tq_values_kernel: CTA = (block of 8 NJ dims, token), four warps over
//   interleaved 16-position k-steps, each with its own cp.async ring of code
//   rows and e tiles. From the chunk maxima: M_h, l = sum_c l_c exp(c - M_h)
//   and the factors exp(c - M_h). A = e * factor (heads x positions, f16, via
//   ldmatrix), B = value centroids (positions x dims): the low (high) nibbles
//   of two positions' code bytes are merged into one byte, whose table entry is
//   exactly the B register pairing those positions for one dim. The warps'
//   partial sums combine in shared memory; u~ = sum / l as f16 hi / lo.
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "kg_async.cuh"
#include "kg_attn.cuh"
#include "kg_dev.cuh"
#include "kg_pdl.cuh"

namespace kg {
namespace attn {
namespace {

constexpr int TQ_CH = 128;     // positions per CTA of the streaming scores kernel; Sp granularity
constexpr int LUT32 = 256 * 32;

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2bits(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ uint32_t hmul2(uint32_t x, __half2 f) {
    __half2 v = __hmul2(*reinterpret_cast<__half2 *>(&x), f);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bar_named(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

// byte b -> (centroid[b & 15], centroid[b >> 4]) as an f16 pair, 32 replicas:
// entry (b, r) at word 32 b + r (centroid tables hold 16 entries, zero-padded
// for 3-bit codebooks)
__device__ __forceinline__ void build_lut32(uint32_t *lut, const float *cent) {
    for (int i = threadIdx.x; i < LUT32 / 4; i += blockDim.x) {
        const int b = i >> 3;
        const uint32_t v = h2bits(__ldg(cent + (b & 15)), __ldg(cent + (b >> 4)));
        reinterpret_cast<uint4 *>(lut)[i] = make_uint4(v, v, v, v);
    }
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];\n" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ float ldsf(uint32_t addr) { return __uint_as_float(lds32(addr)); }
template <typename CW>
__device__ __forceinline__ CW lds_cw(uint32_t addr);
template <>
__device__ __forceinline__ uint2 lds_cw<uint2>(uint32_t addr) { return lds64(addr); }
template <>
__device__ __forceinline__ uint32_t lds_cw<uint32_t>(uint32_t addr) { return lds32(addr); }
// table entry of byte k (0..3) of w for this lane (lut_lane = shared address
// of the table + 4 lane)
__device__ __forceinline__ uint32_t lk(uint32_t lut_lane, uint32_t w, int k) {
    return lds32(lut_lane + (__byte_perm(w, 0u, 0x4440u | (uint32_t)k) << 7));
}
__device__ __forceinline__ uint32_t word_of(const uint2 &v, int wi) { return wi == 0 ? v.x : v.y; }
__device__ __forceinline__ uint32_t word_of(const uint32_t &v, int) { return v; }

// Finalise one (m-tile, head-tile) piece of a 32-position unit: d[e] holds
// rows g + 8 (e >> 1) of the m-tile, heads 8 jj + 2 t + (e & 1). Writes e, the
// 16-position chunk maxima and sums.
__device__ __forceinline__ void finalize_piece(const TqAttnArgs &a, const float (&d)[4], int m, int p, int jj,
                                               int g, int t, int tn, const float (&kn)[2], const float (&vn)[2]) {
    // p = first position of the m-tile
    float s[4];
    bool valid[2];
    valid[0] = p + g < tn;
    valid[1] = p + g + 8 < tn;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        s[e] = d[e] * kn[e >> 1];
        if (valid[e >> 1]) mx[e & 1] = fmaxf(mx[e & 1], s[e]);
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 4));
        mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 8));
        mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 16));
    }
    __half *E = a.E + (int64_t)m * a.nh * a.Sp;
    float sm[2] = {0.0f, 0.0f};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int c = e & 1, h = 8 * jj + 2 * t + c, r = e >> 1;
        const float ev = valid[r] ? __expf(s[e] - mx[c]) : 0.0f;
        sm[c] += ev;
        if (h < a.nh) E[(int64_t)h * a.Sp + p + g + 8 * r] = __float2half_rn(ev * vn[r]);
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        sm[c] += __shfl_xor_sync(0xffffffffu, sm[c], 4);
        sm[c] += __shfl_xor_sync(0xffffffffu, sm[c], 8);
        sm[c] += __shfl_xor_sync(0xffffffffu, sm[c], 16);
    }
    if (g == 0) {
        const int64_t o = ((int64_t)m * a.nc16 + (p >> 4)) * a.nh;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int h = 8 * jj + 2 * t + c;
            if (h < a.nh) {
                a.cmax[o + h] = mx[c];
                a.csum[o + h] = sm[c];
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Scores, q~ resident in registers. Dynamic shared memory: table (32 KB) |
// unit buffers [2 groups][2][32 rows][rsk] | partial sums
// [2 groups][2][G warps][8 NT][32 lanes] f32 | mbarriers [2][2].
template <int NT, int G, int MAXB>
__global__ void __launch_bounds__(64 * G) tq_scores_kernel(const TqAttnArgs a) {
    constexpr int NV = 8 * NT;  // accumulators per lane
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ int s_abort;
    uint32_t *lut = reinterpret_cast<uint32_t *>(dsm);
    const int rsk = a.rsk;
    uint8_t *bufs = dsm + LUT32 * 4;
    float *part = reinterpret_cast<float *>(bufs + 4 * 32 * rsk);
    uint64_t *full = reinterpret_cast<uint64_t *>(part + 2 * 2 * G * NV * 32);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int grp = warp / G, wig = warp % G;
    build_lut32(lut, a.kcent);  // constant input: overlaps the previous kernel
    if (tid == 0) {
        s_abort = 0;
        for (int i = 0; i < 4; ++i) as::mbar_init(full + i, 1);
        as::mbar_fence_init();
    }
    pdl_wait();
    const int m = blockIdx.y;
    const int tn = a.pos[m] + 1;
    const int nu = (tn + 31) >> 5;
    const int per = (nu + gridDim.x - 1) / gridDim.x;
    const int u0 = blockIdx.x * per, u1 = min(nu, u0 + per);
    if (u0 >= u1) return;  // whole CTA
    __syncthreads();
    const int nj = u1 - u0 > grp ? (u1 - u0 - grp + 1) >> 1 : 0;  // units u0 + grp + 2 j of this group
    if (nj == 0) return;  // this group has no unit (its warps take no further barrier)
    const int64_t rbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const uint8_t *codes = a.kcodes + rbase * a.kpl;
    const int nblk = a.kvd >> 6;
    const int bpw = (nblk + G - 1) / G;
    const int b0 = wig * bpw, nbw = max(0, min(nblk, b0 + bpw) - b0);
    // q~ fragments of this warp's blocks: dims 64 b + 16 t .. + 15 of head 8 jj + g
    uint32_t qf[MAXB][NT][8];
    {
        const __half *qb = a.qrot + (int64_t)m * a.nh * a.kvd + 16 * t;
#pragma unroll
        for (int bi = 0; bi < MAXB; ++bi)
#pragma unroll
            for (int jj = 0; jj < NT; ++jj) {
                const int h = 8 * jj + g;
                if (bi < nbw && h < a.nh) {
                    const uint4 *qp = reinterpret_cast<const uint4 *>(qb + (int64_t)h * a.kvd + 64 * (b0 + bi));
                    const uint4 x = __ldg(qp), y = __ldg(qp + 1);
                    qf[bi][jj][0] = x.x; qf[bi][jj][1] = x.y; qf[bi][jj][2] = x.z; qf[bi][jj][3] = x.w;
                    qf[bi][jj][4] = y.x; qf[bi][jj][5] = y.y; qf[bi][jj][6] = y.z; qf[bi][jj][7] = y.w;
                } else {
#pragma unroll
                    for (int k = 0; k < 8; ++k) qf[bi][jj][k] = 0u;
                }
            }
    }
    const uint32_t lutl = as::sa(lut) + 4 * lane;
    uint8_t *gbuf = bufs + grp * 2 * 32 * rsk;
    const uint32_t gbuf_s = as::sa(gbuf) + g * rsk + 8 * t;  // row g, byte 8 t of buffer 0
    uint64_t *gfull = full + 2 * grp;
    float *gpart = part + grp * 2 * G * NV * 32;
    // leader warp: bulk-copy the rows of unit j (one per lane) into buffer j & 1
    auto issue = [&](int j) {
        const int slot = j & 1, p0 = 32 * (u0 + grp + 2 * j), rows = min(32, tn - p0);
        if (lane == 0) as::mbar_expect_tx(gfull + slot, (uint32_t)(rows * a.kpl));
        __syncwarp();
        if (lane < rows)
            as::bulk_load(gbuf + (slot * 32 + lane) * rsk, codes + (int64_t)(p0 + lane) * a.kpl, (uint32_t)a.kpl,
                          gfull + slot);
    };
    if (wig == 0) {
        issue(0);
        if (nj > 1) issue(1);
    }
    for (int j = 0; j < nj; ++j) {
        const int slot = j & 1, p0 = 32 * (u0 + grp + 2 * j);
        // norms of rows p0 + 8 i + g (i = 0..3), loaded while the unit computes
        float kn[4], vn[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int p = min(p0 + 8 * i + g, tn - 1);
            kn[i] = __ldg(a.knorm + rbase + p) * a.scale;
            vn[i] = __ldg(a.vnorm + rbase + p);
        }
        // two accumulator sets (even / odd blocks) keep independent MMA chains in flight
        float acc[2][2][NT][4];
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int jj = 0; jj < NT; ++jj)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[q][mt][jj][e] = 0.0f;
        const bool ok = as::mbar_wait(gfull + slot, (uint32_t)((j >> 1) & 1), &s_abort, a.err);
        if (__all_sync(0xffffffffu, ok)) {
            const uint32_t st = gbuf_s + slot * 32 * rsk + 32 * b0;
#pragma unroll
            for (int bi = 0; bi < MAXB; ++bi) {
                if (bi < nbw) {
                    uint2 c[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) c[i] = lds64(st + 8 * i * rsk + 32 * bi);
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const int k0 = (2 * s) & 3;
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt) {
                            const uint32_t wl = s < 2 ? c[2 * mt].x : c[2 * mt].y;
                            const uint32_t wh = s < 2 ? c[2 * mt + 1].x : c[2 * mt + 1].y;
                            const uint32_t a0 = lk(lutl, wl, k0), a2 = lk(lutl, wl, k0 + 1);
                            const uint32_t a1 = lk(lutl, wh, k0), a3 = lk(lutl, wh, k0 + 1);
#pragma unroll
                            for (int jj = 0; jj < NT; ++jj)
                                mma16816(acc[bi & 1][mt][jj], a0, a1, a2, a3, qf[bi][jj][2 * s], qf[bi][jj][2 * s + 1]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int jj = 0; jj < NT; ++jj)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[0][mt][jj][e] += acc[1][mt][jj][e];
        // exchange partial sums, then refill the buffer
        float *pp = gpart + (j & 1) * G * NV * 32;
        if (G > 1) {
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int jj = 0; jj < NT; ++jj)
#pragma unroll
                    for (int e = 0; e < 4; ++e) pp[(wig * NV + (mt * NT + jj) * 4 + e) * 32 + lane] = acc[0][mt][jj][e];
            bar_named(1 + grp, 32 * G);
        } else {
            __syncwarp();
        }
        if (wig == 0 && j + 2 < nj && !__any_sync(0xffffffffu, s_abort != 0)) issue(j + 2);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int jj = 0; jj < NT; ++jj) {
                if ((mt * NT + jj) % G != wig) continue;
                float d[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    d[e] = acc[0][mt][jj][e];
                    if (G > 1) {
                        float sum = 0.0f;
                        for (int k = 0; k < G; ++k) sum += pp[(k * NV + (mt * NT + jj) * 4 + e) * 32 + lane];
                        d[e] = sum;
                    }
                }
                const float knp[2] = {kn[2 * mt], kn[2 * mt + 1]}, vnp[2] = {vn[2 * mt], vn[2 * mt + 1]};
                finalize_piece(a, d, m, p0 + 16 * mt, jj, g, t, tn, knp, vnp);
            }
    }
}

// Scores for shapes whose q~ does not fit in registers: CTA = (128-position
// chunk, token), warp w streams rows 32 w .. 32 w + 31, PD 64-dim blocks ahead.
template <int NT, int PD>
__global__ void __launch_bounds__(128) tq_scores_stream_kernel(const TqAttnArgs a) {
    __shared__ __align__(16) uint32_t lut[LUT32];
    build_lut32(lut, a.kcent);
    pdl_wait();
    const int m = blockIdx.y;
    const int tn = a.pos[m] + 1;
    const int p0 = blockIdx.x * TQ_CH;
    if (p0 >= tn) return;  // whole CTA
    __syncthreads();
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
    const int pw = p0 + 32 * w;
    if (pw >= tn) return;  // this warp (no barrier follows)
    const uint32_t lutl = as::sa(lut) + 4 * lane;
    const int64_t rbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const int nblk = a.kvd >> 6;
    float acc[2][NT][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.0f;
    const uint8_t *rp[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) rp[i] = a.kcodes + (rbase + min(pw + 8 * i + g, tn - 1)) * a.kpl + 8 * t;
    const __half *qb = a.qrot + (int64_t)m * a.nh * a.kvd + 16 * t;
    uint2 cb[PD][4];
#pragma unroll
    for (int u = 0; u < PD; ++u)
        if (u < nblk)
#pragma unroll
            for (int i = 0; i < 4; ++i) cb[u][i] = __ldcs(reinterpret_cast<const uint2 *>(rp[i] + 32 * u));
    for (int bb = 0; bb < nblk; bb += PD) {
#pragma unroll
        for (int u = 0; u < PD; ++u) {
            const int b = bb + u;
            if (b < nblk) {
                uint32_t qf[NT][8];
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const int h = 8 * j + g;
                    if (h < a.nh) {
                        const uint4 *qp = reinterpret_cast<const uint4 *>(qb + (int64_t)h * a.kvd + 64 * b);
                        const uint4 x = __ldg(qp), y = __ldg(qp + 1);
                        qf[j][0] = x.x; qf[j][1] = x.y; qf[j][2] = x.z; qf[j][3] = x.w;
                        qf[j][4] = y.x; qf[j][5] = y.y; qf[j][6] = y.z; qf[j][7] = y.w;
                    } else {
#pragma unroll
                        for (int k = 0; k < 8; ++k) qf[j][k] = 0u;
                    }
                }
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    const int k0 = (2 * s) & 3;
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        const uint32_t wl = s < 2 ? cb[u][2 * mt].x : cb[u][2 * mt].y;
                        const uint32_t wh = s < 2 ? cb[u][2 * mt + 1].x : cb[u][2 * mt + 1].y;
                        const uint32_t a0 = lk(lutl, wl, k0), a2 = lk(lutl, wl, k0 + 1);
                        const uint32_t a1 = lk(lutl, wh, k0), a3 = lk(lutl, wh, k0 + 1);
#pragma unroll
                        for (int j = 0; j < NT; ++j) mma16816(acc[mt][j], a0, a1, a2, a3, qf[j][2 * s], qf[j][2 * s + 1]);
                    }
                }
                if (b + PD < nblk)
#pragma unroll
                    for (int i = 0; i < 4; ++i) cb[u][i] = __ldcs(reinterpret_cast<const uint2 *>(rp[i] + 32 * (b + PD)));
            }
        }
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
        float kn[2], vn[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int p = min(pw + 16 * mt + 8 * r + g, tn - 1);
            kn[r] = __ldg(a.knorm + rbase + p) * a.scale;
            vn[r] = __ldg(a.vnorm + rbase + p);
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) finalize_piece(a, acc[mt][j], m, pw + 16 * mt, j, g, t, tn, kn, vn);
    }
}

// ---------------------------------------------------------------------------
// Values. Dynamic shared memory: table (32 KB) | rings [4 warps][D][slot] |
// chunk factors [nc16][HP]; a ring slot holds 16 code rows (row stride RS)
// and the e tile [HP heads][16 positions] (row stride 48 bytes).
template <int MT, int NJ>
struct ValuesShape {
    static constexpr int HP = 16 * MT, DB = 8 * NJ, WB = NJ / 2, RB = DB / 2, RS = RB + 16, ES = 48;
    static constexpr int SLOT = 16 * RS + HP * ES;
};

template <int MT, int NJ, int D>
__global__ void __launch_bounds__(128, 3) tq_values_kernel(const TqAttnArgs a) {
    using S = ValuesShape<MT, NJ>;
    constexpr int HP = S::HP, DB = S::DB, WB = S::WB, RB = S::RB, RS = S::RS, ES = S::ES, SLOT = S::SLOT;
    constexpr int NV = MT * NJ * 4;  // accumulators per lane
    using CW = typename std::conditional<WB == 8, uint2, uint32_t>::type;
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ float s_red[128];
    __shared__ float s_M[HP], s_linv[HP];
    uint32_t *lut = reinterpret_cast<uint32_t *>(dsm);
    uint8_t *ring = dsm + LUT32 * 4;
    float *s_f = reinterpret_cast<float *>(ring + 4 * D * SLOT);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
    build_lut32(lut, a.vcent);
    // e rows of heads >= nh stay zero (never copied)
    for (int i = tid; i < 4 * D * (HP - a.nh) * (ES / 4); i += blockDim.x) {
        const int per = (HP - a.nh) * (ES / 4), s = i / per, r = i % per;
        reinterpret_cast<uint32_t *>(ring + s * SLOT + 16 * RS + a.nh * ES)[r] = 0u;
    }
    pdl_wait();
    const int m = blockIdx.y;
    const int tn = a.pos[m] + 1;
    const int nks = (tn + 15) >> 4;
    const int nmy = nks > w ? (nks - w + 3) >> 2 : 0;  // k-steps w, w + 4, ... of this warp
    const int64_t rbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const uint8_t *crow = a.vcodes + rbase * a.vpl + blockIdx.x * RB;
    const __half *Em = a.E + (int64_t)m * a.nh * a.Sp;
    uint8_t *wring = ring + w * D * SLOT;
    // per-lane copy plan: code chunks (row, 16-byte piece) and one e chunk
    constexpr int CPL = RB / 32;
    const uint32_t ring_s = as::sa(wring);
    uint32_t c_dst[CPL];
    int c_row[CPL];
    const uint8_t *c_src[CPL];
#pragma unroll
    for (int r = 0; r < CPL; ++r) {
        const int c = lane + 32 * r, row = c / (RB / 16), piece = c % (RB / 16);
        c_dst[r] = ring_s + row * RS + 16 * piece;
        c_row[r] = row;
        c_src[r] = crow + 16 * piece;
    }
    // e chunks: 2 per head (HP heads, MT per lane); chunk c = lane + 32 r is
    // head c >> 1, 16-byte half c & 1
    bool e_on[MT];
    uint32_t e_dst[MT];
    const __half *e_src[MT];
#pragma unroll
    for (int r = 0; r < MT; ++r) {
        const int c = lane + 32 * r;
        e_on[r] = c < 2 * a.nh;
        e_dst[r] = ring_s + 16 * RS + (c >> 1) * ES + 16 * (c & 1);
        e_src[r] = Em + (int64_t)(e_on[r] ? c >> 1 : 0) * a.Sp + 8 * (c & 1);
    }
    auto issue = [&](int i) {
        const int ks = w + 4 * i;
        const uint32_t so = (uint32_t)(i % D) * SLOT;
#pragma unroll
        for (int r = 0; r < CPL; ++r)
            cp_async16(c_dst[r] + so, c_src[r] + (int64_t)min(16 * ks + c_row[r], tn - 1) * a.vpl);
#pragma unroll
        for (int r = 0; r < MT; ++r)
            if (e_on[r]) cp_async16(e_dst[r] + so, e_src[r] + 16 * ks);
    };
#pragma unroll
    for (int i = 0; i < D - 1; ++i) {
        if (i < nmy) issue(i);
        cp_commit();
    }
    // M_h, factors exp(c - M_h) per chunk and l_h (thread: head tid % HP,
    // chunks tid / HP + RR k, loaded KB at a time), in a fixed order
    {
        constexpr int RR = 128 / HP, KB = 16;
        const int h = tid % HP, r0 = tid / HP;
        const bool hv = h < a.nh;
        const float *cm = a.cmax + (int64_t)m * a.nc16 * a.nh + h;
        const float *cs = a.csum + (int64_t)m * a.nc16 * a.nh + h;
        float mx = -INFINITY;
        for (int c0 = r0; c0 < nks; c0 += RR * KB) {
            float v[KB];
#pragma unroll
            for (int k = 0; k < KB; ++k) {
                const int c = c0 + RR * k;
                v[k] = (hv && c < nks) ? cm[(int64_t)c * a.nh] : -INFINITY;
            }
#pragma unroll
            for (int k = 0; k < KB; ++k) mx = fmaxf(mx, v[k]);
        }
        s_red[tid] = mx;
        __syncthreads();
        if (tid < HP) {
            float v = s_red[tid];
            for (int r = 1; r < RR; ++r) v = fmaxf(v, s_red[r * HP + tid]);
            s_M[tid] = v;
        }
        __syncthreads();
        float l = 0.0f;
        const float M = s_M[h];
        for (int c0 = r0; c0 < nks; c0 += RR * KB) {
            float v[KB], u[KB];
#pragma unroll
            for (int k = 0; k < KB; ++k) {
                const int c = c0 + RR * k;
                const bool ok = hv && c < nks;
                v[k] = ok ? cm[(int64_t)c * a.nh] : 0.0f;
                u[k] = ok ? cs[(int64_t)c * a.nh] : 0.0f;
            }
#pragma unroll
            for (int k = 0; k < KB; ++k) {
                const int c = c0 + RR * k;
                if (c < nks) {
                    const float f = hv ? __expf(v[k] - M) : 0.0f;
                    s_f[c * HP + h] = f;
                    l += u[k] * f;
                }
            }
        }
        s_red[tid] = l;
        __syncthreads();
        if (tid < HP) {
            float v = s_red[tid];
            for (int r = 1; r < RR; ++r) v += s_red[r * HP + tid];
            s_linv[tid] = tid < a.nh ? 1.0f / v : 0.0f;
        }
        __syncthreads();
    }
    float acc[MT][NJ][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][j][e] = 0.0f;
    const uint32_t lutl = as::sa(lut) + 4 * lane;
    // ldmatrix row address: matrix lane >> 3 = (heads + 8 (q & 1), positions 8 (q >> 1))
    const int lq = lane >> 3, lr = lane & 7;
    const uint32_t ld_s = ring_s + 16 * RS + (lr + 8 * (lq & 1)) * ES + 16 * (lq >> 1);
    const uint32_t cw_s = ring_s + (2 * t) * RS + WB * g;
    const uint32_t f_s = as::sa(s_f) + 4 * g;
    for (int i = 0; i < nmy; ++i) {
        if (i + D - 1 < nmy) issue(i + D - 1);
        cp_commit();
        cp_wait<D - 1>();
        __syncwarp();
        const uint32_t so = (uint32_t)(i % D) * SLOT;
        const int ks = w + 4 * i;
        uint32_t af[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            ldsm_x4(ld_s + so + 16 * mt * ES, af[mt][0], af[mt][1], af[mt][2], af[mt][3]);
            const uint32_t fo = f_s + 4 * (ks * HP + 16 * mt);
            const __half2 fa = __float2half2_rn(ldsf(fo));
            const __half2 fb = __float2half2_rn(ldsf(fo + 32));
            af[mt][0] = hmul2(af[mt][0], fa);
            af[mt][1] = hmul2(af[mt][1], fb);
            af[mt][2] = hmul2(af[mt][2], fa);
            af[mt][3] = hmul2(af[mt][3], fb);
        }
        const CW v0 = lds_cw<CW>(cw_s + so);
        const CW v1 = lds_cw<CW>(cw_s + so + RS);
        const CW v2 = lds_cw<CW>(cw_s + so + 8 * RS);
        const CW v3 = lds_cw<CW>(cw_s + so + 9 * RS);
#pragma unroll
        for (int wi = 0; wi < WB / 4; ++wi) {
            const uint32_t w0 = word_of(v0, wi), w1 = word_of(v1, wi), w2 = word_of(v2, wi), w3 = word_of(v3, wi);
            // byte k of lo01 = (low nibble of row 2t's byte k, low nibble of row 2t+1's byte k)
            const uint32_t lo01 = (w0 & 0x0f0f0f0fu) | ((w1 << 4) & 0xf0f0f0f0u);
            const uint32_t hi01 = ((w0 >> 4) & 0x0f0f0f0fu) | (w1 & 0xf0f0f0f0u);
            const uint32_t lo23 = (w2 & 0x0f0f0f0fu) | ((w3 << 4) & 0xf0f0f0f0u);
            const uint32_t hi23 = ((w2 >> 4) & 0x0f0f0f0fu) | (w3 & 0xf0f0f0f0u);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ib = 4 * wi + k;
                const uint32_t b0e = lk(lutl, lo01, k), b1e = lk(lutl, lo23, k);
                const uint32_t b0o = lk(lutl, hi01, k), b1o = lk(lutl, hi23, k);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    mma16816(acc[mt][2 * ib], af[mt][0], af[mt][1], af[mt][2], af[mt][3], b0e, b1e);
                    mma16816(acc[mt][2 * ib + 1], af[mt][0], af[mt][1], af[mt][2], af[mt][3], b0o, b1o);
                }
            }
        }
        __syncwarp();
    }
    cp_wait<0>();
    // combine the four warps: red[w][v][lane], then warp w sums v in [w NV/4, (w+1) NV/4)
    __syncthreads();
    float *red = reinterpret_cast<float *>(dsm);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) red[(w * NV + (mt * NJ + j) * 4 + e) * 32 + lane] = acc[mt][j][e];
    __syncthreads();
    constexpr int NQ = NV / 4;
    float sum[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const int v = w * NQ + q;
        sum[q] = (red[(0 * NV + v) * 32 + lane] + red[(1 * NV + v) * 32 + lane]) +
                 (red[(2 * NV + v) * 32 + lane] + red[(3 * NV + v) * 32 + lane]);
    }
    __syncthreads();
    // normalised tile out[head][dim] (row stride DB + 1), then f16 hi / lo rows
    float *out = red;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const int v = w * NQ + q, e = v & 3, j = (v >> 2) % NJ, mt = (v >> 2) / NJ;
        const int h = 16 * mt + g + 8 * (e >> 1), d = NJ * (2 * t + (e & 1)) + j;
        out[h * (DB + 1) + d] = sum[q] * s_linv[h];
    }
    __syncthreads();
    for (int id = tid; id < HP * DB / 8; id += blockDim.x) {
        const int h = id / (DB / 8), d8 = id % (DB / 8);
        if (h >= a.nh) continue;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float x0 = out[h * (DB + 1) + 8 * d8 + 2 * k], x1 = out[h * (DB + 1) + 8 * d8 + 2 * k + 1];
            const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
            __half2 hh = __halves2half2(h0, h1);
            hi[k] = *reinterpret_cast<uint32_t *>(&hh);
            lo[k] = h2bits(x0 - __half2float(h0), x1 - __half2float(h1));
        }
        const int64_t o = ((int64_t)m * a.nh + h) * a.kvd + blockIdx.x * DB + 8 * d8;
        *reinterpret_cast<uint4 *>(a.U + o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(a.U_lo + o) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// Launch attributes are set (and the occupancy queried) per device on the
// first call of each shape, which is an eager call; graph captures reuse them.
template <int NT, int G, int MAXB>
cudaError_t launch_scores(const TqAttnArgs &a, cudaStream_t s) {
    const size_t smem = (size_t)LUT32 * 4 + 4 * 32 * (size_t)a.rsk + 2 * 2 * G * 8 * NT * 32 * 4 + 4 * 8;
    cudaError_t e = dev::smem(tq_scores_kernel<NT, G, MAXB>, smem);
    if (e != cudaSuccess) return e;
    const int occ = dev::occupancy(tq_scores_kernel<NT, G, MAXB>, 64 * G, smem);
    const int nu_max = (a.B + 31) / 32;
    const int nseg = std::max(1, std::min(nu_max, occ * dev::sm_count() / a.M));
    return launch_pdl(tq_scores_kernel<NT, G, MAXB>, dim3(nseg, a.M), dim3(64 * G), smem, s, a);
}

template <int MT, int NJ>
cudaError_t launch_values(const TqAttnArgs &a, cudaStream_t s) {
    constexpr int D = 4;
    const size_t smem = (size_t)LUT32 * 4 + 4 * D * ValuesShape<MT, NJ>::SLOT + (size_t)a.nc16 * 16 * MT * 4;
    cudaError_t e = dev::smem(tq_values_kernel<MT, NJ, D>, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(tq_values_kernel<MT, NJ, D>, dim3(a.kvd / (8 * NJ), a.M), dim3(128), smem, s, a);
}

}  // namespace

int tq_padded_len(int block_size) { return (block_size + TQ_CH - 1) / TQ_CH * TQ_CH; }

cudaError_t tq_decode_attn(const TqAttnArgs &a0, cudaStream_t s) {
    if (a0.M <= 0) return cudaSuccess;
    if (tc_attn_supported(a0)) return tc_decode_attn(a0, s);  // tcgen05 scores and values
    TqAttnArgs a = a0;
    if (a.kvd % 64 || a.nh < 1 || a.nh > 32 || a.Sp != tq_padded_len(a.B) || a.nc16 != a.Sp / 16 ||
        2 * a.kpl != a.kvd || 2 * a.vpl != a.kvd)
        return cudaErrorInvalidValue;
    // unit-buffer row stride: 8 or 24 (mod 32) words, so the eight rows of a
    // 64-bit read land in distinct banks
    a.rsk = a.kpl + ((a.kpl / 32) % 2 == 0 ? 32 : 0);
    const int nt = (a.nh + 7) / 8;
    const int nblk = a.kvd / 64;
    cudaError_t e;
    if (nt == 1 && nblk <= 12)
        e = launch_scores<1, 1, 12>(a, s);
    else if (nt == 2 && nblk <= 6)
        e = launch_scores<2, 1, 6>(a, s);
    else if (nt == 2 && nblk <= 12)
        e = launch_scores<2, 2, 6>(a, s);
    else if (nt == 2 && nblk <= 24)
        e = launch_scores<2, 4, 6>(a, s);
    else if (nt == 1)
        e = launch_pdl(tq_scores_stream_kernel<1, 4>, dim3(a.Sp / TQ_CH, a.M), dim3(128), 0, s, a);
    else if (nt == 2)
        e = launch_pdl(tq_scores_stream_kernel<2, 4>, dim3(a.Sp / TQ_CH, a.M), dim3(128), 0, s, a);
    else
        e = launch_pdl(tq_scores_stream_kernel<4, 4>, dim3(a.Sp / TQ_CH, a.M), dim3(128), 0, s, a);
    if (e != cudaSuccess) return e;
    if (a.nh > 16) return launch_values<2, 8>(a, s);
    if (a.kvd % 128 == 0) return launch_values<1, 16>(a, s);
    return launch_values<1, 8>(a, s);
}

}  // namespace attn
}  // namespace kg
