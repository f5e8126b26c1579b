// kg_attn.cu — attention over the TurboQuant KV cache, BF16 tensor-core path.
//
// A stored key is k~ = norm * R^T c (src/turboquant/kv_cache.rs:279-317) with
// R the kv_dim x kv_dim rotation shared by all layers and c the centroid vector
// of the codes. Because R mixes all kv_dim coordinates, one head's slice of k~
// depends on every code, so decode attention runs in the rotated domain:
//   q~_h   = R[:, head h columns] q_h                       (GEMM, kg_bf16.cu)
//   s[t,h] = norm_k[t] * scale * <centroid(code_k[t]), q~_h>  (attn_scores)
//   p[t,h] = softmax_t(s) * norm_v[t]                         (attn_softmax)
//   u~_h   = sum_t p[t,h] * centroid(code_v[t])             (attn_values)
//   out_h  = R[:, head h columns]^T u~_h                     (GEMM)
// attn_scores reads the 4-bit codes straight from HBM and turns every byte
// into an f16 hi/lo centroid pair with a 256-entry shared-memory table, in
// registers, feeding mma.sync; attn_values stages a tile of codes in shared memory, dequantizes it
// there and reads it with ldmatrix.trans. Prefill instead dequantizes the
// prompt's K/V once (GEMM with R^T) and runs causal flash attention.
//
// Semantics: forward_quantized attention (src/transformer.rs:4123-4141 over
// the dequantized cache), softmax with 1/sqrt(head_dim) (transformer.rs:333-389).
#include <cuda_bf16.h>

#include <cooperative_groups.h>

#include <algorithm>

#include "kg_async.cuh"
#include "kg_attn.cuh"
#include "kg_pdl.cuh"

namespace kg {
namespace attn {
namespace {

using bf16 = __nv_bfloat16;
namespace cg = cooperative_groups;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}
// f32 pair -> (hi pair, lo pair) of f16
__device__ __forceinline__ void split_h2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    __half2 h = __halves2half2(ha, hb);
    hi = *reinterpret_cast<uint32_t *>(&h);
    lo = pack_h2(a - __half2float(ha), b - __half2float(hb));
}

// byte -> centroid pair (lo nibble, hi nibble) split into f16 hi and lo pairs
__device__ __forceinline__ void build_lut(uint2 *lut, const float *cent) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) {
        uint32_t hi, lo;
        split_h2(cent[b & 15], cent[b >> 4], hi, lo);
        lut[b] = make_uint2(hi, lo);
    }
}

// ---------------------------------------------------------------------------
// 256-entry byte table (byte -> centroid pair of its two nibbles, f16 hi/lo)
// replicated 16 times: entry (b, r) sits at b * 16 + r and lane l reads
// replica l & 15, so the 32 lookups of a warp land in 16 distinct bank pairs
// (two wavefronts for any byte pattern).
constexpr int LUT_ENTRIES = 256 * 16;
__device__ __forceinline__ void build_lut_rep(uint2 *lut, const float *cent) {
    __shared__ uint2 base[256];
    for (int b = threadIdx.x; b < 256; b += blockDim.x) {
        uint32_t hi, lo;
        split_h2(cent[b & 15], cent[b >> 4], hi, lo);
        base[b] = make_uint2(hi, lo);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < LUT_ENTRIES; i += blockDim.x) lut[i] = base[i >> 4];
}
// byte k (0..3) of w through the replicated table (lutl = lut + (lane & 15))
__device__ __forceinline__ uint2 lut_byte(const uint2 *lutl, uint32_t w, int k) {
    return lutl[((w >> (8 * k)) & 0xffu) << 4];
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool pred) {
    const int sz = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(sz));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src));
}
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---------------------------------------------------------------------------
// Decode attention, flash-decoding style, one kernel. The positions [0, tn)
// of a token are cut into ATTEND_CHUNKS equal chunks (multiples of 16); one
// CTA per chunk, and the chunk CTAs of a token form a thread-block cluster.
//  A. scores of the chunk, s[h, t] = norm_k[t] * scale * <centroid(code_k[t]), q~_h>:
//     mma.sync m16n8k16, positions as M, heads as N (NT tiles of 8), kv_dim
//     as K in 64-dim blocks. A thread reads 8 code bytes of each of its rows
//     per block; byte 2st (dims 16c + 4st, +1) feeds k-cols 2c, 2c + 1 of
//     step st, byte 2st + 1 (dims 16c + 4st + 2, +3) k-cols 2c + 8, 2c + 9,
//     so q~ is consumed in natural dim order. Codes of the block and q~ go
//     through a cp.async ring in shared memory.
//  B. local softmax per head: m = max s, l = sum exp(s - m),
//     p = exp(s - m) * norm_v as an f16 hi/lo tile.
//  C. u~_chunk[h, d] = sum_t p[h, t] * centroid(code_v[t, d]): heads as M
//     (A = p via ldmatrix), dims as N, positions as K, over a ring of 16-row
//     code tiles. A thread reads the 4-byte word (dims 8g .. 8g + 7 of a
//     64-dim block) of positions 2c, 2c + 1, 2c + 8, 2c + 9; each byte goes
//     through the table and prmt pairs the two positions of a dim into one
//     B register, so n-tile jj of the block holds dims 8n + jj.
//     The chunks combine through distributed shared memory,
//     u~ = sum_r exp(m_r - M) u~_r / sum_r exp(m_r - M) l_r, written as f16
//     hi/lo, one dim group at a time.
// Every product uses hi*hi + lo*hi + hi*lo of the f16 splits.
constexpr int SSTG = 3, VSTG = 4;
template <int NT, int MT, int MTV, int NBW>
__global__ void __launch_bounds__(128) decode_attn_kernel(const DecodeAttnArgs a) {
    pdl_wait();
    extern __shared__ __align__(16) unsigned char dsm[];
    constexpr int HP = 16 * MTV, QROW = 72;
    const int NCH = gridDim.x, chmax = a.chmax, nbg = a.nbg, DG = 64 * nbg;
    const int SROW = chmax + 4, PROW = chmax + 8, UROW = DG + 4;
    uint2 *lut = reinterpret_cast<uint2 *>(dsm);
    unsigned char *ring = dsm + a.off_ring;
    float *Ss = reinterpret_cast<float *>(dsm + a.off_S);        // [HP][SROW]
    __half *Ph = reinterpret_cast<__half *>(dsm + a.off_P);      // [HP][PROW]
    __half *Pl = Ph + HP * PROW;
    float *part = reinterpret_cast<float *>(dsm + a.off_part);   // [HP][UROW]
    float *mloc = reinterpret_cast<float *>(dsm + a.off_small);  // [HP]
    float *lloc = mloc + HP;                                     // [HP]
    float *wgt = lloc + HP;                                      // [NCH][HP]
    float *kn_s = wgt + NCH * HP;                                // [chmax]
    float *vn_s = kn_s + chmax;                                  // [chmax]

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int m = blockIdx.z;
    const int tn = a.pos[m] + 1;
    const int chl = ((tn + NCH - 1) / NCH + 15) / 16 * 16;
    const int c0 = rank * chl, nloc = max(0, min(tn, c0 + chl) - c0);
    const int nmt = (nloc + 15) / 16;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const uint2 *lutl = lut + (lane & 15);
    const int64_t rowbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;

    // ---- A. scores
    const uint8_t *kcodes = a.kcodes + rowbase * a.kpl;
    const __half *qh = a.qrot + (int64_t)m * a.nh * a.kvd, *ql = a.qrot_lo + (int64_t)m * a.nh * a.kvd;
    const int nblk = a.kvd / 64;
    int mg = 0;  // first m-tile of the current group of 4 * MT
    auto sstage = [&](int q) {
        unsigned char *st = ring + (q % SSTG) * a.sstage;
        const int rows = min(4 * MT, nmt - mg) * 16;
        for (int i = tid; i < rows * 2; i += 128) {  // code rows: 2 x 16 bytes each
            const int r = i >> 1, h16 = i & 1;
            const int t = min(c0 + mg * 16 + r, tn - 1);
            cp_async16(smem_u32(st + r * 32 + h16 * 16), kcodes + (int64_t)t * a.kpl + q * 32 + h16 * 16, true);
        }
        __half *qs = reinterpret_cast<__half *>(st + 4 * MT * 16 * 32);
        for (int i = tid; i < 2 * NT * 8 * 8; i += 128) {
            const int hl = i / (NT * 8 * 8), r = (i / 8) % (NT * 8), ch = i % 8;
            const bool ok = r < a.nh;
            const __half *src = (hl ? ql : qh) + (int64_t)(ok ? r : 0) * a.kvd + q * 64 + ch * 8;
            cp_async16(smem_u32(qs + (hl * NT * 8 + r) * QROW + ch * 8), src, ok);
        }
    };
    auto prologue = [&]() {
#pragma unroll
        for (int s = 0; s < SSTG - 1; ++s) {
            if (s < nblk) sstage(s);
            cp_commit();
        }
    };
    if (nmt > 0) {
        for (int t = tid; t < nloc; t += 128) {
            cp_async4(smem_u32(kn_s + t), a.knorm + rowbase + c0 + t);
            cp_async4(smem_u32(vn_s + t), a.vnorm + rowbase + c0 + t);
        }
        prologue();
    }
    build_lut_rep(lut, a.kcent);
    for (; mg < nmt; mg += 4 * MT) {
        if (mg > 0) prologue();
        const int gm = min(4 * MT, nmt - mg);
        float acc[MT][NT][4];
#pragma unroll
        for (int i = 0; i < MT; ++i)
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;
        for (int q = 0; q < nblk; ++q) {
            cp_wait<SSTG - 2>();
            __syncthreads();
            if (q + SSTG - 1 < nblk) sstage(q + SSTG - 1);
            cp_commit();
            const unsigned char *st = ring + (q % SSTG) * a.sstage;
            const __half *qs = reinterpret_cast<const __half *>(st + 4 * MT * 16 * 32);
            uint32_t bq[NT][8], bl[NT][8];
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const uint4 *sh = reinterpret_cast<const uint4 *>(qs + (j * 8 + g) * QROW + c * 16);
                const uint4 *sl = reinterpret_cast<const uint4 *>(qs + (NT * 8 + j * 8 + g) * QROW + c * 16);
                const uint4 u0 = sh[0], u1 = sh[1], v0 = sl[0], v1 = sl[1];
                bq[j][0] = u0.x; bq[j][1] = u0.y; bq[j][2] = u0.z; bq[j][3] = u0.w;
                bq[j][4] = u1.x; bq[j][5] = u1.y; bq[j][6] = u1.z; bq[j][7] = u1.w;
                bl[j][0] = v0.x; bl[j][1] = v0.y; bl[j][2] = v0.z; bl[j][3] = v0.w;
                bl[j][4] = v1.x; bl[j][5] = v1.y; bl[j][6] = v1.z; bl[j][7] = v1.w;
            }
#pragma unroll
            for (int i = 0; i < MT; ++i) {
                const int mt = warp + 4 * i;
                if (mt < gm) {
                    const uint2 w0 = *reinterpret_cast<const uint2 *>(st + (mt * 16 + g) * 32 + c * 8);
                    const uint2 w1 = *reinterpret_cast<const uint2 *>(st + (mt * 16 + g + 8) * 32 + c * 8);
#pragma unroll
                    for (int s4 = 0; s4 < 4; ++s4) {
                        const uint32_t x0 = s4 < 2 ? w0.x : w0.y, x1 = s4 < 2 ? w1.x : w1.y;
                        const int k = (s4 & 1) * 2;
                        const uint2 e0 = lut_byte(lutl, x0, k), e2 = lut_byte(lutl, x0, k + 1);
                        const uint2 e1 = lut_byte(lutl, x1, k), e3 = lut_byte(lutl, x1, k + 1);
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            mma_f16(acc[i][j], e0.x, e1.x, e2.x, e3.x, bq[j][2 * s4], bq[j][2 * s4 + 1]);
                            mma_f16(acc[i][j], e0.y, e1.y, e2.y, e3.y, bq[j][2 * s4], bq[j][2 * s4 + 1]);
                            mma_f16(acc[i][j], e0.x, e1.x, e2.x, e3.x, bl[j][2 * s4], bl[j][2 * s4 + 1]);
                        }
                    }
                }
            }
        }
        cp_wait<0>();
        __syncthreads();  // norms staged; the ring is free for the next group
#pragma unroll
        for (int i = 0; i < MT; ++i) {
            const int mt = warp + 4 * i;
            if (mt < gm) {
#pragma unroll
                for (int hrow = 0; hrow < 2; ++hrow) {
                    const int t = (mg + mt) * 16 + g + hrow * 8;
                    const float f = t < nloc ? kn_s[t] * a.scale : 0.0f;
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int h = j * 8 + c * 2 + e;
                            if (h < HP) Ss[h * SROW + t] = acc[i][j][hrow * 2 + e] * f;
                        }
                }
            }
        }
    }
    __syncthreads();

    // ---- B. local softmax, one warp per head
    for (int h = warp; h < HP; h += 4) {
        __half *ph = Ph + h * PROW, *pl = Pl + h * PROW;
        const float *srow = Ss + h * SROW;
        const bool live = h < a.nh && nloc > 0;
        float mx = -INFINITY, sum = 0.0f;
        if (live) {
            for (int t = lane; t < nloc; t += 32) mx = fmaxf(mx, srow[t]);
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        for (int t = lane; t < nmt * 16; t += 32) {
            float v = 0.0f;
            if (live && t < nloc) {
                const float e = expf(srow[t] - mx);
                sum += e;
                v = e * vn_s[t];
            }
            const __half hv = __float2half_rn(v);
            ph[t] = hv;
            pl[t] = __float2half_rn(v - __half2float(hv));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            mloc[h] = mx;
            lloc[h] = sum;
        }
    }
    __syncthreads();  // scores phase done with the table
    build_lut_rep(lut, a.vcent);

    // ---- C. values and the cluster combine, one dim group at a time
    const uint8_t *vcodes = a.vcodes + rowbase * a.vpl;
    const int vchunks = DG / 32;  // 16-byte chunks per row of a tile (DG / 2 bytes)
    for (int dg = 0; dg < a.ndg; ++dg) {
        const uint8_t *vsrc = vcodes + dg * (DG / 2);
        auto vstage = [&](int ks) {
            unsigned char *st = ring + (ks % VSTG) * a.vstage;
            for (int i = tid; i < 16 * vchunks; i += 128) {
                const int r = i / vchunks, ch = i % vchunks;
                const int t = min(c0 + ks * 16 + r, tn - 1);
                cp_async16(smem_u32(st + r * a.vrow + ch * 16), vsrc + (int64_t)t * a.vpl + ch * 16, true);
            }
        };
        __syncthreads();  // ring free (scores stages or the previous group's tiles)
#pragma unroll
        for (int s = 0; s < VSTG - 1; ++s) {
            if (s < nmt) vstage(s);
            cp_commit();
        }
        float acc[NBW][MTV][8][4];
#pragma unroll
        for (int b = 0; b < NBW; ++b)
#pragma unroll
            for (int i = 0; i < MTV; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[b][i][j][e] = 0.0f;
        for (int ks = 0; ks < nmt; ++ks) {
            cp_wait<VSTG - 2>();
            __syncthreads();
            if (ks + VSTG - 1 < nmt) vstage(ks + VSTG - 1);
            cp_commit();
            const unsigned char *st = ring + (ks % VSTG) * a.vstage;
            uint32_t ah[MTV][4], al[MTV][4];
#pragma unroll
            for (int i = 0; i < MTV; ++i) {
                const int r = i * 16 + (lane & 15), col = ks * 16 + ((lane >> 4) << 3);
                ldsm_x4(smem_u32(Ph + r * PROW + col), ah[i][0], ah[i][1], ah[i][2], ah[i][3]);
                ldsm_x4(smem_u32(Pl + r * PROW + col), al[i][0], al[i][1], al[i][2], al[i][3]);
            }
#pragma unroll
            for (int b = 0; b < NBW; ++b) {
                if (warp + 4 * b >= nbg) continue;
                const unsigned char *cb = st + (warp + 4 * b) * 32 + 4 * g;
                const uint32_t x0 = *reinterpret_cast<const uint32_t *>(cb + (2 * c) * a.vrow);
                const uint32_t x1 = *reinterpret_cast<const uint32_t *>(cb + (2 * c + 1) * a.vrow);
                const uint32_t x2 = *reinterpret_cast<const uint32_t *>(cb + (2 * c + 8) * a.vrow);
                const uint32_t x3 = *reinterpret_cast<const uint32_t *>(cb + (2 * c + 9) * a.vrow);
#pragma unroll
                uint32_t bh[8][2], bl[8][2];  // B registers of n-tile jj = 2by + hf (dim 8g + jj)
#pragma unroll
                for (int by = 0; by < 4; ++by) {
                    const uint2 e0 = lut_byte(lutl, x0, by), e1 = lut_byte(lutl, x1, by);
                    const uint2 e2 = lut_byte(lutl, x2, by), e3 = lut_byte(lutl, x3, by);
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const uint32_t sel = hf ? 0x7632u : 0x5410u;
                        bh[2 * by + hf][0] = prmt(e0.x, e1.x, sel);
                        bh[2 * by + hf][1] = prmt(e2.x, e3.x, sel);
                        bl[2 * by + hf][0] = prmt(e0.y, e1.y, sel);
                        bl[2 * by + hf][1] = prmt(e2.y, e3.y, sel);
                    }
                }
                // term-major: consecutive MMAs go to different accumulators
#pragma unroll
                for (int i = 0; i < MTV; ++i)
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj)
                        mma_f16(acc[b][i][jj], ah[i][0], ah[i][1], ah[i][2], ah[i][3], bh[jj][0], bh[jj][1]);
#pragma unroll
                for (int i = 0; i < MTV; ++i)
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj)
                        mma_f16(acc[b][i][jj], al[i][0], al[i][1], al[i][2], al[i][3], bh[jj][0], bh[jj][1]);
#pragma unroll
                for (int i = 0; i < MTV; ++i)
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj)
                        mma_f16(acc[b][i][jj], ah[i][0], ah[i][1], ah[i][2], ah[i][3], bl[jj][0], bl[jj][1]);
            }
        }
        cp_wait<0>();
        __syncthreads();  // the partial tile may overlay the table and the ring
        // accumulator (row h, col n = 2c + e) of n-tile jj is dim 8n + jj of block warp + 4b
#pragma unroll
        for (int b = 0; b < NBW; ++b)
            if (warp + 4 * b < nbg)
#pragma unroll
            for (int i = 0; i < MTV; ++i)
#pragma unroll
                for (int hrow = 0; hrow < 2; ++hrow)
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj)
#pragma unroll
                        for (int e = 0; e < 2; ++e)
                            part[(i * 16 + g + hrow * 8) * UROW + (warp + 4 * b) * 64 + 8 * (2 * c + e) + jj] =
                                acc[b][i][jj][hrow * 2 + e];
        cluster.sync();
        if (tid < HP) {
            const int h = tid;
            float M = -INFINITY;
            for (int r = 0; r < NCH; ++r) M = fmaxf(M, *cluster.map_shared_rank(mloc + h, r));
            float L = 0.0f;
            for (int r = 0; r < NCH; ++r) {
                const float mr = *cluster.map_shared_rank(mloc + h, r);
                const float w = mr == -INFINITY ? 0.0f : expf(mr - M);
                wgt[r * HP + h] = w;
                L += w * *cluster.map_shared_rank(lloc + h, r);
            }
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            for (int r = 0; r < NCH; ++r) wgt[r * HP + h] *= inv;
        }
        __syncthreads();
        const int quads = a.nh * (DG / 4);
        const int per = (quads + NCH - 1) / NCH;
        const int q0 = rank * per, q1 = min(quads, q0 + per);
        for (int qd = q0 + tid; qd < q1; qd += 128) {
            const int h = qd / (DG / 4), d = (qd % (DG / 4)) * 4;
            float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < NCH; ++r) {
                const float w = wgt[r * HP + h];
                if (w == 0.0f) continue;  // chunk without positions
                const float4 v = *reinterpret_cast<const float4 *>(cluster.map_shared_rank(part, r) + h * UROW + d);
                u.x += w * v.x; u.y += w * v.y; u.z += w * v.z; u.w += w * v.w;
            }
            uint32_t h01, l01, h23, l23;
            split_h2(u.x, u.y, h01, l01);
            split_h2(u.z, u.w, h23, l23);
            const int64_t o = ((int64_t)m * a.nh + h) * a.kvd + dg * DG + d;
            *reinterpret_cast<uint2 *>(a.U + o) = make_uint2(h01, h23);
            *reinterpret_cast<uint2 *>(a.U_lo + o) = make_uint2(l01, l23);
        }
        cluster.sync();  // peers are done reading this CTA's partial tile
    }
}

// ---------------------------------------------------------------------------
// Decode attention with a TMA producer warp (kv_dim a multiple of 256). Same
// arithmetic and fragment layouts as decode_attn_kernel; the staging differs:
//   warp 4 (one thread) streams every tile through a ring of NS shared-memory
//   stages with cp.async.bulk.tensor: per 64-dim block of the scores phase
//   the chunk's key-code rows ([rows x 32 B], plain) and the q~ hi / lo rows
//   ([heads x 128 B], 128-byte swizzle); per 16-position step of the values
//   phase the value-code rows of the dim group ([16 x 128 B] boxes, 128-byte
//   swizzle, which makes the 4-byte reads of the value step conflict-free).
//   The replicated centroid tables come precomputed from global memory by
//   bulk copy (key table first, value table once the scores are done).
//   Warps 0..3 consume: wait on the stage's full barrier, compute, release it
//   through its empty barrier; no CTA-wide barrier inside the loops.
// Waits are bounded (kg_async.cuh): on a timeout the CTA keeps passing through
// every barrier it owes (named, cluster) with the work skipped, and the
// device error word reports KG_ERR_TIMEOUT.
constexpr int NS = 4;                  // ring stages
// 8 replicas of the byte table (16 KB): lane l reads replica l & 7, at most
// two lanes of a warp share a bank pair (four wavefronts per lookup)
constexpr int LUT8_ENTRIES = 256 * 8;
__device__ __forceinline__ uint2 lut8_byte(const uint2 *lutl, uint32_t w, int k) {
    return lutl[((w >> (8 * k)) & 0xffu) << 3];
}
constexpr int ATTEND_CHUNKS_TMA = 8;   // CTAs per token (one thread-block cluster)
__device__ __forceinline__ void bar_consumers() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

template <int NT, int MT, int MTV, int NBW, bool QRES>
__global__ void __launch_bounds__(160, 2) decode_attn_tma_kernel(const __grid_constant__ AttnMaps maps,
                                                              const DecodeAttnArgs a) {
    pdl_wait();
    extern __shared__ __align__(1024) uint8_t dsm_raw[];
    // 1024-byte alignment for the swizzled tiles, by offsetting the shared
    // array itself (keeps every derived pointer in the shared address space)
    uint8_t *dsm = dsm_raw + ((1024u - (as::sa(dsm_raw) & 1023u)) & 1023u);
    constexpr int HP = 16 * MTV, QB = NT * 8 * 128, ROWS_A = 4 * MT * 16;
    constexpr int DG = 64 * 4 * NBW, NBOX = DG / 256;
    constexpr int NCH = ATTEND_CHUNKS_TMA;
    const int chmax = a.chmax;
    const int SROW = chmax + 4, PROW = chmax + 8, UROW = DG + 4;
    uint2 *lut = reinterpret_cast<uint2 *>(dsm);
    uint8_t *ring = dsm + a.off_ring;
    float *Ss = reinterpret_cast<float *>(dsm + a.off_S);
    __half *Ph = reinterpret_cast<__half *>(dsm + a.off_P);
    __half *Pl = Ph + HP * PROW;
    float *part = reinterpret_cast<float *>(dsm + a.off_part);
    float *mloc = reinterpret_cast<float *>(dsm + a.off_small);
    float *lloc = mloc + HP;
    float *wgt = lloc + HP;
    float *kn_s = wgt + NCH * HP;
    float *vn_s = kn_s + chmax;
    float *hred = vn_s + chmax;                                    // [2][4][HP] per-warp head max / sum
    uint64_t *bars = reinterpret_cast<uint64_t *>(hred + 8 * HP);  // 8-byte aligned: chmax, HP % 16 == 0
    uint64_t *full = bars, *empty = bars + NS, *lutfull = bars + 2 * NS, *lutfree = lutfull + 1;
    uint64_t *fullA = lutfree + 1, *emptyA = fullA + 4, *qfull = emptyA + 4;  // resident-q~ scores phase
    volatile int *abort_flag = reinterpret_cast<volatile int *>(qfull + 1);
    const uint8_t *qres = dsm + a.off_q;                           // [blocks][hi, lo][NT * 8][128 B]

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int m = blockIdx.z;
    const int tn = a.pos[m] + 1;
    const int chl = ((tn + NCH - 1) / NCH + 15) / 16 * 16;
    const int c0 = rank * chl, nloc = max(0, min(tn, c0 + chl) - c0);
    const int nmt = (nloc + 15) / 16;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int64_t rowbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const int nblk = a.kvd / 64;
    const int ngroups = (nmt + 4 * MT - 1) / (4 * MT);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            as::mbar_init(&full[s], 1);
            as::mbar_init(&empty[s], 4);
        }
        as::mbar_init(lutfull, 1);
        as::mbar_init(lutfree, 4);
        for (int w = 0; w < 4; ++w) {
            as::mbar_init(&fullA[w], 1);
            as::mbar_init(&emptyA[w], 1);
        }
        as::mbar_init(qfull, 1);
        *abort_flag = 0;
        as::mbar_fence_init();
    }
    __syncthreads();

    if (warp == 4) {
        // ---- producer
        if (lane == 0) {
            as::mbar_expect_tx(lutfull, LUT8_ENTRIES * 8);
            as::bulk_load(lut, a.lutk, LUT8_ENTRIES * 8, lutfull);
            // the chunk's key and value code rows are contiguous: pull both into
            // L2 now, so the ring's tile loads wait on L2 rather than on DRAM
            if (nloc > 0) {
                const uint32_t kb = (uint32_t)nloc * a.kpl, vb = (uint32_t)nloc * a.vpl;
                as::prefetch_l2(a.kcodes + (rowbase + c0) * a.kpl, (kb + 15) & ~15u);
                as::prefetch_l2(a.vcodes + (rowbase + c0) * a.vpl, (vb + 15) & ~15u);
            }
            if constexpr (QRES) {
                // q~ of the token once, then one 16-position key tile (kpl bytes
                // per row, 128-byte swizzled boxes) per m-tile into its warp's slot
                as::mbar_expect_tx(qfull, 2 * nblk * QB);
                for (int q = 0; q < nblk; ++q) {
                    as::tma_load_2d(dsm + a.off_q + q * 2 * QB, &maps.qh, q * 64, m * a.nh, qfull);
                    as::tma_load_2d(dsm + a.off_q + q * 2 * QB + QB, &maps.ql, q * 64, m * a.nh, qfull);
                }
                const int kb = a.kpl / 128;
                for (int mt = 0; mt < nmt; ++mt) {
                    const int w = mt & 3;
                    if (!as::mbar_wait(&emptyA[w], ((mt >> 2) & 1) ^ 1, abort_flag, a.err)) continue;
                    uint8_t *st = ring + w * a.sstage_a;
                    as::mbar_expect_tx(&fullA[w], kb * 2048);
                    for (int b = 0; b < kb; ++b)
                        as::tma_load_2d(st + b * 2048, &maps.kt, b * 128, (int)(rowbase + c0 + mt * 16), &fullA[w]);
                }
            } else {
                int it = 0;
                for (int mg = 0; mg < ngroups; ++mg)
                    for (int q = 0; q < nblk; ++q, ++it) {
                        const int s = it % NS;
                        if (!as::mbar_wait(&empty[s], ((it / NS) & 1) ^ 1, abort_flag, a.err)) continue;
                        uint8_t *st = ring + s * a.sstage;
                        as::mbar_expect_tx(&full[s], 2 * QB + ROWS_A * 32);
                        as::tma_load_2d(st, &maps.qh, q * 64, m * a.nh, &full[s]);
                        as::tma_load_2d(st + QB, &maps.ql, q * 64, m * a.nh, &full[s]);
                        as::tma_load_2d(st + 2 * QB, &maps.kc, q * 32, (int)(rowbase + c0 + mg * ROWS_A), &full[s]);
                    }
            }
            if (as::mbar_wait(lutfree, 0, abort_flag, a.err)) {
                as::mbar_expect_tx(lutfull, LUT8_ENTRIES * 8);
                as::bulk_load(lut, a.lutv, LUT8_ENTRIES * 8, lutfull);
            }
        }
        __syncwarp();
        int it = QRES ? 0 : ngroups * nblk;
        for (int dg = 0; dg < a.ndg; ++dg) {
            if (lane == 0) {
                for (int ks = 0; ks < nmt; ++ks, ++it) {
                    const int s = it % NS;
                    if (!as::mbar_wait(&empty[s], ((it / NS) & 1) ^ 1, abort_flag, a.err)) continue;
                    uint8_t *st = ring + s * a.sstage;
                    as::mbar_expect_tx(&full[s], NBOX * 16 * 128);
                    for (int b = 0; b < NBOX; ++b)
                        as::tma_load_2d(st + b * 2048, &maps.vc, dg * (DG / 2) + b * 128, (int)(rowbase + c0 + ks * 16),
                                        &full[s]);
                }
            }
            __syncwarp();
            cluster.sync();  // partial tiles written
            cluster.sync();  // combine done
        }
        return;
    }

    // ---- consumers (warps 0..3)
    for (int t = tid; t < nloc; t += 128) {
        kn_s[t] = a.knorm[rowbase + c0 + t];
        vn_s[t] = a.vnorm[rowbase + c0 + t];
    }
    const uint2 *lutl = lut + (lane & 7);
    as::mbar_wait(lutfull, 0, abort_flag, a.err);
    bar_consumers();  // norms staged
    int it = 0;
    if constexpr (QRES) {
        as::mbar_wait(qfull, 0, abort_flag, a.err);
        // scores of this warp's m-tiles (mt = warp + 4i), kept in registers
        float sc[MT][NT][4];
#pragma unroll
        for (int i = 0; i < MT; ++i) {
            const int mt = warp + 4 * i;
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) sc[i][j][e] = -INFINITY;
            if (mt < nmt) {
                const bool ok = as::mbar_wait(&fullA[warp], i & 1, abort_flag, a.err);
                const uint8_t *st = ring + warp * a.sstage_a;
                // hi*hi, lo*hi and hi*lo products in separate accumulators (independent MMA chains)
                float s0[NT][4], s1[NT][4], s2[NT][4];
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) s0[j][e] = s1[j][e] = s2[j][e] = 0.0f;
                if (ok) {
                    for (int q = 0; q < nblk; ++q) {
                        const uint8_t *qh = qres + q * 2 * QB, *ql = qh + QB;
                        uint32_t bq[NT][8], bl[NT][8];
#pragma unroll
                        for (int j = 0; j < NT; ++j) {
                            const uint8_t *rh = qh + (j * 8 + g) * 128, *rl = ql + (j * 8 + g) * 128;
                            const uint4 u0 = *reinterpret_cast<const uint4 *>(rh + (((2 * c) ^ g) << 4));
                            const uint4 u1 = *reinterpret_cast<const uint4 *>(rh + (((2 * c + 1) ^ g) << 4));
                            const uint4 v0 = *reinterpret_cast<const uint4 *>(rl + (((2 * c) ^ g) << 4));
                            const uint4 v1 = *reinterpret_cast<const uint4 *>(rl + (((2 * c + 1) ^ g) << 4));
                            bq[j][0] = u0.x; bq[j][1] = u0.y; bq[j][2] = u0.z; bq[j][3] = u0.w;
                            bq[j][4] = u1.x; bq[j][5] = u1.y; bq[j][6] = u1.z; bq[j][7] = u1.w;
                            bl[j][0] = v0.x; bl[j][1] = v0.y; bl[j][2] = v0.z; bl[j][3] = v0.w;
                            bl[j][4] = v1.x; bl[j][5] = v1.y; bl[j][6] = v1.z; bl[j][7] = v1.w;
                        }
                        // the thread's 8 code bytes of rows g and g + 8: bytes 32q + 8c of each row =
                        // box q / 4, 16-byte chunk 2 (q % 4) + c / 2 (swizzled by row % 8 = g), half c % 2
                        const uint8_t *box = st + (q >> 2) * 2048;
                        const int co = ((((q & 3) << 1) | (c >> 1)) ^ g) << 4 | ((c & 1) << 3);
                        const uint2 w0 = *reinterpret_cast<const uint2 *>(box + g * 128 + co);
                        const uint2 w1 = *reinterpret_cast<const uint2 *>(box + (g + 8) * 128 + co);
#pragma unroll
                        for (int s4 = 0; s4 < 4; ++s4) {
                            const uint32_t x0 = s4 < 2 ? w0.x : w0.y, x1 = s4 < 2 ? w1.x : w1.y;
                            const int kk = (s4 & 1) * 2;
                            const uint2 e0 = lut8_byte(lutl, x0, kk), e2 = lut8_byte(lutl, x0, kk + 1);
                            const uint2 e1 = lut8_byte(lutl, x1, kk), e3 = lut8_byte(lutl, x1, kk + 1);
#pragma unroll
                            for (int j = 0; j < NT; ++j)
                                mma_f16(s0[j], e0.x, e1.x, e2.x, e3.x, bq[j][2 * s4], bq[j][2 * s4 + 1]);
#pragma unroll
                            for (int j = 0; j < NT; ++j)
                                mma_f16(s1[j], e0.y, e1.y, e2.y, e3.y, bq[j][2 * s4], bq[j][2 * s4 + 1]);
#pragma unroll
                            for (int j = 0; j < NT; ++j)
                                mma_f16(s2[j], e0.x, e1.x, e2.x, e3.x, bl[j][2 * s4], bl[j][2 * s4 + 1]);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) as::mbar_arrive(&emptyA[warp]);
#pragma unroll
                for (int hrow = 0; hrow < 2; ++hrow) {
                    const int t = mt * 16 + g + hrow * 8;
                    const float f = t < nloc ? kn_s[t] * a.scale : 0.0f;
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int h = j * 8 + c * 2 + e, x = hrow * 2 + e;
                            if (t < nloc && h < a.nh) sc[i][j][x] = (s0[j][x] + s1[j][x] + s2[j][x]) * f;
                        }
                }
            }
        }
        __syncwarp();
        if (lane == 0) as::mbar_arrive(lutfree);  // the key table is no longer read
        // chunk-local softmax from registers: head h = 8j + 2c + e, rows over g
        float mx[NT][2];
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float v = -INFINITY;
#pragma unroll
                for (int i = 0; i < MT; ++i) v = fmaxf(v, fmaxf(sc[i][j][e], sc[i][j][2 + e]));
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
                mx[j][e] = v;
                if (g == 0) hred[warp * HP + j * 8 + 2 * c + e] = v;
            }
        bar_consumers();
        float ls[NT][2];
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int h = j * 8 + 2 * c + e;
                mx[j][e] = fmaxf(fmaxf(hred[h], hred[HP + h]), fmaxf(hred[2 * HP + h], hred[3 * HP + h]));
                ls[j][e] = 0.0f;
            }
#pragma unroll
        for (int i = 0; i < MT; ++i) {
            const int mt = warp + 4 * i;
            if (mt < nmt) {
#pragma unroll
                for (int hrow = 0; hrow < 2; ++hrow) {
                    const int t = mt * 16 + g + hrow * 8;
                    const float vn = t < nloc ? vn_s[t] : 0.0f;
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int h = j * 8 + 2 * c + e;
                            const float sv = sc[i][j][hrow * 2 + e];
                            const float pe = sv == -INFINITY ? 0.0f : expf(sv - mx[j][e]);
                            ls[j][e] += pe;
                            const float v = pe * vn;
                            const __half hv = __float2half_rn(v);
                            Ph[h * PROW + t] = hv;
                            Pl[h * PROW + t] = __float2half_rn(v - __half2float(hv));
                        }
                }
            }
        }
        if constexpr (NT * 8 < HP) {  // head rows past the MMA tiles stay zero
            for (int x = tid; x < (HP - NT * 8) * nmt * 16; x += 128) {
                const int h = NT * 8 + x / (nmt * 16), t = x % (nmt * 16);
                Ph[h * PROW + t] = Pl[h * PROW + t] = __float2half_rn(0.0f);
            }
        }
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float v = ls[j][e];
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (g == 0) hred[4 * HP + warp * HP + j * 8 + 2 * c + e] = v;
            }
        bar_consumers();
        if (tid < HP) {
            const bool live = tid < a.nh && tid < NT * 8 && nloc > 0;
            mloc[tid] = live ? fmaxf(fmaxf(hred[tid], hred[HP + tid]), fmaxf(hred[2 * HP + tid], hred[3 * HP + tid]))
                             : -INFINITY;
            lloc[tid] = live ? (hred[4 * HP + tid] + hred[5 * HP + tid]) + (hred[6 * HP + tid] + hred[7 * HP + tid])
                             : 0.0f;
        }
    } else {
        for (int mg = 0; mg < ngroups; ++mg) {
            const int gm = min(4 * MT, nmt - mg * 4 * MT);
            float acc[MT][NT][4], acl[MT][NT][4];
    #pragma unroll
            for (int i = 0; i < MT; ++i)
    #pragma unroll
                for (int j = 0; j < NT; ++j)
    #pragma unroll
                    for (int e = 0; e < 4; ++e) acc[i][j][e] = acl[i][j][e] = 0.0f;
            for (int q = 0; q < nblk; ++q, ++it) {
                const int s = it % NS;
                const bool ok = as::mbar_wait(&full[s], (it / NS) & 1, abort_flag, a.err);
                const uint8_t *st = ring + s * a.sstage;
                if (ok) {
                    uint32_t bq[NT][8], bl[NT][8];
    #pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        // q~ row j * 8 + g (row & 7 == g), dims 16c .. 16c + 15 = 16-byte chunks 2c, 2c + 1
                        const uint8_t *rh = st + (j * 8 + g) * 128, *rl = st + QB + (j * 8 + g) * 128;
                        const uint4 u0 = *reinterpret_cast<const uint4 *>(rh + (((2 * c) ^ g) << 4));
                        const uint4 u1 = *reinterpret_cast<const uint4 *>(rh + (((2 * c + 1) ^ g) << 4));
                        const uint4 v0 = *reinterpret_cast<const uint4 *>(rl + (((2 * c) ^ g) << 4));
                        const uint4 v1 = *reinterpret_cast<const uint4 *>(rl + (((2 * c + 1) ^ g) << 4));
                        bq[j][0] = u0.x; bq[j][1] = u0.y; bq[j][2] = u0.z; bq[j][3] = u0.w;
                        bq[j][4] = u1.x; bq[j][5] = u1.y; bq[j][6] = u1.z; bq[j][7] = u1.w;
                        bl[j][0] = v0.x; bl[j][1] = v0.y; bl[j][2] = v0.z; bl[j][3] = v0.w;
                        bl[j][4] = v1.x; bl[j][5] = v1.y; bl[j][6] = v1.z; bl[j][7] = v1.w;
                    }
                    const uint8_t *kc = st + 2 * QB;
    #pragma unroll
                    for (int i = 0; i < MT; ++i) {
                        const int mt = warp + 4 * i;
                        if (mt < gm) {
                            const uint2 w0 = *reinterpret_cast<const uint2 *>(kc + (mt * 16 + g) * 32 + c * 8);
                            const uint2 w1 = *reinterpret_cast<const uint2 *>(kc + (mt * 16 + g + 8) * 32 + c * 8);
    #pragma unroll
                            for (int s4 = 0; s4 < 4; ++s4) {
                                const uint32_t x0 = s4 < 2 ? w0.x : w0.y, x1 = s4 < 2 ? w1.x : w1.y;
                                const int k = (s4 & 1) * 2;
                                const uint2 e0 = lut8_byte(lutl, x0, k), e2 = lut8_byte(lutl, x0, k + 1);
                                const uint2 e1 = lut8_byte(lutl, x1, k), e3 = lut8_byte(lutl, x1, k + 1);
    #pragma unroll
                                for (int j = 0; j < NT; ++j)
                                    mma_f16(acc[i][j], e0.x, e1.x, e2.x, e3.x, bq[j][2 * s4], bq[j][2 * s4 + 1]);
    #pragma unroll
                                for (int j = 0; j < NT; ++j)
                                    mma_f16(acl[i][j], e0.y, e1.y, e2.y, e3.y, bq[j][2 * s4], bq[j][2 * s4 + 1]);
    #pragma unroll
                                for (int j = 0; j < NT; ++j)
                                    mma_f16(acl[i][j], e0.x, e1.x, e2.x, e3.x, bl[j][2 * s4], bl[j][2 * s4 + 1]);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) as::mbar_arrive(&empty[s]);
            }
    #pragma unroll
            for (int i = 0; i < MT; ++i) {
                const int mt = warp + 4 * i;
                if (mt < gm) {
    #pragma unroll
                    for (int hrow = 0; hrow < 2; ++hrow) {
                        const int t = (mg * 4 * MT + mt) * 16 + g + hrow * 8;
                        const float f = t < nloc ? kn_s[t] * a.scale : 0.0f;
    #pragma unroll
                        for (int j = 0; j < NT; ++j)
    #pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int h = j * 8 + c * 2 + e;
                                if (h < HP) Ss[h * SROW + t] = (acc[i][j][hrow * 2 + e] + acl[i][j][hrow * 2 + e]) * f;
                            }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) as::mbar_arrive(lutfree);  // the key table is no longer read
        bar_consumers();                          // all scores in Ss

        // local softmax, one warp per head
        for (int h = warp; h < HP; h += 4) {
            __half *ph = Ph + h * PROW, *pl = Pl + h * PROW;
            const float *srow = Ss + h * SROW;
            const bool live = h < a.nh && nloc > 0;
            float mx = -INFINITY, sum = 0.0f;
            if (live) {
                for (int t = lane; t < nloc; t += 32) mx = fmaxf(mx, srow[t]);
    #pragma unroll
                for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            for (int t = lane; t < nmt * 16; t += 32) {
                float v = 0.0f;
                if (live && t < nloc) {
                    const float e = expf(srow[t] - mx);
                    sum += e;
                    v = e * vn_s[t];
                }
                const __half hv = __float2half_rn(v);
                ph[t] = hv;
                pl[t] = __float2half_rn(v - __half2float(hv));
            }
    #pragma unroll
            for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) {
                mloc[h] = mx;
                lloc[h] = sum;
            }
        }

    }
    as::mbar_wait(lutfull, 1, abort_flag, a.err);  // value table in place
    bar_consumers();                               // P and m / l complete

    for (int dg = 0; dg < a.ndg; ++dg) {
        float acc[NBW][MTV][8][4];
#pragma unroll
        for (int b = 0; b < NBW; ++b)
#pragma unroll
            for (int i = 0; i < MTV; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[b][i][j][e] = 0.0f;
        for (int ks = 0; ks < nmt; ++ks, ++it) {
            const int s = it % NS;
            const bool ok = as::mbar_wait(&full[s], (it / NS) & 1, abort_flag, a.err);
            const uint8_t *st = ring + s * a.sstage;
            if (ok) {
                uint32_t ah[MTV][4], al[MTV][4];
#pragma unroll
                for (int i = 0; i < MTV; ++i) {
                    const int r = i * 16 + (lane & 15), col = ks * 16 + ((lane >> 4) << 3);
                    ldsm_x4(smem_u32(Ph + r * PROW + col), ah[i][0], ah[i][1], ah[i][2], ah[i][3]);
                    ldsm_x4(smem_u32(Pl + r * PROW + col), al[i][0], al[i][1], al[i][2], al[i][3]);
                }
#pragma unroll
                for (int b = 0; b < NBW; ++b) {
                    // dim block db = warp + 4b: box db / 4, 32-byte column (db % 4); the thread's
                    // word (dims 8g ..) sits in 16-byte chunk 2 (db % 4) + g / 4 of each row
                    const int db = warp + 4 * b;
                    const uint8_t *box = st + (db >> 2) * 2048;
                    const int chunk = 2 * (db & 3) + (g >> 2), inb = 4 * (g & 3);
                    auto word = [&](int r) {
                        return *reinterpret_cast<const uint32_t *>(box + r * 128 + ((chunk ^ (r & 7)) << 4) + inb);
                    };
                    const uint32_t x0 = word(2 * c), x1 = word(2 * c + 1), x2 = word(2 * c + 8), x3 = word(2 * c + 9);
                    uint32_t bh[8][2], bl[8][2];
#pragma unroll
                    for (int by = 0; by < 4; ++by) {
                        const uint2 e0 = lut8_byte(lutl, x0, by), e1 = lut8_byte(lutl, x1, by);
                        const uint2 e2 = lut8_byte(lutl, x2, by), e3 = lut8_byte(lutl, x3, by);
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            const uint32_t sel = hf ? 0x7632u : 0x5410u;
                            bh[2 * by + hf][0] = prmt(e0.x, e1.x, sel);
                            bh[2 * by + hf][1] = prmt(e2.x, e3.x, sel);
                            bl[2 * by + hf][0] = prmt(e0.y, e1.y, sel);
                            bl[2 * by + hf][1] = prmt(e2.y, e3.y, sel);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < MTV; ++i)
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj)
                            mma_f16(acc[b][i][jj], ah[i][0], ah[i][1], ah[i][2], ah[i][3], bh[jj][0], bh[jj][1]);
#pragma unroll
                    for (int i = 0; i < MTV; ++i)
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj)
                            mma_f16(acc[b][i][jj], al[i][0], al[i][1], al[i][2], al[i][3], bh[jj][0], bh[jj][1]);
#pragma unroll
                    for (int i = 0; i < MTV; ++i)
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj)
                            mma_f16(acc[b][i][jj], ah[i][0], ah[i][1], ah[i][2], ah[i][3], bl[jj][0], bl[jj][1]);
                }
            }
            __syncwarp();
            if (lane == 0) as::mbar_arrive(&empty[s]);
        }
        bar_consumers();  // the partial tile may overlay the table and the ring (single dim group)
#pragma unroll
        for (int b = 0; b < NBW; ++b)
#pragma unroll
            for (int i = 0; i < MTV; ++i)
#pragma unroll
                for (int hrow = 0; hrow < 2; ++hrow)
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj)
#pragma unroll
                        for (int e = 0; e < 2; ++e)
                            part[(i * 16 + g + hrow * 8) * UROW + (warp + 4 * b) * 64 + 8 * (2 * c + e) + jj] =
                                acc[b][i][jj][hrow * 2 + e];
        cluster.sync();
        if (tid < HP) {
            const int h = tid;
            float mr[NCH], lr[NCH];
#pragma unroll
            for (int r = 0; r < NCH; ++r) {
                mr[r] = *cluster.map_shared_rank(mloc + h, r);
                lr[r] = *cluster.map_shared_rank(lloc + h, r);
            }
            float M = -INFINITY;
#pragma unroll
            for (int r = 0; r < NCH; ++r) M = fmaxf(M, mr[r]);
            float L = 0.0f;
#pragma unroll
            for (int r = 0; r < NCH; ++r) {
                mr[r] = mr[r] == -INFINITY ? 0.0f : expf(mr[r] - M);
                L += mr[r] * lr[r];
            }
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
            for (int r = 0; r < NCH; ++r) wgt[r * HP + h] = mr[r] * inv;
        }
        bar_consumers();
        const int quads = a.nh * (DG / 4);
        const int per = (quads + NCH - 1) / NCH;
        const int q0 = rank * per, q1 = min(quads, q0 + per);
        for (int qd = q0 + tid; qd < q1; qd += 128) {
            const int h = qd / (DG / 4), d = (qd % (DG / 4)) * 4;
            float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
            float4 v[NCH];
#pragma unroll
            for (int r = 0; r < NCH; ++r)  // a chunk without positions has weight 0 and an unwritten tile
                v[r] = wgt[r * HP + h] != 0.0f
                           ? *reinterpret_cast<const float4 *>(cluster.map_shared_rank(part, r) + h * UROW + d)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < NCH; ++r) {
                const float w = wgt[r * HP + h];
                u.x += w * v[r].x; u.y += w * v[r].y; u.z += w * v[r].z; u.w += w * v[r].w;
            }
            uint32_t h01, l01, h23, l23;
            split_h2(u.x, u.y, h01, l01);
            split_h2(u.z, u.w, h23, l23);
            const int64_t o = ((int64_t)m * a.nh + h) * a.kvd + dg * DG + d;
            *reinterpret_cast<uint2 *>(a.U + o) = make_uint2(h01, h23);
            *reinterpret_cast<uint2 *>(a.U_lo + o) = make_uint2(l01, l23);
        }
        cluster.sync();  // peers are done reading this CTA's partial tile
    }
}

// 8-replica byte tables of both codebooks (LUT8_ENTRIES uint2 each)
__global__ void build_luts_kernel(const float *kcent, const float *vcent, uint2 *lutk, uint2 *lutv) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= 2 * LUT8_ENTRIES) return;
    const float *cent = i < LUT8_ENTRIES ? kcent : vcent;
    const int b = (i % LUT8_ENTRIES) >> 3;
    uint32_t hi, lo;
    split_h2(cent[b & 15], cent[b >> 4], hi, lo);
    (i < LUT8_ENTRIES ? lutk : lutv)[i % LUT8_ENTRIES] = make_uint2(hi, lo);
}

// ---------------------------------------------------------------------------
// Standard attention over a bf16 K/V cache (AttentionMode::Standard,
// attention_head, src/transformer.rs:333-389; cache layout of
// MultiLayerKVCache, crates/katgpt-transformer/src/kv_cache.rs:8-124, kept as
// [slot][layer][pos][kv_dim] bf16 on the device).

// New K/V rows of a step into the bf16 cache; for prefill also the f16 hi/lo
// split of the bf16-rounded rows (the flash kernel's operands), so prefill and
// decode attend over the same cached values.
__global__ void kv_store_std_kernel(const float *qkv, int64_t ldx, int64_t koff, int64_t voff, int kvd,
                                    const int32_t *slot, const int32_t *pos, int L, int B, int layer, bf16 *kc,
                                    bf16 *vc, __half *kt, __half *kt2, __half *vt, __half *vt2) {
    pdl_wait();
    const int m = blockIdx.x;
    const int64_t row = ((int64_t)slot[m] * L + layer) * B + pos[m];
    for (int j = threadIdx.x; j < kvd; j += blockDim.x) {
        const bf16 k = __float2bfloat16_rn(qkv[(int64_t)m * ldx + koff + j]);
        const bf16 v = __float2bfloat16_rn(qkv[(int64_t)m * ldx + voff + j]);
        kc[row * kvd + j] = k;
        vc[row * kvd + j] = v;
        if (kt) {
            const float kf = __bfloat162float(k), vf = __bfloat162float(v);
            const __half kh = __float2half_rn(kf), vh = __float2half_rn(vf);
            kt[(int64_t)m * kvd + j] = kh;
            kt2[(int64_t)m * kvd + j] = __float2half_rn(kf - __half2float(kh));
            vt[(int64_t)m * kvd + j] = vh;
            vt2[(int64_t)m * kvd + j] = __float2half_rn(vf - __half2float(vh));
        }
    }
}

// Decode: one CTA per (kv head, token); each of 4 warps streams every 4th
// position (4 positions in flight), lanes own HD / 32 dims, online softmax
// per warp, then the warps combine through shared memory. Query heads that
// share the kv head (GQA) run one after another.
template <int HD>
__global__ void __launch_bounds__(128) std_decode_kernel(const StdDecodeArgs a) {
    pdl_wait();
    constexpr int DPL = HD / 32, U = 4;
    __shared__ float sm_m[4], sm_l[4], sm_o[4][HD];
    const int kh = blockIdx.x, m = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tn = a.pos[m] + 1, G = a.nh / a.nkv;
    const int64_t base = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const bf16 *K = a.kc + base * a.kvd + kh * HD + lane * DPL;
    const bf16 *Vp = a.vc + base * a.kvd + kh * HD + lane * DPL;
    auto load = [&](const bf16 *p, float (&f)[DPL]) {
        if constexpr (DPL == 4) {
            const uint2 w = *reinterpret_cast<const uint2 *>(p);
            const __nv_bfloat162 x0 = *reinterpret_cast<const __nv_bfloat162 *>(&w.x);
            const __nv_bfloat162 x1 = *reinterpret_cast<const __nv_bfloat162 *>(&w.y);
            f[0] = __low2float(x0); f[1] = __high2float(x0); f[2] = __low2float(x1); f[3] = __high2float(x1);
        } else {
            const __nv_bfloat162 x0 = *reinterpret_cast<const __nv_bfloat162 *>(p);
            f[0] = __low2float(x0); f[1] = __high2float(x0);
        }
    };
    for (int qh = 0; qh < G; ++qh) {
        const int h = kh * G + qh;
        float q[DPL];
#pragma unroll
        for (int d = 0; d < DPL; ++d) q[d] = a.Q[(int64_t)m * a.ldq + h * HD + lane * DPL + d] * a.scale;
        float mx = -INFINITY, l = 0.0f, o[DPL];
#pragma unroll
        for (int d = 0; d < DPL; ++d) o[d] = 0.0f;
        for (int t0 = warp * U; t0 < tn; t0 += 4 * U) {
            float kf[U][DPL], vf[U][DPL], s[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int t = min(t0 + u, tn - 1);
                load(K + (int64_t)t * a.kvd, kf[u]);
                load(Vp + (int64_t)t * a.kvd, vf[u]);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float p = 0.0f;
#pragma unroll
                for (int d = 0; d < DPL; ++d) p = fmaf(q[d], kf[u][d], p);
                s[u] = p;
            }
#pragma unroll
            for (int off = 16; off; off >>= 1)
#pragma unroll
                for (int u = 0; u < U; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], off);
            float mnew = mx;
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (t0 + u < tn) mnew = fmaxf(mnew, s[u]);
            const float corr = expf(mx - mnew);
            l *= corr;
#pragma unroll
            for (int d = 0; d < DPL; ++d) o[d] *= corr;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float p = t0 + u < tn ? expf(s[u] - mnew) : 0.0f;
                l += p;
#pragma unroll
                for (int d = 0; d < DPL; ++d) o[d] = fmaf(p, vf[u][d], o[d]);
            }
            mx = mnew;
        }
        if (lane == 0) {
            sm_m[warp] = mx;
            sm_l[warp] = l;
        }
#pragma unroll
        for (int d = 0; d < DPL; ++d) sm_o[warp][lane * DPL + d] = o[d];
        __syncthreads();
        for (int d = threadIdx.x; d < HD; d += 128) {
            float M = -INFINITY;
            for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w]);
            float L = 0.0f, acc = 0.0f;
            for (int w = 0; w < 4; ++w) {
                const float f = sm_m[w] == -INFINITY ? 0.0f : expf(sm_m[w] - M);
                L += f * sm_l[w];
                acc += f * sm_o[w][d];
            }
            a.O[(int64_t)m * a.ldo + h * HD + d] = acc / L;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Prefill: dequantize codes of every prompt token to f16 hi/lo centroid vectors.
__global__ void centroids_kernel(const uint8_t *codes, int pl, int64_t row_stride_codes, const int32_t *slot,
                                 const int32_t *pos, int L, int B, int layer, const float *cent, int kvd, int M,
                                 __half *out, __half *out_lo) {
    pdl_wait();
    __shared__ uint2 lut[256];
    build_lut(lut, cent);
    __syncthreads();
    const int m = blockIdx.x;
    const int64_t row = ((int64_t)slot[m] * L + layer) * B + pos[m];
    const uint8_t *c = codes + row * pl;
    uint32_t *o = reinterpret_cast<uint32_t *>(out + (int64_t)m * kvd);
    uint32_t *ol = reinterpret_cast<uint32_t *>(out_lo + (int64_t)m * kvd);
    for (int b = threadIdx.x; b < kvd / 2; b += blockDim.x) {
        const uint2 e = lut[c[b]];
        o[b] = e.x;
        ol[b] = e.y;
    }
    (void)row_stride_codes;
}
__global__ void gather_norms_kernel(const float *norms, const int32_t *slot, const int32_t *pos, int L, int B,
                                    int layer, int M, float *out) {
    pdl_wait();
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    out[m] = norms[((int64_t)slot[m] * L + layer) * B + pos[m]];
}

// Causal flash attention over one sequence's prompt (rows base..base+T-1).
// Q, K, V are f16 hi/lo splits; every product uses hi*hi + lo*hi + hi*lo, the
// online softmax is f32, output f32. CTA = 64 queries x one head, 4 warps x 16.
template <int HD>
__global__ void __launch_bounds__(128) fa_kernel(const FlashArgs a) {
    pdl_wait();
    constexpr int KT = 64, LD = HD + 8;
    extern __shared__ __align__(16) __half fsm[];
    __half *sKh = fsm, *sKl = fsm + KT * LD, *sVh = fsm + 2 * KT * LD, *sVl = fsm + 3 * KT * LD;
    const int seq = blockIdx.z, h = blockIdx.y, qt0 = blockIdx.x * 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int T = a.T;
    if (qt0 >= T) return;
    const int kvh = h * a.nkv / a.nh;
    const int64_t base = (int64_t)seq * T;
    const int q0 = qt0 + warp * 16;
    uint32_t qh[HD / 16][4], ql[HD / 16][4];
    {
        const int ra = min(q0 + g, T - 1), rb = min(q0 + g + 8, T - 1);
        const int64_t oa = (base + ra) * a.ldq + h * HD, ob = (base + rb) * a.ldq + h * HD;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            const int k0 = ks * 16 + 2 * c;
            qh[ks][0] = *reinterpret_cast<const uint32_t *>(a.Q + oa + k0);
            qh[ks][1] = *reinterpret_cast<const uint32_t *>(a.Q + ob + k0);
            qh[ks][2] = *reinterpret_cast<const uint32_t *>(a.Q + oa + k0 + 8);
            qh[ks][3] = *reinterpret_cast<const uint32_t *>(a.Q + ob + k0 + 8);
            ql[ks][0] = *reinterpret_cast<const uint32_t *>(a.Q_lo + oa + k0);
            ql[ks][1] = *reinterpret_cast<const uint32_t *>(a.Q_lo + ob + k0);
            ql[ks][2] = *reinterpret_cast<const uint32_t *>(a.Q_lo + oa + k0 + 8);
            ql[ks][3] = *reinterpret_cast<const uint32_t *>(a.Q_lo + ob + k0 + 8);
        }
    }
    float o[HD / 8][4];
#pragma unroll
    for (int j = 0; j < HD / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};
    const float sl2 = a.scale * 1.4426950408889634f;
    const int kend = min(T, qt0 + 64);
    for (int k0 = 0; k0 < kend; k0 += KT) {
        __syncthreads();
        for (int e = threadIdx.x; e < KT * HD / 8; e += blockDim.x) {
            const int r = e / (HD / 8), cc = (e % (HD / 8)) * 8;
            const int t = k0 + r;
            uint4 kh = make_uint4(0, 0, 0, 0), kl = kh, vh = kh, vl = kh;
            if (t < T) {
                const int64_t off = (base + t) * a.ldk + kvh * HD + cc;
                kh = *reinterpret_cast<const uint4 *>(a.K + off);
                kl = *reinterpret_cast<const uint4 *>(a.K_lo + off);
                vh = *reinterpret_cast<const uint4 *>(a.V + off);
                vl = *reinterpret_cast<const uint4 *>(a.V_lo + off);
            }
            *reinterpret_cast<uint4 *>(sKh + r * LD + cc) = kh;
            *reinterpret_cast<uint4 *>(sKl + r * LD + cc) = kl;
            *reinterpret_cast<uint4 *>(sVh + r * LD + cc) = vh;
            *reinterpret_cast<uint4 *>(sVl + r * LD + cc) = vl;
        }
        __syncthreads();
        if (k0 > q0 + 15) continue;  // whole tile in the future for this warp
        float s[KT / 8][4];
#pragma unroll
        for (int j = 0; j < KT / 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[j][e] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
#pragma unroll
            for (int j2 = 0; j2 < KT / 16; ++j2) {
                uint32_t b0, b1, b2, b3, d0, d1, d2, d3;
                const int r = j2 * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int col = ks * 16 + (((lane >> 3) & 1) << 3);
                ldsm_x4(smem_u32(sKh + r * LD + col), b0, b1, b2, b3);
                ldsm_x4(smem_u32(sKl + r * LD + col), d0, d1, d2, d3);
                mma_f16(s[2 * j2], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], b0, b1);
                mma_f16(s[2 * j2], ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3], b0, b1);
                mma_f16(s[2 * j2], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], d0, d1);
                mma_f16(s[2 * j2 + 1], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], b2, b3);
                mma_f16(s[2 * j2 + 1], ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3], b2, b3);
                mma_f16(s[2 * j2 + 1], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], d2, d3);
            }
        // causal mask + online softmax (rows g, g+8)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int qi = q0 + g + hr * 8;
            float mx = mrow[hr];
#pragma unroll
            for (int j = 0; j < KT / 8; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int kj = k0 + j * 8 + 2 * c + e;
                    float v = (kj <= qi && kj < T) ? s[j][hr * 2 + e] * sl2 : -INFINITY;
                    s[j][hr * 2 + e] = v;
                    mx = fmaxf(mx, v);
                }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float corr = mrow[hr] == -INFINITY ? 0.0f : exp2f(mrow[hr] - mx);
            float ls = 0.0f;
#pragma unroll
            for (int j = 0; j < KT / 8; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float p = mx == -INFINITY ? 0.0f : exp2f(s[j][hr * 2 + e] - mx);
                    s[j][hr * 2 + e] = p;
                    ls += p;
                }
            ls += __shfl_xor_sync(0xffffffffu, ls, 1);
            ls += __shfl_xor_sync(0xffffffffu, ls, 2);
            lrow[hr] = lrow[hr] * corr + ls;
            mrow[hr] = mx;
#pragma unroll
            for (int j = 0; j < HD / 8; ++j) {
                o[j][hr * 2] *= corr;
                o[j][hr * 2 + 1] *= corr;
            }
        }
        // O += P V  (P split into f16 hi + lo)
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
            uint32_t p0, p1, p2, p3, l0, l1, l2, l3;
            split_h2(s[2 * kk][0], s[2 * kk][1], p0, l0);
            split_h2(s[2 * kk][2], s[2 * kk][3], p1, l1);
            split_h2(s[2 * kk + 1][0], s[2 * kk + 1][1], p2, l2);
            split_h2(s[2 * kk + 1][2], s[2 * kk + 1][3], p3, l3);
#pragma unroll
            for (int j2 = 0; j2 < HD / 16; ++j2) {
                uint32_t b0, b1, b2, b3, d0, d1, d2, d3;
                const int r = kk * 16 + (lane & 15);
                const int col = j2 * 16 + ((lane >> 4) << 3);
                ldsm_x4_t(smem_u32(sVh + r * LD + col), b0, b1, b2, b3);
                ldsm_x4_t(smem_u32(sVl + r * LD + col), d0, d1, d2, d3);
                mma_f16(o[2 * j2], p0, p1, p2, p3, b0, b1);
                mma_f16(o[2 * j2], l0, l1, l2, l3, b0, b1);
                mma_f16(o[2 * j2], p0, p1, p2, p3, d0, d1);
                mma_f16(o[2 * j2 + 1], p0, p1, p2, p3, b2, b3);
                mma_f16(o[2 * j2 + 1], l0, l1, l2, l3, b2, b3);
                mma_f16(o[2 * j2 + 1], p0, p1, p2, p3, d2, d3);
            }
        }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        const int qi = q0 + g + hr * 8;
        if (qi >= T) continue;
        const float inv = 1.0f / lrow[hr];
        float *dst = a.O + (base + qi) * a.ldo + h * HD;
#pragma unroll
        for (int j = 0; j < HD / 8; ++j)
            *reinterpret_cast<float2 *>(dst + j * 8 + 2 * c) = make_float2(o[j][hr * 2] * inv, o[j][hr * 2 + 1] * inv);
    }
}

}  // namespace

namespace {
constexpr int ATTEND_CHUNKS = 8;  // CTAs per token (one thread-block cluster)
int align16(int x) { return (x + 15) / 16 * 16; }
}  // namespace

template <int NT, int NBW>
cudaError_t launch_decode_attn(DecodeAttnArgs a, cudaStream_t s) {
    constexpr int MT = NT <= 2 ? 4 : 2, MTV = (NT * 8 + 15) / 16, HP = 16 * MTV;
    const int NCH = ATTEND_CHUNKS;
    const int DG = 64 * a.nbg;
    a.chmax = ((a.B + NCH - 1) / NCH + 15) / 16 * 16;
    a.sstage = 4 * MT * 16 * 32 + 2 * NT * 8 * 72 * 2;
    a.vrow = DG / 2 + (16 - (DG / 2) % 128 + 128) % 128;  // row stride = 16 mod 128 bytes: conflict-free reads
    a.vstage = 16 * a.vrow;
    const int ring = std::max(SSTG * a.sstage, VSTG * a.vstage);
    const int part = HP * (DG + 4) * 4;
    a.off_ring = LUT_ENTRIES * (int)sizeof(uint2);
    a.off_S = align16(a.off_ring + ring);
    a.off_P = align16(a.off_S + HP * (a.chmax + 4) * 4);
    a.off_small = align16(a.off_P + 2 * HP * (a.chmax + 8) * 2);
    int end = align16(a.off_small + (2 * HP + NCH * HP + 2 * a.chmax) * 4);
    if (a.ndg == 1 && part <= a.off_S) {
        a.off_part = 0;  // the partial tile overlays the table and the ring once they are dead
    } else {
        a.off_part = end;
        end = align16(end + part);
    }
    const int smem = end;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    static int attr = 0;
    if (smem > attr) {
        cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<NT, MT, MTV, NBW>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr = smem;
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(NCH, 1, a.M);
    lc.blockDim = dim3(128);
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = NCH;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 2;
    return cudaLaunchKernelEx(&lc, decode_attn_kernel<NT, MT, MTV, NBW>, a);
}

template <int NT>
cudaError_t decode_attn_nbw(DecodeAttnArgs &a, cudaStream_t s) {
    switch ((a.nbg + 3) / 4) {
        case 1: return launch_decode_attn<NT, 1>(a, s);
        case 2: return launch_decode_attn<NT, 2>(a, s);
        case 3: return launch_decode_attn<NT, 3>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

template <int NT, int NBW, bool QRES>
cudaError_t launch_decode_attn_tma(DecodeAttnArgs a, cudaStream_t s) {
    constexpr int MT = NT <= 2 ? 4 : 2, MTV = (NT * 8 + 15) / 16, HP = 16 * MTV;
    constexpr int DG = 64 * 4 * NBW, QB = NT * 8 * 128;
    const int NCH = ATTEND_CHUNKS_TMA;
    a.nbg = DG / 64;
    a.ndg = a.kvd / DG;
    a.chmax = ((a.B + NCH - 1) / NCH + 15) / 16 * 16;
    const int nblk = a.kvd / 64;
    const int stage_c = (DG / 256) * 2048;
    int ring, end;
    a.off_ring = LUT8_ENTRIES * (int)sizeof(uint2);
    if (QRES) {
        // lut | q~ (all blocks) | ring (one key tile slot per warp / value stages) | P | small
        a.off_q = a.off_ring;
        a.sstage_a = (a.kpl / 128) * 2048;
        a.sstage = stage_c;
        a.off_ring = a.off_q + 2 * nblk * QB;
        ring = std::max(4 * a.sstage_a, NS * a.sstage);
        a.off_S = a.off_ring + ring;  // no score buffer: scores stay in registers
        a.off_P = align16(a.off_S);
    } else {
        const int stage_a = 2 * QB + 4 * MT * 16 * 32;
        a.off_q = 0;
        a.sstage_a = 0;
        a.sstage = (std::max(stage_a, stage_c) + 1023) / 1024 * 1024;
        ring = NS * a.sstage;
        a.off_S = align16(a.off_ring + ring);
        a.off_P = align16(a.off_S + HP * (a.chmax + 4) * 4);
    }
    a.off_small = align16(a.off_P + 2 * HP * (a.chmax + 8) * 2);
    end = align16(a.off_small + (2 * HP + NCH * HP + 2 * a.chmax + 8 * HP) * 4 + (2 * NS + 2 + 9) * 8 + 16);
    const int part = HP * (DG + 4) * 4;
    if (a.ndg == 1 && part <= a.off_ring) {
        a.off_part = 0;  // the partial tile overlays the table (and q~) once they are dead
    } else {
        a.off_part = end;
        end = align16(end + part);
    }
    const int smem = end + 1024;  // slack for the 1024-byte alignment of the swizzled tiles
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    static int attr = 0;
    if (smem > attr) {
        cudaError_t e = cudaFuncSetAttribute(decode_attn_tma_kernel<NT, MT, MTV, NBW, QRES>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr = smem;
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(NCH, 1, a.M);
    lc.blockDim = dim3(160);
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = NCH;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 2;
    return cudaLaunchKernelEx(&lc, decode_attn_tma_kernel<NT, MT, MTV, NBW, QRES>, *a.maps, a);
}

template <int NT, bool QRES>
cudaError_t decode_attn_tma_nbw(const DecodeAttnArgs &a, cudaStream_t s) {
    // dim groups of 256 * NBW dims (NBW <= 2 with two head tiles)
    const int n256 = a.kvd / 256;
    if constexpr (NT <= 2) {
        if (n256 % 3 == 0) return launch_decode_attn_tma<NT, 3, QRES>(a, s);
    }
    if (n256 % 2 == 0) return launch_decode_attn_tma<NT, 2, QRES>(a, s);
    return launch_decode_attn_tma<NT, 1, QRES>(a, s);
}

template <int NT>
cudaError_t decode_attn_tma_q(const DecodeAttnArgs &a, cudaStream_t s) {
    // q~ resident in shared memory when all its blocks fit in 48 KB and a
    // warp's m-tiles cover the longest chunk
    constexpr int MT = NT <= 2 ? 4 : 2;
    const int chmax = ((a.B + ATTEND_CHUNKS_TMA - 1) / ATTEND_CHUNKS_TMA + 15) / 16 * 16;
    if ((a.kvd / 64) * 2 * NT * 8 * 128 <= 48 * 1024 && chmax <= 64 * MT) return decode_attn_tma_nbw<NT, true>(a, s);
    return decode_attn_tma_nbw<NT, false>(a, s);
}

cudaError_t decode_attn(const DecodeAttnArgs &a0, cudaStream_t s) {
    DecodeAttnArgs a = a0;
    if (a.M <= 0) return cudaSuccess;
    if (a.kvd % 64 || a.nh < 1 || a.nh > 32) return cudaErrorInvalidValue;
    if (a.maps && a.lutk && a.lutv && a.kvd % 256 == 0) {
        const int nt = (a.nh + 7) / 8;
        if (nt == 1) return decode_attn_tma_q<1>(a, s);
        if (nt == 2) return decode_attn_tma_q<2>(a, s);
        return decode_attn_tma_q<4>(a, s);
    }
    // 64-dim blocks per dim group: the largest divisor of kv_dim / 64 up to 12
    // (up to 8 with two head tiles, whose accumulators take twice the registers)
    const int nblk = a.kvd / 64;
    const int nt = (a.nh + 7) / 8;
    a.nbg = 1;
    for (int d = nt > 2 ? 8 : 12; d >= 1; --d)
        if (nblk % d == 0) {
            a.nbg = d;
            break;
        }
    a.ndg = nblk / a.nbg;
    if (nt == 1) return decode_attn_nbw<1>(a, s);
    if (nt == 2) return decode_attn_nbw<2>(a, s);
    return decode_attn_nbw<4>(a, s);
}

cudaError_t centroids(const uint8_t *codes, int pl, const int32_t *slot, const int32_t *pos, int L, int B, int layer,
                      const float *cent, int kvd, int M, __half *out, __half *out_lo, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    centroids_kernel<<<M, 128, 0, s>>>(codes, pl, 0, slot, pos, L, B, layer, cent, kvd, M, out, out_lo);
    return cudaGetLastError();
}
cudaError_t gather_norms(const float *norms, const int32_t *slot, const int32_t *pos, int L, int B, int layer, int M,
                         float *out, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    gather_norms_kernel<<<(M + 255) / 256, 256, 0, s>>>(norms, slot, pos, L, B, layer, M, out);
    return cudaGetLastError();
}
template <int HD>
cudaError_t launch_fa(const FlashArgs &a, cudaStream_t s) {
    const int smem = 4 * 64 * (HD + 8) * 2;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(fa_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    dim3 grid((a.T + 63) / 64, a.nh, a.n_seq);
    fa_kernel<HD><<<grid, 128, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t flash_prefill(const FlashArgs &a, cudaStream_t s) {
    switch (a.hd) {
        case 64: return launch_fa<64>(a, s);
        case 128: return launch_fa<128>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

bool decode_attn_maps(AttnMaps *maps, const uint8_t *kcodes, const uint8_t *vcodes, int64_t rows, int kpl, int vpl,
                      const __half *qrot, const __half *qrot_lo, int64_t qrows, int kvd, int nh) {
    if (kvd % 256 || nh < 1 || nh > 32) return false;
    const int nt = (nh + 7) / 8 <= 2 ? (nh + 7) / 8 : 4;
    const int rows_a = 4 * (nt <= 2 ? 4 : 2) * 16;
    return make_tensor_map(&maps->kc, kcodes, rows, kpl, kpl, 1, 32, rows_a, CU_TENSOR_MAP_SWIZZLE_NONE) &&
           make_tensor_map(&maps->kt, kcodes, rows, kpl, kpl, 1, 128, 16, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_tensor_map(&maps->vc, vcodes, rows, vpl, vpl, 1, 128, 16, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_tensor_map(&maps->qh, qrot, qrows, kvd, kvd, 2, 64, nt * 8, CU_TENSOR_MAP_SWIZZLE_128B) &&
           make_tensor_map(&maps->ql, qrot_lo, qrows, kvd, kvd, 2, 64, nt * 8, CU_TENSOR_MAP_SWIZZLE_128B);
}

cudaError_t build_luts(const float *kcent, const float *vcent, uint2 *lutk, uint2 *lutv, cudaStream_t s) {
    build_luts_kernel<<<(2 * LUT8_ENTRIES + 255) / 256, 256, 0, s>>>(kcent, vcent, lutk, lutv);
    return cudaGetLastError();
}

cudaError_t kv_store_std(const float *qkv, int64_t ldx, int64_t koff, int64_t voff, int kvd, int M,
                         const int32_t *slot, const int32_t *pos, int L, int B, int layer, bf16 *kc, bf16 *vc,
                         __half *kt, __half *kt2, __half *vt, __half *vt2, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    return launch_pdl(kv_store_std_kernel, dim3(M), dim3(256), 0, s, qkv, ldx, koff, voff, kvd, slot, pos, L, B, layer,
                      kc, vc, kt, kt2, vt, vt2);
}

cudaError_t std_decode(const StdDecodeArgs &a, cudaStream_t s) {
    if (a.M <= 0) return cudaSuccess;
    if (a.nh % a.nkv) return cudaErrorInvalidValue;
    const dim3 grid(a.nkv, a.M);
    switch (a.hd) {
        case 64: return launch_pdl(std_decode_kernel<64>, grid, dim3(128), 0, s, a);
        case 128: return launch_pdl(std_decode_kernel<128>, grid, dim3(128), 0, s, a);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace attn
}  // namespace kg
