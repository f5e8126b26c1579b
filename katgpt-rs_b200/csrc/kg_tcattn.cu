// kg_tcattn.cu — decode attention over 4-bit / 3-bit TurboQuant codes on the
// 5th-generation tensor cores (tcgen05), in the rotated domain.
//
// Math (forward_quantized attention, src/transformer.rs:4123-4141, softmax
// :333-389; a stored vector is norm * R^T centroid(code),
// src/turboquant/kv_cache.rs:279-317), per token m and head h:
//   s[t,h] = norm_k[t] * scale * <centroid(code_k[t]), q~_h>
//   u~_h   = sum_t softmax_t(s[., h])[t] * norm_v[t] * centroid(code_v[t])
// Three launches per layer:
//  * tc_scores_kernel — CTA = (two 128-position tiles, token). D[128 positions
//    x NHP heads] += A[positions x 16 dims] B[16 dims x heads] with A in
//    tensor memory: decoder thread r owns TMEM lane r (= position r of its
//    tile), turns its row's 32 code bytes per 64-dim block into f16 centroid
//    pairs through a 32-replica shared-memory table (entry (b, l) at word
//    32 b + l, lane l reads replica l: conflict-free) and stores them with
//    tcgen05.st; q~ arrives by TMA (128-byte swizzle) as the B operand. The
//    epilogue scales by norm_k * scale, and per 32-position chunk writes the
//    head maxima c, the sums sum exp(s - c) and e = exp(s - c) * norm_v (f16).
//  * tc_softmax_kernel — per (token, head): the global max M over the chunks,
//    l = sum_c csum_c exp(c - M), 1 / l, and e *= exp(c - M) in place, so the
//    values kernel can load e by TMA as an operand.
//  * tc_values_kernel — CTA = (128 dims, token). D[128 dims x NHP heads] +=
//    A[dims x 16 positions] B[16 positions x heads] with A in tensor memory
//    (lanes = dims, in a fixed permutation the epilogue undoes; columns =
//    position pairs): a decoder thread gathers one code byte of four
//    consecutive rows, and each nibble pair of consecutive positions indexes
//    the same byte -> f16 pair table, stored with tcgen05.st 16x256b. B = e
//    rows by TMA. The epilogue writes u~ = D / l as f16 hi / lo.
// Warp roles (352 threads): warp 0 TMA producer; warps 1 and 2 MMA issuers
// (one thread each: a single thread issues one tcgen05.mma per ~50 ns, so two
// independent MMA streams per CTA, per tile in the scores kernel and per half
// of each K block in the values kernel); warps 3..10 decoders and epilogue.
// Two CTAs per SM. Shared-memory stages (TMA) and tensor-memory A buffers
// (decoders) run as separate rings. Every mbarrier wait is bounded:
// on expiry the CTA raises its abort flag, KG_ERR_TIMEOUT goes to the error
// word, every warp still passes the barriers it owes and the tensor memory is
// released.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

#include "kg_async.cuh"
#include "kg_attn.cuh"
#include "kg_dev.cuh"
#include "kg_pdl.cuh"
#include "kg_tc.cuh"

namespace kg {
namespace attn {
namespace {

constexpr int SCW = 352;        // scores threads per CTA: TMA, two MMA issuers, 8 decoder warps
constexpr int TCW = 352;        // values threads per CTA: TMA, two MMA issuers, 8 decoder warps
constexpr int LUTW = 256 * 32;  // words of the replicated code-byte -> centroid-pair table
constexpr uint32_t FULLM = 0xffffffffu;

// scores
constexpr int S_STG = 6;                             // shared-memory stages (codes + q~)
constexpr int S_AB = 3;                              // A buffers in tensor memory
constexpr int S_TILE = 128;                          // positions per tile (TMEM lanes)
constexpr int S_KB = 64;                             // dims per K block: 32 code bytes per row
constexpr int S_CODE = 2 * S_TILE * 32;              // two tiles of 128 rows x 32 B
constexpr int S_Q = 32 * 128;                        // q~ block: up to 32 heads x 64 dims (f16)
constexpr int S_STAGE = S_CODE + S_Q;                // 12 KB
constexpr int S_CH = 33;                             // padded 32-position chunk in the transpose buffer
constexpr int S_TCOLS = 256;                         // acc (2 x 32) + A (3 buffers x 2 tiles x 32)
static_assert(S_STG * S_STAGE >= 2 * 32 * 4 * S_CH * 4, "the transpose buffer reuses the drained stages");
// values
constexpr int V_STG = 4;
constexpr int V_AB = 3;                              // A buffers in tensor memory
constexpr int V_KB = 128;                            // positions per K block (8 MMA K-steps of 16)
constexpr int V_DG = 128;                            // dims per CTA (64 code bytes per row)
constexpr int V_CODE = V_KB * (V_DG / 2);            // 8 KB, rows in the 64-byte swizzle
constexpr int V_E = 2 * 32 * 128;                    // e block: two 64-position atoms of up to 32 heads (f16)
constexpr int V_STAGE = V_CODE + V_E;                // 16 KB
constexpr int V_TCOLS = 256;                         // acc (2 x 32) + A (3 buffers x 64 columns)

// mul128 = 128 and mul4097 = 4097 arrive as kernel parameters: multiplying by
// a value the compiler cannot see keeps the table-address and index arithmetic
// on the multiply-add pipe (IMAD) instead of shifts on the integer pipe, which
// the decoders otherwise saturate
struct ScoreMaps {
    CUtensorMap codes, q;
    uint32_t mul128;
};
struct ValueMaps {
    CUtensorMap codes, e;
    uint32_t mul128, mul4097;
};

__device__ __forceinline__ uint32_t h2u(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
// byte b -> (centroid[b & 15], centroid[b >> 4]) as an f16 pair, 32 replicas;
// SWAP: (centroid[b >> 4], centroid[b & 15])
template <bool SWAP = false>
__device__ __forceinline__ void lut_build(uint32_t *lut, const float *cent) {
    for (int i = threadIdx.x; i < LUTW / 4; i += blockDim.x) {
        const int b = i >> 3;
        const int lo = SWAP ? b >> 4 : b & 15, hi = SWAP ? b & 15 : b >> 4;
        const uint32_t v = h2u(__ldg(cent + lo), __ldg(cent + hi));
        reinterpret_cast<uint4 *>(lut)[i] = make_uint4(v, v, v, v);
    }
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];\n" : "=r"(v) : "r"(addr));
    return v;
}
// table entry of byte k (0..3) of w for this lane (lut_lane = table address + 4 lane,
// m128 = 128: one table entry spans 32 words)
__device__ __forceinline__ uint32_t lk(uint32_t lut_lane, uint32_t w, int k, uint32_t m128) {
    return lds32(lut_lane + __byte_perm(w, 0u, 0x4440u | (uint32_t)k) * m128);
}
__device__ __forceinline__ void bar_named(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}
// warp-uniform bounded wait
__device__ __forceinline__ bool wait_all(uint64_t *b, uint32_t parity, volatile int *abort_flag, int *err) {
    const bool ok = as::mbar_wait(b, parity, abort_flag, err);
    return __all_sync(FULLM, ok);
}

// ---------------------------------------------------------------------------
template <int NHP>
__global__ void __launch_bounds__(SCW, 2) tc_scores_kernel(const __grid_constant__ ScoreMaps maps, const TqAttnArgs a) {
    extern __shared__ __align__(1024) uint8_t dsm_raw[];
    uint8_t *dsm = dsm_raw + ((1024u - (as::sa(dsm_raw) & 1023u)) & 1023u);
    uint8_t *stages = dsm;
    float *sT = reinterpret_cast<float *>(dsm);  // [2 tiles][NHP][4 chunks][33], over the drained stages
    uint32_t *lut = reinterpret_cast<uint32_t *>(dsm + S_STG * S_STAGE);
    uint64_t *full = reinterpret_cast<uint64_t *>(lut + LUTW);
    uint64_t *empty = full + S_STG;
    uint64_t *afull = empty + S_STG;     // [S_AB][2 tiles]
    uint64_t *aempty = afull + 2 * S_AB;  // [S_AB][2 tiles]
    uint64_t *accfull = aempty + 2 * S_AB;  // [2 tiles]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(accfull + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    lut_build(lut, a.kcent);  // a constant input: overlaps the previous kernel
    if (warp == 0) tc::alloc(tslot, S_TCOLS);
    pdl_wait();
    const int m = blockIdx.y;
    const int tn = a.pos[m] + 1;
    const int p0 = blockIdx.x * 2 * S_TILE;
    const int ntile = p0 >= tn ? 0 : min(2, (tn - p0 + S_TILE - 1) / S_TILE);  // CTA-uniform
    if (threadIdx.x == 0) {
        for (int s = 0; s < S_STG; ++s) {
            as::mbar_init(&full[s], 1);
            as::mbar_init(&empty[s], 5 * ntile + (ntile == 0));  // per live tile: 4 decoder warps + its MMA commit
        }
        for (int i = 0; i < 2 * S_AB; ++i) {
            as::mbar_init(&afull[i], 4);
            as::mbar_init(&aempty[i], 1);
        }
        as::mbar_init(&accfull[0], 1);
        as::mbar_init(&accfull[1], 1);
        *abort_flag = 0;
        as::mbar_fence_init();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tslot;
    const int nkb = a.kvd / S_KB;
    const int64_t rbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const uint32_t acc_col = 0, a_col = 64;  // acc of tile p at p * 32; A of (buffer b, tile p) at 64 + (2b + p) * 32

    if (ntile > 0) {
        if (warp == 0) {
            if (lane == 0) {  // TMA producer
                for (int kb = 0; kb < nkb; ++kb) {
                    const int s = kb % S_STG;
                    if (!as::mbar_wait(&empty[s], ((kb / S_STG) & 1) ^ 1, abort_flag, a.err)) break;
                    uint8_t *st = stages + s * S_STAGE;
                    as::mbar_expect_tx(&full[s], (uint32_t)(ntile * S_TILE * 32 + NHP * 128));
                    for (int p = 0; p < ntile; ++p)
                        as::tma_load_2d(st + p * S_TILE * 32, &maps.codes, 32 * kb, (int)(rbase + p0 + p * S_TILE),
                                        &full[s]);
                    as::tma_load_2d(st + S_CODE, &maps.q, S_KB * kb, m * a.nh, &full[s]);
                }
            }
        } else if (warp <= 2) {
            // MMA issuers: warp 1 + p drives tile p (one accumulator each), so the
            // two tiles' MMA streams issue concurrently
            // (the A barrier also covers the stage's TMA: the decoders waited for it before arriving)
            const int p = warp - 1;
            if (lane == 0 && p < ntile) {
                constexpr uint32_t ID = tc::idesc_f16(0, 128, NHP);
                int s = 0, b = 0;
                uint32_t bph = 0;
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!as::mbar_wait(&afull[2 * b + p], bph, abort_flag, a.err)) break;
                    tc::fence_after();
                    const uint64_t qd = tc::sdesc_k(stages + s * S_STAGE + S_CODE);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        tc::mma_ts(tbase + acc_col + p * 32, tbase + a_col + (2 * b + p) * 32 + 8 * k,
                                   qd + (uint64_t)(2 * k), ID, (kb | k) != 0);
                    tc::commit(&empty[s]);          // q~ of stage s read
                    tc::commit(&aempty[2 * b + p]);  // A of tile p in buffer b read
                    if (++s == S_STG) s = 0;
                    if (++b == S_AB) {
                        b = 0;
                        bph ^= 1;
                    }
                }
                tc::commit(&accfull[p]);
            }
        } else {
            // decoders: warp w handles tile (w - 3) / 4, TMEM lanes 32 (w % 4) .. +31:
            // each thread turns its row's 32 code bytes of the K block into 32 columns
            const int p = (warp - 3) >> 2, quad = warp & 3, r = quad * 32 + lane;
            const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
            const uint32_t lutl = as::sa(lut) + 4 * lane;
            const uint32_t m128 = maps.mul128;
            bool ok = true;
            if (p < ntile) {
                // rows arrive in the 32-byte swizzle: 16-byte half h of row r sits at
                // r * 32 + 16 (h ^ (r / 4 % 2)), so 8 lanes' 16-byte loads cover all banks
                const uint8_t *row0 = stages + p * S_TILE * 32 + r * 32;
                const int hsw = (r >> 2) & 1;
                int s = 0, b = 0;
                uint32_t sph = 0, bph = 0;
                for (int kb = 0; kb < nkb; ++kb) {
                    ok = wait_all(&full[s], sph, abort_flag, a.err) &&
                         wait_all(&aempty[2 * b + p], bph ^ 1, abort_flag, a.err);
                    if (!ok) break;
                    tc::fence_after();
                    const uint8_t *row = row0 + s * S_STAGE;
                    const uint32_t taddr = tbase + lane_off + a_col + (2 * b + p) * 32;
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const uint4 c0 = *reinterpret_cast<const uint4 *>(row + 16 * (hf ^ hsw));
                        uint32_t v[16];
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            v[k] = lk(lutl, c0.x, k, m128);
                            v[4 + k] = lk(lutl, c0.y, k, m128);
                            v[8 + k] = lk(lutl, c0.z, k, m128);
                            v[12 + k] = lk(lutl, c0.w, k, m128);
                        }
                        tc::st16(taddr + 16 * hf, v);
                    }
                    tc::st_wait();
                    tc::fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        as::mbar_arrive(&afull[2 * b + p]);
                        as::mbar_arrive(&empty[s]);
                    }
                    if (++s == S_STG) {
                        s = 0;
                        sph ^= 1;
                    }
                    if (++b == S_AB) {
                        b = 0;
                        bph ^= 1;
                    }
                }
                // epilogue: scaled scores of this lane's position into the transpose buffer
                if (ok) ok = wait_all(&accfull[p], 0, abort_flag, a.err);
                tc::fence_after();
                if (ok) {  // the heads of this lane's position
                    float v[NHP];
                    if constexpr (NHP == 32) {
                        tc::ld32f(tbase + lane_off + acc_col + p * 32, v);
                    } else {
                        tc::ld16f(tbase + lane_off + acc_col + p * 32, v);
                    }
                    const int pos = p0 + p * S_TILE + r;
                    const bool valid = pos < tn;
                    const float kn = valid ? __ldg(a.knorm + rbase + pos) * a.scale : 0.0f;
                    float *col = sT + (p * NHP) * 4 * S_CH + (r >> 5) * S_CH + (r & 31);
#pragma unroll
                    for (int h = 0; h < NHP; ++h) col[h * 4 * S_CH] = valid ? v[h] * kn : -INFINITY;
                }
            }
            bar_named(1, 256);
            ok = ok && !*abort_flag;  // every decoder warp skips the chunks once any wait gave up
            // per (tile, head, 32-position chunk): max, sum of exp, e = exp(s - max) * norm_v (f16)
            const int t = threadIdx.x - 96;  // 0 .. 255 >= 2 tiles x NHP heads x 4 chunks
            const int pt = t / (NHP * 4), h = (t / 4) % NHP, c = t & 3;
            if (ok && pt < ntile && h < a.nh) {
                const int q0 = p0 + pt * S_TILE + c * 32;
                const float *row = sT + (pt * NHP + h) * 4 * S_CH + c * S_CH;
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < 32; ++i) mx = fmaxf(mx, row[i]);
                float sum = 0.0f;
                uint4 *dst = reinterpret_cast<uint4 *>(a.E + ((int64_t)m * a.nh + h) * a.Sp + q0);
#pragma unroll
                for (int j = 0; j < 4; ++j) {  // 8 positions -> one 16-byte store
                    uint32_t pk[4];
#pragma unroll
                    for (int i = 8 * j; i < 8 * j + 8; i += 2) {
                        const float s0 = row[i], s1 = row[i + 1];
                        const float e0 = s0 == -INFINITY ? 0.0f : __expf(s0 - mx);
                        const float e1 = s1 == -INFINITY ? 0.0f : __expf(s1 - mx);
                        sum += e0;
                        sum += e1;
                        const float vn0 = e0 != 0.0f && q0 + i < tn ? __ldg(a.vnorm + rbase + q0 + i) : 0.0f;
                        const float vn1 = e1 != 0.0f && q0 + i + 1 < tn ? __ldg(a.vnorm + rbase + q0 + i + 1) : 0.0f;
                        pk[(i >> 1) & 3] = h2u(e0 * vn0, e1 * vn1);
                    }
                    dst[j] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
                const int64_t ci = ((int64_t)m * a.nc32 + (q0 >> 5)) * a.nh + h;
                a.cmax[ci] = mx;
                a.csum[ci] = sum;
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::dealloc(tbase, S_TCOLS);
    }
}

// ---------------------------------------------------------------------------
// per (head, token): global max, denominator, e rescaled in place
__global__ void __launch_bounds__(128) tc_softmax_kernel(const TqAttnArgs a) {
    pdl_wait();
    __shared__ float red[128];
    __shared__ float fac[6144 / 32];
    const int h = blockIdx.x, m = blockIdx.y, tid = threadIdx.x;
    const int tn = a.pos[m] + 1, nc = (tn + 31) >> 5;
    const float *cm = a.cmax + (int64_t)m * a.nc32 * a.nh + h;
    const float *cs = a.csum + (int64_t)m * a.nc32 * a.nh + h;
    float mx = -INFINITY;
    for (int c = tid; c < nc; c += 128) mx = fmaxf(mx, cm[(int64_t)c * a.nh]);
    red[tid] = mx;
    __syncthreads();
    for (int w = 64; w > 0; w >>= 1) {
        if (tid < w) red[tid] = fmaxf(red[tid], red[tid + w]);
        __syncthreads();
    }
    const float M = red[0];
    __syncthreads();
    float l = 0.0f;
    for (int c = tid; c < nc; c += 128) {
        const float cmv = cm[(int64_t)c * a.nh];
        const float f = cmv == -INFINITY ? 0.0f : __expf(cmv - M);
        fac[c] = f;
        l += cs[(int64_t)c * a.nh] * f;
    }
    red[tid] = l;
    __syncthreads();
    for (int w = 64; w > 0; w >>= 1) {
        if (tid < w) red[tid] += red[tid + w];
        __syncthreads();
    }
    if (tid == 0) a.linv[(int64_t)m * a.nh + h] = 1.0f / red[0];
    __half2 *e = reinterpret_cast<__half2 *>(a.E + ((int64_t)m * a.nh + h) * a.Sp);
    for (int i = tid; i < nc * 16; i += 128) {
        const float f = fac[i >> 4];
        const float2 x = __half22float2(e[i]);
        e[i] = __floats2half2_rn(x.x * f, x.y * f);
    }
}

// ---------------------------------------------------------------------------
// One code byte column over four consecutive positions (byte k of w =
// position k) into a 16x256b tensor-memory store: its low nibbles go to lane
// t/4 of the block and its high nibbles to lane t/4 + 8, two positions per
// column. x * 4097 = x + (x << 12) (no overlapping bits) puts (nibble of
// position 2c + 1) | (nibble of position 2c) << 4 in byte 2c + 1 (c = 0, 1):
// indices into the half-swapped byte -> f16 pair table, whose entry is
// (centroid of position 2c, centroid of position 2c + 1).
__device__ __forceinline__ void decode_column(uint32_t w, uint32_t lutl, uint32_t taddr, uint32_t m128, uint32_t m4097) {
    const uint32_t il = (w & 0x0F0F0F0Fu) * m4097, ih = ((w >> 4) & 0x0F0F0F0Fu) * m4097;
    tc::st16x256(taddr, lk(lutl, il, 1, m128), lk(lutl, il, 3, m128), lk(lutl, ih, 1, m128), lk(lutl, ih, 3, m128));
}

template <int NHP>
__global__ void __launch_bounds__(TCW, 2) tc_values_kernel(const __grid_constant__ ValueMaps maps, const TqAttnArgs a) {
    extern __shared__ __align__(1024) uint8_t dsm_raw[];
    uint8_t *dsm = dsm_raw + ((1024u - (as::sa(dsm_raw) & 1023u)) & 1023u);
    uint8_t *stages = dsm;
    uint32_t *lut = reinterpret_cast<uint32_t *>(dsm + V_STG * V_STAGE);
    uint64_t *full = reinterpret_cast<uint64_t *>(lut + LUTW);
    uint64_t *empty = full + V_STG;
    uint64_t *afull = empty + V_STG;      // [V_AB][2 halves of the K block]
    uint64_t *aempty = afull + 2 * V_AB;  // [V_AB][2 halves]
    uint64_t *accfull = aempty + 2 * V_AB;  // [2 halves]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(accfull + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    lut_build<true>(lut, a.vcent);
    if (threadIdx.x == 0) {
        for (int s = 0; s < V_STG; ++s) {
            as::mbar_init(&full[s], 1);
            as::mbar_init(&empty[s], 10);  // 8 decoder warps (codes read) + the two MMA commits (e read)
        }
        for (int i = 0; i < 2 * V_AB; ++i) {
            as::mbar_init(&afull[i], 4);
            as::mbar_init(&aempty[i], 1);
        }
        as::mbar_init(&accfull[0], 1);
        as::mbar_init(&accfull[1], 1);
        *abort_flag = 0;
        as::mbar_fence_init();
    }
    if (warp == 0) tc::alloc(tslot, V_TCOLS);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tbase = *tslot;
    pdl_wait();

    const int g = blockIdx.x, m = blockIdx.y;
    const int tn = a.pos[m] + 1;
    const int nkb = (tn + V_KB - 1) / V_KB;
    const int64_t rbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    // accumulator of half hh at columns 32 hh; A buffer b at 64 + 64 b (K-steps 0..7, 8 columns each)
    constexpr uint32_t a_col = 64;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % V_STG;
                if (!as::mbar_wait(&empty[s], ((kb / V_STG) & 1) ^ 1, abort_flag, a.err)) break;
                uint8_t *st = stages + s * V_STAGE;
                as::mbar_expect_tx(&full[s], (uint32_t)(V_CODE + 2 * NHP * 128));
                as::tma_load_2d(st, &maps.codes, g * (V_DG / 2), (int)(rbase + kb * V_KB), &full[s]);
                as::tma_load_2d(st + V_CODE, &maps.e, kb * V_KB, m * a.nh, &full[s]);
                as::tma_load_2d(st + V_CODE + NHP * 128, &maps.e, kb * V_KB + 64, m * a.nh, &full[s]);
            }
        }
    } else if (warp <= 2) {
        // MMA issuers: warp 1 + hh takes positions 64 hh .. 64 hh + 63 of every
        // K block (K-steps 4 hh .. +3, e atom hh) into its own accumulator, so the
        // two halves' MMA streams issue concurrently; the epilogue adds them
        // (the A barrier also covers the stage's TMA: the decoders waited for it before arriving)
        const int hh = warp - 1;
        if (lane == 0) {
            constexpr uint32_t ID = tc::idesc_f16(0, 128, NHP);
            int s = 0, b = 0;
            uint32_t bph = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                if (!as::mbar_wait(&afull[2 * b + hh], bph, abort_flag, a.err)) break;
                tc::fence_after();
                const uint64_t ed = tc::sdesc_k(stages + s * V_STAGE + V_CODE + hh * NHP * 128);
#pragma unroll
                for (int k = 0; k < 4; ++k)  // 16 positions: 32 B into the e atom
                    tc::mma_ts(tbase + 32 * hh, tbase + a_col + b * 64 + 8 * (4 * hh + k), ed + (uint64_t)(2 * k), ID,
                               (kb | k) != 0);
                tc::commit(&empty[s]);
                tc::commit(&aempty[2 * b + hh]);
                if (++s == V_STG) s = 0;
                if (++b == V_AB) {
                    b = 0;
                    bph ^= 1;
                }
            }
            tc::commit(&accfull[hh]);
        }
    } else {
        // decoders: warp w writes TMEM lanes 32 q .. +31 (q = w % 4: code bytes
        // 16 q .. 16 q + 15 of each row), K-steps 4 hh .. +3 of each block
        // (hh = (w - 3) / 4). Thread t = 4 j + i takes byte pair 16 q + 2 j,
        // 2 j + 1 of rows 16 ks + 4 i .. +3 (positions), in an order rotated by
        // i / 2 so that the four rows one load instruction touches lie in
        // distinct banks of the 64-byte swizzle; byte 2 j fills lanes j, j + 8
        // and byte 2 j + 1 lanes j + 16, j + 24 of the warp's quarter (dims
        // 4 j + 0, 1, 2, 3).
        const int q = warp & 3, hh = (warp - 3) >> 2, i = lane & 3, j = lane >> 2;
        const int rot = i >> 1;
        const uint32_t selA = rot ? 0x4206u : 0x6420u, selB = rot ? 0x5317u : 0x7531u;
        const uint32_t lutl = as::sa(lut) + 4 * lane;
        const uint32_t lane_off = (uint32_t)(32 * q) << 16;
        const uint32_t m128 = maps.mul128, m4097 = maps.mul4097;
        // byte offsets of this thread's four rows (the K-step adds 16 rows = 1024 B, a
        // whole number of swizzle periods): row 4 i + ((r + rot) & 3) of K-step 4 hh
        int off[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int R = 64 * hh + 4 * i + ((r + rot) & 3);
            off[r] = R * 64 + ((q ^ ((R >> 1) & 3)) << 4) + 2 * j;
        }
        bool ok = true;
        int s = 0, b = 0;
        uint32_t sph = 0, bph = 0;
        for (int kb = 0; kb < nkb; ++kb) {
            ok = wait_all(&full[s], sph, abort_flag, a.err) && wait_all(&aempty[2 * b + hh], bph ^ 1, abort_flag, a.err);
            if (!ok) break;
            tc::fence_after();
            const uint8_t *codes = stages + s * V_STAGE;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                uint32_t h[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) h[r] = *reinterpret_cast<const uint16_t *>(codes + off[r] + 1024 * u);
                const uint32_t x = __byte_perm(h[0], h[1], 0x5410), y = __byte_perm(h[2], h[3], 0x5410);
                const uint32_t taddr = tbase + lane_off + a_col + b * 64 + 8 * (4 * hh + u);
                decode_column(__byte_perm(x, y, selA), lutl, taddr, m128, m4097);
                decode_column(__byte_perm(x, y, selB), lutl, taddr + (16u << 16), m128, m4097);
            }
            tc::st_wait();
            tc::fence_before();
            __syncwarp();
            if (lane == 0) {
                as::mbar_arrive(&afull[2 * b + hh]);
                as::mbar_arrive(&empty[s]);
            }
            if (++s == V_STG) {
                s = 0;
                sph ^= 1;
            }
            if (++b == V_AB) {
                b = 0;
                bph ^= 1;
            }
        }
        // epilogue: warps 3..6 (one per lane quarter) add the two accumulators,
        // TMEM lanes 32 q .. +31 (dims, in the decoders' order)
        if (ok) ok = wait_all(&accfull[0], 0, abort_flag, a.err) && wait_all(&accfull[1], 0, abort_flag, a.err);
        tc::fence_after();
        if (ok && warp < 7) {
            float v[NHP], w[NHP];
            if constexpr (NHP == 32) {
                tc::ld32f(tbase + lane_off, v);
                tc::ld32f(tbase + lane_off + 32, w);
            } else {
                tc::ld16f(tbase + lane_off, v);
                tc::ld16f(tbase + lane_off + 32, w);
            }
            const int d = g * V_DG + 32 * q + 4 * (lane & 7) + 2 * (lane >> 4) + ((lane >> 3) & 1);
#pragma unroll
            for (int h = 0; h < NHP; ++h) {
                if (h < a.nh) {
                    const float u = (v[h] + w[h]) * a.linv[(int64_t)m * a.nh + h];
                    const __half hi = __float2half_rn(u);
                    const int64_t o = ((int64_t)m * a.nh + h) * a.kvd + d;
                    a.U[o] = hi;
                    a.U_lo[o] = __float2half_rn(u - __half2float(hi));
                }
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::dealloc(tbase, V_TCOLS);
    }
}

template <int NHP>
cudaError_t launch_tc(const TqAttnArgs &a, cudaStream_t s) {
    ScoreMaps sm;
    ValueMaps vm;
    std::memset(&sm, 0, sizeof(sm));
    std::memset(&vm, 0, sizeof(vm));
    sm.mul128 = vm.mul128 = 128;
    vm.mul4097 = 4097;
    const int64_t rows = (int64_t)a.n_slots * a.L * a.B;
    if (!make_tensor_map(&sm.codes, a.kcodes, rows, a.kpl, a.kpl, 1, 32, S_TILE, CU_TENSOR_MAP_SWIZZLE_32B) ||
        !make_tensor_map(&sm.q, a.qrot, (int64_t)a.M * a.nh, a.kvd, a.kvd, 2, S_KB, NHP, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tensor_map(&vm.codes, a.vcodes, rows, a.vpl, a.vpl, 1, V_DG / 2, V_KB, CU_TENSOR_MAP_SWIZZLE_64B) ||
        !make_tensor_map(&vm.e, a.E, (int64_t)a.M * a.nh, a.Sp, a.Sp, 2, 64, NHP, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const size_t ssm = 1024 + (size_t)S_STG * S_STAGE + LUTW * 4 + 256;
    const size_t vsm = 1024 + (size_t)V_STG * V_STAGE + LUTW * 4 + 256;
    cudaError_t e = dev::smem(tc_scores_kernel<NHP>, ssm);
    if (e == cudaSuccess) e = dev::smem(tc_values_kernel<NHP>, vsm);
    if (e != cudaSuccess) return e;
    e = launch_pdl(tc_scores_kernel<NHP>, dim3((a.Sp + 2 * S_TILE - 1) / (2 * S_TILE), a.M), dim3(SCW), ssm, s, sm, a);
    if (e == cudaSuccess) e = launch_pdl(tc_softmax_kernel, dim3(a.nh, a.M), dim3(128), 0, s, a);
    if (e == cudaSuccess)
        e = launch_pdl(tc_values_kernel<NHP>, dim3(a.kvd / V_DG, a.M), dim3(TCW), vsm, s, vm, a);
    return e;
}

}  // namespace

bool tc_attn_supported(const TqAttnArgs &a) {
    // from kv_dim 2048 up: below that a CTA's few K blocks do not repay its
    // set-up and the mma.sync kernels of kg_tqattn.cu are faster (measured at
    // kv_dim 768: 0.90 against 0.55 ms per 12-layer step)
    return a.kvd >= 2048 && a.kvd % V_DG == 0 && a.nh >= 1 && a.nh <= 32 && 2 * a.kpl == a.kvd && 2 * a.vpl == a.kvd &&
           a.Sp % S_TILE == 0 && a.Sp <= 6144 && a.nc32 == a.Sp / 32 && a.linv && a.n_slots > 0 &&
           tensor_map_encoder() != nullptr;
}

cudaError_t tc_decode_attn(const TqAttnArgs &a, cudaStream_t s) {
    if (a.M <= 0) return cudaSuccess;
    return a.nh <= 16 ? launch_tc<16>(a, s) : launch_tc<32>(a, s);
}

}  // namespace attn
}  // namespace kg
