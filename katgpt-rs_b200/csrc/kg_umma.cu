// kg_umma.cu — tcgen05 (5th-generation tensor core) GEMM for prefill shapes.
//
// C[M x N] = A[M x K] * B[N x K]^T with the split-operand products of
// kg_bf16.cuh (A = hi + lo activations, B = exact bf16 weights, or f16 hi + lo
// on both sides) and the same fused epilogues, for M in the thousands.
//
// Persistent, warp-specialised CTA (192 threads, one per SM):
//   warp 0      TMA producer: 128B-swizzled A / A_lo / B / B_lo tiles of
//               64 K-elements into a 3-stage shared-memory ring
//               (cp.async.bulk.tensor, completion counted on mbarriers)
//   warp 1      MMA issuer (one thread): tcgen05.mma kind::f16, M = 128,
//               N = BN, K = 16, accumulating in tensor memory; tcgen05.commit
//               releases a ring stage once the MMAs reading it are done and
//               signals a finished accumulator
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32 (w % 4) ..), fused epilogue, stores to global
// Two accumulator buffers of BN TMEM columns let the epilogue of one output
// tile overlap the main loop of the next. Every mbarrier wait is bounded by a
// clock limit; on expiry the kernel records KG_ERR_TIMEOUT in the error word,
// stops issuing work and still releases its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "kg_async.cuh"
#include "kg_bf16.cuh"
#include "kg_dev.cuh"
#include "kg_umma.cuh"

namespace kg {
namespace umma {
namespace {

constexpr int BM = 128, BK = 64, STG = 3, THREADS = 192;
constexpr int STAGE_BYTES = 64 * 1024;
using namespace as;

// shared-memory matrix descriptor: K-major, 128-byte swizzle (8-row x 128 B
// atoms, 1024 B between atoms along M/N), descriptor version 1
__device__ __forceinline__ uint64_t sdesc(const void *p) {
    return (uint64_t)((sa(p) >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// instruction descriptor, kind::f16: f32 accumulator, A and B of `fmt`
// (0 = f16, 1 = bf16), both K-major, shape 128 x BN
__host__ __device__ constexpr uint32_t idesc(int fmt, int bn) {
    return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)(bn >> 3) << 17) |
           ((uint32_t)(BM >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(sa(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T>
__device__ __forceinline__ T to_t(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 to_t<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half to_t<__half>(float v) { return __float2half_rn(v); }
template <typename T>
__device__ __forceinline__ float from_t(T v);
template <>
__device__ __forceinline__ float from_t<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float from_t<__half>(__half v) { return __half2float(v); }

struct Maps {
    CUtensorMap a, a2, b, b2;
};

// The fused epilogue of one output row's 32 columns starting at col (row < M
// and col < N checked by the caller): f32 out (row scale, residual, second
// copy) or 16-bit hi / lo out (ReLU with the alive count, row scale)
// zb: batch index (outputs at z * sC / z * sCb, residual at z * sR).
template <typename T>
__device__ __forceinline__ void epi_chunk(const bf::Gemm &g, int row, int col, float (&v)[32], float rs, int &alive,
                                          int zb = 0) {
    const bool full_row = col + 32 <= g.N;
    switch (g.epi) {
        case bf::EPI_F32:
        case bf::EPI_F32_ROWSCALE:
        case bf::EPI_F32_RESID: {
            float *dst = g.C + zb * g.sC + (int64_t)row * g.ldc + col;
            float *dst2 = g.epi == bf::EPI_F32_RESID && g.C2 ? g.C2 + zb * g.sC + (int64_t)row * g.ldc + col : nullptr;
            const float *r = g.epi == bf::EPI_F32_RESID ? g.R + zb * g.sR + (int64_t)row * g.ldr + col : nullptr;
            if (full_row) {
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    float4 o = make_float4(v[i] * rs, v[i + 1] * rs, v[i + 2] * rs, v[i + 3] * rs);
                    if (r) {
                        const float4 rr = *reinterpret_cast<const float4 *>(r + i);
                        o.x += rr.x; o.y += rr.y; o.z += rr.z; o.w += rr.w;
                    }
                    *reinterpret_cast<float4 *>(dst + i) = o;
                    if (dst2) *reinterpret_cast<float4 *>(dst2 + i) = o;
                }
            } else {
                for (int i = 0; i < 32 && col + i < g.N; ++i) {
                    dst[i] = v[i] * rs + (r ? r[i] : 0.0f);
                    if (dst2) dst2[i] = dst[i];
                }
            }
            break;
        }
        default: {  // 16-bit hi / lo outputs
            T *hi = static_cast<T *>(g.Cb) + zb * g.sCb + (int64_t)row * g.ldcb + col;
            T *lo = g.Cb2 ? static_cast<T *>(g.Cb2) + zb * g.sCb + (int64_t)row * g.ldcb + col : nullptr;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float x = v[i];
                if (g.epi == bf::EPI_RELU) {
                    alive += x > 0.0f ? 1 : 0;
                    x = x > 0.0f ? x : 0.0f;
                } else if (g.epi == bf::EPI_OUT_ROWSCALE) {
                    x *= rs;
                }
                v[i] = x;
            }
            if (full_row) {
#pragma unroll
                for (int i = 0; i < 32; i += 8) {
                    T h[8], l[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        h[e] = to_t<T>(v[i + e]);
                        l[e] = to_t<T>(v[i + e] - from_t<T>(h[e]));
                    }
                    *reinterpret_cast<uint4 *>(hi + i) = *reinterpret_cast<const uint4 *>(h);
                    if (lo) *reinterpret_cast<uint4 *>(lo + i) = *reinterpret_cast<const uint4 *>(l);
                }
            } else {
                for (int i = 0; i < 32 && col + i < g.N; ++i) {
                    const T h = to_t<T>(v[i]);
                    hi[i] = h;
                    if (lo) lo[i] = to_t<T>(v[i] - from_t<T>(h));
                }
            }
        }
    }
}


template <typename T, bool SA, bool SB, int BN>
__global__ void __launch_bounds__(THREADS, 1) umma_gemm_kernel(const __grid_constant__ Maps maps, const bf::Gemm g,
                                                              int *err) {
    extern __shared__ __align__(1024) uint8_t dsm_raw[];
    // 1024-byte alignment for the 128B-swizzled tiles (offsetting the shared
    // array keeps derived pointers in the shared address space)
    uint8_t *dsm = dsm_raw + ((1024u - (sa(dsm_raw) & 1023u)) & 1023u);
    constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
    constexpr uint32_t TX = A_BYTES * (SA ? 2 : 1) + B_BYTES * (SB ? 2 : 1);
    static_assert(TX <= STAGE_BYTES, "stage too large");
    uint64_t *full = reinterpret_cast<uint64_t *>(dsm + STG * STAGE_BYTES);
    uint64_t *empty = full + STG;
    uint64_t *tfull = empty + STG;   // [2] accumulator ready
    uint64_t *tempty = tfull + 2;    // [2] accumulator drained
    uint32_t *tslot = reinterpret_cast<uint32_t *>(tempty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (g.M + BM - 1) / BM, nt = (g.N + BN - 1) / BN, tiles = mt * nt;
    const int kb_n = g.K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STG; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);  // one arrival per epilogue warp
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {  // 2 x BN accumulator columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(sa(tslot)),
                     "r"(2 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            int it = 0;
            for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x) {
                const int m0 = (t / nt) * BM, n0 = (t % nt) * BN;
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s = it % STG;
                    if (!mbar_wait(&empty[s], ((it / STG) & 1) ^ 1, abort_flag, err)) break;
                    uint8_t *st = dsm + s * STAGE_BYTES;
                    mbar_expect_tx(&full[s], TX);
                    tma_load_2d(st, &maps.a, kb * BK, m0, &full[s]);
                    if (SA) tma_load_2d(st + A_BYTES, &maps.a2, kb * BK, m0, &full[s]);
                    uint8_t *sb = st + A_BYTES * (SA ? 2 : 1);
                    tma_load_2d(sb, &maps.b, kb * BK, n0, &full[s]);
                    if (SB) tma_load_2d(sb + B_BYTES, &maps.b2, kb * BK, n0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t ID = idesc(std::is_same<T, __half>::value ? 0 : 1, BN);
            int it = 0, tl = 0;
            for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++tl) {
                const int buf = tl & 1;
                if (!mbar_wait(&tempty[buf], ((tl >> 1) & 1) ^ 1, abort_flag, err)) break;
                tc_fence_after();
                const uint32_t d = tbase + buf * BN;
                bool ok = true;
                for (int kb = 0; kb < kb_n; ++kb, ++it) {
                    const int s = it % STG;
                    if (!mbar_wait(&full[s], (it / STG) & 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint8_t *st = dsm + s * STAGE_BYTES;
                    const uint64_t da = sdesc(st), db = sdesc(st + A_BYTES * (SA ? 2 : 1));
                    const uint64_t da2 = sdesc(st + A_BYTES), db2 = sdesc(st + A_BYTES * (SA ? 2 : 1) + B_BYTES);
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint64_t ko = (uint64_t)(k * 32 >> 4);  // 32 bytes per K step, in 16-byte units
                        umma(d, da + ko, db + ko, ID, (kb | k) != 0);
                        if (SA) umma(d, da2 + ko, db + ko, ID, 1);
                        if (SB) umma(d, da + ko, db2 + ko, ID, 1);
                    }
                    umma_commit(&empty[s]);  // the stage is free once these MMAs are done
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        // epilogue: warp w owns TMEM lanes 32 * (w % 4) .. +31 = tile rows
        const int q = warp & 3;
        int tl = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tl) {
            const int buf = tl & 1;
            if (!mbar_wait(&tfull[buf], (tl >> 1) & 1, abort_flag, err)) break;
            tc_fence_after();
            const int m0 = (t / nt) * BM, n0 = (t % nt) * BN;
            const int row = m0 + q * 32 + lane;
            const bool rok = row < g.M;
            float rs = 1.0f;
            if (rok && (g.epi == bf::EPI_F32_ROWSCALE || g.epi == bf::EPI_OUT_ROWSCALE)) rs = g.row_scale[row];
            int alive = 0;
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float v[32];
                tmem_ld32(tbase + buf * BN + c0 + ((uint32_t)(q * 32) << 16), v);
                const int col = n0 + c0;
                if (!rok || col >= g.N) continue;
                epi_chunk<T>(g, row, col, v, rs, alive);
            }
            if (g.epi == bf::EPI_RELU && rok && alive) atomicAdd(&g.row_alive[row], alive);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(2 * BN));
    }
}

// ---------------------------------------------------------------------------
// Decode-sized GEMMs (M <= 512 rows): the same operands and epilogues, built
// for few output tiles. One thread issues at most one tcgen05.mma per ~50-90 ns
// (measured on B200), so at these shapes the issue rate, not the tensor pipe,
// bounds a single-issuer CTA: two MMA warps each compute one half of the
// tile's columns over every K block (both consume every stage of the ring in
// order, so their barrier waits never run ahead of a phase), tiles are 256
// columns wide when B has no lo half, and the K range is split across CTAs
// (ks parts, a power of two dividing the K blocks) when the tiles alone leave
// SMs idle; split
// parts write f32 partials that splitk_reduce_kernel sums in part order
// before the fused epilogue (deterministic). Batched calls (the per-head
// rotations of the decode attention) are tiles of the same 2-D matrices at
// per-batch row or column offsets (b * sA, b * sB within the maps, b * sC /
// sCb at the output).
// Warps: 0 TMA producer, 1..2 MMA issuers, 3..6 epilogue.
constexpr int DTHREADS = 224;
constexpr int DPF = STG + 3;  // L2 prefetch distance of the weight tiles, in K blocks

template <typename T, bool SA, bool SB, int BN>
__global__ void __launch_bounds__(DTHREADS, 1) umma_dec_kernel(const __grid_constant__ Maps maps, const bf::Gemm g,
                                                              int ks, float *ws, int *err) {
    extern __shared__ __align__(1024) uint8_t dsm_raw[];
    uint8_t *dsm = dsm_raw + ((1024u - (sa(dsm_raw) & 1023u)) & 1023u);
    constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
    constexpr uint32_t TX = A_BYTES * (SA ? 2 : 1) + B_BYTES * (SB ? 2 : 1);
    static_assert(TX <= STAGE_BYTES, "stage too large");
    uint64_t *full = reinterpret_cast<uint64_t *>(dsm + STG * STAGE_BYTES);
    uint64_t *empty = full + STG;   // one commit per issuer
    uint64_t *tfull = empty + STG;  // [2] accumulator ready (one commit per issuer)
    uint64_t *tempty = tfull + 2;   // [2] accumulator drained (one arrival per epilogue warp)
    uint32_t *tslot = reinterpret_cast<uint32_t *>(tempty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nt = (g.N + BN - 1) / BN, mt = (g.M + BM - 1) / BM, tiles = g.batch * mt * nt * ks;
    const int kbs = (g.K / BK) / ks;  // K blocks per part
    // tile t -> (batch zb, row tile, column tile, K part): part fastest
    auto decode_tile = [&](int t, int &zb, int &part, int &m0, int &n0) {
        part = t % ks;
        const int r1 = t / ks;
        n0 = (r1 % nt) * BN;
        const int r2 = r1 / nt;
        m0 = (r2 % mt) * BM;
        zb = r2 / mt;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STG; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 2);
            mbar_init(&tempty[b], 4);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {  // two BN-column accumulator buffers (issuer i writes columns i BN/2 .. of each)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(sa(tslot)),
                     "r"(2 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tslot;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer: the tile's K part, block by block
            int it = 0;
            for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x) {
                int zb, part, m0, n0;
                decode_tile(t, zb, part, m0, n0);
                // batch offsets inside the 2-D maps: whole rows or a column shift
                const int64_t ao = zb * g.sA, bo = zb * g.sB;
                const int ay = m0 + (int)(ao / g.lda), ax = (int)(ao % g.lda);
                const int by = n0 + (int)(bo / g.ldb), bx = (int)(bo % g.ldb);
                for (int j = 0; j < kbs; ++j, ++it) {
                    const int s = it % STG, kb = part * kbs + j;
                    // weight tiles DPF blocks ahead into L2 (the ring holds STG of them)
                    for (int pj = (j == 0 ? STG : DPF); pj <= DPF; ++pj)
                        if (j + pj < kbs) {
                            tma_prefetch_2d(&maps.b, bx + (kb + pj) * BK, by);
                            if (SB) tma_prefetch_2d(&maps.b2, bx + (kb + pj) * BK, by);
                        }
                    if (!mbar_wait(&empty[s], ((it / STG) & 1) ^ 1, abort_flag, err)) break;
                    uint8_t *st = dsm + s * STAGE_BYTES;
                    mbar_expect_tx(&full[s], TX);
                    tma_load_2d(st, &maps.a, ax + kb * BK, ay, &full[s]);
                    if (SA) tma_load_2d(st + A_BYTES, &maps.a2, ax + kb * BK, ay, &full[s]);
                    uint8_t *sb = st + A_BYTES * (SA ? 2 : 1);
                    tma_load_2d(sb, &maps.b, bx + kb * BK, by, &full[s]);
                    if (SB) tma_load_2d(sb + B_BYTES, &maps.b2, bx + kb * BK, by, &full[s]);
                }
            }
        }
    } else if (warp <= 2) {
        if (lane == 0) {  // MMA issuer i: columns i BN/2 .. (i + 1) BN/2 of the tile, every K block
            const int i = warp - 1;
            constexpr int HN = BN / 2;
            constexpr uint32_t ID = idesc(std::is_same<T, __half>::value ? 0 : 1, HN);
            // the B tile's rows HN i .. (K-major, 128-byte rows; 8-row atoms of 1024 B)
            const uint64_t bofs = (uint64_t)(i * HN * 128 >> 4);
            int it = 0, tl = 0;
            for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++tl) {
                const int buf = tl & 1;
                if (!mbar_wait(&tempty[buf], ((tl >> 1) & 1) ^ 1, abort_flag, err)) break;
                tc_fence_after();
                const uint32_t d = tbase + buf * BN + i * HN;
                bool ok = true;
                for (int j = 0; j < kbs; ++j, ++it) {
                    const int s = it % STG;
                    if (!mbar_wait(&full[s], (it / STG) & 1, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint8_t *st = dsm + s * STAGE_BYTES;
                    const uint64_t da = sdesc(st), db = sdesc(st + A_BYTES * (SA ? 2 : 1)) + bofs;
                    const uint64_t da2 = sdesc(st + A_BYTES), db2 = sdesc(st + A_BYTES * (SA ? 2 : 1) + B_BYTES) + bofs;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint64_t ko = (uint64_t)(k * 32 >> 4);
                        umma(d, da + ko, db + ko, ID, (j | k) != 0);
                        if (SA) umma(d, da2 + ko, db + ko, ID, 1);
                        if (SB) umma(d, da + ko, db2 + ko, ID, 1);
                    }
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        // epilogue: warp w owns TMEM lanes 32 (w % 4) .. +31 = tile rows
        const int q = warp & 3;
        int tl = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tl) {
            const int buf = tl & 1;
            if (!mbar_wait(&tfull[buf], (tl >> 1) & 1, abort_flag, err)) break;
            tc_fence_after();
            int zb, part, m0, n0;
            decode_tile(t, zb, part, m0, n0);
            const int row = m0 + q * 32 + lane;
            const bool rok = row < g.M;
            float rs = 1.0f;
            if (ks == 1 && rok && (g.epi == bf::EPI_F32_ROWSCALE || g.epi == bf::EPI_OUT_ROWSCALE))
                rs = g.row_scale[row];
            int alive = 0;
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float v[32];
                tmem_ld32(tbase + buf * BN + c0 + ((uint32_t)(q * 32) << 16), v);
                const int col = n0 + c0;
                if (!rok || col >= g.N) continue;
                if (ks > 1) {  // f32 partial of this part: ws[batch][part][row][col]
                    float *dst = ws + (((int64_t)zb * ks + part) * g.M + row) * g.N + col;
                    if (col + 32 <= g.N) {
#pragma unroll
                        for (int e = 0; e < 32; e += 4)
                            *reinterpret_cast<float4 *>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                    } else {
                        for (int e = 0; e < 32 && col + e < g.N; ++e) dst[e] = v[e];
                    }
                } else {
                    epi_chunk<T>(g, row, col, v, rs, alive, zb);
                }
            }
            if (g.epi == bf::EPI_RELU && rok && alive) atomicAdd(&g.row_alive[row], alive);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tbase), "r"(2 * BN));
    }
}

// sum of the ks partials (part order) + the fused epilogue; one thread per
// (batch, row, 32-column chunk)
template <typename T>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const bf::Gemm g, int ks, const float *ws) {
    const int chunks = (g.N + 31) / 32;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (int64_t)g.batch * g.M * chunks) return;
    const int zb = (int)(idx / ((int64_t)g.M * chunks));
    const int64_t rc = idx - (int64_t)zb * g.M * chunks;
    const int row = (int)(rc / chunks), col = (int)(rc % chunks) * 32;
    float v[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) v[e] = 0.0f;
    const bool full_row = col + 32 <= g.N;
    for (int p = 0; p < ks; ++p) {
        const float *src = ws + (((int64_t)zb * ks + p) * g.M + row) * g.N + col;
        if (full_row) {
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
                const float4 x = *reinterpret_cast<const float4 *>(src + e);
                v[e] += x.x;
                v[e + 1] += x.y;
                v[e + 2] += x.z;
                v[e + 3] += x.w;
            }
        } else {
            for (int e = 0; e < 32 && col + e < g.N; ++e) v[e] += src[e];
        }
    }
    const float rs = (g.epi == bf::EPI_F32_ROWSCALE || g.epi == bf::EPI_OUT_ROWSCALE) ? g.row_scale[row] : 1.0f;
    int alive = 0;
    epi_chunk<T>(g, row, col, v, rs, alive, zb);
    if (g.epi == bf::EPI_RELU && alive) atomicAdd(&g.row_alive[row], alive);
}

template <typename T, bool SA, bool SB, int BN>
cudaError_t launch_bn(const bf::Gemm &g, cudaStream_t s, int *err, int nsm) {
    Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;  // 16-bit elements either way: the map only moves bytes
    if (!make_tensor_map(&maps.a, g.A, g.M, g.K, g.lda, 2, BK, BM, SW) ||
        (SA && !make_tensor_map(&maps.a2, g.A2, g.M, g.K, g.lda, 2, BK, BM, SW)) ||
        !make_tensor_map(&maps.b, g.B, g.N, g.K, g.ldb, 2, BK, BN, SW) ||
        (SB && !make_tensor_map(&maps.b2, g.B2, g.N, g.K, g.ldb, 2, BK, BN, SW)))
        return cudaErrorInvalidValue;
    const int smem = 1024 + STG * STAGE_BYTES + 256;
    {
        cudaError_t e = dev::smem(umma_gemm_kernel<T, SA, SB, BN>, smem);
        if (e != cudaSuccess) return e;
    }
    const int tiles = ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
    umma_gemm_kernel<T, SA, SB, BN><<<std::min(tiles, nsm), THREADS, smem, s>>>(maps, g, err);
    return cudaGetLastError();
}

template <typename T, bool SA, bool SB, int BN>
cudaError_t launch_dec(const bf::Gemm &g, cudaStream_t s, int *err, int nsm, int ks) {
    Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
    // batched calls: the maps cover every batch's rows / columns of the 2-D matrices
    const int64_t arows = g.M + (g.batch > 1 ? (int64_t)(g.batch - 1) * g.sA / g.lda : 0);
    const int64_t brows = g.N + (g.batch > 1 ? (int64_t)(g.batch - 1) * g.sB / g.ldb : 0);
    const int64_t acols = g.batch > 1 ? g.lda : g.K, bcols = g.batch > 1 ? g.ldb : g.K;
    if (!make_tensor_map(&maps.a, g.A, arows, acols, g.lda, 2, BK, BM, SW) ||
        (SA && !make_tensor_map(&maps.a2, g.A2, arows, acols, g.lda, 2, BK, BM, SW)) ||
        !make_tensor_map(&maps.b, g.B, brows, bcols, g.ldb, 2, BK, BN, SW) ||
        (SB && !make_tensor_map(&maps.b2, g.B2, brows, bcols, g.ldb, 2, BK, BN, SW)))
        return cudaErrorInvalidValue;
    const int smem = 1024 + STG * STAGE_BYTES + 256;
    {
        cudaError_t e = dev::smem(umma_dec_kernel<T, SA, SB, BN>, smem);
        if (e != cudaSuccess) return e;
    }
    const int tiles = g.batch * ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN) * ks;
    umma_dec_kernel<T, SA, SB, BN><<<std::min(tiles, nsm), DTHREADS, smem, s>>>(maps, g, ks, g.ws, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || ks == 1) return e;
    const int64_t work = (int64_t)g.batch * g.M * ((g.N + 31) / 32);
    splitk_reduce_kernel<T><<<(unsigned)((work + 255) / 256), 256, 0, s>>>(g, ks, g.ws);
    return cudaGetLastError();
}

// Tile width: 256 (128 with split B), 128 or 64 columns. Up to 2048 rows (a
// 512-sequence decode step) the widest that still gives every SM a tile;
// above, 128 when it raises the share of busy SMs over the launch's waves by
// at least 10 points (a pass whose last wave would be mostly empty).
template <typename T, bool SA, bool SB>
cudaError_t launch(const bf::Gemm &g, cudaStream_t s, int *err) {
    const int nsm = dev::sm_count();
    const int mt = (g.M + BM - 1) / BM;
    if (g.M <= 512 && g.K / BK >= 2) {  // decode-sized: two issuers, wide tiles, split K
        constexpr int DBN = SB ? 128 : 256;
        const int kb_n = g.K / BK, tiles = g.batch * mt * ((g.N + DBN - 1) / DBN);
        int ks = 1;
        while (tiles * ks * 2 <= nsm && kb_n % (ks * 2) == 0 && kb_n / (ks * 2) >= 4 && g.ws &&
               (int64_t)ks * 2 * g.batch * g.M * g.N * 4 <= g.ws_bytes)
            ks *= 2;
        return launch_dec<T, SA, SB, DBN>(g, s, err, nsm, ks);
    }
    auto busy = [&](int bn) {
        const int t = mt * ((g.N + bn - 1) / bn);
        return (double)t / ((double)((t + nsm - 1) / nsm) * nsm);
    };
    int bn = SB ? 128 : 256;
    if (g.M <= 2048) {  // few rows: the widest tile that still gives every SM a tile
        auto tiles = [&](int w) { return mt * ((g.N + w - 1) / w); };
        if (tiles(bn) < nsm) bn = 128;
        if (tiles(bn) < nsm) bn = 64;
    } else if (!SB && busy(128) >= busy(256) + 0.10) {  // many rows: a small last wave
        bn = 128;
    }
    if constexpr (!SB) {
        if (bn == 256) return launch_bn<T, SA, SB, 256>(g, s, err, nsm);
    }
    if (bn == 128) return launch_bn<T, SA, SB, 128>(g, s, err, nsm);
    return launch_bn<T, SA, SB, 64>(g, s, err, nsm);
}

}  // namespace

bool supported(const bf::Gemm &g) {
    // K in whole 64-element blocks, 16-byte aligned rows and bases, and the
    // hi-only B form only for bf16 weights; batches only in the decode-sized
    // GEMM (M <= 512, at least 2 K blocks), as whole-row or in-row column
    // shifts (16-byte aligned) of the 2-D operands
    if (g.batch < 1 || g.K % BK || g.lda % 8 || g.ldb % 8) return false;
    if (g.batch > 1) {
        if (g.M > 512 || g.K / BK < 2) return false;
        auto shift_ok = [&](int64_t s, int64_t ld) {
            return s >= 0 && (s % ld == 0 || ((int64_t)(g.batch - 1) * s + g.K <= ld && s % 8 == 0));
        };
        if (!shift_ok(g.sA, g.lda) || !shift_ok(g.sB, g.ldb)) return false;
        const bool f32_out = g.epi == bf::EPI_F32 || g.epi == bf::EPI_F32_RESID || g.epi == bf::EPI_F32_ROWSCALE;
        if (f32_out ? (g.sC % 4 != 0 || g.sR % 4 != 0) : (g.sCb % 8 != 0)) return false;
        if (g.epi == bf::EPI_RELU || g.epi == bf::EPI_F32_ROWSCALE || g.epi == bf::EPI_OUT_ROWSCALE) return false;
    }
    if (g.Qh || g.Dacc || g.epi == bf::EPI_BF16_SPLIT) return false;  // fused extras: mma.sync epilogue only
    if ((reinterpret_cast<uintptr_t>(g.A) | reinterpret_cast<uintptr_t>(g.B)) & 15) return false;
    if (g.A2 && (reinterpret_cast<uintptr_t>(g.A2) & 15)) return false;
    if (g.B2 && (reinterpret_cast<uintptr_t>(g.B2) & 15)) return false;
    if (g.epi == bf::EPI_F32 || g.epi == bf::EPI_F32_RESID || g.epi == bf::EPI_F32_ROWSCALE) {
        if (g.ldc % 4 || (g.epi == bf::EPI_F32_RESID && g.ldr % 4)) return false;
        if (reinterpret_cast<uintptr_t>(g.C) & 15) return false;
    } else if (g.ldcb % 8 || (reinterpret_cast<uintptr_t>(g.Cb) & 15)) {
        return false;
    }
    return tensor_map_encoder() != nullptr;
}

cudaError_t gemm(const bf::Gemm &g, cudaStream_t s, int *err) {
    if (g.M <= 0 || g.N <= 0) return cudaSuccess;
    const bool sa = g.A2 != nullptr, sb = g.B2 != nullptr;
    if (g.dtype == bf::DT_BF16) {
        if (sb) return cudaErrorInvalidValue;
        return sa ? launch<__nv_bfloat16, true, false>(g, s, err) : launch<__nv_bfloat16, false, false>(g, s, err);
    }
    if (sa && sb) return launch<__half, true, true>(g, s, err);
    if (sa) return launch<__half, true, false>(g, s, err);
    if (sb) return launch<__half, false, true>(g, s, err);
    return launch<__half, false, false>(g, s, err);
}

}  // namespace umma

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool make_tensor_map(CUtensorMap *m, const void *base, int64_t rows, int64_t cols, int64_t ld, int elem,
                     int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
    auto fn = tensor_map_encoder();
    if (!fn || !base) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(ld * elem)};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUtensorMapDataType dt = elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
    return fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace kg
