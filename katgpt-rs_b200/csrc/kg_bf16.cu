// kg_bf16.cu — BF16 tensor-core GEMM and the small per-token kernels of the
// large-model path (embedding, RMSNorm, delta routing, TwELL sparse W2,
// temperature softmax).
//
// The GEMM is C = A * B^T with A [M x K] activations and B [N x K] weights,
// both K-contiguous (the reference's row-major [out, in] weight layout), f32
// accumulation and fused epilogues (residual add, ReLU + alive count, row
// scale). Tiles of 128 x 128 x 32 go through a 4-stage cp.async pipeline into
// XOR-swizzled shared memory and feed mma.sync m16n8k16 via ldmatrix.
#include <algorithm>

#include <cooperative_groups.h>

#include "kg_bf16.cuh"
#include "kg_dev.cuh"
#include "kg_pdl.cuh"

namespace kg {
namespace bf {
namespace {

namespace cg = cooperative_groups;

constexpr int BK = 32, STAGES = 4;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool pred) {
    int sz = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(sz));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<bf16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <typename T>
__device__ __forceinline__ T to_t(float v);
template <>
__device__ __forceinline__ bf16 to_t<bf16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half to_t<__half>(float v) { return __float2half_rn(v); }
template <typename T>
__device__ __forceinline__ float from_t(T v);
template <>
__device__ __forceinline__ float from_t<bf16>(bf16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float from_t<__half>(__half v) { return __half2float(v); }

// 16-byte chunk (row, c) of a [rows x 32] 16-bit tile: 4 chunks per row,
// swizzled so the 8 rows an ldmatrix reads fall in distinct banks.
__device__ __forceinline__ int swz(int row, int c) { return row * 4 + (c ^ ((row >> 1) & 3)); }

// one output element through the epilogue; returns 1 when a ReLU output is alive
template <typename T>
__device__ __forceinline__ int epi_store(const Gemm &g, int z, int row, int cc, float v, float rs) {
    switch (g.epi) {
        case EPI_F32: {
            g.C[z * g.sC + (int64_t)row * g.ldc + cc] = v;
            if (g.Qh && cc < g.qcols) {
                const __half h = __float2half_rn(v);
                g.Qh[(int64_t)row * g.ldq + cc] = h;
                g.Ql[(int64_t)row * g.ldq + cc] = __float2half_rn(v - __half2float(h));
            }
            return 0;
        }
        case EPI_F32_RESID: {
            const int64_t i = z * g.sC + (int64_t)row * g.ldc + cc;
            const float o = v + g.R[z * g.sR + (int64_t)row * g.ldr + cc];
            g.C[i] = o;
            if (g.C2) g.C2[i] = o;
            if (g.Dacc) g.Dacc[i] += o - g.R3[i];
            return 0;
        }
        case EPI_BF16_SPLIT: {
            const int64_t ob = z * g.sCb + (int64_t)row * g.ldcb + cc;
            const bf16 hi = __float2bfloat16_rn(v);
            static_cast<bf16 *>(g.Cb)[ob] = hi;
            if (g.Cb2) static_cast<bf16 *>(g.Cb2)[ob] = __float2bfloat16_rn(v - __bfloat162float(hi));
            return 0;
        }
        case EPI_F32_ROWSCALE: g.C[z * g.sC + (int64_t)row * g.ldc + cc] = v * rs; return 0;
        default: {
            int alive = 0;
            if (g.epi == EPI_RELU) {
                alive = v > 0.0f ? 1 : 0;
                v = v > 0.0f ? v : 0.0f;
            } else if (g.epi == EPI_OUT_ROWSCALE) {
                v = v * rs;
            }
            const int64_t ob = z * g.sCb + (int64_t)row * g.ldcb + cc;
            const T hi = to_t<T>(v);
            static_cast<T *>(g.Cb)[ob] = hi;
            if (g.Cb2) static_cast<T *>(g.Cb2)[ob] = to_t<T>(v - from_t<T>(hi));
            return alive;
        }
    }
}

// Tile shapes: 128 x 128 with 2 x 4 warps (warp tile 64 x 32) for prefill
// shapes, 64 x 64 with 2 x 2 warps (warp tile 32 x 32) for decode shapes
// (few rows: more tiles in flight over the weight stream).
template <int BM_, int BN_, int WM_, int WN_>
struct Tile {
    static constexpr int BM = BM_, BN = BN_, WM = WM_, WN = WN_, THREADS = 32 * WM_ * WN_;
    static constexpr int MI = BM_ / WM_ / 16, NJ = BN_ / WN_ / 8;
};
using TileL = Tile<128, 128, 2, 4>;
using TileS = Tile<64, 64, 2, 2>;

template <typename CF, bool SA, bool SB>
constexpr int gemm_smem() {
    return std::max(STAGES * (CF::BM * (SA ? 2 : 1) + CF::BN * (SB ? 2 : 1)) * BK * 2, CF::BM * (CF::BN + 4) * 4);
}

template <typename CF, typename T, bool SA, bool SB>
__global__ void __launch_bounds__(CF::THREADS) gemm_kernel(const Gemm g) {
    pdl_wait();
    constexpr int BM_ = CF::BM, BN_ = CF::BN, NT_ = CF::THREADS, MI = CF::MI, NJ = CF::NJ;
    extern __shared__ uint4 sm[];
    constexpr int TA = BM_ * 4, TB = BN_ * 4;  // 16-byte chunks per tile
    constexpr int PER_STAGE = TA * (SA ? 2 : 1) + TB * (SB ? 2 : 1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp / CF::WN, wn = warp % CF::WN;
    const int bm = blockIdx.y * BM_, bn = blockIdx.x * BN_;
    const int ks = blockIdx.z % g.ksplit, z = blockIdx.z / g.ksplit;
    const T *A = static_cast<const T *>(g.A) + z * g.sA;
    const T *A2 = SA ? static_cast<const T *>(g.A2) + z * g.sA : nullptr;
    const T *B = static_cast<const T *>(g.B) + z * g.sB;
    const T *B2 = SB ? static_cast<const T *>(g.B2) + z * g.sB : nullptr;
    const int KT_all = g.K / BK;
    const int kt_per = (KT_all + g.ksplit - 1) / g.ksplit;
    const int kt0 = ks * kt_per;
    const int KT = max(0, min(KT_all, kt0 + kt_per) - kt0);

    auto tileA = [&](int st, int part) { return sm + st * PER_STAGE + part * TA; };
    auto tileB = [&](int st, int part) { return sm + st * PER_STAGE + TA * (SA ? 2 : 1) + part * TB; };

    auto load = [&](int stage, int kt) {
        const int k0 = (kt0 + kt) * BK;
#pragma unroll
        for (int idx = tid; idx < TA; idx += NT_) {
            const int row = idx >> 2, c = idx & 3, gr = bm + row;
            const int64_t ao = (int64_t)min(gr, g.M - 1) * g.lda + k0 + c * 8;
            cp_async16(smem_u32(tileA(stage, 0) + swz(row, c)), A + ao, gr < g.M);
            if (SA) cp_async16(smem_u32(tileA(stage, 1) + swz(row, c)), A2 + ao, gr < g.M);
        }
#pragma unroll
        for (int idx = tid; idx < TB; idx += NT_) {
            const int row = idx >> 2, c = idx & 3, gn = bn + row;
            const int64_t bo = (int64_t)min(gn, g.N - 1) * g.ldb + k0 + c * 8;
            cp_async16(smem_u32(tileB(stage, 0) + swz(row, c)), B + bo, gn < g.N);
            if (SB) cp_async16(smem_u32(tileB(stage, 1) + swz(row, c)), B2 + bo, gn < g.N);
        }
    };

    float acc[MI][NJ][4];
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < KT) load(s, s);
        cp_commit();
    }
    for (int kt = 0; kt < KT; ++kt) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        if (kt + STAGES - 1 < KT) load((kt + STAGES - 1) % STAGES, kt + STAGES - 1);
        cp_commit();
        const int st = kt % STAGES;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {  // two k16 steps per BK = 32
            uint32_t bfr[2][NJ][2];
#pragma unroll
            for (int part = 0; part < (SB ? 2 : 1); ++part)
#pragma unroll
                for (int j2 = 0; j2 < NJ / 2; ++j2) {
                    const int row = wn * (BN_ / CF::WN) + j2 * 16 + (lane & 7) + ((lane >> 4) << 3);
                    const int c = kk * 2 + ((lane >> 3) & 1);
                    ldsm_x4(smem_u32(tileB(st, part) + swz(row, c)), bfr[part][j2 * 2][0], bfr[part][j2 * 2][1],
                            bfr[part][j2 * 2 + 1][0], bfr[part][j2 * 2 + 1][1]);
                }
            uint32_t af[2][MI][4];
#pragma unroll
            for (int part = 0; part < (SA ? 2 : 1); ++part)
#pragma unroll
                for (int i = 0; i < MI; ++i) {
                    const int row = wm * (BM_ / CF::WM) + i * 16 + (lane & 15);
                    const int c = kk * 2 + (lane >> 4);
                    ldsm_x4(smem_u32(tileA(st, part) + swz(row, c)), af[part][i][0], af[part][i][1], af[part][i][2],
                            af[part][i][3]);
                }
            // term-major order: consecutive MMAs go to different accumulators
#pragma unroll
            for (int i = 0; i < MI; ++i)
#pragma unroll
                for (int j = 0; j < NJ; ++j) mma16816<T>(acc[i][j], af[0][i], bfr[0][j][0], bfr[0][j][1]);
            if (SA) {
#pragma unroll
                for (int i = 0; i < MI; ++i)
#pragma unroll
                    for (int j = 0; j < NJ; ++j) mma16816<T>(acc[i][j], af[SA ? 1 : 0][i], bfr[0][j][0], bfr[0][j][1]);
            }
            if (SB) {
#pragma unroll
                for (int i = 0; i < MI; ++i)
#pragma unroll
                    for (int j = 0; j < NJ; ++j) mma16816<T>(acc[i][j], af[0][i], bfr[SB ? 1 : 0][j][0], bfr[SB ? 1 : 0][j][1]);
            }
        }
    }
    cp_wait<0>();
    const int g8 = lane >> 2, c4 = lane & 3;

    if (g.ksplit > 1) {
        // Split-K: the ksplit CTAs of one output tile form a thread-block
        // cluster. Each parks its partial tile in its own shared memory, then
        // each reduces a 1/ksplit slice of the tile over all peers' shared
        // memory (in split order, so results are deterministic) and runs the
        // epilogue on it.
        cg::cluster_group cluster = cg::this_cluster();
        constexpr int LDR = BN_ + 4;
        float *red = reinterpret_cast<float *>(sm);
        __syncthreads();  // every warp is done with the pipeline buffers
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
            for (int hrow = 0; hrow < 2; ++hrow)
#pragma unroll
                for (int j = 0; j < NJ; ++j) {
                    const int r = wm * (BM_ / CF::WM) + i * 16 + g8 + hrow * 8;
                    const int cl = wn * (BN_ / CF::WN) + j * 8 + c4 * 2;
                    *reinterpret_cast<float2 *>(red + r * LDR + cl) =
                        make_float2(acc[i][j][hrow * 2], acc[i][j][hrow * 2 + 1]);
                }
        cluster.sync();
        const int rank = (int)cluster.block_rank();
        const int mrows = min(BM_, g.M - bm);
        const int quads = mrows * (BN_ / 4);  // float4 groups of the valid rows
        const int per = (quads + g.ksplit - 1) / g.ksplit;
        const int q0 = rank * per, q1 = min(quads, q0 + per);
        for (int qd = q0 + tid; qd < q1; qd += NT_) {
            const int r = qd / (BN_ / 4), cl = (qd % (BN_ / 4)) * 4;
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p = 0; p < g.ksplit; ++p) {
                const float4 v = *reinterpret_cast<const float4 *>(cluster.map_shared_rank(red, p) + r * LDR + cl);
                sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
            }
            const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
            const int row = bm + r;
            float rs = 1.0f;
            if (g.epi == EPI_F32_ROWSCALE || g.epi == EPI_OUT_ROWSCALE) rs = g.row_scale[z * g.sRs + row];
            int alive = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (bn + cl + e < g.N) alive += epi_store<T>(g, z, row, bn + cl + e, vals[e], rs);
            if (g.epi == EPI_RELU) {
                // one atomic per row and warp: lanes of the same row pool their counts
                const unsigned grp = __match_any_sync(__activemask(), row);
                alive = __reduce_add_sync(grp, alive);
                if (alive && lane == __ffs(grp) - 1) atomicAdd(&g.row_alive[row], alive);
            }
        }
        cluster.sync();  // peers may still be reading this CTA's shared memory
        return;
    }

    // ---- epilogue
#pragma unroll
    for (int i = 0; i < MI; ++i) {
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow) {
            const int row = bm + wm * (BM_ / CF::WM) + i * 16 + g8 + hrow * 8;
            const bool rok = row < g.M;
            int alive = 0;
            float rs = 1.0f;
            if (rok && (g.epi == EPI_F32_ROWSCALE || g.epi == EPI_OUT_ROWSCALE)) rs = g.row_scale[z * g.sRs + row];
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const int col = bn + wn * (BN_ / CF::WN) + j * 8 + c4 * 2;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int cc = col + e;
                    if (rok && cc < g.N) alive += epi_store<T>(g, z, row, cc, acc[i][j][hrow * 2 + e], rs);
                }
            }
            if (g.epi == EPI_RELU) {
                alive += __shfl_xor_sync(0xffffffffu, alive, 1);
                alive += __shfl_xor_sync(0xffffffffu, alive, 2);
                if (rok && c4 == 0 && alive) atomicAdd(&g.row_alive[row], alive);
            }
        }
    }
}

// ---- small kernels ---------------------------------------------------------

__global__ void embed_kernel(const int32_t *tok, const int32_t *pos, const bf16 *wte, const bf16 *wpe, int n,
                             int M, float *x, float *zero_rows) {
    pdl_wait();
    const int m = blockIdx.x;
    if (m >= M) return;
    const bf16 *a = wte + (int64_t)tok[m] * n, *b = wpe + (int64_t)pos[m] * n;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        x[(int64_t)m * n + j] = __bfloat162float(a[j]) + __bfloat162float(b[j]);
        if (zero_rows) zero_rows[(int64_t)m * n + j] = 0.0f;
    }
}

__device__ __forceinline__ float block_sum(float v, float *red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
    return s;
}
__device__ __forceinline__ float block_max(float v, float *red) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float s = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s = fmaxf(s, red[i]);
    return s;
}

__device__ __forceinline__ void put_split(bf16 *yb, bf16 *yb2, int64_t i, float v) {
    const bf16 hi = __float2bfloat16_rn(v);
    if (yb) yb[i] = hi;
    if (yb2) yb2[i] = __float2bfloat16_rn(v - __bfloat162float(hi));
}

__global__ void rmsnorm_kernel(const float *x, int n, int M, float *yf, bf16 *yb, bf16 *yb2, int twice,
                               int *zero_count, const float *gamma) {
    pdl_wait();
    __shared__ float red[32];
    const int m = blockIdx.x;
    if (zero_count && threadIdx.x == 0) zero_count[m] = 0;
    const float *xr = x + (int64_t)m * n;
    float ss = 0.0f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) ss += xr[j] * xr[j];
    ss = block_sum(ss, red);
    float inv = 1.0f / sqrtf(ss / (float)n + 1e-5f);
    if (twice) {
        float ss2 = 0.0f;
        for (int j = threadIdx.x; j < n; j += blockDim.x) {
            float v = xr[j] * inv;
            ss2 += v * v;
        }
        ss2 = block_sum(ss2, red);
        float inv2 = 1.0f / sqrtf(ss2 / (float)n + 1e-5f);
        for (int j = threadIdx.x; j < n; j += blockDim.x) {
            float v = (xr[j] * inv) * inv2;
            if (yf) yf[(int64_t)m * n + j] = v;
            put_split(yb, yb2, (int64_t)m * n + j, v);
        }
        return;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        float v = xr[j] * inv;
        if (gamma) v = gamma[j] * v;
        if (yf) yf[(int64_t)m * n + j] = v;
        put_split(yb, yb2, (int64_t)m * n + j, v);
    }
}

__global__ void to_bf16_kernel(const float *x, int64_t ldx, int n, int M, bf16 *y, bf16 *y2, int64_t ldy) {
    pdl_wait();
    const int m = blockIdx.x;
    for (int j = threadIdx.x; j < n; j += blockDim.x) put_split(y, y2, (int64_t)m * ldy + j, x[(int64_t)m * ldx + j]);
}

__global__ void to_f16_kernel(const float *x, int64_t ldx, int n, __half *hi, __half *lo, int64_t ldy) {
    pdl_wait();
    const int m = blockIdx.x;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float v = x[(int64_t)m * ldx + j];
        const __half h = __float2half_rn(v);
        hi[(int64_t)m * ldy + j] = h;
        lo[(int64_t)m * ldy + j] = __float2half_rn(v - __half2float(h));
    }
}

__global__ void f16_split_kernel(const float *x, int64_t count, __half *hi, __half *lo) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        const __half h = __float2half_rn(x[i]);
        hi[i] = h;
        lo[i] = __float2half_rn(x[i] - __half2float(h));
    }
}

__global__ void flat_bf16_kernel(const float *x, int64_t count, bf16 *y) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __float2bfloat16_rn(x[i]);
}

// delta routing for one token (one block per token)
__global__ void delta_route_kernel(float *x, const float *xr, float *delta, const float *query, const float *normw,
                                   int n, int layer) {
    pdl_wait();
    __shared__ float red[32];
    const int m = blockIdx.x;
    float *xm = x + (int64_t)m * n, *dm = delta + (int64_t)m * n;
    const float *xrm = xr + (int64_t)m * n;
    for (int j = threadIdx.x; j < n; j += blockDim.x) dm[j] = dm[j] + (xm[j] - xrm[j]);
    if ((layer & 3) != 3) return;
    const int b = layer >> 2;  // sources: b zeroed blocks and the current block
    __syncthreads();
    float ss = 0.0f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) ss += dm[j] * dm[j];
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)n + 1e-5f);
    const float inv0 = 1.0f / sqrtf(1e-5f);
    float lg = 0.0f, lz = 0.0f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        lg += normw[j] * (dm[j] * inv) * query[j];
        lz += normw[j] * (0.0f * inv0) * query[j];
    }
    lg = block_sum(lg, red);
    lz = block_sum(lz, red);
    float mx = lg;
    if (b > 0) mx = fmaxf(mx, lz);
    const float eo = expf(lg - mx), ez = expf(lz - mx);
    const float w = eo / (eo + (float)b * ez);
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        xm[j] = xm[j] + w * dm[j];
        dm[j] = 0.0f;
    }
}

// TwELL sparse W2 for one token (one block per row); skips rows over threshold
__global__ void twell_kernel(const bf16 *hidden, const bf16 *hidden_lo, const int *row_alive, const bf16 *w2t,
                             const float *resid, float *out, int n, int m, float threshold) {
    pdl_wait();
    extern __shared__ int s_idx[];
    __shared__ int s_off[256];
    const int r = blockIdx.x;
    const int alive = row_alive[r];
    if (!((float)alive / (float)m <= 1.0f - threshold)) return;  // dense result stands
    const bf16 *h = hidden + (int64_t)r * m;
    const bf16 *hl = hidden_lo ? hidden_lo + (int64_t)r * m : nullptr;
    float *s_val = reinterpret_cast<float *>(s_idx + m);
    // pack alive (> 0) indices in ascending order (simd_sparse_matmul_rows'
    // packing): each thread scans a contiguous strip, a block scan places it
    const int strip = (m + blockDim.x - 1) / blockDim.x, j0 = threadIdx.x * strip, j1 = min(m, j0 + strip);
    int cnt = 0;
    for (int j = j0; j < j1; ++j) cnt += (__bfloat162float(h[j]) + (hl ? __bfloat162float(hl[j]) : 0.0f)) > 0.0f;
    s_off[threadIdx.x] = cnt;
    __syncthreads();
    for (int d = 1; d < (int)blockDim.x; d <<= 1) {  // inclusive scan of the strip counts
        const int v = threadIdx.x >= d ? s_off[threadIdx.x - d] : 0;
        __syncthreads();
        s_off[threadIdx.x] += v;
        __syncthreads();
    }
    int k = s_off[threadIdx.x] - cnt;
    for (int j = j0; j < j1; ++j) {
        const float v = __bfloat162float(h[j]) + (hl ? __bfloat162float(hl[j]) : 0.0f);
        if (v > 0.0f) {
            s_idx[k] = j;
            s_val[k] = v;
            ++k;
        }
    }
    const int na = s_off[blockDim.x - 1];
    __syncthreads();
    for (int c = threadIdx.x; c < n; c += blockDim.x) {
        float acc = 0.0f;
        for (int a = 0; a < na; ++a) acc += s_val[a] * __bfloat162float(w2t[(int64_t)s_idx[a] * n + c]);
        out[(int64_t)r * n + c] = acc + resid[(int64_t)r * n + c];
    }
}

// Benchmark hook: hidden activations after W1 replaced by a per-token
// Bernoulli(keep) mask with |N(0, 1)| survivors (the c4 workload's ~90%-zero
// hidden layer), deterministic in (seed, layer, slot, position, index); the
// alive counts follow.
__device__ __forceinline__ uint64_t mix64(uint64_t x) {
    x ^= x >> 30;
    x *= 0xbf58476d1ce4e5b9ull;
    x ^= x >> 27;
    x *= 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}
// one block per row; a thread draws 8 consecutive entries (one hash each for
// the Bernoulli draw, a second for a survivor's Box-Muller value) and stores
// them as one 16-byte vector per half
__global__ void mlp_hook_kernel(bf16 *hid, bf16 *hid2, int *row_alive, const int32_t *slot, const int32_t *pos, int m,
                                float keep, uint64_t seed, int layer) {
    pdl_wait();
    __shared__ int s_cnt;
    const int r = blockIdx.x;
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    const uint64_t key = mix64(seed ^ mix64(((uint64_t)layer << 48) ^ ((uint64_t)slot[r] << 24) ^ (uint64_t)pos[r]));
    int cnt = 0;
    for (int j0 = 8 * threadIdx.x; j0 < m; j0 += 8 * blockDim.x) {
        uint32_t hv[4], lv[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            float v[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const uint64_t j = (uint64_t)(j0 + e + q);
                const float u = (float)(mix64(key + 2 * j) >> 40) * (1.0f / 16777216.0f);
                v[q] = 0.0f;
                if (u < keep) {  // Box-Muller on two more uniforms
                    const uint64_t b2 = mix64(key + 2 * j + 1);
                    const float u1 = ((float)(b2 >> 40) + 0.5f) * (1.0f / 16777216.0f);
                    const float u2 = (float)((b2 >> 16) & 0xffffff) * (1.0f / 16777216.0f);
                    v[q] = fabsf(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));  // post-ReLU: non-negative
                    cnt += v[q] > 0.0f;
                }
            }
            const bf16 h0 = __float2bfloat16_rn(v[0]), h1 = __float2bfloat16_rn(v[1]);
            const bf16 l0 = __float2bfloat16_rn(v[0] - __bfloat162float(h0)), l1 = __float2bfloat16_rn(v[1] - __bfloat162float(h1));
            hv[e / 2] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
            lv[e / 2] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
        }
        *reinterpret_cast<uint4 *>(hid + (int64_t)r * m + j0) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        *reinterpret_cast<uint4 *>(hid2 + (int64_t)r * m + j0) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&s_cnt, cnt);
    __syncthreads();
    if (threadIdx.x == 0) row_alive[r] = s_cnt;
}

__global__ void softmax_kernel(const float *logits, float *probs, int V, int64_t ld, float inv_temp) {
    pdl_wait();
    __shared__ float red[32];
    const int m = blockIdx.x;
    const float *l = logits + (int64_t)m * ld;
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < V; j += blockDim.x) mx = fmaxf(mx, l[j]);
    mx = block_max(mx, red);
    float s = 0.0f;
    for (int j = threadIdx.x; j < V; j += blockDim.x) s += expf((l[j] - mx) * inv_temp);
    s = block_sum(s, red);
    const float inv = 1.0f / s;
    for (int j = threadIdx.x; j < V; j += blockDim.x) probs[(int64_t)m * ld + j] = expf((l[j] - mx) * inv_temp) * inv;
}

}  // namespace

template <typename CF, typename T, bool SA, bool SB>
cudaError_t launch_gemm(Gemm g, cudaStream_t s) {
    constexpr int smem = gemm_smem<CF, SA, SB>();
    {
        cudaError_t e = dev::smem(gemm_kernel<CF, T, SA, SB>, smem);
        if (e != cudaSuccess) return e;
    }
    const int64_t tiles = (int64_t)((g.N + CF::BN - 1) / CF::BN) * ((g.M + CF::BM - 1) / CF::BM) * g.batch;
    if (g.ksplit == 0) {
        // split K when the output has too few tiles to fill the GPU: at least
        // 3 K tiles per split, at most 8 CTAs per cluster, stop at two waves
        const int kt = g.K / BK;
        g.ksplit = 1;
        while (tiles * g.ksplit < 2 * 148 && g.ksplit * 2 * 3 <= kt && g.ksplit * 2 <= 8) g.ksplit *= 2;
    }
    if (g.ksplit > 8 || (g.ksplit & (g.ksplit - 1)) || (g.K / BK) < g.ksplit) return cudaErrorInvalidValue;
    dim3 grid((g.N + CF::BN - 1) / CF::BN, (g.M + CF::BM - 1) / CF::BM, g.batch * g.ksplit);
    if (g.ksplit == 1) {
        return launch_pdl(gemm_kernel<CF, T, SA, SB>, grid, dim3(CF::THREADS), smem, s, g);
    }
    return launch_pdl_cluster(gemm_kernel<CF, T, SA, SB>, grid, dim3(CF::THREADS), smem, s, dim3(1, 1, g.ksplit), g);
}

template <typename T, bool SA, bool SB>
cudaError_t launch_gemm_shape(const Gemm &g, cudaStream_t s) {
    return g.M <= 64 ? launch_gemm<TileS, T, SA, SB>(g, s) : launch_gemm<TileL, T, SA, SB>(g, s);
}

cudaError_t gemm(const Gemm &g, cudaStream_t s) {
    if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return cudaSuccess;
    if (g.K % BK != 0 || g.lda % 8 != 0 || g.ldb % 8 != 0) return cudaErrorInvalidValue;
    const bool sa = g.A2 != nullptr, sb = g.B2 != nullptr;
    if (g.dtype == DT_BF16) {
        if (sb) return cudaErrorInvalidValue;  // bf16 B operands are exact weights
        return sa ? launch_gemm_shape<bf16, true, false>(g, s) : launch_gemm_shape<bf16, false, false>(g, s);
    }
    if (sa && sb) return launch_gemm_shape<__half, true, true>(g, s);
    if (sa) return launch_gemm_shape<__half, true, false>(g, s);
    if (sb) return launch_gemm_shape<__half, false, true>(g, s);
    return launch_gemm_shape<__half, false, false>(g, s);
}

cudaError_t embed(const int32_t *tok, const int32_t *pos, const bf16 *wte, const bf16 *wpe, int n, int M, float *x,
                  cudaStream_t s, float *zero_rows) {
    if (M <= 0) return cudaSuccess;
    return launch_pdl(embed_kernel, dim3(M), dim3(256), 0, s, tok, pos, wte, wpe, n, M, x, zero_rows);
}
cudaError_t rmsnorm(const float *x, int n, int M, float *yf, bf16 *yb, bf16 *yb2, bool twice, cudaStream_t s,
                    int *zero_count, const float *gamma) {
    if (M <= 0) return cudaSuccess;
    return launch_pdl(rmsnorm_kernel, dim3(M), dim3(256), 0, s, x, n, M, yf, yb, yb2, twice ? 1 : 0, zero_count,
                      gamma);
}
cudaError_t to_bf16(const float *x, int64_t ldx, int n, int M, bf16 *y, bf16 *y2, int64_t ldy, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    return launch_pdl(to_bf16_kernel, dim3(M), dim3(256), 0, s, x, ldx, n, M, y, y2, ldy);
}
cudaError_t to_f16(const float *x, int64_t ldx, int n, int M, __half *hi, __half *lo, int64_t ldy, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    return launch_pdl(to_f16_kernel, dim3(M), dim3(256), 0, s, x, ldx, n, hi, lo, ldy);
}
cudaError_t f32_to_f16_split(const float *x, int64_t count, __half *hi, __half *lo, cudaStream_t s) {
    if (count <= 0) return cudaSuccess;
    f16_split_kernel<<<1184, 256, 0, s>>>(x, count, hi, lo);
    return cudaGetLastError();
}
cudaError_t f32_to_bf16_flat(const float *x, int64_t count, bf16 *y, cudaStream_t s) {
    if (count <= 0) return cudaSuccess;
    flat_bf16_kernel<<<1184, 256, 0, s>>>(x, count, y);
    return cudaGetLastError();
}
cudaError_t delta_route(float *x, const float *xr, float *delta, const float *query, const float *normw, int n,
                        int M, int layer, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    return launch_pdl(delta_route_kernel, dim3(M), dim3(256), 0, s, x, xr, delta, query, normw, n, layer);
}
cudaError_t twell_sparse_w2(const bf16 *hidden, const bf16 *hidden_lo, const int *row_alive, const bf16 *w2t,
                            const float *resid, float *out, int n, int m, int M, float threshold, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    const size_t smem = (size_t)m * 8;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(twell_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(twell_kernel, dim3(M), dim3(256), smem, s, hidden, hidden_lo, row_alive, w2t, resid, out, n, m, threshold);
}
cudaError_t mlp_hook(bf16 *hid, bf16 *hid2, int *row_alive, const int32_t *slot, const int32_t *pos, int m, int M,
                     float keep, uint64_t seed, int layer, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (m % 8) return cudaErrorInvalidValue;  // 16-byte row vectors
    return launch_pdl(mlp_hook_kernel, dim3(M), dim3(256), 0, s, hid, hid2, row_alive, slot, pos, m, keep, seed, layer);
}
cudaError_t softmax_rows(const float *logits, float *probs, int V, int M, int64_t ld, float inv_temp, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    return launch_pdl(softmax_kernel, dim3(M), dim3(256), 0, s, logits, probs, V, ld, inv_temp);
}

}  // namespace bf
}  // namespace kg
