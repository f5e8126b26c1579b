// kg_tq.cu — TurboQuant codec kernels in the reference's exact operation order.
//
// * Rotation build: modified Gram-Schmidt of the seeded Gaussian matrix
//   (src/turboquant/rotation.rs:11-52). The reference is left-looking (column i
//   subtracts its projections on q_0..q_{i-1}, each dot a sequential f32 sum);
//   this is the right-looking order of the same operations: at step j every
//   column i > j subtracts its projection on q_j. Column i sees the same
//   operands in the same sequence, so the result is bit-identical, and the
//   columns update in parallel (one thread per column).
// * Encode (store_key / store_value, src/turboquant/kv_cache.rs:156-237):
//   norm = sqrt(simd_sum_sq), x/norm, R*x with simd_dot_f32 order, boundary
//   count, pack. A warp computes one dot: lane L owns the chain of elements
//   k = L (mod 32) (AVX2 accumulator L/8, lane L%8), and the chains are
//   reduced with shuffles in the fixed ((acc0+acc1)+(acc2+acc3)) +
//   horizontal_sum_256 tree.
//
// Compiled with -fmad=false.
#include <mutex>
#include <string>

#include "kg_dev.cuh"
#include "kg_exact.cuh"
#include "kg_internal.h"
#include "kg_pdl.cuh"

namespace kg {
namespace {

// Fixed-order reduction of 32 lane chains (see file header).
__device__ __forceinline__ float tree32(float a) {
    float u = a + __shfl_down_sync(0xffffffffu, a, 8);   // acc0+acc1 (lanes 0-7), acc2+acc3 (16-23)
    float t = u + __shfl_down_sync(0xffffffffu, u, 16);  // (acc0+acc1)+(acc2+acc3), lanes 0-7
    float s = t + __shfl_down_sync(0xffffffffu, t, 4);   // lo128 + hi128, lanes 0-3
    float w = s + __shfl_down_sync(0xffffffffu, s, 1);   // v0+v1 (lane 0), v2+v3 (lane 2)
    float r = w + __shfl_down_sync(0xffffffffu, w, 2);   // (v0+v1)+(v2+v3), lane 0
    return __shfl_sync(0xffffffffu, r, 0);
}
// hsum8 of lanes 0..7 (an 8-lane accumulator), result broadcast.
__device__ __forceinline__ float tree8(float a) {
    float s = a + __shfl_down_sync(0xffffffffu, a, 4);
    float w = s + __shfl_down_sync(0xffffffffu, s, 1);
    float r = w + __shfl_down_sync(0xffffffffu, w, 2);
    return __shfl_sync(0xffffffffu, r, 0);
}

// simd_sum_sq over x[0..len) by one warp (result in every lane).
__device__ float warp_sum_sq(const float *x, int len, int stride) {
    const int lane = threadIdx.x & 31;
    const int c2 = len / 16;
    float acc = 0.0f;
    if (lane < 16) {
        int c = 0;
        for (; c + 8 <= c2; c += 8) {  // loads first, then the chain in order
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = x[(int64_t)(16 * (c + u) + lane) * stride];
#pragma unroll
            for (int u = 0; u < 8; ++u) acc = fmaf(v[u], v[u], acc);
        }
        for (; c < c2; ++c) {
            float v = x[(int64_t)(16 * c + lane) * stride];
            acc = fmaf(v, v, acc);
        }
    }
    // t[l] = a0[l] + a1[l] = chain l + chain l+8, then hsum8
    float t = acc + __shfl_down_sync(0xffffffffu, acc, 8);
    float sum = tree8(t);
    const int rem = (len - c2 * 16) / 8;
    float r = 0.0f;
    if (lane < 8 && rem > 0) {
        float v = x[(int64_t)(c2 * 16 + lane) * stride];
        r = fmaf(v, v, r);
    }
    sum = sum + tree8(r);
    for (int i = c2 * 16 + rem * 8; i < len; ++i) {
        float v = x[(int64_t)i * stride];
        sum = sum + v * v;
    }
    return sum;
}

// simd_dot_f32(a, b, len) by one warp (result in every lane).
__device__ __forceinline__ float warp_dot(const float *a, const float *b, int len) {
    const int lane = threadIdx.x & 31;
    const int c4 = len / 32;
    float acc = 0.0f;
    for (int c = 0; c < c4; ++c) acc = fmaf(a[32 * c + lane], b[32 * c + lane], acc);
    float sum = tree32(acc);
    const int rem = (len - c4 * 32) / 8;
    float r = 0.0f;
    if (lane < 8)
        for (int c = 0; c < rem; ++c) r = fmaf(a[c4 * 32 + 8 * c + lane], b[c4 * 32 + 8 * c + lane], r);
    sum = sum + tree8(r);
    for (int i = c4 * 32 + rem * 8; i < len; ++i) sum = sum + a[i] * b[i];
    return sum;
}

// One MGS step j. V is row-major (V[k*dim + i] = row k of column i) so that
// the per-column threads read coalesced rows.
__global__ void mgs_step(int dim, int j, float *V, float *Q) {
    extern __shared__ float qj[];
    __shared__ float s_norm;
    if (threadIdx.x < 32) {
        float ss = warp_sum_sq(V + j, dim, dim);
        if (threadIdx.x == 0) s_norm = sqrtf(ss);
    }
    __syncthreads();
    const float nrm = s_norm;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) {
        float qv = nrm > 1e-8f ? V[(int64_t)k * dim + j] / nrm : 0.0f;
        qj[k] = qv;
        if (blockIdx.x == 0 && nrm > 1e-8f) Q[(int64_t)k * dim + j] = qv;
    }
    __syncthreads();
    const int i = j + 1 + blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= dim) return;
    float d = -0.0f;  // Iterator::<f32>::sum starts from -0.0
    int k = 0;
    for (; k + 16 <= dim; k += 16) {  // loads first, then the sequential sum in order
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] = V[(int64_t)(k + u) * dim + i];
#pragma unroll
        for (int u = 0; u < 16; ++u) d = d + qj[k + u] * v[u];
    }
    for (; k < dim; ++k) d = d + qj[k] * V[(int64_t)k * dim + i];
#pragma unroll 8
    for (int kk = 0; kk < dim; ++kk) V[(int64_t)kk * dim + i] = V[(int64_t)kk * dim + i] - d * qj[kk];
}

__global__ void transpose_sq(int dim, const float *a, float *t) {
    __shared__ float tile[32][33];
    int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        int row = by + r, col = bx + threadIdx.x;
        if (row < dim && col < dim) tile[r][threadIdx.x] = a[(int64_t)row * dim + col];
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        int row = bx + r, col = by + threadIdx.x;
        if (row < dim && col < dim) t[(int64_t)row * dim + col] = tile[threadIdx.x][r];
    }
}

// Encode: one warp per vector, rows in sequence. smem per warp: xn[dim] + codes[dim].
__global__ void tq_encode_warp(int dim, int bits, int64_t n_vec, const float *x, int64_t ldx, const float *rot,
                               const float *bnd, uint8_t *packed, int64_t pstride, float *norms,
                               int64_t nstride, const int32_t *slot, const int32_t *pos, int L, int B,
                               int layer) {
    extern __shared__ float smf[];
    const int warps = blockDim.x / 32, w = threadIdx.x / 32, lane = threadIdx.x & 31;
    float *xn = smf + (size_t)w * dim;
    uint8_t *cd = reinterpret_cast<uint8_t *>(smf + (size_t)warps * dim) + (size_t)w * dim;
    const int nb = (1 << bits) - 1;
    for (int64_t v = (int64_t)blockIdx.x * warps + w; v < n_vec; v += (int64_t)gridDim.x * warps) {
        const float *xv = x + v * ldx;
        // destination row: v itself, or the arena row of token v
        const int64_t drow = slot ? ((int64_t)slot[v] * L + layer) * B + pos[v] : v;
        float norm = sqrtf(warp_sum_sq(xv, dim, 1));
        if (lane == 0) norms[drow * nstride] = norm;
        if (norm < 1e-8f) continue;  // indices untouched (reference quirk)
        const float inv = 1.0f / norm;
        for (int k = lane; k < dim; k += 32) xn[k] = xv[k] * inv;
        __syncwarp();
        for (int i = 0; i < dim; ++i) {
            float r = warp_dot(rot + (int64_t)i * dim, xn, dim);
            if (lane == 0) {
                int c = 0;
                for (int b = 0; b < nb; ++b) c += (r >= bnd[b]) ? 1 : 0;
                cd[i] = (uint8_t)c;
            }
        }
        __syncwarp();
        uint8_t *out = packed + drow * pstride;
        if (bits == 2) {
            for (int b = lane; b < (dim + 3) / 4; b += 32) {
                uint8_t o = 0;
                for (int s = 0; s < 4; ++s)
                    if (4 * b + s < dim) o |= (uint8_t)((cd[4 * b + s] & 3) << (2 * s));
                out[b] = o;
            }
        } else if (bits == 3 || bits == 4) {
            for (int b = lane; b < (dim + 1) / 2; b += 32) {
                uint8_t o = cd[2 * b] & 15;
                if (2 * b + 1 < dim) o |= (uint8_t)((cd[2 * b + 1] & 15) << 4);
                out[b] = o;
            }
        } else if (bits == 8) {
            for (int b = lane; b < dim; b += 32) out[b] = cd[b];
        } else {
            if (lane == 0) {
                const int pl = (dim * bits + 7) / 8;
                for (int b = 0; b < pl; ++b) out[b] = 0;
                int64_t bp = 0;
                for (int i = 0; i < dim; ++i, bp += bits) {
                    int byte = (int)(bp / 8), sh = (int)(bp % 8);
                    out[byte] |= (uint8_t)(cd[i] << sh);
                    if (sh + bits > 8) out[byte + 1] |= (uint8_t)(cd[i] >> (8 - sh));
                }
            }
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// Tiled exact encoder. Phase 1 (norm_kernel): per vector, norm = sqrt(simd_sum_sq)
// and xn = x * (1/norm) in the reference order; vectors with norm < 1e-8 are
// flagged (their codes stay untouched). Phase 2 (rotate_kernel): r = R xn for a
// tile of 64 rows x 16 vectors per CTA (8 warps of 16 x 8); lane L of a warp
// owns the AVX2 lane chain k = L (mod 32) of all 128 outputs of the warp, so
// each output's FMAs run in the reference order, then tree32 reduces it.
// Requires dim % 128 == 0.
constexpr int ER = 64, EV = 16, EK = 128;  // rows, vectors, columns per stage

__global__ void norm_kernel(int dim, int64_t n_vec, const float *x, int64_t ldx, float *xn, uint8_t *skip,
                            float *norms, const int32_t *slot, const int32_t *pos, int L, int B, int layer) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t v = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (v >= n_vec) return;
    const float *xv = x + v * ldx;
    const float norm = sqrtf(warp_sum_sq(xv, dim, 1));
    const int64_t drow = slot ? ((int64_t)slot[v] * L + layer) * B + pos[v] : v;
    if (lane == 0) {
        norms[drow] = norm;
        skip[v] = norm < 1e-8f ? 1 : 0;
    }
    const float inv = norm < 1e-8f ? 0.0f : 1.0f / norm;
    for (int k = lane; k < dim; k += 32) xn[v * dim + k] = xv[k] * inv;
}

__device__ __forceinline__ void cp16(void *dst, const void *src, bool pred) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(pred ? 16 : 0));
}

// blockIdx.z selects the second side (the V rows of a K + V launch): its xn
// and flags follow the first side's n_vec rows, with its own codebook,
// bit width and code arena.
struct RotSide {
    const float *bnd;
    uint8_t *packed;
    int64_t pstride;
    int bits;
};
__global__ void __launch_bounds__(256) rotate_kernel(int dim, int bits, int64_t n_vec, const float *xn,
                                                     const uint8_t *skip, const float *rot, const float *bnd,
                                                     uint8_t *packed, int64_t pstride, const int32_t *slot,
                                                     const int32_t *pos, int L, int B, int layer, RotSide side2) {
    pdl_wait();
    if (blockIdx.z) {
        xn += n_vec * dim;
        skip += n_vec;
        bnd = side2.bnd;
        packed = side2.packed;
        pstride = side2.pstride;
        bits = side2.bits;
    }
    extern __shared__ float4 esm[];
    float *Rs = reinterpret_cast<float *>(esm);   // [2][ER][EK]
    float *Xs = Rs + 2 * ER * EK;                 // [2][EV][EK]
    __shared__ uint8_t codes[EV][ER];
    __shared__ float s_bnd[256];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int b = tid; b < (1 << bits) - 1; b += blockDim.x) s_bnd[b] = bnd[b];
    const int wr = warp >> 1, wv = warp & 1;  // 4 x 2 warps: 16 rows x 8 vectors each
    const int r0 = blockIdx.x * ER;
    const int64_t v0 = (int64_t)blockIdx.y * EV;
    const int nst = dim / EK;
    auto stage = [&](int buf, int st) {
        const int c0 = st * EK;
        for (int e = tid; e < ER * EK / 4; e += 256) {  // R rows: 32 chunks of 16 B per row
            const int r = e / (EK / 4), ch = e % (EK / 4);
            cp16(Rs + (buf * ER + r) * EK + ch * 4, rot + (int64_t)(r0 + r) * dim + c0 + ch * 4, true);
        }
        for (int e = tid; e < EV * EK / 4; e += 256) {
            const int vv = e / (EK / 4), ch = e % (EK / 4);
            const int64_t gv = v0 + vv;
            cp16(Xs + (buf * EV + vv) * EK + ch * 4, xn + min(gv, n_vec - 1) * dim + c0 + ch * 4, gv < n_vec);
        }
        asm volatile("cp.async.commit_group;\n" ::);
    };
    float acc[16][8];
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
        for (int v = 0; v < 8; ++v) acc[i][v] = 0.0f;
    stage(0, 0);
    for (int st = 0; st < nst; ++st) {
        const int buf = st & 1;
        if (st + 1 < nst) {
            stage(buf ^ 1, st + 1);
            asm volatile("cp.async.wait_group 1;\n" ::);
        } else {
            asm volatile("cp.async.wait_group 0;\n" ::);
        }
        __syncthreads();
        const float *Rb = Rs + (buf * ER + wr * 16) * EK;
        const float *Xb = Xs + (buf * EV + wv * 8) * EK;
#pragma unroll
        for (int cc = 0; cc < EK / 32; ++cc) {  // one 32-wide chunk: lane L holds element 32*c + L
            float xv[8];
#pragma unroll
            for (int v = 0; v < 8; ++v) xv[v] = Xb[v * EK + cc * 32 + lane];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float r = Rb[i * EK + cc * 32 + lane];
#pragma unroll
                for (int v = 0; v < 8; ++v) acc[i][v] = fmaf(r, xv[v], acc[i][v]);
            }
        }
        __syncthreads();  // buffer reused by the stage after next
    }
    // Fixed-order reduction of all 128 outputs at once: a transposed butterfly
    // over the lane masks 8, 16, 4, 1, 2 — the pairing order of the reference
    // tree ((acc0+acc1)+(acc2+acc3), then horizontal_sum_256) — halves the
    // values per lane at each step, so every output gets exactly that tree and
    // each lane ends with 4 finished outputs. The remaining-8-chunk and tail
    // terms are empty (dim % 32 == 0): sum = tree + hsum(0) = tree + 0.
    float *v = &acc[0][0];  // flat view: output o = i * 8 + q lives in v[o]
    int obase = 0;
#define KG_BFLY(MASK, HALF)                                                        \
    {                                                                              \
        const bool hi = (lane & (MASK)) != 0;                                      \
        _Pragma("unroll") for (int k = 0; k < (HALF); ++k) {                       \
            const float send = hi ? v[k] : v[k + (HALF)];                          \
            const float keep = hi ? v[k + (HALF)] : v[k];                          \
            v[k] = keep + __shfl_xor_sync(0xffffffffu, send, (MASK));              \
        }                                                                          \
        if (hi) obase += (HALF);                                                   \
    }
    KG_BFLY(8, 64)
    KG_BFLY(16, 32)
    KG_BFLY(4, 16)
    KG_BFLY(1, 8)
    KG_BFLY(2, 4)
#undef KG_BFLY
    const int nb = (1 << bits) - 1;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float r = v[k] + 0.0f;
        int c = 0;
        for (int b = 0; b < nb; ++b) c += (r >= s_bnd[b]) ? 1 : 0;
        const int o = obase + k;  // o = i * 8 + q
        codes[wv * 8 + (o & 7)][wr * 16 + (o >> 3)] = (uint8_t)c;
    }
    __syncthreads();
    // pack 64 codes per vector: 32 bytes (3/4-bit) at byte offset r0/2
    for (int e = tid; e < EV * (ER / 2); e += 256) {
        const int vv = e / (ER / 2), b = e % (ER / 2);
        const int64_t gv = v0 + vv;
        if (gv >= n_vec || skip[gv]) continue;
        const int64_t drow = slot ? ((int64_t)slot[gv] * L + layer) * B + pos[gv] : gv;
        packed[drow * pstride + r0 / 2 + b] = (uint8_t)((codes[vv][2 * b] & 15) | ((codes[vv][2 * b + 1] & 15) << 4));
    }
}

// ---------------------------------------------------------------------------
// Tensor-core encoder with exact fix-up (bit-identical codes).
//
// The reference code of coordinate j is count(y_j >= b) over the sorted
// boundaries b, with y_j = simd_dot(R[j, :], xn) in the AVX2 order. A
// split-precision GEMM (xn and R as f16 hi + lo, three products, f32
// accumulation) gives y'_j with |y'_j - y_j| <= eps, eps bounding both
// roundings (the reference dot's and the tensor core's) for a unit vector
// against a unit row: whenever every boundary is farther than eps from
// y'_j, y'_j yields the reference code. The few coordinates closer than eps
// are recomputed exactly (warp_dot, the same order as the exact encoder).
// K and V rows of a step go through one norm launch, one GEMM and one
// quantize launch: vector v < Mk is a K row, the rest V rows.

// Per vector: norm (exact order) to the arena, xn = x * (1 / norm), and its
// f16 hi / lo split (row v of xh / xl, zero for vectors the reference skips).
__global__ void norm_split_kernel(int dim, int Mk, int Mv, const float *qkv, int64_t ldx, int64_t koff,
                                  int64_t voff, float *xn, __half *xh, __half *xl, uint8_t *skip, float *knorm,
                                  float *vnorm, const int32_t *slot, const int32_t *pos, int L, int B, int layer) {
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int v = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (v >= Mk + Mv) return;
    const int M = Mk;
    const int t = v < M ? v : v - M;
    const float *xv = qkv + (int64_t)t * ldx + (v < M ? koff : voff);
    const float norm = sqrtf(warp_sum_sq(xv, dim, 1));
    const int64_t drow = slot ? ((int64_t)slot[t] * L + layer) * B + pos[t] : t;
    if (lane == 0) {
        (v < M ? knorm : vnorm)[drow] = norm;
        skip[v] = norm < 1e-8f ? 1 : 0;
    }
    const float inv = norm < 1e-8f ? 0.0f : 1.0f / norm;
    for (int k = lane; k < dim; k += 32) {
        const float y = xv[k] * inv;
        xn[(int64_t)v * dim + k] = y;
        if (xh) {
            const __half h = __float2half_rn(y);
            xh[(int64_t)v * dim + k] = h;
            xl[(int64_t)v * dim + k] = __float2half_rn(y - __half2float(h));
        }
    }
}

// One CTA per vector (K or V row): codes from y' where no boundary is within
// eps, then exact recomputation of the others, then 4-bit packing (two codes
// per byte, low first). The vector's xn is staged in shared memory once; the
// near-boundary coordinates (about 4% of them at kv_dim 4096, so ~160 per
// vector) go to a shared list that the CTA's warps drain, so each warp
// streams rotation rows with many loads in flight and no warp idles while
// another holds a long run of recomputations.
constexpr int kFixWarps = 8;

// simd_dot_f32(row, xs, dim) by one warp with xs in shared memory: lane l
// accumulates elements l + 32c in order (the AVX2 body's 32 lanes), the row
// loaded 32 deep per lane before the FMA chain consumes it. dim % 32 == 0.
__device__ __forceinline__ float warp_dot_row(const float *__restrict__ row, const float *xs, int dim) {
    const int lane = threadIdx.x & 31;
    const int c4 = dim / 32;
    float acc = 0.0f;
    int c = 0;
    for (; c + 32 <= c4; c += 32) {
        float ra[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) ra[u] = __ldg(row + 32 * (c + u) + lane);
        asm volatile("" ::: "memory");  // all 32 loads issue before the chain's first shared read
#pragma unroll
        for (int u = 0; u < 32; ++u) acc = fmaf(ra[u], xs[32 * (c + u) + lane], acc);
    }
#pragma unroll 8
    for (; c < c4; ++c) acc = fmaf(__ldg(row + 32 * c + lane), xs[32 * c + lane], acc);
    const float sum = tree32(acc);
    return sum + 0.0f;  // warp_dot adds the (here empty) 8-chunk remainder
}

__global__ void __launch_bounds__(kFixWarps * 32, 4)
quantize_fixup_kernel(int dim, int Mk, int Mv, const float *Y, const float *xn, const uint8_t *skip,
                      const float *rot, const float *kb, const float *vb, int kbits, int vbits, uint8_t *kcodes,
                      uint8_t *vcodes, int64_t kpl, int64_t vpl, const int32_t *slot, const int32_t *pos, int L,
                      int B, int layer, float eps, int *nfix) {
    pdl_wait();
    extern __shared__ float4 fix_sm4[];
    float *xs = reinterpret_cast<float *>(fix_sm4);                 // [dim]
    uint16_t *list = reinterpret_cast<uint16_t *>(xs + dim);       // [dim] near-boundary coordinates
    uint8_t *cbuf = reinterpret_cast<uint8_t *>(list + dim);       // [dim] codes
    __shared__ float bnd[15];
    __shared__ int nlist;
    const int64_t v = blockIdx.x;
    if (v >= Mk + Mv || skip[v]) return;  // skipped vectors keep their codes (reference quirk); CTA-uniform
    const int which = v < Mk ? 0 : 1;
    const int bits = which ? vbits : kbits;
    const int nb = (1 << bits) - 1;
    if (threadIdx.x < 15) bnd[threadIdx.x] = threadIdx.x < nb ? (which ? vb : kb)[threadIdx.x] : INFINITY;
    if (threadIdx.x == 0) nlist = 0;
    __syncthreads();
    const float *yv = Y + v * dim, *xv = xn + v * dim;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) {
        xs[j] = xv[j];
        const float y = yv[j];
        int c = 0;
        bool near = false;
        for (int k = 0; k < nb; ++k) {
            c += y >= bnd[k] ? 1 : 0;
            near |= fabsf(y - bnd[k]) <= eps;
        }
        cbuf[j] = (uint8_t)c;
        if (near) list[atomicAdd(&nlist, 1)] = (uint16_t)j;
    }
    __syncthreads();
    const int n_near = nlist;
    const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
    for (int f = w; f < n_near; f += kFixWarps) {  // exact recomputation in the reference order
        const int j = list[f];
        const float r = warp_dot_row(rot + (int64_t)j * dim, xs, dim);
        if (lane == 0) {
            int c = 0;
            for (int k = 0; k < nb; ++k) c += r >= bnd[k] ? 1 : 0;
            cbuf[j] = (uint8_t)c;
        }
    }
    __syncthreads();
    const int64_t t = which ? v - Mk : v;
    const int64_t drow = slot ? ((int64_t)slot[t] * L + layer) * B + pos[t] : t;
    uint8_t *out = (which ? vcodes : kcodes) + drow * (which ? vpl : kpl);
    for (int b = threadIdx.x; b < dim / 2; b += blockDim.x)
        out[b] = (uint8_t)((cbuf[2 * b] & 15) | ((cbuf[2 * b + 1] & 15) << 4));
    if (nfix && threadIdx.x == 0 && n_near) atomicAdd(nfix, n_near);
}

// ---- SpectralQuant codec at any kv_dim (store_vector / dequantize_*_into,
// src/spectralquant/spectral_kv_cache.rs:399-470, 567-672). A layer's tables:
// eig [kvd*kvd] (V[i][j] at i*kvd + j, columns = eigenvectors), meta [kvd]
// (width | levels << 8), cent [kvd][64], offs [kvd] (bit offset of dimension j
// in the pack: the prefix sum of the widths), and the pack's byte count.

// One CTA per vector: norm (simd_sum_sq order), x / norm, y_j = sum over i in
// order of V[i][j] x_i (rotate_into: one thread per output, separate multiply
// and add), the nearest centroid by the reference's bisection, and the index
// ORed into the pack at its bit offset (LSB-first stream). A vector with norm
// < 1e-8 stores norm 0 and leaves its bytes as they were.
__global__ void sq_encode_kernel(int kvd, const float *x, const float *eig, const int *meta, const float *cent,
                                 const int *offs, int nbytes, uint8_t *packed, int64_t pstride, float *norms) {
    extern __shared__ float sq_sm[];
    float *xn = sq_sm;                                          // [kvd]
    uint32_t *words = reinterpret_cast<uint32_t *>(xn + kvd);  // [nbytes / 4 + 2]
    __shared__ float s_norm;
    const int64_t v = blockIdx.x;
    const float *xv = x + v * kvd;
    if (threadIdx.x < 32) {
        const float ss = warp_sum_sq(xv, kvd, 1);
        if (threadIdx.x == 0) s_norm = sqrtf(ss);
    }
    for (int w = threadIdx.x; w < nbytes / 4 + 2; w += blockDim.x) words[w] = 0u;
    __syncthreads();
    const float norm = s_norm;
    if (norm < 1e-8f) {  // CTA-uniform
        if (threadIdx.x == 0) norms[v] = 0.0f;
        return;
    }
    if (threadIdx.x == 0) norms[v] = norm;
    const float inv = 1.0f / norm;
    for (int i = threadIdx.x; i < kvd; i += blockDim.x) xn[i] = xv[i] * inv;
    __syncthreads();
    for (int j = threadIdx.x; j < kvd; j += blockDim.x) {
        float y = 0.0f;
        for (int i = 0; i < kvd; ++i) y = y + eig[(int64_t)i * kvd + j] * xn[i];
        const int n = meta[j] >> 8;
        const float *c = cent + (int64_t)j * 64;
        int q = 0;  // quantize_to_idx (spectral_kv_cache.rs:1079-1111)
        if (n > 1) {
            int lo = 0, hi = n - 1;
            if (y <= c[lo]) q = lo;
            else if (y >= c[hi]) q = hi;
            else {
                while (lo + 1 < hi) {
                    const int mid = lo + (hi - lo) / 2;
                    if (c[mid] <= y) lo = mid;
                    else hi = mid;
                }
                q = fabsf(y - c[lo]) <= fabsf(c[hi] - y) ? lo : hi;
            }
        }
        const int o = offs[j];
        const uint64_t sh = (uint64_t)q << (o & 31);  // pack_variable_bits (:1125-1164)
        atomicOr(&words[o >> 5], (uint32_t)sh);
        if (sh >> 32) atomicOr(&words[(o >> 5) + 1], (uint32_t)(sh >> 32));
    }
    __syncthreads();
    const uint8_t *wb = reinterpret_cast<const uint8_t *>(words);
    uint8_t *out = packed + v * pstride;
    for (int b = threadIdx.x; b < nbytes; b += blockDim.x) out[b] = wb[b];
}

// One CTA per vector: unpack (unpack_variable_bits, :1167-1187), centroids,
// out_i = simd_dot(V row i, c) (simd_matmul_rows: one warp per row, the AVX2
// order) * norm; zeros when norm < 1e-8.
__global__ void sq_decode_kernel(int kvd, const uint8_t *packed, int64_t pstride, const float *norms, const float *eig,
                                 const int *meta, const float *cent, const int *offs, int nbytes, float *out) {
    extern __shared__ float sq_sm[];
    float *c = sq_sm;  // [kvd]
    const int64_t v = blockIdx.x;
    const float norm = norms[v];
    float *ov = out + v * kvd;
    if (norm < 1e-8f) {
        for (int i = threadIdx.x; i < kvd; i += blockDim.x) ov[i] = 0.0f;
        return;
    }
    const uint8_t *p = packed + v * pstride;
    for (int j = threadIdx.x; j < kvd; j += blockDim.x) {
        const int m = meta[j], bits = m & 255, n = m >> 8, o = offs[j];
        uint32_t w = 0;
        for (int b = 0; b < 3; ++b) {
            const int bi = (o >> 3) + b;
            if (bi < nbytes) w |= (uint32_t)p[bi] << (8 * b);
        }
        const int idx = (int)((w >> (o & 7)) & ((1u << bits) - 1u));
        c[j] = idx < n ? cent[(int64_t)j * 64 + idx] : 0.0f;
    }
    __syncthreads();
    const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int i = wp; i < kvd; i += nw) {
        const float r = warp_dot(eig + (int64_t)i * kvd, c, kvd);
        if (lane == 0) ov[i] = r * norm;
    }
}

}  // namespace

// Bound on |y' - y| for the fix-up: both roundings of a dim-term dot of a unit
// vector with a unit row (the AVX2 order's ~dim/32 + 8 roundings and the
// tensor core's per-k-step accumulation), with a 4x margin.
float tq_fixup_eps(int dim) { return 4.0f * (16.0f + (float)dim / 16.0f) * 5.96e-8f; }

cudaError_t tq_norm_split(int dim, int Mk, int Mv, const float *qkv, int64_t ldx, int64_t koff, int64_t voff,
                          float *xn, __half *xh, __half *xl, uint8_t *skip, float *knorm, float *vnorm,
                          const int32_t *slot, const int32_t *pos, int L, int B, int layer, cudaStream_t s) {
    if (Mk + Mv <= 0) return cudaSuccess;
    return launch_pdl(norm_split_kernel, dim3((Mk + Mv + 7) / 8), dim3(256), 0, s, dim, Mk, Mv, qkv, ldx, koff, voff,
                      xn, xh, xl, skip, knorm, vnorm, slot, pos, L, B, layer);
}

cudaError_t tq_quantize_fixup(int dim, int Mk, int Mv, const float *Y, const float *xn, const uint8_t *skip,
                              const float *rot, const float *kb, const float *vb, int kbits, int vbits,
                              uint8_t *kcodes, uint8_t *vcodes, int64_t kpl, int64_t vpl, const int32_t *slot,
                              const int32_t *pos, int L, int B, int layer, int *nfix, cudaStream_t s) {
    if (Mk + Mv <= 0) return cudaSuccess;
    if (dim % 32 || dim > 32768 || kbits < 3 || kbits > 4 || vbits < 3 || vbits > 4) return cudaErrorInvalidValue;
    const size_t smem = (size_t)dim * (sizeof(float) + sizeof(uint16_t) + 1);
    const cudaError_t e = dev::smem(quantize_fixup_kernel, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(quantize_fixup_kernel, dim3((unsigned)(Mk + Mv)), dim3(kFixWarps * 32), smem, s, dim, Mk, Mv, Y,
                      xn, skip, rot, kb, vb, kbits, vbits, kcodes, vcodes, kpl, vpl, slot, pos, L, B, layer,
                      tq_fixup_eps(dim), nfix);
}

namespace {
}  // namespace

cudaError_t sq_encode_device(int kvd, int64_t n_vec, const float *x, const float *eig, const int *meta,
                             const float *cent, const int *offs, int nbytes, uint8_t *packed, int64_t pstride,
                             float *norms, cudaStream_t s) {
    if (n_vec <= 0) return cudaSuccess;
    if (kvd < 2 || nbytes < 1 || nbytes > kvd) return cudaErrorInvalidValue;
    const size_t smem = (size_t)kvd * 4 + (size_t)(nbytes / 4 + 2) * 4;
    cudaError_t e = dev::smem(sq_encode_kernel, smem);
    if (e != cudaSuccess) return e;
    sq_encode_kernel<<<(unsigned)n_vec, 256, smem, s>>>(kvd, x, eig, meta, cent, offs, nbytes, packed, pstride, norms);
    return cudaGetLastError();
}

cudaError_t sq_decode_device(int kvd, int64_t n_vec, const uint8_t *packed, int64_t pstride, const float *norms,
                             const float *eig, const int *meta, const float *cent, const int *offs, int nbytes,
                             float *out, cudaStream_t s) {
    if (n_vec <= 0) return cudaSuccess;
    if (kvd < 2 || nbytes < 1 || nbytes > kvd) return cudaErrorInvalidValue;
    const size_t smem = (size_t)kvd * 4;
    cudaError_t e = dev::smem(sq_decode_kernel, smem);
    if (e != cudaSuccess) return e;
    sq_decode_kernel<<<(unsigned)n_vec, 256, smem, s>>>(kvd, packed, pstride, norms, eig, meta, cent, offs, nbytes, out);
    return cudaGetLastError();
}

cudaError_t tq_rotation_device(int dim, const float *g, float *rot, float *rot_t, float *work,
                               cudaStream_t s) {
    // V (row-major, V[k*dim+i] = column i) is the Gaussian matrix itself:
    // the reference fills column vectors v_col[row] = mat[row][col].
    cudaError_t e = cudaMemcpyAsync(work, g, (size_t)dim * dim * sizeof(float),
                                    cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(rot, 0, (size_t)dim * dim * sizeof(float), s);
    if (e != cudaSuccess) return e;
    const int threads = 128;
    const size_t smem = (size_t)dim * sizeof(float);
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(mgs_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    for (int j = 0; j < dim; ++j) {
        int cols = dim - j - 1;
        int blocks = cols > 0 ? (cols + threads - 1) / threads : 1;
        mgs_step<<<blocks, threads, smem, s>>>(dim, j, work, rot);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    dim3 tb(32, 8), gb((dim + 31) / 32, (dim + 31) / 32);
    transpose_sq<<<gb, tb, 0, s>>>(dim, rot, rot_t);
    return cudaGetLastError();
}

cudaError_t tq_encode_device(int dim, int bits, int64_t n_vec, const float *x, const float *rot,
                             const float *bnd, uint8_t *packed, int64_t pstride, float *norms,
                             int64_t nstride, cudaStream_t s) {
    return tq_encode_scatter(dim, bits, n_vec, x, dim, rot, bnd, packed, pstride, norms, nstride, nullptr,
                             nullptr, 0, 0, 0, s);
}

cudaError_t tq_encode_tiled(int dim, int bits, int64_t n_vec, const float *x, int64_t ldx, const float *rot,
                            const float *bnd, uint8_t *packed, int64_t pstride, float *norms,
                            const int32_t *slot, const int32_t *pos, int L, int B, int layer, float *xn_scratch,
                            uint8_t *skip_scratch, cudaStream_t s) {
    if (n_vec <= 0) return cudaSuccess;
    if (dim % EK || (bits != 3 && bits != 4)) return cudaErrorInvalidValue;
    norm_kernel<<<(unsigned)((n_vec + 7) / 8), 256, 0, s>>>(dim, n_vec, x, ldx, xn_scratch, skip_scratch, norms, slot,
                                                             pos, L, B, layer);
    const int smem = 2 * (ER + EV) * EK * 4;
    {
        cudaError_t e = dev::smem(rotate_kernel, smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid(dim / ER, (unsigned)((n_vec + EV - 1) / EV));
    rotate_kernel<<<grid, 256, smem, s>>>(dim, bits, n_vec, xn_scratch, skip_scratch, rot, bnd, packed, pstride, slot,
                                          pos, L, B, layer, RotSide{});
    return cudaGetLastError();
}

cudaError_t tq_encode_tiled_kv(int dim, int kbits, int vbits, int M, const float *qkv, int64_t ldx, int64_t koff,
                               int64_t voff, const float *rot, const float *kb, const float *vb, uint8_t *kcodes,
                               int64_t kpl, float *knorm, uint8_t *vcodes, int64_t vpl, float *vnorm,
                               const int32_t *slot, const int32_t *pos, int L, int B, int layer, float *xn_scratch,
                               uint8_t *skip_scratch, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    if (dim % EK || kbits < 3 || kbits > 4 || vbits < 3 || vbits > 4) return cudaErrorInvalidValue;
    cudaError_t e0 = launch_pdl(norm_split_kernel, dim3((2 * M + 7) / 8), dim3(256), 0, s, dim, M, M, qkv, ldx, koff,
                                voff, xn_scratch, (__half *)nullptr, (__half *)nullptr, skip_scratch, knorm, vnorm,
                                slot, pos, L, B, layer);
    if (e0 != cudaSuccess) return e0;
    const int smem = 2 * (ER + EV) * EK * 4;
    {
        cudaError_t e = dev::smem(rotate_kernel, smem);
        if (e != cudaSuccess) return e;
    }
    dim3 grid(dim / ER, (unsigned)((M + EV - 1) / EV), 2);
    return launch_pdl(rotate_kernel, grid, dim3(256), smem, s, dim, kbits, (int64_t)M, (const float *)xn_scratch,
                      (const uint8_t *)skip_scratch, rot, kb, kcodes, kpl, slot, pos, L, B, layer,
                      RotSide{vb, vcodes, vpl, vbits});
}

cudaError_t tq_encode_scatter(int dim, int bits, int64_t n_vec, const float *x, int64_t ldx, const float *rot,
                              const float *bnd, uint8_t *packed, int64_t pstride, float *norms, int64_t nstride,
                              const int32_t *slot, const int32_t *pos, int L, int B, int layer, cudaStream_t s) {
    if (n_vec <= 0) return cudaSuccess;
    int warps = 4;
    size_t smem = (size_t)warps * dim * (sizeof(float) + 1);
    while (smem > 200 * 1024 && warps > 1) {
        warps /= 2;
        smem = (size_t)warps * dim * (sizeof(float) + 1);
    }
    cudaError_t e = dev::smem(tq_encode_warp, smem);
    if (e != cudaSuccess) return e;
    int64_t blocks = (n_vec + warps - 1) / warps;
    if (blocks > 148 * 16) blocks = 148 * 16;
    tq_encode_warp<<<(unsigned)blocks, warps * 32, smem, s>>>(dim, bits, n_vec, x, ldx, rot, bnd, packed,
                                                             pstride, norms, nstride, slot, pos, L, B, layer);
    return cudaGetLastError();
}

}  // namespace kg

// ---------------------------------------------------------------------------
// Allocation-free encoder entry point.
//
// Some callers cannot allocate device memory at the moment they encode: code
// running between the stages of a captured or latency-critical decode loop
// (cudaMalloc and cudaFree synchronise the whole device), and hosts that hand
// the library a fixed memory budget up front and forbid growth afterwards
// (the zero-alloc discipline of the reference's TurboQuant hot path). For
// them kg_tq_encode_noalloc takes device pointers for its inputs and outputs
// and keeps the encoder's scratch (normalised rows and zero-norm flags) in the
// file-scope arrays below, which every GPU that loads this library holds
// until the process exits.
namespace kg {
namespace {
constexpr int64_t kNoAllocMaxFloats = int64_t(1) << 20;  // 4 MiB of normalised rows (n_vec * kv_dim)
constexpr int64_t kNoAllocMaxVectors = int64_t(1) << 16;  // zero-norm flags
static __device__ __align__(256) float g_noalloc_xn[kNoAllocMaxFloats];
static __device__ __align__(256) uint8_t g_noalloc_skip[kNoAllocMaxVectors];

// Device addresses of the arrays above, looked up once per device with that
// device current (the host-side names are stand-ins, not device addresses).
std::mutex g_noalloc_mu;
float *g_noalloc_xn_ptr[64] = {};
uint8_t *g_noalloc_skip_ptr[64] = {};

cudaError_t noalloc_scratch(int device, float **xn, uint8_t **skip) {
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_xn_ptr[device]) {
        void *a = nullptr, *b = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&a, g_noalloc_xn);
        if (e != cudaSuccess) return e;
        e = cudaGetSymbolAddress(&b, g_noalloc_skip);
        if (e != cudaSuccess) return e;
        g_noalloc_xn_ptr[device] = static_cast<float *>(a);
        g_noalloc_skip_ptr[device] = static_cast<uint8_t *>(b);
    }
    *xn = g_noalloc_xn_ptr[device];
    *skip = g_noalloc_skip_ptr[device];
    return cudaSuccess;
}
}  // namespace
}  // namespace kg

extern "C" int kg_tq_encode_noalloc(kg_ctx *ctx, int32_t which, int64_t n_vec, const float *x, uint8_t *packed,
                                    float *norms, void *stream) {
    if (!ctx || !x || !packed || !norms || n_vec < 0 || (which != 0 && which != 1)) return KG_ERR_INVALID_ARG;
    if (!kg::kv_is_tq(ctx->cfg.kv_mode)) {
        ctx->err = "context has no TurboQuant codec";
        return KG_ERR_INVALID_ARG;
    }
    const int64_t kvd = ctx->kvd;
    // bound n_vec before forming n_vec * kv_dim (a huge n_vec would overflow the product)
    if (n_vec > kg::kNoAllocMaxVectors || n_vec > kg::kNoAllocMaxFloats / kvd) {
        ctx->err = "kg_tq_encode_noalloc: n_vec * kv_dim exceeds the fixed scratch of " +
                   std::to_string(kg::kNoAllocMaxFloats) + " floats (at most " +
                   std::to_string(kg::kNoAllocMaxFloats / kvd) + " vectors at this kv_dim)";
        return KG_ERR_INVALID_ARG;
    }
    if (n_vec == 0) return KG_OK;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) {
        ctx->err = std::string("cudaSetDevice: ") + cudaGetErrorString(e);
        return KG_ERR_CUDA;
    }
    float *xn = nullptr;
    uint8_t *skip = nullptr;
    e = kg::noalloc_scratch(ctx->device, &xn, &skip);
    if (e != cudaSuccess) {
        ctx->err = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
        return KG_ERR_CUDA;
    }
    const int bits = which == 0 ? ctx->cfg.key_bits : ctx->cfg.val_bits;
    const float *bnd = which == 0 ? ctx->kb : ctx->vb;
    const int64_t pl = (bits == 2) ? (kvd + 3) / 4 : (bits == 3 || bits == 4) ? (kvd + 1) / 2 : (bits == 8) ? kvd
                                                                                               : (kvd * bits + 7) / 8;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (kvd % 128 == 0 && (bits == 3 || bits == 4))
        e = kg::tq_encode_tiled((int)kvd, bits, n_vec, x, kvd, ctx->rot, bnd, packed, pl, norms, nullptr, nullptr, 0, 0,
                                0, xn, skip, s);
    else
        e = kg::tq_encode_device((int)kvd, bits, n_vec, x, ctx->rot, bnd, packed, pl, norms, 1, s);
    if (e != cudaSuccess) {
        ctx->err = std::string("kg_tq_encode_noalloc: ") + cudaGetErrorString(e);
        return KG_ERR_CUDA;
    }
    return KG_OK;
}

