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

#include "kg_attn.cuh"

namespace kg {
namespace attn {
namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
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
// Decode scores: one warp = 16 positions x all heads, K = kv_dim.
// The k dimension is permuted per 64-dim block so that each thread reads 8
// contiguous code bytes of a row (see file notes); q~ is permuted the same way.
template <int NT>  // n-tiles of 8 heads
__global__ void __launch_bounds__(128) scores_kernel(const ScoreArgs a) {
    __shared__ uint2 lut[256];
    build_lut(lut, a.kcent);
    __syncthreads();
    const int m = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int pos = a.pos[m];
    const int tn = pos + 1;
    const int t0 = blockIdx.x * 64 + warp * 16;
    if (t0 >= tn) return;
    const int slot = a.slot[m];
    const int64_t rowbase = ((int64_t)slot * a.L + a.layer) * a.B;
    const uint8_t *codes = a.kcodes + rowbase * a.kpl;
    const int r0 = min(t0 + g, tn - 1), r1 = min(t0 + g + 8, tn - 1);
    const uint8_t *c0 = codes + (int64_t)r0 * a.kpl, *c1 = codes + (int64_t)r1 * a.kpl;
    const __half *qt = a.qrot + (int64_t)m * a.nh * a.kvd;
    const __half *ql = a.qrot_lo + (int64_t)m * a.nh * a.kvd;
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.0f;
    const int nblk = a.kvd / 64;
    for (int q = 0; q < nblk; ++q) {
        const uint2 w0 = *reinterpret_cast<const uint2 *>(c0 + q * 32 + c * 8);
        const uint2 w1 = *reinterpret_cast<const uint2 *>(c1 + q * 32 + c * 8);
        uint32_t bq[NT][8], bl[NT][8];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int h = j * 8 + g;
            if (h < a.nh) {
                const int64_t off = (int64_t)h * a.kvd + q * 64 + c * 16;
                const uint4 *src = reinterpret_cast<const uint4 *>(qt + off);
                const uint4 *srl = reinterpret_cast<const uint4 *>(ql + off);
                uint4 u0 = src[0], u1 = src[1], v0 = srl[0], v1 = srl[1];
                bq[j][0] = u0.x; bq[j][1] = u0.y; bq[j][2] = u0.z; bq[j][3] = u0.w;
                bq[j][4] = u1.x; bq[j][5] = u1.y; bq[j][6] = u1.z; bq[j][7] = u1.w;
                bl[j][0] = v0.x; bl[j][1] = v0.y; bl[j][2] = v0.z; bl[j][3] = v0.w;
                bl[j][4] = v1.x; bl[j][5] = v1.y; bl[j][6] = v1.z; bl[j][7] = v1.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) bq[j][e] = bl[j][e] = 0u;
            }
        }
#pragma unroll
        for (int st = 0; st < 4; ++st) {
            // step st uses bytes 2st (k-cols 2c,2c+1) and 2st+1 (k-cols 8+2c, 9+2c)
            const uint32_t lo0 = st < 2 ? w0.x : w0.y, lo1 = st < 2 ? w1.x : w1.y;
            const int sh = (st & 1) * 16;
            const uint2 e0 = lut[(lo0 >> sh) & 0xff], e2 = lut[(lo0 >> (sh + 8)) & 0xff];
            const uint2 e1 = lut[(lo1 >> sh) & 0xff], e3 = lut[(lo1 >> (sh + 8)) & 0xff];
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                mma_f16(acc[j], e0.x, e1.x, e2.x, e3.x, bq[j][2 * st], bq[j][2 * st + 1]);
                mma_f16(acc[j], e0.y, e1.y, e2.y, e3.y, bq[j][2 * st], bq[j][2 * st + 1]);
                mma_f16(acc[j], e0.x, e1.x, e2.x, e3.x, bl[j][2 * st], bl[j][2 * st + 1]);
            }
        }
    }
    // epilogue: s = acc * norm_k[t] * scale; positions >= tn are -inf
    const float *kn = a.knorm + rowbase;
    float *S = a.S + (int64_t)m * a.nh * a.Tpad;
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
        const int t = t0 + g + hrow * 8;
        const float f = t < tn ? kn[t] * a.scale : 0.0f;
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int h = j * 8 + c * 2 + e;
                if (h < a.nh && t < a.Tpad) S[(int64_t)h * a.Tpad + t] = t < tn ? acc[j][hrow * 2 + e] * f : -INFINITY;
            }
    }
}

// softmax over positions per (token, head); p = softmax(s) * norm_v as f16 hi/lo, zero-padded
__global__ void softmax_kernel(const SoftmaxArgs a) {
    __shared__ float red[32];
    const int m = blockIdx.y, h = blockIdx.x;
    const int tn = a.pos[m] + 1;
    const float *s = a.S + ((int64_t)m * a.nh + h) * a.Tpad;
    __half *p = a.P + ((int64_t)m * a.nhp + h) * a.Tpad;
    __half *pl = a.P_lo + ((int64_t)m * a.nhp + h) * a.Tpad;
    const int64_t rowbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const float *vn = a.vnorm + rowbase;
    float mx = -INFINITY;
    for (int t = threadIdx.x; t < tn; t += blockDim.x) mx = fmaxf(mx, s[t]);
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
    __syncthreads();
    float sum = 0.0f;
    for (int t = threadIdx.x; t < tn; t += blockDim.x) sum += expf(s[t] - mx);
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    sum = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) sum += red[i];
    const float inv = 1.0f / sum;
    for (int t = threadIdx.x; t < a.Tpad; t += blockDim.x) {
        const float v = t < tn ? expf(s[t] - mx) * inv * vn[t] : 0.0f;
        const __half hv = __float2half_rn(v);
        p[t] = hv;
        pl[t] = __float2half_rn(v - __half2float(hv));
    }
}

// zero the padded head rows of P (heads nh..nhp-1) once per call
__global__ void zero_rows_kernel(__half *P, __half *P_lo, int nh, int nhp, int Tpad) {
    const int m = blockIdx.y, h = nh + blockIdx.x;
    __half *p = P + ((int64_t)m * nhp + h) * Tpad, *pl = P_lo + ((int64_t)m * nhp + h) * Tpad;
    for (int t = threadIdx.x; t < Tpad; t += blockDim.x) p[t] = pl[t] = __float2half_rn(0.0f);
}

// ---------------------------------------------------------------------------
// Decode values: u~[h, i] = sum_t p[h, t] * centroid(code_v[t, i]).
// CTA = 64 dims x all heads; 4 warps x 16 dims; positions in tiles of 32.
template <int MT>  // m-tiles of 16 heads
__global__ void __launch_bounds__(128) values_kernel(const ValueArgs a) {
    __shared__ uint2 lut[256];
    __shared__ __align__(16) __half tile[2][32][72];  // hi / lo: 32 positions x 64 dims (+8 pad)
    build_lut(lut, a.vcent);
    const int m = blockIdx.y, d0 = blockIdx.x * 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int tn = a.pos[m] + 1;
    const int64_t rowbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const uint8_t *codes = a.vcodes + rowbase * a.vpl + d0 / 2;
    const __half *P = a.P + (int64_t)m * a.nhp * a.Tpad;
    const __half *Pl = a.P_lo + (int64_t)m * a.nhp * a.Tpad;
    float acc[MT][2][4];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;
    const int ntile = (tn + 31) / 32;
    for (int tt = 0; tt < ntile; ++tt) {
        __syncthreads();  // lut ready / previous tile consumed
        {   // stage: thread -> (position tid/4, 8 bytes = 16 dims)
            const int pr = threadIdx.x >> 2, part = threadIdx.x & 3;
            const int t = tt * 32 + pr;
            uint2 w = make_uint2(0u, 0u);
            if (t < tn) w = *reinterpret_cast<const uint2 *>(codes + (int64_t)t * a.vpl + part * 8);
            uint32_t oh[8], ol[8];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint2 e0 = lut[(w.x >> (8 * b)) & 0xff], e1 = lut[(w.y >> (8 * b)) & 0xff];
                oh[b] = e0.x; ol[b] = e0.y;
                oh[4 + b] = e1.x; ol[4 + b] = e1.y;
            }
            uint4 *dh = reinterpret_cast<uint4 *>(&tile[0][pr][part * 16]);
            uint4 *dl = reinterpret_cast<uint4 *>(&tile[1][pr][part * 16]);
            dh[0] = make_uint4(oh[0], oh[1], oh[2], oh[3]);
            dh[1] = make_uint4(oh[4], oh[5], oh[6], oh[7]);
            dl[0] = make_uint4(ol[0], ol[1], ol[2], ol[3]);
            dl[1] = make_uint4(ol[4], ol[5], ol[6], ol[7]);
        }
        __syncthreads();
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {  // two k16 steps (positions)
            const int tk = tt * 32 + ks * 16;
            uint32_t bh[4], bw[4];
            {
                const int r = ks * 16 + (lane & 15);
                const int col = warp * 16 + ((lane >> 4) << 3);
                ldsm_x4_t(smem_u32(&tile[0][r][col]), bh[0], bh[1], bh[2], bh[3]);
                ldsm_x4_t(smem_u32(&tile[1][r][col]), bw[0], bw[1], bw[2], bw[3]);
            }
#pragma unroll
            for (int i = 0; i < MT; ++i) {
                const int64_t o0 = (int64_t)(i * 16 + g) * a.Tpad + tk, o1 = o0 + 8 * (int64_t)a.Tpad;
                const uint32_t a0 = *reinterpret_cast<const uint32_t *>(P + o0 + 2 * c);
                const uint32_t a1 = *reinterpret_cast<const uint32_t *>(P + o1 + 2 * c);
                const uint32_t a2 = *reinterpret_cast<const uint32_t *>(P + o0 + 8 + 2 * c);
                const uint32_t a3 = *reinterpret_cast<const uint32_t *>(P + o1 + 8 + 2 * c);
                const uint32_t l0 = *reinterpret_cast<const uint32_t *>(Pl + o0 + 2 * c);
                const uint32_t l1 = *reinterpret_cast<const uint32_t *>(Pl + o1 + 2 * c);
                const uint32_t l2 = *reinterpret_cast<const uint32_t *>(Pl + o0 + 8 + 2 * c);
                const uint32_t l3 = *reinterpret_cast<const uint32_t *>(Pl + o1 + 8 + 2 * c);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    mma_f16(acc[i][j], a0, a1, a2, a3, bh[2 * j], bh[2 * j + 1]);
                    mma_f16(acc[i][j], l0, l1, l2, l3, bh[2 * j], bh[2 * j + 1]);
                    mma_f16(acc[i][j], a0, a1, a2, a3, bw[2 * j], bw[2 * j + 1]);
                }
            }
        }
    }
    // write u~ as f16 hi/lo [m][h][kvd]
    __half *U = a.U + (int64_t)m * a.nh * a.kvd, *Ul = a.U_lo + (int64_t)m * a.nh * a.kvd;
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow) {
            const int h = i * 16 + g + hrow * 8;
            if (h >= a.nh) continue;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int d = d0 + warp * 16 + j * 8 + c * 2;
                uint32_t hi, lo;
                split_h2(acc[i][j][hrow * 2], acc[i][j][hrow * 2 + 1], hi, lo);
                *reinterpret_cast<uint32_t *>(U + (int64_t)h * a.kvd + d) = hi;
                *reinterpret_cast<uint32_t *>(Ul + (int64_t)h * a.kvd + d) = lo;
            }
        }
}

// ---------------------------------------------------------------------------
// Prefill: dequantize codes of every prompt token to f16 hi/lo centroid vectors.
__global__ void centroids_kernel(const uint8_t *codes, int pl, int64_t row_stride_codes, const int32_t *slot,
                                 const int32_t *pos, int L, int B, int layer, const float *cent, int kvd, int M,
                                 __half *out, __half *out_lo) {
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
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    out[m] = norms[((int64_t)slot[m] * L + layer) * B + pos[m]];
}

// Causal flash attention over one sequence's prompt (rows base..base+T-1).
// Q, K, V are f16 hi/lo splits; every product uses hi*hi + lo*hi + hi*lo, the
// online softmax is f32, output f32. CTA = 64 queries x one head, 4 warps x 16.
template <int HD>
__global__ void __launch_bounds__(128) fa_kernel(const FlashArgs a) {
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

cudaError_t scores(const ScoreArgs &a, cudaStream_t s) {
    dim3 grid((a.Tmax + 63) / 64, a.M);
    const int nt = (a.nh + 7) / 8;
    if (a.kvd % 64) return cudaErrorInvalidValue;
    switch (nt) {
        case 1: scores_kernel<1><<<grid, 128, 0, s>>>(a); break;
        case 2: scores_kernel<2><<<grid, 128, 0, s>>>(a); break;
        case 3: scores_kernel<3><<<grid, 128, 0, s>>>(a); break;
        case 4: scores_kernel<4><<<grid, 128, 0, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t softmax(const SoftmaxArgs &a, cudaStream_t s) {
    softmax_kernel<<<dim3(a.nh, a.M), 256, 0, s>>>(a);
    if (a.nhp > a.nh) zero_rows_kernel<<<dim3(a.nhp - a.nh, a.M), 128, 0, s>>>(a.P, a.P_lo, a.nh, a.nhp, a.Tpad);
    return cudaGetLastError();
}

cudaError_t values(const ValueArgs &a, cudaStream_t s) {
    if (a.kvd % 64) return cudaErrorInvalidValue;
    dim3 grid(a.kvd / 64, a.M);
    const int mt = a.nhp / 16;
    switch (mt) {
        case 1: values_kernel<1><<<grid, 128, 0, s>>>(a); break;
        case 2: values_kernel<2><<<grid, 128, 0, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
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

}  // namespace attn
}  // namespace kg
