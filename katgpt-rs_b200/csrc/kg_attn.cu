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
// into a bf16 pair with a 256-entry shared-memory table, in registers, feeding
// mma.sync; attn_values stages a tile of codes in shared memory, dequantizes it
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
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
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
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// byte -> (centroid[lo nibble], centroid[hi nibble]) as a bf16 pair
__device__ __forceinline__ void build_lut(uint32_t *lut, const float *cent) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) lut[b] = pack_bf16(cent[b & 15], cent[b >> 4]);
}

// ---------------------------------------------------------------------------
// Decode scores: one warp = 16 positions x all heads, K = kv_dim.
// The k dimension is permuted per 64-dim block so that each thread reads 8
// contiguous code bytes of a row (see file notes); q~ is permuted the same way.
template <int NT>  // n-tiles of 8 heads
__global__ void __launch_bounds__(128) scores_kernel(const ScoreArgs a) {
    __shared__ uint32_t lut[256];
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
    const bf16 *qt = a.qrot + (int64_t)m * a.nh * a.kvd;
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.0f;
    const int nblk = a.kvd / 64;
    for (int q = 0; q < nblk; ++q) {
        const uint2 w0 = *reinterpret_cast<const uint2 *>(c0 + q * 32 + c * 8);
        const uint2 w1 = *reinterpret_cast<const uint2 *>(c1 + q * 32 + c * 8);
        uint32_t bq[NT][8];
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            const int h = j * 8 + g;
            if (h < a.nh) {
                const uint4 *src = reinterpret_cast<const uint4 *>(qt + (int64_t)h * a.kvd + q * 64 + c * 16);
                uint4 u0 = src[0], u1 = src[1];
                bq[j][0] = u0.x; bq[j][1] = u0.y; bq[j][2] = u0.z; bq[j][3] = u0.w;
                bq[j][4] = u1.x; bq[j][5] = u1.y; bq[j][6] = u1.z; bq[j][7] = u1.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) bq[j][e] = 0u;
            }
        }
#pragma unroll
        for (int st = 0; st < 4; ++st) {
            // step st uses bytes 2st (k-cols 2c,2c+1) and 2st+1 (k-cols 8+2c, 9+2c)
            const uint32_t lo0 = st < 2 ? w0.x : w0.y, lo1 = st < 2 ? w1.x : w1.y;
            const int sh = (st & 1) * 16;
            const uint32_t a0 = lut[(lo0 >> sh) & 0xff], a2 = lut[(lo0 >> (sh + 8)) & 0xff];
            const uint32_t a1 = lut[(lo1 >> sh) & 0xff], a3 = lut[(lo1 >> (sh + 8)) & 0xff];
#pragma unroll
            for (int j = 0; j < NT; ++j) mma_bf16(acc[j], a0, a1, a2, a3, bq[j][2 * st], bq[j][2 * st + 1]);
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

// softmax over positions per (token, head); p = softmax(s) * norm_v, bf16, zero-padded
__global__ void softmax_kernel(const SoftmaxArgs a) {
    __shared__ float red[32];
    const int m = blockIdx.y, h = blockIdx.x;
    const int tn = a.pos[m] + 1;
    const float *s = a.S + ((int64_t)m * a.nh + h) * a.Tpad;
    bf16 *p = a.P + ((int64_t)m * a.nhp + h) * a.Tpad;
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
    for (int t = threadIdx.x; t < tn; t += blockDim.x) sum += __expf(s[t] - mx);
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    sum = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) sum += red[i];
    const float inv = 1.0f / sum;
    for (int t = threadIdx.x; t < a.Tpad; t += blockDim.x)
        p[t] = __float2bfloat16_rn(t < tn ? __expf(s[t] - mx) * inv * vn[t] : 0.0f);
}

// zero the padded head rows of P (heads nh..nhp-1) once per call
__global__ void zero_rows_kernel(bf16 *P, int nh, int nhp, int Tpad) {
    const int m = blockIdx.y, h = nh + blockIdx.x;
    bf16 *p = P + ((int64_t)m * nhp + h) * Tpad;
    for (int t = threadIdx.x; t < Tpad; t += blockDim.x) p[t] = __float2bfloat16_rn(0.0f);
}

// ---------------------------------------------------------------------------
// Decode values: u~[h, i] = sum_t p[h, t] * centroid(code_v[t, i]).
// CTA = 64 dims x all heads; 4 warps x 16 dims; positions in tiles of 32.
template <int MT>  // m-tiles of 16 heads
__global__ void __launch_bounds__(128) values_kernel(const ValueArgs a) {
    __shared__ uint32_t lut[256];
    __shared__ __align__(16) bf16 tile[32][72];  // 32 positions x 64 dims (+8 pad)
    build_lut(lut, a.vcent);
    const int m = blockIdx.y, d0 = blockIdx.x * 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int tn = a.pos[m] + 1;
    const int64_t rowbase = ((int64_t)a.slot[m] * a.L + a.layer) * a.B;
    const uint8_t *codes = a.vcodes + rowbase * a.vpl + d0 / 2;
    const bf16 *P = a.P + (int64_t)m * a.nhp * a.Tpad;
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
            uint32_t o[8];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                o[b] = lut[(w.x >> (8 * b)) & 0xff];
                o[4 + b] = lut[(w.y >> (8 * b)) & 0xff];
            }
            uint4 *dst = reinterpret_cast<uint4 *>(&tile[pr][part * 16]);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
        __syncthreads();
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {  // two k16 steps (positions)
            const int tk = tt * 32 + ks * 16;
            // B fragments (k = positions, n = 16 dims of this warp) via ldmatrix.trans
            uint32_t b0, b1, b2, b3;
            {
                const int r = ks * 16 + (lane & 15);
                const int col = warp * 16 + ((lane >> 4) << 3);
                ldsm_x4_t(smem_u32(&tile[r][col]), b0, b1, b2, b3);
            }
#pragma unroll
            for (int i = 0; i < MT; ++i) {
                const bf16 *pr0 = P + (int64_t)(i * 16 + g) * a.Tpad + tk;
                const bf16 *pr1 = P + (int64_t)(i * 16 + g + 8) * a.Tpad + tk;
                const uint32_t a0 = *reinterpret_cast<const uint32_t *>(pr0 + 2 * c);
                const uint32_t a1 = *reinterpret_cast<const uint32_t *>(pr1 + 2 * c);
                const uint32_t a2 = *reinterpret_cast<const uint32_t *>(pr0 + 8 + 2 * c);
                const uint32_t a3 = *reinterpret_cast<const uint32_t *>(pr1 + 8 + 2 * c);
                mma_bf16(acc[i][0], a0, a1, a2, a3, b0, b1);
                mma_bf16(acc[i][1], a0, a1, a2, a3, b2, b3);
            }
        }
    }
    // write u~ as bf16 [m][h][kvd]
    bf16 *U = a.U + (int64_t)m * a.nh * a.kvd;
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow) {
            const int h = i * 16 + g + hrow * 8;
            if (h >= a.nh) continue;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int d = d0 + warp * 16 + j * 8 + c * 2;
                *reinterpret_cast<uint32_t *>(U + (int64_t)h * a.kvd + d) =
                    pack_bf16(acc[i][j][hrow * 2], acc[i][j][hrow * 2 + 1]);
            }
        }
}

// ---------------------------------------------------------------------------
// Prefill: dequantize codes of every prompt token to bf16 centroid vectors.
__global__ void centroids_kernel(const uint8_t *codes, int pl, int64_t row_stride_codes, const int32_t *slot,
                                 const int32_t *pos, int L, int B, int layer, const float *cent, int kvd, int M,
                                 bf16 *out) {
    __shared__ uint32_t lut[256];
    build_lut(lut, cent);
    __syncthreads();
    const int m = blockIdx.x;
    const int64_t row = ((int64_t)slot[m] * L + layer) * B + pos[m];
    const uint8_t *c = codes + row * pl;
    uint32_t *o = reinterpret_cast<uint32_t *>(out + (int64_t)m * kvd);
    for (int b = threadIdx.x; b < kvd / 2; b += blockDim.x) o[b] = lut[c[b]];
    (void)row_stride_codes;
}
__global__ void gather_norms_kernel(const float *norms, const int32_t *slot, const int32_t *pos, int L, int B,
                                    int layer, int M, float *out) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    out[m] = norms[((int64_t)slot[m] * L + layer) * B + pos[m]];
}

// Causal flash attention over one sequence's prompt (rows base..base+T-1),
// bf16 Q/K/V, f32 online softmax. CTA = 64 queries x one head, 4 warps x 16.
template <int HD>
__global__ void __launch_bounds__(128) fa_kernel(const FlashArgs a) {
    constexpr int KT = 64;
    __shared__ __align__(16) bf16 sK[KT][HD + 8];
    __shared__ __align__(16) bf16 sV[KT][HD + 8];
    const int seq = blockIdx.z, h = blockIdx.y, qt0 = blockIdx.x * 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, c = lane & 3;
    const int T = a.T;
    if (qt0 >= T) return;
    const int kvh = h * a.nkv / a.nh;
    const int64_t base = (int64_t)seq * T;
    const int q0 = qt0 + warp * 16;
    // Q fragments (rows q0+g, q0+g+8), all HD/16 k-steps
    uint32_t qf[HD / 16][4];
    {
        const int ra = min(q0 + g, T - 1), rb = min(q0 + g + 8, T - 1);
        const bf16 *qa = a.Q + (base + ra) * a.ldq + h * HD, *qb = a.Q + (base + rb) * a.ldq + h * HD;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
            qf[ks][0] = *reinterpret_cast<const uint32_t *>(qa + ks * 16 + 2 * c);
            qf[ks][1] = *reinterpret_cast<const uint32_t *>(qb + ks * 16 + 2 * c);
            qf[ks][2] = *reinterpret_cast<const uint32_t *>(qa + ks * 16 + 8 + 2 * c);
            qf[ks][3] = *reinterpret_cast<const uint32_t *>(qb + ks * 16 + 8 + 2 * c);
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
            uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
            if (t < T) {
                kv = *reinterpret_cast<const uint4 *>(a.K + (base + t) * a.ldk + kvh * HD + cc);
                vv = *reinterpret_cast<const uint4 *>(a.V + (base + t) * a.ldk + kvh * HD + cc);
            }
            *reinterpret_cast<uint4 *>(&sK[r][cc]) = kv;
            *reinterpret_cast<uint4 *>(&sV[r][cc]) = vv;
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
                uint32_t b0, b1, b2, b3;
                const int r = j2 * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int col = ks * 16 + (((lane >> 3) & 1) << 3);
                ldsm_x4(smem_u32(&sK[r][col]), b0, b1, b2, b3);
                mma_bf16(s[2 * j2], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
                mma_bf16(s[2 * j2 + 1], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b2, b3);
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
        // O += P V
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk) {
            const uint32_t p0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
            const uint32_t p1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
            const uint32_t p2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            const uint32_t p3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int j2 = 0; j2 < HD / 16; ++j2) {
                uint32_t b0, b1, b2, b3;
                const int r = kk * 16 + (lane & 15);
                const int col = j2 * 16 + ((lane >> 4) << 3);
                ldsm_x4_t(smem_u32(&sV[r][col]), b0, b1, b2, b3);
                mma_bf16(o[2 * j2], p0, p1, p2, p3, b0, b1);
                mma_bf16(o[2 * j2 + 1], p0, p1, p2, p3, b2, b3);
            }
        }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        const int qi = q0 + g + hr * 8;
        if (qi >= T) continue;
        const float inv = 1.0f / lrow[hr];
        bf16 *dst = a.O + (base + qi) * a.ldo + h * HD;
#pragma unroll
        for (int j = 0; j < HD / 8; ++j)
            *reinterpret_cast<uint32_t *>(dst + j * 8 + 2 * c) = pack_bf16(o[j][hr * 2] * inv, o[j][hr * 2 + 1] * inv);
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
    if (a.nhp > a.nh) zero_rows_kernel<<<dim3(a.nhp - a.nh, a.M), 128, 0, s>>>(a.P, a.nh, a.nhp, a.Tpad);
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
                      const float *cent, int kvd, int M, bf16 *out, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    centroids_kernel<<<M, 128, 0, s>>>(codes, pl, 0, slot, pos, L, B, layer, cent, kvd, M, out);
    return cudaGetLastError();
}
cudaError_t gather_norms(const float *norms, const int32_t *slot, const int32_t *pos, int L, int B, int layer, int M,
                         float *out, cudaStream_t s) {
    if (M <= 0) return cudaSuccess;
    gather_norms_kernel<<<(M + 255) / 256, 256, 0, s>>>(norms, slot, pos, L, B, layer, M, out);
    return cudaGetLastError();
}
cudaError_t flash_prefill(const FlashArgs &a, cudaStream_t s) {
    dim3 grid((a.T + 63) / 64, a.nh, a.n_seq);
    switch (a.hd) {
        case 64: fa_kernel<64><<<grid, 128, 0, s>>>(a); break;
        case 128: fa_kernel<128><<<grid, 128, 0, s>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace attn
}  // namespace kg
