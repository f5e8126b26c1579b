// kg_attn.cu — attention kernels of the BF16 tensor-core path other than the
// quantized-KV decode (kg_tqattn.cu):
//   - prefill over the TurboQuant cache: the prompt's codes are dequantized
//     once (centroids_kernel, then k~ = norm * c R^T as a GEMM in kg_big.cu)
//     and causal flash attention runs over f16 hi/lo rows (fa_kernel);
//   - standard attention (AttentionMode::Standard): bf16 K/V cache rows
//     (kv_store_std_kernel) and a streaming decode kernel (std_decode_kernel).
//
// Semantics: forward_quantized attention (src/transformer.rs:4123-4141 over
// the dequantized cache), attention_head softmax with 1/sqrt(head_dim)
// (src/transformer.rs:333-389).
#include <cuda_bf16.h>

#include <algorithm>

#include "kg_attn.cuh"
#include "kg_dev.cuh"
#include "kg_pdl.cuh"

namespace kg {
namespace attn {
namespace {

using bf16 = __nv_bfloat16;

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
// Standard attention over a bf16 K/V cache (AttentionMode::Standard,
// attention_head, src/transformer.rs:333-389; cache layout of
// MultiLayerKVCache, crates/katgpt-transformer/src/kv_cache.rs:8-124, kept as
// [slot][layer][pos][kv_dim] bf16 on the device).

// New K/V rows of a step into the bf16 cache; for prefill also the f16 hi/lo
// split of the bf16-rounded rows (the flash kernel's operands), so prefill and
// decode attend over the same cached values.
__global__ void kv_store_std_kernel(const float *qkv, int64_t ldx, int64_t koff, int64_t voff, int kvd,
                                    const int32_t *slot, const int32_t *pos, int L, int B, int layer, bf16 *kc,
                                    bf16 *vc, __half *kt, __half *kt2, __half *vt, __half *vt2, const int32_t *ptab,
                                    int maxp, int S, int n_pages, int *err) {
    pdl_wait();
    const int m = blockIdx.x;
    int64_t krow = ((int64_t)slot[m] * L + layer) * B + pos[m], vrow = krow;
    if (ptab) {  // PagedKVCache::write_kv (kv_cache.rs:298-309): the page that holds pos
        const int pg = ptab[((int64_t)layer * S + slot[m]) * maxp + (pos[m] >> 4)];
        if (pg < 0 || pg >= n_pages) {  // no page: nothing is written, the call reports it
            if (threadIdx.x == 0 && err) atomicExch(err, 1);
            return;
        }
        krow = (int64_t)pg * 32 + (pos[m] & 15);
        vrow = krow + 16;
    }
    for (int j = threadIdx.x; j < kvd; j += blockDim.x) {
        const bf16 k = __float2bfloat16_rn(qkv[(int64_t)m * ldx + koff + j]);
        const bf16 v = __float2bfloat16_rn(qkv[(int64_t)m * ldx + voff + j]);
        kc[krow * kvd + j] = k;
        vc[vrow * kvd + j] = v;
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
    // paged cache: row t of this sequence's layer lives at page tab[t / 16]
    const int32_t *tab = a.ptab ? a.ptab + ((int64_t)a.layer * a.S + a.slot[m]) * a.maxp : nullptr;
    if (tab) {
        bool bad = false;
        for (int q = threadIdx.x; q <= (tn - 1) >> 4; q += blockDim.x)
            bad |= q >= a.maxp || tab[q] < 0 || tab[q] >= a.n_pages;
        if (__syncthreads_or(bad)) {  // CTA-uniform: no page to read, the call reports it
            if (threadIdx.x == 0 && a.err) atomicExch(a.err, 1);
            return;
        }
    }
    auto krow = [&](int t) -> const bf16 * {
        if (tab) return a.kc + ((int64_t)tab[t >> 4] * 32 + (t & 15)) * a.kvd + kh * HD + lane * DPL;
        return K + (int64_t)t * a.kvd;
    };
    auto vrow = [&](int t) -> const bf16 * {
        if (tab) return a.vc + ((int64_t)tab[t >> 4] * 32 + 16 + (t & 15)) * a.kvd + kh * HD + lane * DPL;
        return Vp + (int64_t)t * a.kvd;
    };
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
                load(krow(t), kf[u]);
                load(vrow(t), vf[u]);
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
    const int kend = a.bidir ? T : min(T, qt0 + 64);
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
        if (!a.bidir && k0 > q0 + 15) continue;  // whole tile in the future for this warp
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
                    float v = ((a.bidir || kj <= qi) && kj < T) ? s[j][hr * 2 + e] * sl2 : -INFINITY;
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
    {
        cudaError_t e = dev::smem(fa_kernel<HD>, smem);
        if (e != cudaSuccess) return e;
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

cudaError_t kv_store_std(const float *qkv, int64_t ldx, int64_t koff, int64_t voff, int kvd, int M,
                         const int32_t *slot, const int32_t *pos, int L, int B, int layer, bf16 *kc, bf16 *vc,
                         __half *kt, __half *kt2, __half *vt, __half *vt2, cudaStream_t s, const int32_t *ptab,
                         int maxp, int S, int n_pages, int *err) {
    if (M <= 0) return cudaSuccess;
    return launch_pdl(kv_store_std_kernel, dim3(M), dim3(256), 0, s, qkv, ldx, koff, voff, kvd, slot, pos, L, B, layer,
                      kc, vc, kt, kt2, vt, vt2, ptab, maxp, S, n_pages, err);
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
