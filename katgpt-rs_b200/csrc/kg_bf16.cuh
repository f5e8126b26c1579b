// kg_bf16.cuh — interfaces of the BF16 tensor-core path (kg_bf16.cu: GEMMs, norms, TwELL, small kernels).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace kg {
namespace bf {

using bf16 = __nv_bfloat16;

enum Epi : int {
    EPI_F32 = 0,           // C = acc
    EPI_F32_RESID = 1,     // C = acc + R
    EPI_RELU = 2,          // Cb(+Cb2) = split(max(acc, 0)); row_alive[row] += #(acc > 0)
    EPI_OUT = 3,           // Cb(+Cb2) = split(acc)
    EPI_F32_ROWSCALE = 4,  // C = acc * row_scale[row]
    EPI_OUT_ROWSCALE = 5,  // Cb(+Cb2) = split(acc * row_scale[row])
    EPI_BF16_SPLIT = 6     // Cb(+Cb2) = bf16 hi / lo split of acc, whatever the operand type
};
enum DType : int { DT_BF16 = 0, DT_F16 = 1 };

// C[M x N] = A[M x K] * B[N x K]^T (+ epilogue), A/B row-major with K contiguous,
// f32 accumulation. Operands are bf16 or f16 (`dtype`, the same for A and B).
// A2 / B2 optional "lo" parts: an operand is then hi + lo (a split of an f32
// value into two 16-bit floats), and the product is hi*hi + lo*hi + hi*lo,
// which carries about 16 (bf16) or 22 (f16) mantissa bits. Outputs Cb / Cb2
// receive the hi / lo split of the result (Cb2 may be null).
// Batched over blockIdx.z with element strides sA/sB/sC/sR/sCb/sRs.
struct Gemm {
    const void *A, *A2;
    int64_t lda, sA;
    const void *B, *B2;
    int64_t ldb, sB;
    int M, N, K, batch;
    int epi, dtype;
    float *C;
    int64_t ldc, sC;
    const float *R;
    int64_t ldr, sR;
    void *Cb, *Cb2;
    int64_t ldcb, sCb;
    int *row_alive;
    const float *row_scale;
    int64_t sRs;
    float *C2;  // EPI_F32_RESID: optional second copy of C (same ldc / sC)
    // EPI_F32: optional f16 hi / lo copy of columns [0, qcols) into Qh / Ql
    // (row stride ldq); EPI_F32_RESID: optional Dacc[i] += C[i] - R3[i] (same
    // indexing as C). mma.sync path only (M < 256).
    __half *Qh, *Ql;
    int64_t ldq;
    int qcols;
    float *Dacc;
    const float *R3;
    // split-K (1, 2, 4 or 8; 0 = chosen from the shape): the K range is cut
    // into ksplit parts computed by the CTAs of one thread-block cluster and
    // reduced through distributed shared memory in part order (deterministic)
    int ksplit;
    // tcgen05 decode-sized GEMMs: f32 workspace for split-K partials (null: no
    // split), ws_bytes its size
    float *ws;
    int64_t ws_bytes;
};

cudaError_t gemm(const Gemm &g, cudaStream_t s);

// x[m, :] = wte[tok[m], :] + wpe[pos[m], :] (bf16 tables, f32 out); zero_rows
// (optional, [M][n]) is cleared on the way
cudaError_t embed(const int32_t *tok, const int32_t *pos, const bf16 *wte, const bf16 *wpe, int n, int M,
                  float *x, cudaStream_t s, float *zero_rows = nullptr);
// per row: y = x / sqrt(mean(x^2) + 1e-5); `twice` applies it twice (sp_kv double norm).
// Writes f32 (if yf) and the bf16 hi/lo split (if yb / yb2). In-place allowed (yf == x).
// zero_count (optional, [M]) is cleared on the way (the next ReLU GEMM's alive counts).
// gamma (optional, [n]): rmsnorm_with_gamma, y = gamma * (x * inv_rms) (math.rs:218-233).
cudaError_t rmsnorm(const float *x, int n, int M, float *yf, bf16 *yb, bf16 *yb2, bool twice, cudaStream_t s,
                    int *zero_count = nullptr, const float *gamma = nullptr);
// f32 -> bf16 hi (+ lo) split (strided rows)
cudaError_t to_bf16(const float *x, int64_t ldx, int n, int M, bf16 *y, bf16 *y2, int64_t ldy, cudaStream_t s);
// f32 -> f16 hi + lo split (strided rows)
cudaError_t to_f16(const float *x, int64_t ldx, int n, int M, __half *hi, __half *lo, int64_t ldy, cudaStream_t s);
// f32 -> f16 hi + lo split of a flat array
cudaError_t f32_to_f16_split(const float *x, int64_t count, __half *hi, __half *lo, cudaStream_t s);
// round a flat f32 array to bf16 (nearest-even)
cudaError_t f32_to_bf16_flat(const float *x, int64_t count, bf16 *y, cudaStream_t s);
// delta routing (src/transformer.rs:1707-1765, 2129-2158) for one layer l:
// delta += x - xr; at l % 4 == 3 route over b = l/4 zeroed blocks + delta, then zero delta.
cudaError_t delta_route(float *x, const float *xr, float *delta, const float *query, const float *normw,
                        int n, int M, int layer, cudaStream_t s);
// TwELL (math.rs:315-355): for rows whose alive fraction <= 1 - threshold, recompute
// out = sum over alive j of h[j] * W2[:, j] + resid (gather over W2^T rows) in f32.
// Benchmark hook: replace post-ReLU hidden activations by a Bernoulli(keep)
// mask with |N(0,1)| survivors (the hidden activation is post-ReLU, and the
// gather counts only entries > 0; deterministic per layer, slot, position) and
// recount alive entries.
cudaError_t mlp_hook(bf16 *hid, bf16 *hid2, int *row_alive, const int32_t *slot, const int32_t *pos, int m, int M,
                     float keep, uint64_t seed, int layer, cudaStream_t s);
cudaError_t twell_sparse_w2(const bf16 *hidden, const bf16 *hidden_lo, const int *row_alive, const bf16 *w2t, const float *resid,
                            float *out, int n, int m, int M, float threshold, cudaStream_t s);
// softmax_scaled (math.rs:36-50) per row of logits [M x V], rows `ld` floats apart
cudaError_t softmax_rows(const float *logits, float *probs, int V, int M, int64_t ld, float inv_temp, cudaStream_t s);

}  // namespace bf
}  // namespace kg
