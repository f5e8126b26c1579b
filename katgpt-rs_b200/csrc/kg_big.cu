// kg_big.cu — the BF16 tensor-core forward for full-size models (host side).
//
// Reproduces forward_quantized (src/transformer.rs:4042-4233; KG_KV_TQ) and
// forward_sp_kv_quant (src/sp_kv/forward.rs:610-822; KG_KV_SPKV_TQ) on f32
// arithmetic over bf16-rounded weights, with bf16 GEMM inputs:
//   per layer: RMSNorm -> fused QKV GEMM (Kog layout: [Wq; Wk; Wv] rows,
//   weights.rs:236-249) -> exact TurboQuant encode of K and V into the code
//   arena -> attention over the codes -> Wo GEMM + residual -> RMSNorm ->
//   W1 GEMM + ReLU (+ alive count) -> W2 GEMM + residual (TwELL sparse rows
//   recomputed by gather) -> delta routing; then lm_head GEMM (+ softmax).
// Decode (T = 1) attends in the rotated domain straight from the codes;
// prefill (T > 1 from position 0) dequantizes the prompt's K/V once and runs
// causal flash attention; T > 1 from other positions runs decode rows.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "kg_attn.cuh"
#include "kg_pdl.cuh"
#include "kg_umma.cuh"
#include "kg_bf16.cuh"
#include "kg_internal.h"

namespace kg {

using bf::bf16;

namespace {

__global__ void expand_tokens_kernel(const int32_t *seq_ids, const int32_t *start_pos, int T, int n_seq, int B,
                                     int n_slots, int V, const int32_t *tokens, int32_t *slot_of, int32_t *pos_of,
                                     int *err) {
    pdl_wait();
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= n_seq * T) return;
    const int i = m / T, t = m - i * T;
    const int s = seq_ids[i];
    const int p = (start_pos ? start_pos[i] : 0) + t;
    const int tok = tokens[m];
    if (s < 0 || s >= n_slots || p < 0 || p >= B || tok < 0 || tok >= V) {
        atomicExch(err, 1);
        slot_of[m] = 0;
        pos_of[m] = 0;
        return;
    }
    slot_of[m] = s;
    pos_of[m] = p;
}

__global__ void transpose_bf16_kernel(const bf16 *a, int rows, int cols, bf16 *t) {
    __shared__ bf16 tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int row = by + r, col = bx + threadIdx.x;
        if (row < rows && col < cols) tile[r][threadIdx.x] = a[(int64_t)row * cols + col];
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int row = bx + r, col = by + threadIdx.x;
        if (row < cols && col < rows) t[(int64_t)row * rows + col] = tile[threadIdx.x][r];
    }
}

// One position offset t of a multi-position call from arbitrary start
// positions: row i = (sequence i, position start_pos[i] + t, token i*T + t).
__global__ void expand_offset_kernel(const int32_t *seq_ids, const int32_t *start_pos, int T, int t, int n_seq, int B,
                                     int n_slots, int V, const int32_t *tokens, int32_t *slot_of, int32_t *pos_of,
                                     int32_t *tok_of, int *err) {
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_seq) return;
    const int s = seq_ids[i], p = start_pos[i] + t, tok = tokens[(int64_t)i * T + t];
    if (s < 0 || s >= n_slots || p < 0 || p >= B || tok < 0 || tok >= V) {
        atomicExch(err, 1);
        slot_of[i] = 0;
        pos_of[i] = 0;
        tok_of[i] = 0;
        return;
    }
    slot_of[i] = s;
    pos_of[i] = p;
    tok_of[i] = tok;
}

__global__ void sanitize_tokens_kernel(const int32_t *tokens, int M, int V, int32_t *out) {
    pdl_wait();
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m < M) out[m] = min(max(tokens[m], 0), V - 1);
}

template <typename T>
cudaError_t dalloc(T **p, size_t count, std::vector<void *> &owned) {
    void *q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T));
    if (e != cudaSuccess) return e;
    owned.push_back(q);
    *p = static_cast<T *>(q);
    return cudaSuccess;
}

#define BIG_TRY(call)                            \
    do {                                         \
        cudaError_t e_ = (call);                 \
        if (e_ != cudaSuccess) return e_;        \
    } while (0)

}  // namespace

int big_supported(const kg_config &c, std::string &why) {
    if (c.weight_dtype != KG_W_BF16) return why = "the tensor-core path runs bf16 weights (KG_W_BF16)", -1;
    if (c.kv_mode == KG_KV_SQ) return why = "the SpectralQuant forward runs on the exact micro path", -1;
    if (c.kv_mode != KG_KV_F32)
        for (int b : {c.key_bits, c.val_bits})
            if (b != 3 && b != 4) return why = "the bf16 path packs 3/4-bit codes", -1;
    if (c.kv_mode != KG_KV_F32 && c.block_size > 6144) return why = "quantized-KV decode attention: block_size <= 6144", -1;
    if (c.n_kv_head < 1 || c.n_head % c.n_kv_head) return why = "n_head must be a multiple of n_kv_head", -1;
    const int kvd = c.n_kv_head * c.head_dim;
    if (kvd % 64) return why = "kv_dim must be a multiple of 64", -1;
    if (c.head_dim != 64 && c.head_dim != 128) return why = "head_dim must be 64 or 128", -1;
    if (c.n_embd % 32 || c.mlp_hidden % 32) return why = "n_embd and mlp_hidden must be multiples of 32", -1;
    if (c.n_head > 32) return why = "at most 32 heads", -1;
    if ((c.n_head + 15) / 16 > 2) return why = "at most 32 heads", -1;
    return 0;
}

cudaError_t big_init(kg_ctx *ctx) {
    BigState &g = ctx->big;
    const kg_config &c = ctx->cfg;
    const int64_t n = ctx->n, kvd = ctx->kvd, m = ctx->m, V = ctx->V, L = ctx->L, B = ctx->B, S = c.max_seqs;
    // workspace rows: prefill runs in passes of whole sequences up to this many
    // tokens (large passes keep the tcgen05 GEMMs' last wave small); about
    // 75 KB per row at n_embd 768, 200 KB at 2048
    g.ws_tokens = std::max<int64_t>(S, n <= 2048 ? 32768 : 16384);
    g.Tpad = (B + 31) / 32 * 32;
    auto &own = ctx->allocs;
    // weights (bf16), one block in the flat reference order
    g.nbf = V * n + B * n + L * (2 * n * n + 2 * kvd * n + 2 * m * n) + V * n;
    BIG_TRY(dalloc(&g.wall, g.nbf, own));
    g.wte = g.wall;
    g.wpe = g.wte + V * n;
    g.layers = g.wpe + B * n;
    g.lm = g.layers + L * (2 * n * n + 2 * kvd * n + 2 * m * n);
    BIG_TRY(dalloc(&g.w2t, L * m * n, own));
    BIG_TRY(dalloc(&g.dq, L * n, own));
    BIG_TRY(dalloc(&g.dn, L * n, own));
    BIG_TRY(dalloc(&g.ag, L * n, own));
    BIG_TRY(dalloc(&g.mg, L * n, own));
    BIG_TRY(dalloc(&g.pdelta, S * n, own));
    g.std_kv = c.kv_mode == KG_KV_F32 || c.kv_mode == KG_KV_PAGED;
    g.paged = c.kv_mode == KG_KV_PAGED;  // K/V rows in the page pool instead (kg_paged.cu)
    if (g.std_kv && !g.paged) {  // standard attention: bf16 K/V arena
        BIG_TRY(dalloc(&g.kcache, (size_t)S * L * B * kvd, own));
        BIG_TRY(dalloc(&g.vcache, (size_t)S * L * B * kvd, own));
    } else {
        BIG_TRY(dalloc(&g.rot_h, kvd * kvd, own));
        BIG_TRY(dalloc(&g.rot_l, kvd * kvd, own));
        BIG_TRY(dalloc(&g.rot_th, kvd * kvd, own));
        BIG_TRY(dalloc(&g.rot_tl, kvd * kvd, own));
        // code arena
        BIG_TRY(dalloc(&g.kcodes, (size_t)S * L * B * ctx->kpl, own));
        BIG_TRY(dalloc(&g.vcodes, (size_t)S * L * B * ctx->vpl, own));
        BIG_TRY(dalloc(&g.knorm, (size_t)S * L * B, own));
        BIG_TRY(dalloc(&g.vnorm, (size_t)S * L * B, own));
    }
    // workspace (ws_tokens rows)
    const int64_t W = g.ws_tokens;
    const int64_t nqkv = n + 2 * kvd;
    BIG_TRY(dalloc(&g.x, W * n, own));
    BIG_TRY(dalloc(&g.xr, W * n, own));
    BIG_TRY(dalloc(&g.xr2, W * n, own));
    BIG_TRY(dalloc(&g.delta, W * n, own));
    BIG_TRY(dalloc(&g.attf, W * n, own));
    BIG_TRY(dalloc(&g.xb, W * n, own));
    BIG_TRY(dalloc(&g.xb2, W * n, own));
    BIG_TRY(dalloc(&g.attb, W * n, own));
    BIG_TRY(dalloc(&g.attb2, W * n, own));
    BIG_TRY(dalloc(&g.qkv, W * nqkv, own));
    BIG_TRY(dalloc(&g.qh, W * n, own));
    BIG_TRY(dalloc(&g.ql, W * n, own));
    BIG_TRY(dalloc(&g.hid, W * m, own));
    BIG_TRY(dalloc(&g.hid2, W * m, own));
    BIG_TRY(dalloc(&g.alive, W, own));
    BIG_TRY(dalloc(&g.slot_of, W, own));
    BIG_TRY(dalloc(&g.pos_of, W, own));
    BIG_TRY(dalloc(&g.tok_of, W, own));
    // prefill attention scratch
    BIG_TRY(dalloc(&g.cent, W * kvd, own));
    BIG_TRY(dalloc(&g.cent2, W * kvd, own));
    BIG_TRY(dalloc(&g.kt, W * kvd, own));
    BIG_TRY(dalloc(&g.kt2, W * kvd, own));
    BIG_TRY(dalloc(&g.vt, W * kvd, own));
    BIG_TRY(dalloc(&g.vt2, W * kvd, own));
    BIG_TRY(dalloc(&g.nrm, W, own));
    BIG_TRY(dalloc(&g.xn, 2 * W * kvd, own));
    BIG_TRY(dalloc(&g.skip, 2 * W, own));
    BIG_TRY(dalloc(&g.xnh, 2 * W * kvd, own));
    BIG_TRY(dalloc(&g.xnl, 2 * W * kvd, own));
    BIG_TRY(dalloc(&g.yrot, 2 * W * kvd, own));
    // decode attention scratch (max_seqs rows)
    BIG_TRY(dalloc(&g.qrot, S * ctx->nh * kvd, own));
    BIG_TRY(dalloc(&g.qrot2, S * ctx->nh * kvd, own));
    BIG_TRY(dalloc(&g.U, S * ctx->nh * kvd, own));
    BIG_TRY(dalloc(&g.U2, S * ctx->nh * kvd, own));
    if (g.std_kv) {
        BIG_TRY(cudaStreamSynchronize(ctx->stream));
        return cudaSuccess;
    }
    g.Sp = attn::tq_padded_len((int)B);
    BIG_TRY(dalloc(&g.pe, S * ctx->nh * g.Sp, own));
    BIG_TRY(dalloc(&g.pmax, S * (g.Sp / 16) * ctx->nh, own));
    BIG_TRY(dalloc(&g.psum, S * (g.Sp / 16) * ctx->nh, own));
    BIG_TRY(dalloc(&g.linv, S * ctx->nh, own));
    {
        constexpr size_t kSplitWsFloats = (size_t)8 << 20;  // 32 MiB: split-K partials of decode GEMMs
        BIG_TRY(dalloc(&g.splitk_ws, kSplitWsFloats, own));
        g.splitk_ws_bytes = (int64_t)kSplitWsFloats * 4;
    }
    // centroid tables
    BIG_TRY(dalloc(&g.kcent, 16, own));
    BIG_TRY(dalloc(&g.vcent, 16, own));
    std::vector<float> kc(16, 0.0f), vc(16, 0.0f);
    std::copy(ctx->h_kc.begin(), ctx->h_kc.end(), kc.begin());
    std::copy(ctx->h_vc.begin(), ctx->h_vc.end(), vc.begin());
    BIG_TRY(cudaMemcpy(g.kcent, kc.data(), 64, cudaMemcpyHostToDevice));
    BIG_TRY(cudaMemcpy(g.vcent, vc.data(), 64, cudaMemcpyHostToDevice));
    // f16 hi/lo splits of the rotation for the tensor-core GEMMs
    BIG_TRY(bf::f32_to_f16_split(ctx->rot, kvd * kvd, g.rot_h, g.rot_l, ctx->stream));
    BIG_TRY(bf::f32_to_f16_split(ctx->rot_t, kvd * kvd, g.rot_th, g.rot_tl, ctx->stream));
    BIG_TRY(cudaStreamSynchronize(ctx->stream));
    return cudaSuccess;
}

cudaError_t big_reset(kg_ctx *ctx, int64_t slot0, int64_t nslots) {
    BigState &g = ctx->big;
    const size_t rows = (size_t)ctx->L * ctx->B;
    cudaStream_t s = ctx->stream;
    if (g.paged) return cudaSuccess;  // pages are zeroed when they are handed out
    if (g.std_kv) {
        const size_t e = rows * ctx->kvd;
        BIG_TRY(cudaMemsetAsync(g.kcache + slot0 * e, 0, nslots * e * 2, s));
        BIG_TRY(cudaMemsetAsync(g.vcache + slot0 * e, 0, nslots * e * 2, s));
        return cudaStreamSynchronize(s);
    }
    BIG_TRY(cudaMemsetAsync(g.kcodes + slot0 * rows * ctx->kpl, 0, nslots * rows * ctx->kpl, s));
    BIG_TRY(cudaMemsetAsync(g.vcodes + slot0 * rows * ctx->vpl, 0, nslots * rows * ctx->vpl, s));
    BIG_TRY(cudaMemsetAsync(g.knorm + slot0 * rows, 0, nslots * rows * 4, s));
    BIG_TRY(cudaMemsetAsync(g.vnorm + slot0 * rows, 0, nslots * rows * 4, s));
    return cudaStreamSynchronize(s);
}

// Convert flat f32 weights [offset, offset+count) (device pointer) into the bf16 block.
cudaError_t big_upload_chunk(kg_ctx *ctx, const float *dsrc, int64_t offset, int64_t count) {
    BigState &g = ctx->big;
    if (offset < 0 || offset + count > g.nbf) return cudaErrorInvalidValue;
    return bf::f32_to_bf16_flat(dsrc, count, g.wall + offset, ctx->stream);
}

// The f32 tail of the flat layout (delta-routing query and norm, attention and
// MLP norm gammas: [4][L][n]) and W2^T for the TwELL gather.
cudaError_t big_finish_upload(kg_ctx *ctx, const float *dq_dn_dev) {
    BigState &g = ctx->big;
    const int64_t n = ctx->n, kvd = ctx->kvd, m = ctx->m, L = ctx->L;
    cudaStream_t s = ctx->stream;
    const int64_t per_layer = 2 * n * n + 2 * kvd * n + 2 * m * n;
    if (dq_dn_dev) {
        BIG_TRY(cudaMemcpyAsync(g.dq, dq_dn_dev, L * n * 4, cudaMemcpyDeviceToDevice, s));
        BIG_TRY(cudaMemcpyAsync(g.dn, dq_dn_dev + L * n, L * n * 4, cudaMemcpyDeviceToDevice, s));
        BIG_TRY(cudaMemcpyAsync(g.ag, dq_dn_dev + 2 * L * n, L * n * 4, cudaMemcpyDeviceToDevice, s));
        BIG_TRY(cudaMemcpyAsync(g.mg, dq_dn_dev + 3 * L * n, L * n * 4, cudaMemcpyDeviceToDevice, s));
    }
    for (int64_t l = 0; l < L; ++l) {
        const bf16 *w2 = g.layers + l * per_layer + 2 * n * n + 2 * kvd * n + m * n;  // [n x m]
        dim3 tb(32, 8), gb((m + 31) / 32, (n + 31) / 32);
        transpose_bf16_kernel<<<gb, tb, 0, s>>>(w2, (int)n, (int)m, g.w2t + l * m * n);
    }
    BIG_TRY(cudaGetLastError());
    return cudaStreamSynchronize(s);
}

namespace {
// counter-based normal generator for synthetic benchmark weights
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
__global__ void random_bf16_kernel(bf16 *w, int64_t count, uint64_t seed, float std_) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t r = mix64(seed ^ mix64((uint64_t)i));
        float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
        float u2 = ((float)((r >> 16) & 0xFFFFFF)) * (1.0f / 16777216.0f);
        float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        w[i] = __float2bfloat16_rn(z * std_);
    }
}
__global__ void fill_kernel(float *p, int64_t count, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}
__global__ void bf16_to_f32_kernel(const bf16 *a, int64_t count, float *o) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        o[i] = __bfloat162float(a[i]);
}
}  // namespace

// Synthetic weights N(0, std) for every bf16 tensor; delta query 0, norm and gammas 1.
cudaError_t big_random_weights(kg_ctx *ctx, uint64_t seed, float std_) {
    BigState &g = ctx->big;
    cudaStream_t s = ctx->stream;
    random_bf16_kernel<<<2048, 256, 0, s>>>(g.wall, g.nbf, seed, std_);
    fill_kernel<<<64, 256, 0, s>>>(g.dq, ctx->L * ctx->n, 0.0f);
    fill_kernel<<<64, 256, 0, s>>>(g.dn, ctx->L * ctx->n, 1.0f);
    fill_kernel<<<64, 256, 0, s>>>(g.ag, ctx->L * ctx->n, 1.0f);
    fill_kernel<<<64, 256, 0, s>>>(g.mg, ctx->L * ctx->n, 1.0f);
    BIG_TRY(cudaGetLastError());
    return big_finish_upload(ctx, nullptr);
}

// bf16 block [offset, offset+count) back to f32 (device pointer)
cudaError_t big_download(kg_ctx *ctx, float *dst, int64_t offset, int64_t count) {
    BigState &g = ctx->big;
    if (offset < 0 || offset + count > g.nbf) return cudaErrorInvalidValue;
    bf16_to_f32_kernel<<<1024, 256, 0, ctx->stream>>>(g.wall + offset, count, dst);
    return cudaGetLastError();
}

namespace {

constexpr int kTwellMaxRows = 32;  // rows per call up to which sparse rows take the gather path

bf::Gemm gemm0() {
    bf::Gemm q;
    std::memset(&q, 0, sizeof(q));
    q.batch = 1;
    q.ksplit = 1;
    return q;
}

// Weight matrices of at least this many elements take the tcgen05 GEMM from
// kMinUmmaRows rows on (decode steps of a wide model); smaller ones keep the
// mma.sync cluster kernel below 256 rows (its fused decode epilogues win
// there).
constexpr int64_t kWideGemm = (int64_t)8 << 20;
constexpr int kMinUmmaRows = 32;

// Launch a GEMM: tcgen05 for prefill-sized M and for decode-sized M over wide
// weights (the decode variant splits K across CTAs through the context's
// workspace: main-stream calls only, one GEMM at a time), otherwise the
// mma.sync kernel (with K split across a cluster when the output has few
// tiles).
cudaError_t gemm_split(kg_ctx *ctx, bf::Gemm q, cudaStream_t s) {
    const bool wide = (int64_t)q.batch * q.N * q.K >= kWideGemm;  // all batches' weights
    if ((q.M >= 256 || (q.M >= kMinUmmaRows && wide)) && umma::supported(q)) {
        if (s != ctx->aux) {
            q.ws = ctx->big.splitk_ws;
            q.ws_bytes = ctx->big.splitk_ws_bytes;
        }
        return umma::gemm(q, s, ctx->d_err);
    }
    q.ksplit = 0;
    return bf::gemm(q, s);
}

// One pass over all layers for M tokens (rows of the workspace). Every GEMM
// operand that is not an exact bf16 weight is a 16-bit hi/lo split, so the
// products keep about f32 accuracy (the 4-bit KV codes are discontinuous in
// their inputs: plain bf16 activations move rotated coordinates across
// codebook boundaries).
cudaError_t run_layers(kg_ctx *ctx, int M, bool prefill, int n_seq, int T, cudaStream_t s) {
    BigState &g = ctx->big;
    const kg_config &c = ctx->cfg;
    const int n = (int)ctx->n, kvd = (int)ctx->kvd, m = (int)ctx->m, L = (int)ctx->L, B = (int)ctx->B;
    const int nh = (int)ctx->nh, hd = (int)ctx->hd;
    const int nqkv = n + 2 * kvd;
    const int64_t per_layer = 2 * (int64_t)n * n + 2 * (int64_t)kvd * n + 2 * (int64_t)m * n;
    const bool spkv = c.kv_mode == KG_KV_SPKV_TQ;
    const float scale = 1.0f / sqrtf((float)hd);
    // g.delta (delta-routing accumulator) was cleared by the embedding kernel
    for (int l = 0; l < L; ++l) {
        const bf16 *wqkv = g.layers + l * per_layer;
        const bf16 *wo = wqkv + (int64_t)(n + 2 * kvd) * n;
        const bf16 *w1 = wo + (int64_t)n * n;
        const bf16 *w2 = w1 + (int64_t)m * n;
        // pre-attention norm: residual xr = norm(x); sp_kv normalises a second time
        // forward_base (standard attention) applies attn_norm_gamma at run time
        // (kog_cpu_fusion, src/transformer.rs:1893-1895); forward_quantized and
        // forward_sp_kv_quant use plain rmsnorm (:4076, sp_kv/forward.rs:649-651)
        // forward_paged normalises twice too, without gammas (src/transformer.rs:3361-3364)
        if (spkv || g.paged) {
            BIG_TRY(bf::rmsnorm(g.x, n, M, g.xr, nullptr, nullptr, false, s));
            BIG_TRY(bf::rmsnorm(g.xr, n, M, nullptr, g.xb, g.xb2, false, s));
        } else {
            BIG_TRY(bf::rmsnorm(g.x, n, M, g.xr, g.xb, g.xb2, false, s, nullptr,
                                g.std_kv ? g.ag + (int64_t)l * n : nullptr));
        }
        // decode steps of fewer than 256 rows over narrow weights run the
        // mma.sync GEMMs, whose epilogues also produce q's f16 split, the
        // attention output's bf16 split and the delta-routing accumulation (no
        // separate kernels); wide models take the tcgen05 GEMMs instead
        const bool fuse = !prefill && M < 256 && (M < kMinUmmaRows || (int64_t)n * n < kWideGemm);
        const bool fuse_q = fuse && !g.std_kv;
        // fused QKV projection
        bf::Gemm q = gemm0();
        q.A = g.xb; q.A2 = g.xb2; q.lda = n; q.B = wqkv; q.ldb = n; q.M = M; q.N = nqkv; q.K = n;
        q.epi = bf::EPI_F32; q.C = g.qkv; q.ldc = nqkv;
        if (fuse_q) {
            q.Qh = g.qh; q.Ql = g.ql; q.ldq = n; q.qcols = n;
        }
        prof_mark(ctx, KG_PROF_GEMM, 0, s);
        BIG_TRY(gemm_split(ctx, q, s));
        prof_mark(ctx, KG_PROF_GEMM, 1, s);
        // decode over codes: q~_h = R[:, head cols] q_h (batched over heads) on the
        // side stream while this stream encodes K and V; joined before attention
        const bool fork = fuse_q && ctx->aux && !ctx->prof;
        auto qrot_gemm = [&](cudaStream_t st) {
            bf::Gemm r = gemm0();
            r.dtype = bf::DT_F16;
            r.A = g.qh; r.A2 = g.ql; r.lda = n; r.sA = hd;
            r.B = g.rot_h; r.B2 = g.rot_l; r.ldb = kvd; r.sB = hd;
            r.M = M; r.N = kvd; r.K = hd; r.batch = nh;
            r.epi = bf::EPI_OUT; r.Cb = g.qrot; r.Cb2 = g.qrot2; r.ldcb = (int64_t)nh * kvd; r.sCb = kvd;
            return gemm_split(ctx, r, st);
        };
        if (fork) {
            BIG_TRY(cudaEventRecord(ctx->ev_fork, s));
            BIG_TRY(cudaStreamWaitEvent(ctx->aux, ctx->ev_fork, 0));
            BIG_TRY(qrot_gemm(ctx->aux));
            BIG_TRY(cudaEventRecord(ctx->ev_join, ctx->aux));
        }
        // TurboQuant encode of K and V into the arena (exact reference order)
        prof_mark(ctx, KG_PROF_ENCODE, 0, s);
        if (g.std_kv) {
            // standard attention: K/V rows into the bf16 cache (and the prompt's
            // f16 hi/lo copies for the flash kernel)
            if (g.paged) {  // write_kv into the sequence's page (kv_cache.rs:298-309)
                bf16 *pool = static_cast<bf16 *>(ctx->paged.pool);
                BIG_TRY(attn::kv_store_std(g.qkv, nqkv, n, n + kvd, kvd, M, g.slot_of, g.pos_of, L, B, l, pool, pool,
                                           prefill ? g.kt : nullptr, g.kt2, g.vt, g.vt2, s, ctx->paged.d_tab,
                                           ctx->paged.maxp, c.max_seqs, (int)ctx->paged.cap, ctx->d_err));
            } else {
                BIG_TRY(attn::kv_store_std(g.qkv, nqkv, n, n + kvd, kvd, M, g.slot_of, g.pos_of, L, B, l, g.kcache,
                                           g.vcache, prefill ? g.kt : nullptr, g.kt2, g.vt, g.vt2, s));
            }
        } else if (M >= 256) {
            // prefill-sized: K and V rows together, exact norms and xn, rotation
            // on the tensor cores, codes with exact recomputation next to the
            // boundaries
            BIG_TRY(tq_norm_split(kvd, M, M, g.qkv, nqkv, n, n + kvd, g.xn, g.xnh, g.xnl, g.skip, g.knorm, g.vnorm,
                                  g.slot_of, g.pos_of, L, B, l, s));
            bf::Gemm rg = gemm0();
            rg.dtype = bf::DT_F16;
            rg.A = g.xnh; rg.A2 = g.xnl; rg.lda = kvd; rg.B = g.rot_h; rg.B2 = g.rot_l; rg.ldb = kvd;
            rg.M = 2 * M; rg.N = kvd; rg.K = kvd;
            rg.epi = bf::EPI_F32; rg.C = g.yrot; rg.ldc = kvd;
            BIG_TRY(gemm_split(ctx, rg, s));
            BIG_TRY(tq_quantize_fixup(kvd, M, M, g.yrot, g.xn, g.skip, ctx->rot, ctx->kb, ctx->vb, c.key_bits,
                                      c.val_bits, g.kcodes, g.vcodes, ctx->kpl, ctx->vpl, g.slot_of, g.pos_of, L, B,
                                      l, nullptr, s));
        } else if (kvd % 128 == 0) {  // decode-sized: the exact tiled encoder is faster
            BIG_TRY(tq_encode_tiled_kv(kvd, c.key_bits, c.val_bits, M, g.qkv, nqkv, n, n + kvd, ctx->rot, ctx->kb,
                                       ctx->vb, g.kcodes, ctx->kpl, g.knorm, g.vcodes, ctx->vpl, g.vnorm, g.slot_of,
                                       g.pos_of, L, B, l, g.xn, g.skip, s));
        } else {
            BIG_TRY(tq_encode_scatter(kvd, c.key_bits, M, g.qkv + n, nqkv, ctx->rot, ctx->kb, g.kcodes, ctx->kpl,
                                      g.knorm, 1, g.slot_of, g.pos_of, L, B, l, s));
            BIG_TRY(tq_encode_scatter(kvd, c.val_bits, M, g.qkv + n + kvd, nqkv, ctx->rot, ctx->vb, g.vcodes,
                                      ctx->vpl, g.vnorm, 1, g.slot_of, g.pos_of, L, B, l, s));
        }
        prof_mark(ctx, KG_PROF_ENCODE, 1, s);
        if ((prefill || !g.std_kv) && !fuse_q) BIG_TRY(bf::to_f16(g.qkv, nqkv, n, M, g.qh, g.ql, n, s));
        if (g.std_kv && !prefill) {
            attn::StdDecodeArgs sa;
            sa.Q = g.qkv; sa.ldq = nqkv; sa.kc = g.kcache; sa.vc = g.vcache; sa.slot = g.slot_of; sa.pos = g.pos_of;
            sa.O = g.attf; sa.ldo = n; sa.M = M; sa.nh = nh; sa.nkv = (int)ctx->nkv; sa.hd = hd; sa.kvd = kvd;
            sa.L = L; sa.B = B; sa.layer = l; sa.scale = scale;
            if (g.paged) {  // read_kv of positions 0..pos through the page table
                sa.kc = sa.vc = static_cast<const bf16 *>(ctx->paged.pool);
                sa.ptab = ctx->paged.d_tab; sa.maxp = ctx->paged.maxp; sa.S = c.max_seqs;
                sa.n_pages = (int)ctx->paged.cap; sa.err = ctx->d_err;
            }
            prof_mark(ctx, KG_PROF_ATTN, 0, s);
            BIG_TRY(attn::std_decode(sa, s));
            prof_mark(ctx, KG_PROF_ATTN, 1, s);
        } else if (prefill) {
            // dequantize the prompt's K and V: k~ = norm * (c R) (standard
            // attention already has its f16 hi / lo rows from kv_store_std)
            for (int kv = 0; kv < (g.std_kv ? 0 : 2); ++kv) {
                const uint8_t *codes = kv ? g.vcodes : g.kcodes;
                const int pl = (int)(kv ? ctx->vpl : ctx->kpl);
                BIG_TRY(attn::centroids(codes, pl, g.slot_of, g.pos_of, L, B, l, kv ? g.vcent : g.kcent, kvd, M,
                                        g.cent, g.cent2, s));
                BIG_TRY(attn::gather_norms(kv ? g.vnorm : g.knorm, g.slot_of, g.pos_of, L, B, l, M, g.nrm, s));
                bf::Gemm d = gemm0();
                d.dtype = bf::DT_F16;
                d.A = g.cent; d.A2 = g.cent2; d.lda = kvd; d.B = g.rot_th; d.B2 = g.rot_tl; d.ldb = kvd;
                d.M = M; d.N = kvd; d.K = kvd;
                d.epi = bf::EPI_OUT_ROWSCALE; d.Cb = kv ? g.vt : g.kt; d.Cb2 = kv ? g.vt2 : g.kt2; d.ldcb = kvd;
                d.row_scale = g.nrm;
                BIG_TRY(gemm_split(ctx, d, s));
            }
            attn::FlashArgs fa;
            fa.Q = g.qh; fa.Q_lo = g.ql; fa.K = g.kt; fa.K_lo = g.kt2; fa.V = g.vt; fa.V_lo = g.vt2; fa.O = g.attf;
            fa.ldq = n; fa.ldk = kvd; fa.ldo = n;
            fa.n_seq = n_seq; fa.T = T; fa.nh = nh; fa.nkv = (int)ctx->nkv; fa.hd = hd; fa.scale = scale;
            fa.bidir = 0;
            BIG_TRY(attn::flash_prefill(fa, s));
        } else {
            if (fork)
                BIG_TRY(cudaStreamWaitEvent(s, ctx->ev_join, 0));
            else
                BIG_TRY(qrot_gemm(s));
            attn::TqAttnArgs ta;
            ta.kcodes = g.kcodes; ta.vcodes = g.vcodes; ta.knorm = g.knorm; ta.vnorm = g.vnorm;
            ta.kcent = g.kcent; ta.vcent = g.vcent; ta.qrot = g.qrot;
            ta.slot = g.slot_of; ta.pos = g.pos_of; ta.E = g.pe; ta.cmax = g.pmax; ta.csum = g.psum;
            ta.U = g.U; ta.U_lo = g.U2;
            ta.M = M; ta.nh = nh; ta.kvd = kvd; ta.kpl = (int)ctx->kpl; ta.vpl = (int)ctx->vpl;
            ta.L = L; ta.B = B; ta.layer = l; ta.Sp = g.Sp; ta.nc16 = g.Sp / 16; ta.scale = scale;
            ta.err = ctx->d_err;
            ta.nc32 = g.Sp / 32; ta.linv = g.linv; ta.n_slots = c.max_seqs;
            prof_mark(ctx, KG_PROF_ATTN, 0, s);
            BIG_TRY(attn::tq_decode_attn(ta, s));
            prof_mark(ctx, KG_PROF_ATTN, 1, s);
            // out_h = R[:, head cols]^T u~_h
            bf::Gemm o = gemm0();
            o.dtype = bf::DT_F16;
            o.A = g.U; o.A2 = g.U2; o.lda = (int64_t)nh * kvd; o.sA = kvd;
            o.B = g.rot_th; o.B2 = g.rot_tl; o.ldb = kvd; o.sB = (int64_t)hd * kvd;
            o.M = M; o.N = hd; o.K = kvd; o.batch = nh;
            if (fuse) {  // straight to the Wo GEMM's bf16 hi / lo operand
                o.epi = bf::EPI_BF16_SPLIT; o.Cb = g.attb; o.Cb2 = g.attb2; o.ldcb = n; o.sCb = hd;
            } else {
                o.epi = bf::EPI_F32; o.C = g.attf; o.ldc = n; o.sC = hd;
            }
            BIG_TRY(gemm_split(ctx, o, s));
        }
        if (!(fuse && !g.std_kv)) BIG_TRY(bf::to_bf16(g.attf, n, n, M, g.attb, g.attb2, n, s));
        // output projection + residual: x = Wo att + xr
        bf::Gemm w = gemm0();
        w.A = g.attb; w.A2 = g.attb2; w.lda = n; w.B = wo; w.ldb = n; w.M = M; w.N = n; w.K = n;
        w.epi = bf::EPI_F32_RESID; w.C = g.x; w.ldc = n; w.R = g.xr; w.ldr = n; w.C2 = g.xr2;  // xr2: MLP residual
        prof_mark(ctx, KG_PROF_GEMM, 0, s);
        BIG_TRY(gemm_split(ctx, w, s));
        prof_mark(ctx, KG_PROF_GEMM, 1, s);
        // MLP
        // also clears alive counts; mlp_norm_gamma for forward_base (src/transformer.rs:2023-2026)
        BIG_TRY(bf::rmsnorm(g.x, n, M, nullptr, g.xb, g.xb2, false, s, g.alive,
                            g.std_kv && !g.paged ? g.mg + (int64_t)l * n : nullptr));
        bf::Gemm u = gemm0();
        u.A = g.xb; u.A2 = g.xb2; u.lda = n; u.B = w1; u.ldb = n; u.M = M; u.N = m; u.K = n;
        u.epi = bf::EPI_RELU; u.Cb = g.hid; u.Cb2 = g.hid2; u.ldcb = m; u.row_alive = g.alive;
        prof_mark(ctx, KG_PROF_GEMM, 0, s);
        BIG_TRY(gemm_split(ctx, u, s));
        prof_mark(ctx, KG_PROF_GEMM, 1, s);
        if (ctx->hook_keep > 0.0f)  // benchmark hook: ~(1 - keep) of the hidden activations exactly zero
            BIG_TRY(bf::mlp_hook(g.hid, g.hid2, g.alive, g.slot_of, g.pos_of, m, M, ctx->hook_keep, ctx->hook_seed, l,
                                 s));
        bf::Gemm dn = gemm0();
        dn.A = g.hid; dn.A2 = g.hid2; dn.lda = m; dn.B = w2; dn.ldb = m; dn.M = M; dn.N = n; dn.K = m;
        dn.epi = bf::EPI_F32_RESID; dn.C = g.x; dn.ldc = n; dn.R = g.xr2; dn.ldr = n;
        // delta routing's per-layer accumulation (delta += x - xr) in the
        // epilogue, except at routing layers (3, 7, ..: the routing kernel
        // accumulates) and when the TwELL gather may still rewrite x
        const bool fuse_delta = fuse && !spkv && (l & 3) != 3 && M > kTwellMaxRows;
        if (fuse_delta) {
            dn.Dacc = g.delta; dn.R3 = g.xr;
        }
        prof_mark(ctx, KG_PROF_GEMM, 0, s);
        BIG_TRY(gemm_split(ctx, dn, s));
        prof_mark(ctx, KG_PROF_GEMM, 1, s);
        // TwELL (math.rs:315-355): rows at or under the alive threshold are
        // recomputed as a compressed-index gather over W2^T rows. With many rows
        // per call the dense product (one weight stream for all rows) stands:
        // it is the same sum in another order, and cheaper than one gather of
        // ~alive rows of W2^T per token.
        if (M <= kTwellMaxRows)
            BIG_TRY(bf::twell_sparse_w2(g.hid, g.hid2, g.alive, g.w2t + (int64_t)l * m * n, g.xr2, g.x, n, m, M,
                                        c.sparse_threshold, s));
        if (!spkv && !fuse_delta)
            BIG_TRY(bf::delta_route(g.x, g.xr, g.delta, g.dq + (int64_t)l * n, g.dn + (int64_t)l * n, n, M, l, s));
    }
    return cudaSuccess;
}

// lm_head + softmax_scaled; output rows are `ld` floats apart (V unless a
// pass writes every T-th row of a [n_seq][T][V] output)
cudaError_t lm_head(kg_ctx *ctx, int M, float *logits, float *probs, int64_t ld, cudaStream_t s) {
    BigState &g = ctx->big;
    const int n = (int)ctx->n, V = (int)ctx->V;
    if (!logits && !probs) return cudaSuccess;
    BIG_TRY(bf::to_bf16(g.x, n, n, M, g.xb, g.xb2, n, s));
    float *lo = logits ? logits : probs;  // logits land in the probs buffer when only probs are wanted
    bf::Gemm q = gemm0();
    q.A = g.xb; q.A2 = g.xb2; q.lda = n; q.B = g.lm; q.ldb = n; q.M = M; q.N = V; q.K = n;
    q.epi = bf::EPI_F32; q.C = lo; q.ldc = ld;
    prof_mark(ctx, KG_PROF_GEMM, 0, s);
    BIG_TRY(gemm_split(ctx, q, s));
    prof_mark(ctx, KG_PROF_GEMM, 1, s);
    if (probs) BIG_TRY(bf::softmax_rows(lo, probs, V, M, ld, 1.0f / ctx->cfg.temperature, s));
    return cudaSuccess;
}

}  // namespace

cudaError_t big_forward(kg_ctx *ctx, int n_seq, const int32_t *seq_ids, const int32_t *tokens,
                        const int32_t *start_pos, int T, float *logits, float *probs, cudaStream_t s) {
    BigState &g = ctx->big;
    const int n = (int)ctx->n;
    const int64_t V = ctx->V;
    if (T > 1 && start_pos) {
        // T positions per sequence from arbitrary start positions (chunked
        // prefill, batched verification of a speculative path; the semantics
        // of forward_batched, src/transformer.rs:461-517): every (sequence,
        // offset) is a decode row. Each layer encodes all rows' K/V into the
        // arena before its attention runs and a row attends positions up to
        // its own, so a row sees exactly the cache of T sequential calls.
        // Decode scratch holds max_seqs rows: larger calls run one offset per
        // pass, in offset order.
        const int S = (int)std::min<int64_t>(g.ws_tokens, ctx->cfg.max_seqs);
        if ((int64_t)n_seq * T <= S) {
            const int M = n_seq * T;
            BIG_TRY(launch_pdl(expand_tokens_kernel, dim3((M + 255) / 256), dim3(256), 0, s, seq_ids, start_pos, T,
                               n_seq, (int)ctx->B, ctx->cfg.max_seqs, (int)V, tokens, g.slot_of, g.pos_of,
                               ctx->d_err));
            BIG_TRY(launch_pdl(sanitize_tokens_kernel, dim3((M + 255) / 256), dim3(256), 0, s, tokens, M, (int)V,
                               g.tok_of));
            BIG_TRY(bf::embed(g.tok_of, g.pos_of, g.wte, g.wpe, n, M, g.x, s, g.delta));
            BIG_TRY(run_layers(ctx, M, false, M, 1, s));
            BIG_TRY(lm_head(ctx, M, logits, probs, V, s));
            return cudaGetLastError();
        }
        if (n_seq > S) return cudaErrorInvalidValue;
        for (int t = 0; t < T; ++t) {
            BIG_TRY(launch_pdl(expand_offset_kernel, dim3((n_seq + 255) / 256), dim3(256), 0, s, seq_ids, start_pos,
                               T, t, n_seq, (int)ctx->B, ctx->cfg.max_seqs, (int)V, tokens, g.slot_of, g.pos_of,
                               g.tok_of, ctx->d_err));
            BIG_TRY(bf::embed(g.tok_of, g.pos_of, g.wte, g.wpe, n, n_seq, g.x, s, g.delta));
            BIG_TRY(run_layers(ctx, n_seq, false, n_seq, 1, s));
            BIG_TRY(lm_head(ctx, n_seq, logits ? logits + t * V : nullptr, probs ? probs + t * V : nullptr, T * V, s));
        }
        return cudaGetLastError();
    }
    if (T == 1) {
        // decode: tokens of up to ws_tokens sequences per pass
        for (int i0 = 0; i0 < n_seq; i0 += (int)std::min<int64_t>(g.ws_tokens, ctx->cfg.max_seqs)) {
            const int cnt = std::min<int>(n_seq - i0, (int)std::min<int64_t>(g.ws_tokens, ctx->cfg.max_seqs));
            BIG_TRY(launch_pdl(expand_tokens_kernel, dim3((cnt + 255) / 256), dim3(256), 0, s, seq_ids + i0,
                               start_pos ? start_pos + i0 : nullptr, 1, cnt, (int)ctx->B, ctx->cfg.max_seqs, (int)V,
                               tokens + i0, g.slot_of, g.pos_of, ctx->d_err));
            BIG_TRY(launch_pdl(sanitize_tokens_kernel, dim3((cnt + 255) / 256), dim3(256), 0, s, tokens + i0, cnt,
                               (int)V, g.tok_of));
            BIG_TRY(bf::embed(g.tok_of, g.pos_of, g.wte, g.wpe, n, cnt, g.x, s, g.delta));
            BIG_TRY(run_layers(ctx, cnt, false, cnt, 1, s));
            BIG_TRY(lm_head(ctx, cnt, logits ? logits + (int64_t)i0 * V : nullptr,
                            probs ? probs + (int64_t)i0 * V : nullptr, V, s));
        }
        return cudaGetLastError();
    }
    // prefill: whole sequences per pass
    const int per = (int)std::max<int64_t>(1, g.ws_tokens / T);
    for (int i0 = 0; i0 < n_seq; i0 += per) {
        const int cnt = std::min(per, n_seq - i0);
        const int M = cnt * T;
        expand_tokens_kernel<<<(M + 255) / 256, 256, 0, s>>>(seq_ids + i0, nullptr, T, cnt, (int)ctx->B,
                                                            ctx->cfg.max_seqs, (int)V, tokens + (int64_t)i0 * T,
                                                            g.slot_of, g.pos_of, ctx->d_err);
        sanitize_tokens_kernel<<<(M + 255) / 256, 256, 0, s>>>(tokens + (int64_t)i0 * T, M, (int)V, g.tok_of);
        BIG_TRY(bf::embed(g.tok_of, g.pos_of, g.wte, g.wpe, n, M, g.x, s, g.delta));
        BIG_TRY(run_layers(ctx, M, true, cnt, T, s));
        BIG_TRY(lm_head(ctx, M, logits ? logits + (int64_t)i0 * T * V : nullptr,
                        probs ? probs + (int64_t)i0 * T * V : nullptr, V, s));
    }
    return cudaGetLastError();
}

namespace {

__device__ __forceinline__ float block_sum_f(float v, float *red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
    return t;
}

// forward_prefill's delta routing for one layer (src/transformer.rs:2954-2982):
// one CTA per sequence keeps the sequence's block-delta accumulator D and walks
// the positions in order: D += x_p - xr_p; at a routing layer (l % 4 == 3) the
// position routes with D as it stands (blocks 0..b-1 are zero by then, the
// routing softmax over them and D, transformer.rs:1707-1765) and D is zeroed.
__global__ void prefill_route_kernel(float *x, const float *xr, float *D, const float *query, const float *normw,
                                     int n, int T, int layer) {
    pdl_wait();
    __shared__ float red[32];
    const int seq = blockIdx.x, tid = threadIdx.x;
    float *d = D + (int64_t)seq * n;
    const bool routing = (layer & 3) == 3;
    const int b = layer >> 2;
    for (int p = 0; p < T; ++p) {
        float *xp = x + ((int64_t)seq * T + p) * n;
        const float *rp = xr + ((int64_t)seq * T + p) * n;
        for (int j = tid; j < n; j += blockDim.x) d[j] = d[j] + (xp[j] - rp[j]);
        if (!routing) continue;  // no cross-thread reads in this pass: each thread owns its j
        __syncthreads();
        float ss = 0.0f;
        for (int j = tid; j < n; j += blockDim.x) ss += d[j] * d[j];
        ss = block_sum_f(ss, red);
        const float inv = 1.0f / sqrtf(ss / (float)n + 1e-5f);
        float dt = 0.0f;
        for (int j = tid; j < n; j += blockDim.x) dt += normw[j] * (d[j] * inv) * query[j];
        const float own = block_sum_f(dt, red);
        // b zero sources with logit 0 and the accumulator with logit `own`
        const float mx = b > 0 ? fmaxf(0.0f, own) : own;
        const float ez = expf(-mx), eo = expf(own - mx);
        const float w = eo / ((float)b * ez + eo);
        for (int j = tid; j < n; j += blockDim.x) {
            xp[j] = xp[j] + w * d[j];
            d[j] = 0.0f;
        }
        __syncthreads();
    }
}

}  // namespace

// forward_prefill (src/transformer.rs:2606-3004) on the bf16 path, standard
// attention: per layer a double rmsnorm (no gamma), the fused QKV GEMM, K/V
// into the bf16 cache, attention of every position over the whole prompt
// (bidirectional), Wo + residual, rmsnorm, W1 / W2 + residual, then the
// position-ordered delta routing. Writes the last position's logits per
// sequence (logits [n_seq][V]) and leaves positions 0..T-1 in the cache.
cudaError_t big_forward_prefill(kg_ctx *ctx, int n_seq, const int32_t *seq_ids, const int32_t *tokens, int T,
                                float *logits, cudaStream_t s) {
    BigState &g = ctx->big;
    if (!g.std_kv) return cudaErrorNotSupported;
    const int n = (int)ctx->n, kvd = (int)ctx->kvd, m = (int)ctx->m, L = (int)ctx->L, B = (int)ctx->B;
    const int nh = (int)ctx->nh, hd = (int)ctx->hd, V = (int)ctx->V, nqkv = n + 2 * kvd;
    const int64_t per_layer = 2 * (int64_t)n * n + 2 * (int64_t)kvd * n + 2 * (int64_t)m * n;
    const float scale = 1.0f / sqrtf((float)hd);
    const int per = (int)std::max<int64_t>(1, std::min<int64_t>(g.ws_tokens / T, ctx->cfg.max_seqs));
    for (int i0 = 0; i0 < n_seq; i0 += per) {
        const int cnt = std::min(per, n_seq - i0), M = cnt * T;
        BIG_TRY(launch_pdl(expand_tokens_kernel, dim3((M + 255) / 256), dim3(256), 0, s, seq_ids + i0,
                           (const int32_t *)nullptr, T, cnt, B, ctx->cfg.max_seqs, V, tokens + (int64_t)i0 * T,
                           g.slot_of, g.pos_of, ctx->d_err));
        BIG_TRY(launch_pdl(sanitize_tokens_kernel, dim3((M + 255) / 256), dim3(256), 0, s, tokens + (int64_t)i0 * T,
                           M, V, g.tok_of));
        BIG_TRY(bf::embed(g.tok_of, g.pos_of, g.wte, g.wpe, n, M, g.x, s));
        BIG_TRY(cudaMemsetAsync(g.pdelta, 0, (size_t)cnt * n * sizeof(float), s));
        for (int l = 0; l < L; ++l) {
            const bf16 *wqkv = g.layers + l * per_layer;
            const bf16 *wo = wqkv + (int64_t)nqkv * n, *w1 = wo + (int64_t)n * n, *w2 = w1 + (int64_t)m * n;
            // phase A: xr = rmsnorm(x); the projections read rmsnorm(xr) (:2674-2677)
            BIG_TRY(bf::rmsnorm(g.x, n, M, g.xr, nullptr, nullptr, false, s));
            BIG_TRY(bf::rmsnorm(g.xr, n, M, nullptr, g.xb, g.xb2, false, s));
            bf::Gemm q = gemm0();
            q.A = g.xb; q.A2 = g.xb2; q.lda = n; q.B = wqkv; q.ldb = n; q.M = M; q.N = nqkv; q.K = n;
            q.epi = bf::EPI_F32; q.C = g.qkv; q.ldc = nqkv;
            BIG_TRY(gemm_split(ctx, q, s));
            BIG_TRY(attn::kv_store_std(g.qkv, nqkv, n, n + kvd, kvd, M, g.slot_of, g.pos_of, L, B, l, g.kcache,
                                       g.vcache, g.kt, g.kt2, g.vt, g.vt2, s));
            BIG_TRY(bf::to_f16(g.qkv, nqkv, n, M, g.qh, g.ql, n, s));
            // phase B: every position attends the whole prompt (:2863, :2892)
            attn::FlashArgs fa;
            fa.Q = g.qh; fa.Q_lo = g.ql; fa.K = g.kt; fa.K_lo = g.kt2; fa.V = g.vt; fa.V_lo = g.vt2; fa.O = g.attf;
            fa.ldq = n; fa.ldk = kvd; fa.ldo = n;
            fa.n_seq = cnt; fa.T = T; fa.nh = nh; fa.nkv = (int)ctx->nkv; fa.hd = hd; fa.scale = scale; fa.bidir = 1;
            BIG_TRY(attn::flash_prefill(fa, s));
            BIG_TRY(bf::to_bf16(g.attf, n, n, M, g.attb, g.attb2, n, s));
            bf::Gemm w = gemm0();
            w.A = g.attb; w.A2 = g.attb2; w.lda = n; w.B = wo; w.ldb = n; w.M = M; w.N = n; w.K = n;
            w.epi = bf::EPI_F32_RESID; w.C = g.x; w.ldc = n; w.R = g.xr; w.ldr = n; w.C2 = g.xr2;
            BIG_TRY(gemm_split(ctx, w, s));
            BIG_TRY(bf::rmsnorm(g.x, n, M, nullptr, g.xb, g.xb2, false, s, g.alive));
            bf::Gemm u = gemm0();
            u.A = g.xb; u.A2 = g.xb2; u.lda = n; u.B = w1; u.ldb = n; u.M = M; u.N = m; u.K = n;
            u.epi = bf::EPI_RELU; u.Cb = g.hid; u.Cb2 = g.hid2; u.ldcb = m; u.row_alive = g.alive;
            BIG_TRY(gemm_split(ctx, u, s));
            bf::Gemm dn = gemm0();
            dn.A = g.hid; dn.A2 = g.hid2; dn.lda = m; dn.B = w2; dn.ldb = m; dn.M = M; dn.N = n; dn.K = m;
            dn.epi = bf::EPI_F32_RESID; dn.C = g.x; dn.ldc = n; dn.R = g.xr2; dn.ldr = n;
            BIG_TRY(gemm_split(ctx, dn, s));
            if (M <= kTwellMaxRows)
                BIG_TRY(bf::twell_sparse_w2(g.hid, g.hid2, g.alive, g.w2t + (int64_t)l * m * n, g.xr2, g.x, n, m, M,
                                            ctx->cfg.sparse_threshold, s));
            BIG_TRY(launch_pdl(prefill_route_kernel, dim3(cnt), dim3(256), 0, s, g.x, (const float *)g.xr, g.pdelta,
                               (const float *)(g.dq + (int64_t)l * n), (const float *)(g.dn + (int64_t)l * n), n, T,
                               l));
        }
        // lm_head of each sequence's last position
        BIG_TRY(bf::to_bf16(g.x + (int64_t)(T - 1) * n, (int64_t)T * n, n, cnt, g.xb, g.xb2, n, s));
        bf::Gemm q = gemm0();
        q.A = g.xb; q.A2 = g.xb2; q.lda = n; q.B = g.lm; q.ldb = n; q.M = cnt; q.N = V; q.K = n;
        q.epi = bf::EPI_F32; q.C = logits + (int64_t)i0 * V; q.ldc = V;
        BIG_TRY(gemm_split(ctx, q, s));
    }
    return cudaGetLastError();
}

cudaError_t gemm_auto(kg_ctx *ctx, const void *gemm_args, cudaStream_t s) {
    return gemm_split(ctx, *static_cast<const bf::Gemm *>(gemm_args), s);
}

}  // namespace kg
