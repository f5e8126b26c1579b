// kg_sample.cu — token sampling on the device: sample_token_into
// (crates/katgpt-types/src/math.rs:398-422) with the reference Rng
// (crates/katgpt-types/src/rng.rs:26-72), one generator per sequence slot.
//
// The reference draws r = Rng::uniform() (again while r == 0), builds the CDF
// as a running f32 sum in index order and returns the first index whose CDF
// value exceeds r (partition_point on a non-decreasing sequence), at most
// V - 1. The running sum is sequential f32 arithmetic, so the kernel keeps that
// order: one CTA per row, the warp stages 1024-entry chunks of the row in
// shared memory (coalesced, double-buffered) and lane 0 adds them in order,
// stopping at the first crossing (the CDF never decreases, so every later
// entry also exceeds r and the partition point is that index).
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "kg_internal.h"
#include "kg_pdl.cuh"

namespace kg {
namespace {

constexpr int kChunk = 1024;

// Rng::next (XorShift64 13/7/17) and Rng::uniform (24 bits -> [0, 1)).
__device__ __forceinline__ uint64_t rng_next(uint64_t &s) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s;
}
__device__ __forceinline__ float rng_uniform(uint64_t &s) {
    const uint32_t bits = ((uint32_t)(rng_next(s) >> 40) & 0x007fffffu) | 0x3f800000u;
    return __uint_as_float(bits) - 1.0f;
}

__global__ void __launch_bounds__(32) sample_kernel(const float *probs, int64_t ldp, int V, int n_rows,
                                                    const int32_t *slots, int n_slots, uint64_t *rng_state,
                                                    int32_t *out, int *err) {
    pdl_wait();
    __shared__ __align__(16) float buf[2][kChunk];
    __shared__ float s_r;
    __shared__ int s_slot;
    const int row = blockIdx.x, lane = threadIdx.x;
    if (row >= n_rows) return;
    if (lane == 0) {
        const int s = slots ? slots[row] : row;
        s_slot = s;
        if (s < 0 || s >= n_slots) {
            atomicExch(err, 1);
            s_r = 0.0f;
        } else {
            uint64_t st = rng_state[s];
            float r = rng_uniform(st);
            while (r == 0.0f) r = rng_uniform(st);  // redraw on exactly 0 (math.rs:400-404)
            rng_state[s] = st;
            s_r = r;
        }
    }
    __syncwarp();
    if (s_slot < 0 || s_slot >= n_slots) {
        if (lane == 0) out[row] = 0;
        return;
    }
    const float r = s_r;
    const float *p = probs + (int64_t)row * ldp;
    auto stage = [&](int c, int b) {
        const int base = c * kChunk;
        for (int j = lane; j < kChunk; j += 32) buf[b][j] = base + j < V ? __ldg(p + base + j) : 0.0f;
    };
    const int nchunks = (V + kChunk - 1) / kChunk;
    float sum = 0.0f;
    int idx = V;
    stage(0, 0);
    __syncwarp();
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) stage(c + 1, (c + 1) & 1);  // the next chunk loads while lane 0 scans
        int found = 0;
        if (lane == 0) {
            const float *q = buf[c & 1];
            const int cnt = min(kChunk, V - c * kChunk);
            for (int j = 0; j < cnt; ++j) {
                sum = sum + q[j];  // cdf[i] = running f32 sum in index order (math.rs:407-413)
                if (sum > r) {     // partition_point(|c| c <= r)
                    idx = c * kChunk + j;
                    found = 1;
                    break;
                }
            }
        }
        found = __shfl_sync(0xffffffffu, found, 0);
        __syncwarp();
        if (found) break;
    }
    if (lane == 0) out[row] = min(idx, V - 1);
}

// ---------------------------------------------------------------------------
// Speculative verification (speculative_step_rollback, src/speculative/step.rs:150-222,
// with sample_from_distribution / sample_residual_distribution_into,
// crates/katgpt-core/src/speculative/sampling.rs:26-116).

// First index whose running f32 sum (index order) of value(i) exceeds r, or -1:
// the warp stages 1024-entry chunks of p (and q) in shared memory, lane 0 adds.
// value(i) = p[i] when q is null, else max(p[i] - q[i], 0) * scale.
__device__ int staged_scan(const float *p, const float *q, float scale, int V, float r, float (*bp)[kChunk],
                           float (*bq)[kChunk]) {
    const int lane = threadIdx.x;
    auto stage = [&](int c, int b) {
        const int base = c * kChunk;
        for (int j = lane; j < kChunk; j += 32) {
            bp[b][j] = base + j < V ? __ldg(p + base + j) : 0.0f;
            if (q) bq[b][j] = base + j < V ? __ldg(q + base + j) : 0.0f;
        }
    };
    const int nchunks = (V + kChunk - 1) / kChunk;
    float sum = 0.0f;
    int idx = -1;
    stage(0, 0);
    __syncwarp();
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) stage(c + 1, (c + 1) & 1);
        int found = 0;
        if (lane == 0) {
            const float *x = bp[c & 1], *y = bq[c & 1];
            const int cnt = min(kChunk, V - c * kChunk);
            for (int j = 0; j < cnt; ++j) {
                sum = sum + (q ? fmaxf(x[j] - y[j], 0.0f) * scale : x[j]);
                if (r < sum) {
                    idx = c * kChunk + j;
                    found = 1;
                    break;
                }
            }
        }
        found = __shfl_sync(0xffffffffu, found, 0);
        __syncwarp();
        if (found) break;
    }
    return __shfl_sync(0xffffffffu, idx, 0);
}

// sum of max(p - q, 0) in the residual sampler's order: 4-wide chunks summed as
// (r0 + r1) + (r2 + r3) into a running total, then the tail one by one
__device__ float residual_sum(const float *p, const float *q, int V, float (*bp)[kChunk], float (*bq)[kChunk]) {
    const int lane = threadIdx.x;
    float sum = 0.0f;
    for (int base = 0; base < V; base += kChunk) {  // kChunk is a multiple of 4: chunks never straddle
        for (int j = lane; j < kChunk; j += 32) {
            bp[0][j] = base + j < V ? __ldg(p + base + j) : 0.0f;
            bq[0][j] = base + j < V ? __ldg(q + base + j) : 0.0f;
        }
        __syncwarp();
        if (lane == 0) {
            const int cnt = min(kChunk, V - base), full4 = (V / 4) * 4 - base;
            int j = 0;
            for (; j + 4 <= cnt && j + 4 <= full4; j += 4) {
                const float r0 = fmaxf(bp[0][j] - bq[0][j], 0.0f), r1 = fmaxf(bp[0][j + 1] - bq[0][j + 1], 0.0f);
                const float r2 = fmaxf(bp[0][j + 2] - bq[0][j + 2], 0.0f), r3 = fmaxf(bp[0][j + 3] - bq[0][j + 3], 0.0f);
                sum += (r0 + r1) + (r2 + r3);
            }
            for (; j < cnt; ++j) sum += fmaxf(bp[0][j] - bq[0][j], 0.0f);
        }
        __syncwarp();
    }
    return __shfl_sync(0xffffffffu, sum, 0);
}

// one warp per row: the acceptance loop over the row's k draft tokens
__global__ void __launch_bounds__(32) verify_kernel(const float *p, const float *q, const int32_t *drafts, int k, int V,
                                                    int n_rows, const int32_t *slots, int n_slots, uint64_t *rng_state,
                                                    int32_t *out, int32_t *n_out, int *err) {
    pdl_wait();
    __shared__ __align__(16) float bp[2][kChunk], bq[2][kChunk];
    __shared__ uint64_t s_state;
    const int row = blockIdx.x, lane = threadIdx.x;
    if (row >= n_rows) return;
    const int slot = slots ? slots[row] : row;
    if (slot < 0 || slot >= n_slots) {
        if (lane == 0) {
            atomicExch(err, 1);
            n_out[row] = 0;
        }
        return;
    }
    if (lane == 0) s_state = rng_state[slot];
    __syncwarp();
    const float *prow = p + (int64_t)row * k * V, *qrow = q + (int64_t)row * k * V;
    int32_t *o = out + (int64_t)row * (k + 1);
    int count = 0, cur = 0;  // cur: row of p holding the target distribution in use
    bool all = true;
    for (int i = 0; i < k; ++i) {
        const int d = drafts[(int64_t)row * k + i];
        const bool inr = d >= 0 && d < V;
        const float qi = inr ? __ldg(qrow + (int64_t)i * V + d) : 0.0f;
        const float pi = inr ? __ldg(prow + (int64_t)cur * V + d) : 0.0f;
        const float acc = qi > 0.0f ? fminf(pi / qi, 1.0f) : 1.0f;
        float u = 0.0f;
        if (lane == 0) {
            uint64_t st = s_state;
            u = rng_uniform(st);
            s_state = st;
        }
        u = __shfl_sync(0xffffffffu, u, 0);
        __syncwarp();
        if (u <= acc) {
            if (lane == 0) o[count] = d;
            ++count;
            if (i + 1 < k) cur = i + 1;  // the path's next forward position
        } else {
            // residual distribution normalize(max(0, p - q)), else p itself
            const float *pr = prow + (int64_t)cur * V, *qr = qrow + (int64_t)i * V;
            const float sum = residual_sum(pr, qr, V, bp, bq);
            float r = 0.0f;
            if (lane == 0) {
                uint64_t st = s_state;
                r = rng_uniform(st);
                while (r == 0.0f) r = rng_uniform(st);
                s_state = st;
            }
            r = __shfl_sync(0xffffffffu, r, 0);
            __syncwarp();
            int idx = sum > 0.0f ? staged_scan(pr, qr, 1.0f / sum, V, r, bp, bq) : staged_scan(pr, nullptr, 1.0f, V, r, bp, bq);
            if (idx < 0) idx = V - 1;
            if (lane == 0) o[count] = idx;
            ++count;
            all = false;
            break;
        }
    }
    if (all && k > 0) {  // bonus token from the last distribution in use
        float r = 0.0f;
        if (lane == 0) {
            uint64_t st = s_state;
            r = rng_uniform(st);
            while (r == 0.0f) r = rng_uniform(st);
            s_state = st;
        }
        r = __shfl_sync(0xffffffffu, r, 0);
        __syncwarp();
        int idx = staged_scan(prow + (int64_t)cur * V, nullptr, 1.0f, V, r, bp, bq);
        if (idx < 0) idx = V - 1;
        if (lane == 0) o[count] = idx;
        ++count;
    }
    if (lane == 0) {
        n_out[row] = count;
        rng_state[slot] = s_state;
    }
}

// the path's forward tokens: [current token, d_0 .. d_{k-2}] per row
__global__ void verify_tokens_kernel(const int32_t *tokens, const int32_t *drafts, int k, int n_rows, int32_t *out) {
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * k) return;
    const int row = i / k, t = i - row * k;
    out[i] = t == 0 ? tokens[row] : drafts[(int64_t)row * k + t - 1];
}

// Rng::new (rng.rs:34-49): SplitMix64 finaliser, state 0 replaced by 1.
uint64_t rng_new(uint64_t seed) {
    uint64_t z = seed + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    const uint64_t s = z ^ (z >> 31);
    return s == 0 ? 1 : s;
}

int set_err(kg_ctx *ctx, int code, const std::string &m) {
    ctx->err = m;
    return code;
}

}  // namespace

// Seed every slot's generator with Rng::new(slot) (called at context creation).
cudaError_t sampler_init(kg_ctx *ctx) {
    const int S = ctx->cfg.max_seqs;
    std::vector<uint64_t> h(S);
    for (int i = 0; i < S; ++i) h[i] = rng_new((uint64_t)i);
    cudaError_t e = cudaMalloc(&ctx->rng, (size_t)S * sizeof(uint64_t));
    if (e != cudaSuccess) return e;
    ctx->allocs.push_back(ctx->rng);
    return cudaMemcpy(ctx->rng, h.data(), (size_t)S * sizeof(uint64_t), cudaMemcpyHostToDevice);
}

}  // namespace kg

extern "C" {

int kg_rng_seed(kg_ctx *ctx, int32_t seq, uint64_t seed) {
    if (!ctx || !ctx->rng || seq < 0 || seq >= ctx->cfg.max_seqs) return KG_ERR_INVALID_ARG;
    const uint64_t st = kg::rng_new(seed);
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = cudaMemcpy(ctx->rng + seq, &st, sizeof(st), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, std::string("kg_rng_seed: ") + cudaGetErrorString(e));
    return KG_OK;
}

int kg_rng_state(kg_ctx *ctx, int32_t seq, uint64_t *state_out) {
    if (!ctx || !ctx->rng || !state_out || seq < 0 || seq >= ctx->cfg.max_seqs) return KG_ERR_INVALID_ARG;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = cudaMemcpy(state_out, ctx->rng + seq, sizeof(uint64_t), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, std::string("kg_rng_state: ") + cudaGetErrorString(e));
    return KG_OK;
}

int kg_sample_dev(kg_ctx *ctx, int32_t n_rows, const int32_t *seq_ids, const float *probs, int64_t ld_probs,
                  int32_t *tokens_out, void *stream) {
    if (!ctx || !ctx->rng || n_rows < 0 || !probs || !tokens_out || ld_probs < ctx->V) return KG_ERR_INVALID_ARG;
    if (n_rows == 0) return KG_OK;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess)
        e = kg::launch_pdl(kg::sample_kernel, dim3(n_rows), dim3(32), 0, static_cast<cudaStream_t>(stream), probs,
                       ld_probs, (int)ctx->V, (int)n_rows, seq_ids, ctx->cfg.max_seqs, ctx->rng, tokens_out,
                       ctx->d_err);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, std::string("kg_sample_dev: ") + cudaGetErrorString(e));
    return KG_OK;
}

int kg_verify_dev(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *start_pos,
                  const int32_t *tokens, const int32_t *drafts, int32_t k, const float *draft_probs, int32_t *accepted,
                  int32_t *n_accepted, void *stream) {
    if (!ctx || !ctx->rng || n_seq < 1 || n_seq > ctx->cfg.max_seqs || k < 1 || !seq_ids || !start_pos || !tokens ||
        !drafts || !draft_probs || !accepted || !n_accepted)
        return KG_ERR_INVALID_ARG;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, cudaGetErrorString(e));
    const int64_t need = (int64_t)n_seq * k;
    if (need > ctx->verify_rows) {  // scratch for the path's probabilities and tokens (grows, not per call)
        if (ctx->verify_probs) cudaFree(ctx->verify_probs);
        if (ctx->verify_tok) cudaFree(ctx->verify_tok);
        ctx->verify_probs = nullptr;
        ctx->verify_tok = nullptr;
        ctx->verify_rows = 0;
        e = cudaMalloc(&ctx->verify_probs, (size_t)need * ctx->V * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&ctx->verify_tok, (size_t)need * sizeof(int32_t));
        if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_OOM, std::string("kg_verify_dev: ") + cudaGetErrorString(e));
        ctx->verify_rows = need;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    e = kg::launch_pdl(kg::verify_tokens_kernel, dim3((unsigned)((need + 255) / 256)), dim3(256), 0, s, tokens, drafts,
                       (int)k, (int)n_seq, ctx->verify_tok);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, cudaGetErrorString(e));
    const int rc = kg_forward_batch_dev(ctx, n_seq, seq_ids, ctx->verify_tok, start_pos, k, nullptr, ctx->verify_probs,
                                        stream);
    if (rc) return rc;
    e = kg::launch_pdl(kg::verify_kernel, dim3(n_seq), dim3(32), 0, s, (const float *)ctx->verify_probs, draft_probs,
                       drafts, (int)k, (int)ctx->V, (int)n_seq, seq_ids, ctx->cfg.max_seqs, ctx->rng, accepted,
                       n_accepted, ctx->d_err);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, std::string("kg_verify_dev: ") + cudaGetErrorString(e));
    return KG_OK;
}

int kg_verify(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *start_pos, const int32_t *tokens,
              const int32_t *drafts, int32_t k, const float *draft_probs, int32_t *accepted, int32_t *n_accepted) {
    if (!ctx || n_seq < 1 || n_seq > ctx->cfg.max_seqs || k < 1 || !seq_ids || !start_pos || !tokens || !drafts ||
        !draft_probs || !accepted || !n_accepted)
        return KG_ERR_INVALID_ARG;
    for (int32_t i = 0; i < n_seq; ++i) {
        if (seq_ids[i] < 0 || seq_ids[i] >= ctx->cfg.max_seqs)
            return kg::set_err(ctx, KG_ERR_INVALID_ARG, "sequence id out of range");
        if (start_pos[i] < 0 || start_pos[i] + k > ctx->B)
            return kg::set_err(ctx, KG_ERR_INVALID_ARG, "position beyond block_size");
    }
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, cudaGetErrorString(e));
    cudaStream_t s = ctx->stream;
    const size_t nb = (size_t)n_seq * 4, db = (size_t)n_seq * k * 4, qb = (size_t)n_seq * k * ctx->V * 4;
    char *buf = nullptr;
    e = cudaMallocAsync(&buf, 3 * nb + db + qb + (size_t)n_seq * (k + 1) * 4 + nb, s);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_OOM, cudaGetErrorString(e));
    int32_t *d_ids = reinterpret_cast<int32_t *>(buf), *d_pos = d_ids + n_seq, *d_tok = d_pos + n_seq;
    int32_t *d_dr = d_tok + n_seq;
    float *d_q = reinterpret_cast<float *>(d_dr + (size_t)n_seq * k);
    int32_t *d_acc = reinterpret_cast<int32_t *>(d_q + (size_t)n_seq * k * ctx->V), *d_n = d_acc + (size_t)n_seq * (k + 1);
    e = cudaMemcpyAsync(d_ids, seq_ids, nb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_pos, start_pos, nb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_tok, tokens, nb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_dr, drafts, db, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_q, draft_probs, qb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_err, 0, 4, s);
    int rc = KG_OK;
    if (e == cudaSuccess) rc = kg_verify_dev(ctx, n_seq, d_ids, d_pos, d_tok, d_dr, k, d_q, d_acc, d_n, s);
    if (e == cudaSuccess && rc == KG_OK) {
        e = cudaMemcpyAsync(accepted, d_acc, (size_t)n_seq * (k + 1) * 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(n_accepted, d_n, nb, cudaMemcpyDeviceToHost, s);
    }
    int herr = 0;
    if (e == cudaSuccess && rc == KG_OK) e = cudaMemcpyAsync(&herr, ctx->d_err, 4, cudaMemcpyDeviceToHost, s);
    cudaFreeAsync(buf, s);
    const cudaError_t e2 = cudaStreamSynchronize(s);
    if (rc) return rc;
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, std::string("kg_verify: ") + cudaGetErrorString(e));
    if (herr) return kg::set_err(ctx, KG_ERR_INVALID_ARG, "device rejected a token, position or slot");
    return KG_OK;
}

int kg_sample(kg_ctx *ctx, int32_t n_rows, const int32_t *seq_ids, const float *probs, int32_t *tokens_out) {
    if (!ctx || !ctx->rng || n_rows < 0 || !seq_ids || !probs || !tokens_out) return KG_ERR_INVALID_ARG;
    if (n_rows == 0) return KG_OK;
    for (int32_t i = 0; i < n_rows; ++i)
        if (seq_ids[i] < 0 || seq_ids[i] >= ctx->cfg.max_seqs)
            return kg::set_err(ctx, KG_ERR_INVALID_ARG, "sequence id out of range");
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, cudaGetErrorString(e));
    const size_t pb = (size_t)n_rows * ctx->V * 4;
    float *dp = nullptr;
    int32_t *dids = nullptr, *dout = nullptr;
    cudaStream_t s = ctx->stream;
    e = cudaMallocAsync(&dp, pb, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&dids, (size_t)n_rows * 4, s);
    if (e == cudaSuccess) e = cudaMallocAsync(&dout, (size_t)n_rows * 4, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dp, probs, pb, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dids, seq_ids, (size_t)n_rows * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = kg::launch_pdl(kg::sample_kernel, dim3(n_rows), dim3(32), 0, s, (const float *)dp, (int64_t)ctx->V,
                       (int)ctx->V, (int)n_rows, (const int32_t *)dids, ctx->cfg.max_seqs, ctx->rng, dout, ctx->d_err);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tokens_out, dout, (size_t)n_rows * 4, cudaMemcpyDeviceToHost, s);
    if (dp) cudaFreeAsync(dp, s);
    if (dids) cudaFreeAsync(dids, s);
    if (dout) cudaFreeAsync(dout, s);
    const cudaError_t e2 = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) return kg::set_err(ctx, KG_ERR_CUDA, std::string("kg_sample: ") + cudaGetErrorString(e));
    return KG_OK;
}

}  // extern "C"
