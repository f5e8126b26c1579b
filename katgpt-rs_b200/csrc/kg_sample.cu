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
