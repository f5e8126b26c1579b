// kg_attn.cuh — attention kernels over the TurboQuant KV cache (kg_attn.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace kg {
namespace attn {

// Arena layout: codes [slot][layer][pos][pl], norms [slot][layer][pos].
// Operands marked hi/lo are f16 splits of f32 values (x = hi + lo).
struct ScoreArgs {
    const uint8_t *kcodes;
    const float *knorm;
    const float *kcent;               // 16 key centroids (4-bit)
    const __half *qrot, *qrot_lo;     // [M][nh][kvd]
    const int32_t *slot, *pos;        // per token
    float *S;                         // [M][nh][Tpad]
    int M, nh, kvd, kpl, L, B, layer, Tpad, Tmax;
    float scale;
};
struct SoftmaxArgs {
    const float *S;
    const float *vnorm;
    const int32_t *slot, *pos;
    __half *P, *P_lo;  // [M][nhp][Tpad]
    int M, nh, nhp, L, B, layer, Tpad;
};
struct ValueArgs {
    const uint8_t *vcodes;
    const float *vcent;
    const __half *P, *P_lo;  // [M][nhp][Tpad]
    const int32_t *slot, *pos;
    __half *U, *U_lo;        // [M][nh][kvd]
    int M, nh, nhp, kvd, vpl, L, B, layer, Tpad;
};
struct FlashArgs {
    const __half *Q, *Q_lo, *K, *K_lo, *V, *V_lo;  // rows = tokens (sequence-major, T per sequence)
    float *O;
    int64_t ldq, ldk, ldo;
    int n_seq, T, nh, nkv, hd;
    float scale;
};

cudaError_t scores(const ScoreArgs &a, cudaStream_t s);
cudaError_t softmax(const SoftmaxArgs &a, cudaStream_t s);
cudaError_t values(const ValueArgs &a, cudaStream_t s);
cudaError_t centroids(const uint8_t *codes, int pl, const int32_t *slot, const int32_t *pos, int L, int B, int layer,
                      const float *cent, int kvd, int M, __half *out, __half *out_lo, cudaStream_t s);
cudaError_t gather_norms(const float *norms, const int32_t *slot, const int32_t *pos, int L, int B, int layer, int M,
                         float *out, cudaStream_t s);
cudaError_t flash_prefill(const FlashArgs &a, cudaStream_t s);

}  // namespace attn
}  // namespace kg
