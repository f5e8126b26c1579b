// kg_attn.cuh — attention kernels (kg_attn.cu, kg_tqattn.cu).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace kg {
namespace attn {

// Arena layout: codes [slot][layer][pos][pl], norms [slot][layer][pos].
// Operands marked hi/lo are f16 splits of f32 values (x = hi + lo).
struct FlashArgs {
    const __half *Q, *Q_lo, *K, *K_lo, *V, *V_lo;  // rows = tokens (sequence-major, T per sequence)
    float *O;
    int64_t ldq, ldk, ldo;
    int n_seq, T, nh, nkv, hd;
    float scale;
    int bidir;  // 1: every query attends all T keys (forward_prefill); 0: causal
};

// Decode attention of M single-token queries over 4-bit / 3-bit codes as two
// streaming kernels (kg_tqattn.cu): scores per 32-position unit, then values
// per block of dims. E, cmax and csum are scratch of [M][nh][Sp] f16 and
// [M][nc16][nh] f32 (one entry per 16 positions), Sp = tq_padded_len(B),
// nc16 = Sp / 16.
struct TqAttnArgs {
    const uint8_t *kcodes, *vcodes;   // [slot][layer][pos][kvd / 2]
    const float *knorm, *vnorm;       // [slot][layer][pos]
    const float *kcent, *vcent;       // 16 centroids each (zero-padded)
    const __half *qrot;               // q~ [M][nh][kvd] (f16)
    const int32_t *slot, *pos;        // per token
    __half *E;                        // exp(s - chunk max) * norm_v [M][nh][Sp]
    float *cmax, *csum;               // chunk maxima and sums [M][nc16][nh]
    __half *U, *U_lo;                 // u~ [M][nh][kvd], f16 hi / lo
    int *err;                         // device error word (timeouts)
    int M, nh, kvd, kpl, vpl, L, B, layer, Sp, nc16;
    float scale;
    int rsk;                          // set by the launcher
    // tcgen05 path (kg_tcattn.cu): 32-position chunk statistics in cmax / csum
    // ([M][nc32][nh]), 1 / softmax denominator per (token, head), arena slots
    int nc32;
    float *linv;                      // [M][nh]
    int n_slots;
};
int tq_padded_len(int block_size);
cudaError_t tq_decode_attn(const TqAttnArgs &a, cudaStream_t s);
// The tcgen05 form (kg_tcattn.cu): 4-bit / nibble-packed codes, kv_dim a
// multiple of 256 and at least 2048, at most 32 heads, block_size <= 6144.
bool tc_attn_supported(const TqAttnArgs &a);
cudaError_t tc_decode_attn(const TqAttnArgs &a, cudaStream_t s);

// Standard attention over a bf16 K/V cache [slot][layer][pos][kvd].
struct StdDecodeArgs {
    const float *Q;              // f32 query rows (column 0 of qkv), scaled inside
    int64_t ldq;
    const __nv_bfloat16 *kc, *vc;
    const int32_t *slot, *pos;
    float *O;                    // [M][n] f32 attention output
    int64_t ldo;
    int M, nh, nkv, hd, kvd, L, B, layer;
    float scale;
    // paged cache (forward_paged): kc = vc = the page pool [page][K 16 rows |
    // V 16 rows][kv_dim]; ptab [L][S][maxp] page indices; a missing page sets *err
    const int32_t *ptab = nullptr;
    int maxp = 0, S = 0, n_pages = 0;
    int *err = nullptr;
};
cudaError_t std_decode(const StdDecodeArgs &a, cudaStream_t s);
// new K / V rows into the bf16 cache; kt.. (optional) receive the f16 hi / lo
// split of the bf16-rounded rows for the prefill flash kernel
cudaError_t kv_store_std(const float *qkv, int64_t ldx, int64_t koff, int64_t voff, int kvd, int M,
                         const int32_t *slot, const int32_t *pos, int L, int B, int layer, __nv_bfloat16 *kc,
                         __nv_bfloat16 *vc, __half *kt, __half *kt2, __half *vt, __half *vt2, cudaStream_t s,
                         const int32_t *ptab = nullptr, int maxp = 0, int S = 0, int n_pages = 0, int *err = nullptr);
cudaError_t centroids(const uint8_t *codes, int pl, const int32_t *slot, const int32_t *pos, int L, int B, int layer,
                      const float *cent, int kvd, int M, __half *out, __half *out_lo, cudaStream_t s);
cudaError_t gather_norms(const float *norms, const int32_t *slot, const int32_t *pos, int L, int B, int layer, int M,
                         float *out, cudaStream_t s);
cudaError_t flash_prefill(const FlashArgs &a, cudaStream_t s);

}  // namespace attn
}  // namespace kg
