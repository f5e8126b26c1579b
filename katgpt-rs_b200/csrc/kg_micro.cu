// kg_micro.cu — exact-order f32 forward for the reference's micro model family
// (launchers; the kernel itself is in kg_micro_kernel.cuh).
//
// One thread owns one (sequence, position). All T new positions of a sequence
// sit in one CTA, so a teacher-forced prefill of every position and every
// layer is a single launch: per layer, each thread projects its own token,
// writes K/V (f32, or TurboQuant codes + dequantized cache) to the device
// arena, the CTA synchronises, and each thread attends over positions
// 0..pos of its sequence. Weights, rotation tables and the SP-KV predictor
// (about 20 KB for Config::micro()) are staged in shared memory; every
// warp reads the same weight element at once (broadcast).
//
// Arithmetic follows the reference's x86-64 AVX2 operation order (see
// kg_exact.cuh), so logits and codes are bit-identical to the CPU path for
// forward_base / forward_quantized; forward_sp_kv_quant calls libm expf,
// reproduced to the correctly rounded value.
//
// References (katgpt-rs):
//   forward_base          src/transformer.rs:1821-2200
//   attention_head        src/transformer.rs:333-389
//   forward_quantized     src/transformer.rs:4042-4233
//   forward_sp_kv_quant   src/sp_kv/forward.rs:610-822, attention_head_core :166-245
//   utility predictor     src/sp_kv/utility_predictor.rs:51-87
//   TurboQuant store/deq  src/turboquant/kv_cache.rs:156-317
//   delta routing         src/transformer.rs:1707-1765, 2129-2158
//   softmax_scaled        crates/katgpt-types/src/math.rs:36-50
#include <algorithm>

#include "kg_dev.cuh"
#include "kg_internal.h"
#include "kg_micro_kernel.cuh"

namespace kg {
namespace {

template <int MODE, int BLK = 16, bool LORA = false>
cudaError_t launch_mode(const MicroArgs &a, cudaStream_t s) {
    const int T = a.T;
    const int SB = 128 / T;
    const int threads = SB * T;
    const int blocks = (a.n_seq + SB - 1) / SB;
    const size_t smem =
        ((size_t)a.pack_floats + 128 * (BLK + 1) + (MODE == MODE_PREFILL ? 128 * 16 : 0)) * sizeof(float);
    auto kfn = micro_forward<16, 4, 4, 4, 64, 27, BLK, MODE, LORA>;
    cudaError_t e = dev::smem(kfn, smem);
    if (e != cudaSuccess) return e;
    const int n_sm = dev::sm_count(), per_sm = dev::occupancy(kfn, 128, smem);
    const int grid = std::min(blocks, n_sm * per_sm);
    kfn<<<grid, threads, smem, s>>>(a);
    return cudaGetLastError();
}

__global__ void zero_pages_kernel(float *pool, const int32_t *idx, int64_t page_floats) {
    float4 *pg = reinterpret_cast<float4 *>(pool + (int64_t)idx[blockIdx.x] * page_floats);
    for (int64_t e = threadIdx.x; e < page_floats / 4; e += blockDim.x) pg[e] = make_float4(0.f, 0.f, 0.f, 0.f);
}

}  // namespace

// alloc_page's fill(0.0) of reused pages (kv_cache.rs:244-247), batched: one
// CTA per listed page (page_floats is a multiple of 4).
cudaError_t zero_pages(float *pool, const int32_t *idx, int n, int64_t page_floats, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    zero_pages_kernel<<<n, 128, 0, s>>>(pool, idx, page_floats);
    return cudaGetLastError();
}

int micro_supported(const kg_config &c) {
    // Instantiated shape: Config::micro() widths (any n_layer).
    // forward_paged also at block_size 64, so page lists of several pages run
    const bool blk_ok = c.block_size == 16 || (c.kv_mode == KG_KV_PAGED && c.block_size == 64);
    bool ok = c.n_embd == 16 && c.n_head == 4 && c.head_dim == 4 && c.n_kv_head == 4 &&
              c.mlp_hidden == 64 && c.vocab_size == 27 && blk_ok &&
              c.weight_dtype == KG_W_F32 && c.n_layer >= 1 && c.n_layer <= 60;
    if (c.kv_mode == KG_KV_SPKV_TQ) ok = ok && c.spkv_window >= c.block_size;
    return ok ? 0 : -1;
}

// forward_prefill over positions 0..T-1 of each sequence (forward_base family: f32 K/V)
cudaError_t launch_micro_prefill(const kg_config &c, const MicroArgs &a, cudaStream_t s) {
    if (a.n_seq <= 0) return cudaSuccess;
    if (a.T < 1 || a.T > 16 || c.kv_mode != KG_KV_F32 || a.start_pos) return cudaErrorInvalidValue;
    return a.lora_rank[0] > 0 ? launch_mode<MODE_PREFILL, 16, true>(a, s) : launch_mode<MODE_PREFILL>(a, s);
}

cudaError_t launch_micro(const kg_config &c, const MicroArgs &a, cudaStream_t s) {
    if (a.n_seq <= 0) return cudaSuccess;
    if (a.T < 1 || a.T > 16) return cudaErrorInvalidValue;
    switch (c.kv_mode) {
        case KG_KV_F32: return a.lora_rank[1] > 0 ? launch_mode<MODE_BASE, 16, true>(a, s) : launch_mode<MODE_BASE>(a, s);
        case KG_KV_TQ: return launch_mode<MODE_QUANT>(a, s);
        case KG_KV_SPKV_TQ: return a.lora_rank[1] > 0 ? launch_mode<MODE_SPKV, 16, true>(a, s) : launch_mode<MODE_SPKV>(a, s);
        case KG_KV_PAGED:
            return c.block_size == 64 ? launch_mode<MODE_PAGED, 64>(a, s) : launch_mode<MODE_PAGED, 16>(a, s);
        case KG_KV_SQ: return launch_mode<MODE_SQ>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace kg
