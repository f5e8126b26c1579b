// kg_micro_args.h — arguments of the exact-order micro forward kernel
// (kg_micro_kernel.cuh). Plain C++ types only, so the kernel source also
// compiles for the host, where the CPU tests run it against the oracle.
#pragma once
#include <cstdint>

namespace kg {

// Arguments of the exact-order micro forward kernel (kg_micro_kernel.cuh).
struct MicroArgs {
    // packed read-only data copied to shared memory: weights (flat reference
    // layout), TurboQuant tables, SP-KV predictor
    const float *pack;
    int pack_floats;
    int off_wte, off_wpe, off_layers, layer_stride, off_lm, off_dq, off_dn, off_ag, off_mg;
    int off_rot, off_rot_t, off_kc, off_kb, off_vc, off_vb;
    int off_pw1, off_pb1, off_pw2, off_pb2;
    int off_sq_eig, off_sq_cent, off_sq_meta;  // SpectralQuant: [L][kvd*kvd], [L][kvd][64], [L][kvd] (bits | levels << 8)
    int L;
    int kbits, vbits, kpl, vpl;
    float sparse_threshold, inv_temp;
    // batch
    int n_seq, T;
    const int32_t *seq_ids, *tokens, *start_pos;
    float *logits, *probs;
    // per-sequence device state, [slot][layer][pos][...]
    float *Kf, *Vf;          // f32 K/V (forward_base) or dequantized K/V cache (TurboQuant modes)
    uint8_t *codes;          // [.. ][kpl + vpl]
    float *norms;            // [.. ][2]
    float *util;             // [.. ]
    int n_slots;
    int *err;                // set to a nonzero code on an invalid token/position/slot
    // forward_paged: page pool [n_pages][2][16][kvd] and page tables [L][n_slots][maxp]
    float *pool;
    const int32_t *ptab;
    int maxp, n_pages;
    // LoraPair (crates/katgpt-types/src/lora.rs:470-490): [0] the reader
    // (forward_prefill), [1] the writer (forward_base); A [rank][in_dim] at
    // off_lora_a, B [out_dim][rank] at off_lora_b in the pack; rank 0 = none
    int lora_rank[2], lora_in[2], lora_out[2], off_lora_a[2], off_lora_b[2];
    float lora_scale[2];  // alpha / rank
};
constexpr int kLoraMax = 16;  // rank, in_dim and out_dim of a micro-path adapter
constexpr int kSqLevels = 64;  // centroids per dimension in the SpectralQuant tables

}  // namespace kg
