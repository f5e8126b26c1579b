// kg_internal.h — host/device shared structures of libkgcuda (not part of the ABI).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "../../include/kg_abi.h"
#include "kg_attn.cuh"
#include "kg_micro_args.h"

namespace kg {


inline bool kv_is_tq(int kv_mode) { return kv_mode == KG_KV_TQ || kv_mode == KG_KV_SPKV_TQ; }
// modes that keep packed codes and norms per (layer, position)
inline bool kv_has_codes(int kv_mode) { return kv_is_tq(kv_mode) || kv_mode == KG_KV_SQ; }

// PagedKVCache bookkeeping (crates/katgpt-transformer/src/kv_cache.rs:187-420)
// on the host, pages in a device pool.
struct PagedState {
    std::vector<std::vector<std::vector<int32_t>>> tables;  // [layer][seq] -> page list
    std::vector<int32_t> free_pages;                        // LIFO
    std::vector<int32_t> refs;                              // per page index < total
    int64_t total = 0;                                      // pages ever handed out
    int64_t cap = 0;                                        // device pool capacity (pages)
    int maxp = 0;                                           // device table width (pages per list)
    void *pool = nullptr;                                   // [cap][2][16][kvd] f32 (micro) or bf16
    int32_t *d_tab = nullptr;                               // [L][max_seqs][maxp], -1 = none
    std::vector<int32_t> h_tab;
    std::vector<int32_t> zero_list;                         // reused pages to zero before the next use
    int32_t *d_zero = nullptr;                              // [cap]
    bool dirty = true;
};
cudaError_t zero_pages(float *pool, const int32_t *idx, int n, int64_t page_floats, cudaStream_t s);

// Returns 0 if the model shape has a compiled micro kernel.
int micro_supported(const kg_config &c);
cudaError_t launch_micro(const kg_config &c, const MicroArgs &a, cudaStream_t s);
// forward_prefill (bidirectional, src/transformer.rs:2606-3004) of positions
// 0..T-1; writes one logits row per sequence (the last position's)
cudaError_t launch_micro_prefill(const kg_config &c, const MicroArgs &a, cudaStream_t s);

// TurboQuant device helpers (kg_tq.cu)
// Modified Gram-Schmidt of a row-major dim x dim Gaussian matrix `g`
// (device) into `rot` (row-major Q, columns = basis), bit-identical to
// generate_rotation_matrix (src/turboquant/rotation.rs:11-52). `work` holds
// dim*dim floats.
cudaError_t tq_rotation_device(int dim, const float *g, float *rot, float *rot_t, float *work,
                               cudaStream_t s);
// Encode n_vec vectors [n_vec][dim] (exact reference order).
cudaError_t tq_encode_device(int dim, int bits, int64_t n_vec, const float *x, const float *rot,
                             const float *bnd, uint8_t *packed, int64_t packed_stride,
                             float *norms, int64_t norm_stride, cudaStream_t s);
// Tiled form for many vectors (dim % 128 == 0, 3/4-bit): same codes and norms;
// xn_scratch holds n_vec*dim floats and skip_scratch n_vec bytes.
cudaError_t tq_encode_tiled(int dim, int bits, int64_t n_vec, const float *x, int64_t ldx, const float *rot,
                            const float *bnd, uint8_t *packed, int64_t pstride, float *norms,
                            const int32_t *slot, const int32_t *pos, int L, int B, int layer, float *xn_scratch,
                            uint8_t *skip_scratch, cudaStream_t s);
// Same, reading row v at x + v*ldx and writing arena row (slot[v]*L + layer)*B + pos[v].
// Tensor-core encoder with exact fix-up (kg_tq.cu): norms + xn + f16 split of
// the K and V rows of qkv (2M vectors), then after the caller's rotation GEMM
// Y = xn R^T, codes from Y with exact recomputation near boundaries.
float tq_fixup_eps(int dim);
// SpectralQuant store / dequantize at any kv_dim with one layer's device tables
// (eig [kvd*kvd], meta [kvd] = width | levels << 8, cent [kvd][64], offs [kvd]
// bit offsets, nbytes = the pack's length); packed rows pstride bytes apart.
cudaError_t sq_encode_device(int kvd, int64_t n_vec, const float *x, const float *eig, const int *meta,
                             const float *cent, const int *offs, int nbytes, uint8_t *packed, int64_t pstride,
                             float *norms, cudaStream_t s);
cudaError_t sq_decode_device(int kvd, int64_t n_vec, const uint8_t *packed, int64_t pstride, const float *norms,
                             const float *eig, const int *meta, const float *cent, const int *offs, int nbytes,
                             float *out, cudaStream_t s);
// Vectors v < Mk are K rows (x + t * ldx + koff), the next Mv are V rows.
cudaError_t tq_norm_split(int dim, int Mk, int Mv, const float *qkv, int64_t ldx, int64_t koff, int64_t voff,
                          float *xn, __half *xh, __half *xl, uint8_t *skip, float *knorm, float *vnorm,
                          const int32_t *slot, const int32_t *pos, int L, int B, int layer, cudaStream_t s);
cudaError_t tq_quantize_fixup(int dim, int Mk, int Mv, const float *Y, const float *xn, const uint8_t *skip,
                              const float *rot, const float *kb, const float *vb, int kbits, int vbits,
                              uint8_t *kcodes, uint8_t *vcodes, int64_t kpl, int64_t vpl, const int32_t *slot,
                              const int32_t *pos, int L, int B, int layer, int *nfix, cudaStream_t s);
// exact tiled encoder for the K and V rows of qkv in one norm and one rotate
// launch (kv_dim % 128 == 0); xn / skip scratch of 2M rows
cudaError_t tq_encode_tiled_kv(int dim, int kbits, int vbits, int M, const float *qkv, int64_t ldx, int64_t koff,
                               int64_t voff, const float *rot, const float *kb, const float *vb, uint8_t *kcodes,
                               int64_t kpl, float *knorm, uint8_t *vcodes, int64_t vpl, float *vnorm,
                               const int32_t *slot, const int32_t *pos, int L, int B, int layer, float *xn_scratch,
                               uint8_t *skip_scratch, cudaStream_t s);
// the rotation GEMM of the fast encoder (tcgen05 or mma.sync by size)
cudaError_t gemm_auto(kg_ctx *ctx, const void *gemm_args, cudaStream_t s);
cudaError_t tq_encode_scatter(int dim, int bits, int64_t n_vec, const float *x, int64_t ldx, const float *rot,
                              const float *bnd, uint8_t *packed, int64_t pstride, float *norms, int64_t nstride,
                              const int32_t *slot, const int32_t *pos, int L, int B, int layer, cudaStream_t s);

}  // namespace kg

namespace kg {
// Device state of the BF16 tensor-core path (kg_big.cu).
struct BigState {
    __nv_bfloat16 *wall = nullptr;  // [wte | wpe | layers | lm_head] in flat reference order
    __nv_bfloat16 *wte = nullptr, *wpe = nullptr, *layers = nullptr, *lm = nullptr, *w2t = nullptr;
    float *dq = nullptr, *dn = nullptr;                // delta routing query / norm [L][n]
    float *ag = nullptr, *mg = nullptr;                // attn_norm_gamma / mlp_norm_gamma [L][n]
    float *pdelta = nullptr;                           // forward_prefill block-delta accumulator [max_seqs][n]
    __half *rot_h = nullptr, *rot_l = nullptr, *rot_th = nullptr, *rot_tl = nullptr;  // f16 hi/lo of R, R^T
    float *kcent = nullptr, *vcent = nullptr;          // 16 centroids each
    uint8_t *kcodes = nullptr, *vcodes = nullptr;      // [slot][layer][pos][pl]
    float *knorm = nullptr, *vnorm = nullptr;          // [slot][layer][pos]
    int64_t ws_tokens = 0, Tpad = 0, nbf = 0;
    // workspace (hi/lo pairs are 16-bit splits of f32 values)
    float *x = nullptr, *xr = nullptr, *xr2 = nullptr, *delta = nullptr, *qkv = nullptr, *nrm = nullptr,
          *attf = nullptr;
    __nv_bfloat16 *xb = nullptr, *xb2 = nullptr, *attb = nullptr, *attb2 = nullptr, *hid = nullptr, *hid2 = nullptr;
    __half *qh = nullptr, *ql = nullptr, *cent = nullptr, *cent2 = nullptr, *kt = nullptr, *kt2 = nullptr,
           *vt = nullptr, *vt2 = nullptr, *qrot = nullptr, *qrot2 = nullptr, *U = nullptr, *U2 = nullptr;
    float *xn = nullptr;  // normalised K and V rows of a step [2 * ws_tokens][kv_dim]
    uint8_t *skip = nullptr;
    __half *xnh = nullptr, *xnl = nullptr;  // their f16 hi / lo split (rotation GEMM operand)
    float *yrot = nullptr;                  // rotated rows from the GEMM, before the fix-up
    int *alive = nullptr;
    int32_t *slot_of = nullptr, *pos_of = nullptr, *tok_of = nullptr;
    // standard attention (kv_mode KG_KV_F32): bf16 K/V cache [slot][layer][pos][kv_dim]
    bool std_kv = false;
    bool paged = false;  // std_kv rows in the PagedKVCache pool (kv_mode KG_KV_PAGED)
    __nv_bfloat16 *kcache = nullptr, *vcache = nullptr;
    // two-kernel decode attention scratch: e rows [max_seqs][nh][Sp] and
    // 16-position chunk maxima / sums [max_seqs][Sp / 16][nh]
    __half *pe = nullptr;
    float *pmax = nullptr, *psum = nullptr, *linv = nullptr;
    float *splitk_ws = nullptr;  // f32 split-K partials of decode-sized tcgen05 GEMMs
    int64_t splitk_ws_bytes = 0;
    int Sp = 0;
};
int big_supported(const kg_config &c, std::string &why);
}  // namespace kg

// Host-side context (InferenceBackend state for one device).
struct kg_ctx {
    kg_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    std::string dev_name;
    bool compiled = false;
    bool micro = false;     // shape has the exact-order micro kernel
    bool big_path = false;  // shape runs on the BF16 tensor-core path
    kg::BigState big;
    // phase timing (kg_profile): CUDA event pairs recorded on the launching stream
    bool prof = false;
    std::vector<cudaEvent_t> prof_ev[KG_PROF_N][2];
    size_t prof_used[KG_PROF_N] = {};
    int64_t n = 0, nh = 0, hd = 0, nkv = 0, kvd = 0, m = 0, V = 0, L = 0, B = 0;
    int64_t kpl = 0, vpl = 0, ph = 0;
    int64_t w_count = 0;
    // device buffers
    float *pack = nullptr;  // micro pack: weights + tables + predictor
    int64_t pack_floats = 0;
    kg::MicroArgs margs{};
    float *Kf = nullptr, *Vf = nullptr, *norms = nullptr, *util = nullptr;
    uint8_t *codes = nullptr;
    float *rot = nullptr, *rot_t = nullptr, *kc = nullptr, *kb = nullptr, *vc = nullptr, *vb = nullptr;
    int *d_err = nullptr;
    // host copies of the TurboQuant tables
    std::vector<float> h_rot, h_kc, h_kb, h_vc, h_vb, h_pred;
    // decode step graphs (bf16 path, T == 1): inputs are copied into the
    // g_* buffers, the graph replays the whole forward; keyed by batch shape
    // and output pointers. A key runs eagerly once before it is captured (the
    // first run sets kernel attributes, which capture cannot).
    struct DecodeGraph {
        int n_seq;
        bool has_pos;
        float *logits, *probs;
        cudaStream_t stream;
        cudaGraphExec_t exec;
        int64_t kernels;
        bool captured;
        uint64_t last_use;
    };
    static constexpr size_t kMaxDecodeGraphs = 8;
    std::vector<DecodeGraph> graphs;
    uint64_t graph_clock = 0;
    int32_t *g_ids = nullptr, *g_tok = nullptr, *g_pos = nullptr;
    int64_t last_graph_kernels = 0;
    // staging for host-pointer calls
    void *stage = nullptr;
    size_t stage_bytes = 0;
    std::vector<void *> allocs;
    std::vector<uint8_t> slot_used;  // kg_seq_alloc / kg_seq_free bookkeeping
    __half *enc_rh = nullptr, *enc_rl = nullptr;  // f16 hi / lo of R for kg_tq_encode (codec contexts)
    float hook_keep = 0.0f;                       // kg_set_mlp_hook (benchmark input), 0 = off
    uint64_t hook_seed = 0;
    // side stream of the decode layers (q~ GEMM alongside the K/V encoder),
    // forked from and joined back to the calling stream through events
    cudaStream_t aux = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    // per-slot Rng state of sample_token_into on the device (kg_sample.cu)
    uint64_t *rng = nullptr;
    // multi-GPU sequence shards (kg_comm.cu): NCCL communicator, this rank,
    // and the probabilities buffer of the sampled-token gather
    void *comm = nullptr;
    int world = 1, rank = 0;
    float *probs_buf = nullptr;
    // speculative verification scratch (kg_verify_dev): the path's target
    // probabilities and forward tokens, grown to the largest n_seq * k seen
    float *verify_probs = nullptr;
    int32_t *verify_tok = nullptr;
    int64_t verify_rows = 0;
    // kv_mode KG_KV_PAGED: PagedKVCache state (kg_paged.cu)
    kg::PagedState paged;
    // kv_mode KG_KV_SQ: host copies of the SpectralQuant tables (kg_sq.cpp), set by calibration
    bool sq_ready = false;
    std::vector<float> h_sq_eig, h_sq_cent;
    std::vector<uint8_t> h_sq_bits;
    std::vector<int32_t> h_sq_lev, h_sq_deff;
    // the same tables for the codec entry points at any kv_dim: [L] layers of
    // eig [kvd*kvd], meta [kvd], cent [kvd][64], bit offsets [kvd]; pack bytes per layer
    float *sq_eig_d = nullptr, *sq_cent_d = nullptr;
    int *sq_meta_d = nullptr, *sq_offs_d = nullptr;
    std::vector<int> sq_nbytes;
};

namespace kg {
void prof_mark(kg_ctx *ctx, int phase, int end, cudaStream_t s);
cudaError_t big_init(kg_ctx *ctx);
cudaError_t big_reset(kg_ctx *ctx, int64_t slot0, int64_t nslots);
cudaError_t big_upload_chunk(kg_ctx *ctx, const float *dsrc, int64_t offset, int64_t count);
cudaError_t big_finish_upload(kg_ctx *ctx, const float *dq_dn_dev);
cudaError_t big_random_weights(kg_ctx *ctx, uint64_t seed, float std_);
cudaError_t big_download(kg_ctx *ctx, float *dst_dev, int64_t offset, int64_t count);
cudaError_t big_forward(kg_ctx *ctx, int n_seq, const int32_t *seq_ids, const int32_t *tokens,
                        const int32_t *start_pos, int T, float *logits, float *probs, cudaStream_t s);
cudaError_t big_forward_prefill(kg_ctx *ctx, int n_seq, const int32_t *seq_ids, const int32_t *tokens, int T,
                                float *logits, cudaStream_t s);
// per-slot sampler generators, Rng::new(slot) (kg_sample.cu)
cudaError_t sampler_init(kg_ctx *ctx);
}  // namespace kg
