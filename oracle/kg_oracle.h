/*
 * kg_oracle.h — CPU oracle for the katgpt-rs per-token transformer forward.
 *
 * TEST INFRASTRUCTURE ONLY. This library restates, in C++ with the same AVX2
 * intrinsics and the same operation order, the x86-64 code path that the
 * reference (katopz/katgpt-rs, Rust) takes under its default features plus
 * `turboquant` + `sp_kv`. It is the parity checker for the CUDA library and the
 * timed CPU baseline. Nothing in the product (libkgcuda) links or calls it.
 *
 * Parity pin: the reference cannot be compiled here (no Rust toolchain) and has
 * no golden files; the oracle is checked against the structural asserts of its
 * unit tests and, to three or four significant digits, against published
 * reconstruction-quality tables (.benchmarks/022_octopus_goat.md: TurboQuant
 * and SpectralQuant on seeded keys); the older TurboQuant table of
 * .docs/04_performance.md:323-328 is not reproduced. See the test files under
 * tests/ for each pin.
 *
 * All functions are plain C ABI (ctypes-friendly): pointers + sizes.
 */
#ifndef KG_ORACLE_H
#define KG_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Subset of the reference `Config` (crates/katgpt-types/src/config.rs:14-180)
 * that the forward path reads. */
typedef struct {
    int32_t vocab_size;
    int32_t block_size;
    int32_t n_embd;
    int32_t n_head;
    int32_t head_dim;
    int32_t n_kv_head;
    int32_t mlp_hidden;
    int32_t n_layer;
    int32_t bos_token;
    float temperature;
    float sparse_threshold;
} or_config;

/* SpectralQuantKVCacheConfig fields the codec build reads
 * (src/spectralquant/types.rs:97-126). */
typedef struct {
    uint64_t seed;
    int32_t lloyd_max_iter;
    int32_t calibration_samples;
    float avg_bits;
    int32_t min_tail_bits;
    int32_t max_bits;
    int32_t wf_min_bits;
    int32_t wf_max_bits;
    int32_t use_water_fill;
} or_sq_params;

/* Forward flavours (one per reference entry point). */
enum {
    OR_MODE_BASE = 0,      /* transformer::forward -> forward_base (src/transformer.rs:398-429,1821-2200) */
    OR_MODE_QUANT = 1,     /* transformer::forward_quantized<TurboQuantKVCache> (:4042-4233) */
    OR_MODE_SPKV_QUANT = 2 /* sp_kv::forward::forward_sp_kv_quant, Hard gate (src/sp_kv/forward.rs:610-800) */
};

/* ---- Rng (crates/katgpt-types/src/rng.rs:26-72) ---- */
void or_rng_uniforms(uint64_t seed, int64_t n, float *out);
void or_rng_normals(uint64_t seed, int64_t n, float *out);

/* ---- weights (crates/katgpt-transformer/src/weights.rs:76-177) ----
 * Flat layout, reference init order: wte[V*n], wpe[block*n], per layer
 * {wq[n*n], wk[kvd*n], wv[kvd*n], wo[n*n], w1[m*n], w2[n*m]}, lm_head[V*n],
 * then delta-routing query[L*n] (zeros) and norm[L*n] (ones). */
int64_t or_weights_count(const or_config *c);
/* scale_mode 0: reference scales sqrt(2/n), sqrt(2/(n*L)); 1: fixed std `std`. */
void or_weights_init(const or_config *c, uint64_t seed, int scale_mode, float std_, float *out);

/* ---- SIMD kernels, exposed for the SIMD-vs-scalar parity tests ---- */
float or_dot(const float *a, const float *b, int64_t len);
float or_sum_sq(const float *x, int64_t len);
float or_sum(const float *x, int64_t len);
float or_max(const float *x, int64_t len);
void or_exp_inplace(float *x, int64_t len);
float or_exp_sum_inplace(float *x, int64_t len);
float or_sparse_dot(const float *w_row, const int64_t *idx, const float *val, int64_t alive);
void or_softmax_scaled(float *x, int64_t len, float inv_temp);
int64_t or_sample_token(const float *probs, int64_t n, uint64_t seed);
/* k successive sample_token_into draws from one Rng::new(seed): row j of
 * probs[k][n] -> out[j] */
void or_sample_tokens(const float *probs, int64_t n, int64_t k, uint64_t seed, int64_t *out);
/* speculative_step_rollback's acceptance loop (src/speculative/step.rs:150-222)
 * for one path with Rng::new(seed): p [k][n] target distributions, q [k][n]
 * draft marginals, drafts [k]; writes out [k+1], returns the count */
int32_t or_verify_path(const float *p, const float *q, const int32_t *drafts, int32_t k, int64_t n, uint64_t seed,
                       int32_t *out);
/* scalar (non-SIMD) restatements used to cross-check the AVX2 ones */
float or_scalar_exp(float x);

/* ---- TurboQuant (src/turboquant/...) ---- */
int64_t or_tq_packed_len(int64_t dim, int bits);
/* centroids[2^bits], boundaries[2^bits-1], *mse */
void or_tq_codebook(int64_t dim, int bits, float *centroids, float *boundaries, float *mse);
/* row-major dim*dim orthogonal Q (columns = MGS basis) */
void or_tq_rotation(int64_t dim, uint64_t seed, float *rot);
/* same, from a caller-supplied row-major dim*dim Gaussian matrix */
void or_tq_rotation_from(int64_t dim, const float *gauss, float *rot);
/* normals from the pre-SplitMix64 Rng (state = seed), used to reproduce the
 * reference's published TurboQuant table, which predates that change */
void or_rng_normals_rawstate(uint64_t state, int64_t n, float *out);
/* encode one vector: codes packed into `packed`, norm into *norm */
void or_tq_store(const float *rot, const float *boundaries, int bits, int64_t dim,
                 const float *x, uint8_t *packed, float *norm);
/* decode one vector through rotation_t (row-major transpose of rot) */
void or_tq_dequant(const float *rot_t, const float *centroids, int bits, int64_t dim,
                   const uint8_t *packed, float norm, float *out);
/* allocating decode through the scalar column loop (mat_vec_t) */
void or_tq_dequant_scalar(const float *rot, const float *centroids, int bits, int64_t dim,
                          const uint8_t *packed, float norm, float *out);
void or_tq_pack(const uint8_t *idx, int64_t n, int bits, uint8_t *out);
void or_tq_unpack(const uint8_t *packed, int64_t n, int bits, uint8_t *out);
float or_cosine(const float *a, const float *b, int64_t len);

/* ---- teacher-forced sequence runners ----
 * Runs positions 0..T-1 of one sequence through the chosen forward and writes
 * logits[T*V]. For the quantized modes, codes[L][T][2][packed] and
 * norms[L][T][2] (K then V) are written when non-NULL; utilities[L][T] for
 * SP-KV. weights: flat layout above. key_bits/val_bits for quantized modes.
 * Returns 0 on success. */
int or_run_sequence(const or_config *c, int mode, int key_bits, int val_bits,
                    const float *weights, const int32_t *tokens, int32_t T,
                    float *logits, uint8_t *codes, float *norms, float *utilities);

/* Same for the quantized modes, also writing the rotated unit coordinates
 * each TurboQuant store quantizes: rot_out[L][T][2][kvd] (K then V; rows of
 * zero-norm vectors untouched). */
/* One forward_paged token (src/transformer.rs:3305-3504) over caller-ensured
 * PagedKVCache pages: pool = pages of [K 16 x kvd | V 16 x kvd] f32, table =
 * the sequence's [n_layer][maxp] page indices. */
int or_forward_paged(const or_config *c, const float *weights, float *pool, const int64_t *table, int64_t maxp,
                     int32_t token, int32_t pos, float *logits);
/* SpectralQuant (src/spectralquant/): calibrate_eigenbasis, the per-layer
 * tables of SpectralQuantKVCache::from_calibration ([L][kvd*kvd] eigenvectors,
 * [L][kvd] bits, [L][kvd][64] centroids, [L][kvd] level counts, [L] d_eff),
 * one store+dequantize round trip, and forward_quantized over the codec. */
int or_set_lora(int which, int64_t rank, int64_t in_dim, int64_t out_dim, float alpha, const float *a,
                const float *b);
void or_lora_apply(int64_t rank, int64_t in_dim, int64_t out_dim, float alpha, const float *a, const float *b,
                   const float *in, float *out);
void or_spkv_predict(int64_t d_model, int64_t hidden, int64_t nkv, float init_bias, const float *h, float *util);
void or_spkv_predictor_weights(int64_t d_model, int64_t hidden, int64_t nkv, float init_bias, float *out);
void or_attention_head_gated(const float *q, const float *K, const float *V, float *out, float *scores, int64_t qoff,
                             int64_t kvoff, int64_t kvd, int64_t hd, int64_t tn, float scale, const float *bias);
int or_sq_jacobi(const double *m, int64_t dim, float *evals, float *evecs);
void or_sq_allocate(float d_eff, float avg_bits, int64_t head_dim, int max_bits, int32_t *b_high, int32_t *b_low);
void or_sq_waterfill(const double *ev, int64_t d, int64_t total, int min_bits, int max_bits, uint8_t *out);
void or_sq_lloyd_fit(const float *data, int64_t n, int bits, int max_iter, uint64_t seed, float *centroids);
int64_t or_sq_nearest(float x, const float *centroids, int64_t n);
int64_t or_sq_pack(const uint8_t *idx, const uint8_t *bits, int64_t n, uint8_t *out);
void or_sq_unpack(const uint8_t *p, int64_t plen, const uint8_t *bits, int64_t n, uint8_t *out);
int or_sq_calibrate_eigenbasis(const float *samples, int64_t n, int64_t dim, float *eigvecs, float *eigvals,
                               float *d_eff);
int or_sq_build(const or_sq_params *P, int64_t kvd, int32_t L, const float *eig_in, const float *eval_in,
                const float *deff_in, float *eig_out, uint8_t *bits_out, float *cent_out, int32_t *nlev_out,
                int32_t *deff_out);
int64_t or_sq_roundtrip(int64_t kvd, const float *eig, const uint8_t *bits, const float *cent, const int32_t *nlev,
                        const float *x, uint8_t *packed, float *norm, float *deq);
int or_sq_quality_keys(const or_sq_params *P, int64_t dim, const float *keys, int64_t n_keys, int64_t n_calib,
                       float *recon);
int or_run_sequence_sq(const or_config *c, const float *weights, const float *eig, const uint8_t *bits,
                       const float *cent, const int32_t *nlev, const int32_t *tokens, int32_t T, float *logits,
                       uint8_t *codes, float *norms);
int or_run_sequence_rot(const or_config *c, int mode, int key_bits, int val_bits, const float *weights,
                        const int32_t *tokens, int32_t T, float *logits, uint8_t *codes, float *norms,
                        float *rot_out);

/* forward_quantized with the K/V codes imposed: every TurboQuant store keeps
 * its own norm but takes its codes from codes_in[L][T][kpl + vpl] (K then V,
 * the layout `codes` has above). Replays another implementation's
 * quantization decisions, so the continuous arithmetic of the two can be
 * compared where a rounding difference next to a codebook boundary would
 * otherwise pick a different code. */
int or_run_sequence_forced(const or_config *c, int key_bits, int val_bits, const float *weights,
                           const int32_t *tokens, int32_t T, const uint8_t *codes_in, float *logits);

/* forward_prefill (src/transformer.rs:2606-3004: bidirectional attention over
 * the prompt, double rmsnorm, delta-routing state across positions) over
 * prompt[0..P), then forward_base of cont[0..n_cont) at positions P.. on the
 * prefill's f32 cache. logits_out [1 + n_cont][V]: the prefill's (last
 * position) logits, then each continuation token's. */
int or_prefill_then_decode(const or_config *c, const float *weights, const int32_t *prompt, int32_t P,
                           const int32_t *cont, int32_t n_cont, float *logits_out);

/* Multi-sequence runner: n_seq sequences of T tokens each (row-major),
 * spread over n_threads std::threads (one per core, as the reference's rayon
 * generate_batch). logits may be NULL (discarded) for timing runs. */
int or_run_batch(const or_config *c, int mode, int key_bits, int val_bits,
                 const float *weights, const int32_t *tokens, int32_t n_seq, int32_t T,
                 float *logits, int n_threads);

/* Same, but only positions [t0, T) of each sequence are kept in `logits`
 * (logits laid out [n_seq][T - t0][V]); all positions are still computed. */
int or_run_batch_tail(const or_config *c, int mode, int key_bits, int val_bits,
                      const float *weights, const int32_t *tokens, int32_t n_seq, int32_t T,
                      int32_t t0, float *logits, int n_threads);

/* CPU-baseline timing harness (not a reference function): tokens/s of
 * forward_quantized (mode 1) or forward_base (mode 0) decode at positions
 * ctx .. ctx+n_pos-1, one sequence per thread, over a cache whose first ctx
 * positions hold synthetic codes / rows.
 * w_one_layer: the flat layout of the model with n_layer = 1, its layer
 * shared by all c->n_layer layers. Returns < 0 on bad arguments. */
double or_time_decode(const or_config *c, int mode, int key_bits, int val_bits, const float *w_one_layer,
                      int32_t ctx, int32_t n_pos, int n_threads);

#ifdef __cplusplus
}
#endif
#endif
