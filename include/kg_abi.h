/*
 * kg_abi.h — C ABI of libkgcuda, the B200 (sm_100a) backend for katgpt-rs's
 * per-token transformer forward (prefill + batched decode).
 *
 * The reference's only plugin seam for this path is the `InferenceBackend`
 * trait (src/inference_backend.rs:45-92): one `forward(ctx, weights, cache,
 * token, pos, config) -> &mut [f32]` per token, plus device_name /
 * supports_stateful / reset / compile / is_compiled / recompile_hint. A Rust
 * `CudaBackend` implementing that trait binds the entry points below through
 * a thin `extern "C"` block over these declarations; the batched entry points are
 * the extension the trait lacks (prefill over T positions, decode over many
 * sequences).
 *
 * Conventions: every call returns an int status (0 = ok, negative = kg_status)
 * and never transfers ownership. Host buffers are caller-allocated. The `_dev`
 * variants take device pointers and a cudaStream_t (as void*) and do not
 * synchronise. Calls on one context must be serialised by the caller (the
 * trait takes &mut self). There is no CPU fallback: a context needs a B200,
 * and forward entry points return KG_ERR_UNSUPPORTED for a model shape that
 * has no device kernel (the TurboQuant codec still works for any shape).
 */
#ifndef KG_ABI_H
#define KG_ABI_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kg_ctx kg_ctx;

/* Status codes. Mirrors CompileError (src/inference_backend.rs:14-40):
 * KG_ERR_INVALID_WEIGHTS ~ InvalidWeights, KG_ERR_UNSUPPORTED ~
 * UnsupportedBackend, KG_ERR_CUDA/KG_ERR_OOM ~ DeviceError. */
typedef enum {
    KG_OK = 0,
    KG_ERR_INVALID_ARG = -1,
    KG_ERR_OOM = -2,
    KG_ERR_CUDA = -3,
    KG_ERR_TIMEOUT = -4,
    KG_ERR_NOT_COMPILED = -5,
    KG_ERR_UNSUPPORTED = -6,
    KG_ERR_INVALID_WEIGHTS = -7
} kg_status;

/* Which reference forward a context reproduces. */
typedef enum {
    KG_KV_F32 = 0,     /* transformer::forward -> forward_base, f32 KV (src/transformer.rs:398-429,1821-2200) */
    KG_KV_TQ = 1,      /* transformer::forward_quantized<TurboQuantKVCache> (src/transformer.rs:4042-4233) */
    KG_KV_SPKV_TQ = 2, /* sp_kv::forward::forward_sp_kv_quant, SpKvGateMode::Hard (src/sp_kv/forward.rs:610-822) */
    KG_KV_PAGED = 3,   /* transformer::forward_paged over a PagedKVCache (src/transformer.rs:3305-3504,
                          crates/katgpt-transformer/src/kv_cache.rs:187-420); see the paged section */
    KG_KV_SQ = 4       /* transformer::forward_quantized<SpectralQuantKVCache> (src/transformer.rs:4042-4233,
                          src/spectralquant/spectral_kv_cache.rs); see the SpectralQuant section */
} kg_kv_mode;

typedef enum {
    KG_W_F32 = 0,  /* f32 weights, reference operation order (exact path) */
    KG_W_BF16 = 1  /* bf16 weights, tensor-core path */
} kg_weight_dtype;

/* Fields of the reference `Config` (crates/katgpt-types/src/config.rs:14-180)
 * that the path reads, plus backend knobs. */
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
    float sparse_threshold; /* TwELL switch: dense W2 recompute when alive/m > 1 - this */
    int32_t kv_mode;        /* kg_kv_mode */
    int32_t key_bits;       /* TurboQuant bits (2,3,4,8) for KG_KV_TQ / KG_KV_SPKV_TQ */
    int32_t val_bits;
    int32_t weight_dtype;   /* kg_weight_dtype */
    int32_t max_seqs;       /* sequence slots in the device KV arena */
    int32_t spkv_window;    /* SpKvConfig::window (src/sp_kv/types.rs:44-56), default 128 */
    float spkv_threshold;   /* SpKvConfig::threshold, default 0.5 */
    float spkv_init_bias;   /* SpKvConfig::predictor_init_bias, default 5.0 */
    uint64_t tq_seed;       /* rotation seed, 42 in TurboQuantKVCache::new (src/turboquant/kv_cache.rs:63-77) */
} kg_config;

/* Fill `c` with Config::micro() (config.rs:226-316) and the defaults above. */
void kg_config_micro(kg_config *c);

/* ---- context lifecycle (InferenceBackend::compile / is_compiled) ---- */

/* Create a context on CUDA device `device`: allocates the KV arena for
 * cfg->max_seqs sequences and builds the TurboQuant tables (codebook,
 * rotation) bit-identically to TurboQuantKVCache::new. */
int kg_ctx_create(const kg_config *cfg, int device, kg_ctx **out);
void kg_ctx_destroy(kg_ctx *ctx);
/* Last error message of this context ("" if none). */
const char *kg_last_error(const kg_ctx *ctx);
const char *kg_status_string(int status);
/* InferenceBackend::device_name */
const char *kg_device_name(const kg_ctx *ctx);

/* Number of floats in the flat weight layout: wte[V*n], wpe[block*n], per
 * layer {wq[n*n], wk[kvd*n], wv[kvd*n], wo[n*n], w1[m*n], w2[n*m]},
 * lm_head[V*n], delta_routing_query[L*n], delta_routing_norm[L*n],
 * attn_norm_gamma[L*n], mlp_norm_gamma[L*n] — the TransformerWeights field
 * order (crates/katgpt-transformer/src/weights.rs:12-30, 76-177), the two
 * kog_cpu_fusion gammas last. forward_base (KG_KV_F32) applies both gammas at
 * run time (src/transformer.rs:1893-1895, 2023-2026); forward_quantized and
 * forward_sp_kv_quant normalise without them, as the reference does. A model
 * whose MLP gamma was folded into w1 (weights.rs:205-221) passes ones. */
int64_t kg_weights_count(const kg_config *cfg);

/* TransformerWeights::new(config, Rng::new(seed)) (weights.rs:76-177) into a
 * host buffer of kg_weights_count floats. scale_mode 0: the reference's
 * scales; 1: every tensor ~ N(0, std_) drawn in the same order. */
int kg_reference_weights(const kg_config *cfg, uint64_t seed, int scale_mode, float std_,
                         float *out);

/* Upload weights (flat layout above, host f32). For KG_W_BF16 contexts the
 * values are rounded to bf16 (nearest-even) on the device. Marks the context
 * compiled (InferenceBackend::compile). */
int kg_upload_weights(kg_ctx *ctx, const float *host_weights, int64_t count);
/* Same, from a device f32 buffer. */
int kg_upload_weights_dev(kg_ctx *ctx, const float *dev_weights, int64_t count);
/* InferenceBackend::is_compiled */
int kg_is_compiled(const kg_ctx *ctx);
/* Synthetic benchmark weights for the bf16 path, generated on the device:
 * every bf16 tensor ~ N(0, std_) from a counter-based generator keyed by
 * `seed`, delta-routing query 0 and norm 1 (no reference counterpart: the
 * reference draws its weights on the host with Rng, weights.rs:76-177). */
int kg_random_weights(kg_ctx *ctx, uint64_t seed, float std_);
/* Copy the context's weights back to host f32 in the flat layout (bf16 path),
 * e.g. so a CPU checker runs on exactly the device's bf16-rounded values. */
int kg_download_weights(kg_ctx *ctx, float *host_out, int64_t count);

/* ---- sequences (InferenceBackend::reset) ---- */

/* Clear sequence slot `seq` (KV codes, norms, caches) for a new sequence,
 * as MultiLayerKVCache::reset / TurboQuantKVCache::reset / SpKvQuantCache::reset. */
int kg_seq_reset(kg_ctx *ctx, int32_t seq);
int kg_seq_reset_all(kg_ctx *ctx);
/* Sequence slots: kg_seq_alloc hands out a free slot id in [0, max_seqs)
 * (reset, ready for position 0) or KG_ERR_OOM when all are taken;
 * kg_seq_free returns one. Slots may also be addressed directly by id. */
int kg_seq_alloc(kg_ctx *ctx, int32_t *seq_out);
int kg_seq_free(kg_ctx *ctx, int32_t seq);

/* ---- KV snapshot / restore (MultiLayerKVCache::snapshot / restore,
 * crates/katgpt-transformer/src/kv_cache.rs:89-122): the device cache state of
 * one sequence for positions [0, pos) of every layer, kept in caller-owned
 * DEVICE memory of kg_kv_snapshot_bytes(ctx, pos) bytes. Restore writes it
 * back and zeroes positions [pos, block_size) like the reference. Both are
 * enqueued on `stream` (NULL = the legacy default stream). ---- */
int64_t kg_kv_snapshot_bytes(const kg_ctx *ctx, int32_t pos);
int kg_kv_snapshot(kg_ctx *ctx, int32_t seq, int32_t pos, void *dst_dev, void *stream);
int kg_kv_restore(kg_ctx *ctx, int32_t seq, int32_t pos, const void *src_dev, void *stream);

/* ---- forward ---- */

/* InferenceBackend::forward: one token of sequence `seq` at position `pos`;
 * writes vocab_size logits to host `logits_out`. */
int kg_forward_token(kg_ctx *ctx, int32_t seq, int32_t token, int32_t pos, float *logits_out);

/* Teacher-forced batch: for each i < n_seq, sequence seq_ids[i] runs tokens
 * [i*T .. i*T+T) at positions start_pos[i] .. start_pos[i]+T-1 (start_pos may
 * be NULL = all zero). Equals T successive `forward` calls per sequence.
 * logits_out [n_seq][T][V] and probs_out [n_seq][T][V] (softmax_scaled with
 * 1/temperature, math.rs:36-50) are written when non-NULL. Host pointers. */
int kg_forward_batch(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens,
                     const int32_t *start_pos, int32_t T, float *logits_out, float *probs_out);

/* Device-pointer form of kg_forward_batch, enqueued on `stream` (a
 * cudaStream_t; NULL is the CUDA legacy default stream). All pointers are
 * device pointers; no host synchronisation. Device-side argument checks set a
 * flag that the next host-pointer call on the context reports. */
int kg_forward_batch_dev(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids,
                         const int32_t *tokens, const int32_t *start_pos, int32_t T,
                         float *logits_out, float *probs_out, void *stream);

/* ---- sampling (sample_token_into, crates/katgpt-types/src/math.rs:398-422) ---- */

/* Seed sequence slot `seq`'s generator with Rng::new(seed)
 * (crates/katgpt-types/src/rng.rs:34-49). Every slot starts as Rng::new(slot). */
int kg_rng_seed(kg_ctx *ctx, int32_t seq, uint64_t seed);
/* Current XorShift64 state of slot `seq`'s generator. */
int kg_rng_state(kg_ctx *ctx, int32_t seq, uint64_t *state_out);
/* For each row i < n_rows: r = Rng::uniform() of slot seq_ids[i]'s generator,
 * redrawn while r == 0; tokens_out[i] = the first index whose running f32 sum
 * of probs[i][0..vocab) (index order) exceeds r, at most vocab - 1 — the
 * reference's CDF + partition_point. probs rows are ld_probs floats apart
 * (e.g. the probs_out of kg_forward_batch_dev); seq_ids NULL means row i uses
 * slot i. Device pointers, enqueued on `stream`; each row advances its slot's
 * generator by the draws it took. */
int kg_sample_dev(kg_ctx *ctx, int32_t n_rows, const int32_t *seq_ids, const float *probs, int64_t ld_probs,
                  int32_t *tokens_out, void *stream);
/* Host-pointer form (probs [n_rows][vocab]); synchronises. */
int kg_sample(kg_ctx *ctx, int32_t n_rows, const int32_t *seq_ids, const float *probs, int32_t *tokens_out);

/* Speculative verification of one draft path per sequence on the device —
 * speculative_step_rollback's loop (src/speculative/step.rs:150-222) with
 * Leviathan acceptance and residual resampling
 * (crates/katgpt-core/src/speculative/sampling.rs:26-116). Sequence i stands at
 * start_pos[i] with its current token tokens[i] and k draft tokens
 * drafts[i][0..k) whose draft-model probabilities are draft_probs[i][k][vocab].
 * One multi-position forward scores the path (tokens[i], d_0 .. d_{k-2} at
 * positions start_pos[i] ..); then for j < k, with u = Rng::uniform() of the
 * slot's generator, d_j is accepted while u <= min(p(d_j) / q(d_j), 1) (1 when
 * q(d_j) = 0), p being the target's softmax_scaled distribution at the path's
 * current position; the first rejection draws from normalize(max(0, p - q))
 * (p itself when that is all zero) and ends the path; a fully accepted path
 * adds a bonus draw from the last distribution used. accepted[i][0..k] receives
 * the emitted tokens, n_accepted[i] their count (1..k+1). The KV cache then
 * holds the path's forwarded positions; positions past the accepted ones are
 * rewritten by the next call before any read. Device pointers on `stream`. */
int kg_verify_dev(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *start_pos,
                  const int32_t *tokens, const int32_t *drafts, int32_t k, const float *draft_probs, int32_t *accepted,
                  int32_t *n_accepted, void *stream);
/* Host-pointer form; synchronises. */
int kg_verify(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *start_pos, const int32_t *tokens,
              const int32_t *drafts, int32_t k, const float *draft_probs, int32_t *accepted, int32_t *n_accepted);

/* ---- multi-GPU sequence shards (one context per GPU) ----
 * Sequences shard across GPUs with replicated weights; the one exchange is an
 * all-gather of every shard's decode outputs, done here over NCCL on the
 * caller's stream (the reference has no multi-device path: its batch path is a
 * per-sequence par_iter on one host, src/transformer.rs:3588-3606). NCCL is
 * loaded at run time; without it these return KG_ERR_UNSUPPORTED. */

/* A 128-byte NCCL unique id, made on one rank and handed to every rank by the
 * caller's own channel (a store, a broadcast, a file). */
int kg_comm_unique_id(uint8_t *id_out);
/* Join the `world`-rank communicator as `rank` (collective over all ranks). */
int kg_comm_init(kg_ctx *ctx, const uint8_t *id, int32_t world, int32_t rank);
/* Leave it (also done by kg_ctx_destroy). */
int kg_comm_destroy(kg_ctx *ctx);
/* One decode step of this rank's n_seq sequences (seq_ids, tokens, positions
 * as in kg_forward_batch_dev with T = 1), then the all-gather: logits_all
 * [world][n_seq][vocab] f32 and/or tokens_all [world][n_seq] int32 (tokens
 * sampled on the device from softmax_scaled probabilities, as kg_sample_dev)
 * receive every rank's rows, this rank's at offset rank. Every rank passes the
 * same n_seq and the same choice of outputs. Device pointers, enqueued on
 * `stream`; without a communicator it is the local step only. A rank whose
 * local step fails still joins the gathers (its rows are then stale) and
 * returns the error, so no other rank is left waiting in its gather. */
int kg_decode_gather_dev(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens,
                         const int32_t *positions, float *logits_all, int32_t *tokens_all, void *stream);

/* ---- forward_prefill (src/transformer.rs:2606-3004) ----
 * The reference's prefill variant: over the prompt tokens[i][0..T) of each
 * sequence (from position 0) every layer normalises twice (rmsnorm without
 * gammas), writes K/V of every position into the cache, lets every position
 * attend the WHOLE prompt (bidirectional), and runs delta routing with one
 * block-delta accumulator shared by the prompt's positions in order. Writes
 * the last position's logits, logits_out [n_seq][vocab]; the cache then holds
 * positions 0..T-1, and decoding continues with kg_forward_batch at position T
 * (generate_with_prefill, :3010-3106). Contexts with kv_mode KG_KV_F32. */
int kg_forward_prefill(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens, int32_t T,
                       float *logits_out);
/* Device-pointer form, enqueued on `stream`. */
int kg_forward_prefill_dev(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens, int32_t T,
                           float *logits_out, void *stream);

/* LoraPair (crates/katgpt-types/src/lora.rs:470-490) of generate_with_prefill:
 * which 0 = the reader, applied by kg_forward_prefill (forward_prefill's
 * `lora`), 1 = the writer, applied by kg_forward_batch / kg_forward_token
 * (forward_base's `lora`, the decode half). The adapter is a LoraAdapter:
 * A [rank][in_dim], B [out_dim][rank] (host f32, copied), alpha; lora_apply
 * (lora.rs:452-467) adds (alpha / rank) * B @ (A @ input) after each of the
 * six projections (Q, K, V, O, the post-ReLU W1 activations, W2), to the
 * first out_dim outputs from the first in_dim inputs, in the reference's
 * operation order. rank 0 removes the adapter (None: the plain forward).
 * Exact micro path: kv_mode KG_KV_F32, or KG_KV_SPKV_TQ for the writer
 * (forward_sp_kv_quant's `lora`, src/sp_kv/forward.rs:610-822); rank, in_dim <= n_embd and out_dim <=
 * min(n_embd, kv_dim) at most 16 each (the reference indexes past a
 * projection's output otherwise). Synchronises the device. */
int kg_set_lora(kg_ctx *ctx, int32_t which, int32_t rank, int32_t in_dim, int32_t out_dim, float alpha,
                const float *a, const float *b);

/* ---- PagedKVCache + forward_paged (contexts with kv_mode KG_KV_PAGED) ----
 * The reference's copy-on-write page store for DDTree branch exploration
 * (crates/katgpt-transformer/src/kv_cache.rs:187-420): f32 K/V in pages of 16
 * positions, [K 16 x kv_dim | V 16 x kv_dim] per page, per-layer page lists per
 * sequence, a LIFO free list and per-page reference counts. The bookkeeping
 * lives on the host inside the context (the same integer state as the
 * reference: page indices, counts and free-list order match it call for call);
 * the pages live in a device pool of max(initial, 2 * max_seqs * n_layer *
 * (block_size/16 + 1)) pages, bounded by 90% of the device memory left free
 * at creation less 2 GiB, and an allocation past it returns KG_ERR_OOM (the
 * reference grows its Vec instead). A page taken from the free list is
 * zeroed, as alloc_page does. Sequence indices run from 0 to the paged
 * sequence count (grown by ensure and fork), at most max_seqs.
 * kg_forward_batch / kg_forward_token on such a context are forward_paged
 * (src/transformer.rs:3305-3504): rmsnorm, residual, rmsnorm (no gammas),
 * write_kv at the position, attention over positions 0..pos read back from
 * the pages, the MLP and delta routing as forward; for each sequence in batch
 * order they call ensure_pages(seq, p) for every position p of the call
 * first. kg_forward_batch_dev expects the caller to have done those ensures
 * with kg_paged_ensure. Two device forms: the exact f32 path at the micro
 * widths (Config::micro(), block_size 16 or 64; f32 pages, logits
 * bit-identical to the reference order), and the bf16 tensor-core path at
 * model widths (KG_W_BF16 weights, standard attention over bf16 pages). */

/* PagedKVCache::new(config, max_sequences) (:215-238): drop every page and
 * sequence, then max_sequences empty sequences and (block_size/16 + 1) *
 * n_layer free pages. Contexts start as kg_paged_init(ctx, 1). */
int kg_paged_init(kg_ctx *ctx, int32_t max_sequences);
/* PagedKVCache::ensure_pages (:268-296): pages for positions 0..pos of every layer. */
int kg_paged_ensure(kg_ctx *ctx, int32_t seq, int32_t pos);
/* PagedKVCache::fork (:334-350): a new sequence sharing seq's first
 * fork_at_pos/16 pages of each layer; its index goes to *new_seq. */
int kg_paged_fork(kg_ctx *ctx, int32_t seq, int32_t fork_at_pos, int32_t *new_seq);
/* PagedKVCache::rollback (:360-378): keep pages covering [0, pos/16*16), free
 * the pages whose reference count drops to zero. */
int kg_paged_rollback(kg_ctx *ctx, int32_t seq, int32_t pos);
/* PagedKVCache::reset (:381-390): every sequence's pages back to the free list. */
int kg_paged_reset(kg_ctx *ctx);
/* write_kv / read_kv (:298-329): kv_dim floats of K and V at (layer, seq, pos),
 * host pointers; the page must exist (kg_paged_ensure). Synchronises. */
int kg_paged_write_kv(kg_ctx *ctx, int32_t layer, int32_t seq, int32_t pos, const float *k, const float *v);
int kg_paged_read_kv(kg_ctx *ctx, int32_t layer, int32_t seq, int32_t pos, float *k, float *v);
/* The page list of (layer, seq): up to cap indices into pages_out, its length
 * into *len_out (layer_page_tables[layer][seq]). */
int kg_paged_table(const kg_ctx *ctx, int32_t layer, int32_t seq, int32_t *pages_out, int32_t cap,
                   int32_t *len_out);
/* total_pages, free_pages.len(), the sequence count, and (when refs is not
 * NULL) page_ref_counts[0 .. min(total_pages, refs_cap)). */
int kg_paged_stats(const kg_ctx *ctx, int64_t *total_pages, int64_t *free_pages, int32_t *n_sequences,
                   int32_t *refs, int64_t refs_cap);

/* ---- SpectralQuant (contexts with kv_mode KG_KV_SQ) ----
 * The calibrated-eigenbasis KV codec (src/spectralquant/): each K/V vector is
 * normalised, rotated by the layer's eigenvectors (V^T x), quantized per
 * dimension with Lloyd-Max codebooks (b_high bits on the first d_eff
 * "semantic" dimensions, or water-filled widths, b_low on the tail), and
 * packed LSB-first at those widths; keys and values share the layer's tables,
 * as the reference does. kg_kv_codes returns the pack at the front of a
 * kv_dim-byte row. A KG_KV_SQ context needs one of the two calibration calls
 * before its first forward or codec call (KG_ERR_NOT_COMPILED otherwise). The
 * forward runs the micro widths (Config::micro()); kg_sq_encode / kg_sq_decode
 * run any kv_dim. Codebooks of at most 64 centroids (6 bits) per dimension. */

/* SpectralQuantKVCacheConfig (src/spectralquant/types.rs:97-126), the fields
 * the codec build reads. */
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
} kg_sq_params;

/* The reference's test configuration (spectral_kv_cache.rs:1214-1234): seed
 * 42, 30 Lloyd-Max iterations, 100 calibration samples, 3 bits on average,
 * tail >= 1, at most 8, water-fill off (1..6 when on). */
void kg_sq_params_default(kg_sq_params *p);
/* SpectralQuantKVCache::from_keys (spectral_kv_cache.rs:349-385): calibrate
 * the eigenbasis from key_samples [n_samples][kv_dim] (calibrate_eigenbasis,
 * spectral.rs:226-278) and build every layer's tables from it. */
int kg_sq_calibrate(kg_ctx *ctx, const kg_sq_params *p, const float *key_samples, int64_t n_samples);
/* SpectralQuantKVCache::from_calibration (spectral_kv_cache.rs:99-347): per
 * layer calibrations, eigenvectors [n_layer][kv_dim*kv_dim] (row-major,
 * columns = eigenvectors; an identity matrix selects a seeded random
 * rotation), eigenvalues [n_layer][kv_dim], d_eff [n_layer]. */
int kg_sq_calibrate_from(kg_ctx *ctx, const kg_sq_params *p, const float *eigenvectors, const float *eigenvalues,
                         const float *d_eff);
/* Host-only forms (no context, no device): calibrate_eigenbasis of samples
 * [n_samples][dim] (eigenvectors [dim*dim], eigenvalues [dim], d_eff), and the
 * tables kg_sq_calibrate_from would install for n_layers calibrations (outputs
 * laid out as kg_sq_tables, one layer after another), e.g. to store them with
 * a model. KG_ERR_UNSUPPORTED when a codebook exceeds 64 centroids. */
int kg_sq_calibrate_eigenbasis(const float *samples, int64_t n_samples, int64_t dim, float *eigenvectors,
                               float *eigenvalues, float *d_eff);
int kg_sq_build_tables(const kg_sq_params *p, int64_t kv_dim, int32_t n_layers, const float *eigenvectors,
                       const float *eigenvalues, const float *d_eff, float *eig_out, uint8_t *bits_out,
                       float *centroids_out, int32_t *n_levels_out, int32_t *d_eff_out);
/* The codec at any kv_dim (a KG_KV_SQ context whose shape has no forward
 * kernel is a codec context, like a TurboQuant one): store_vector of n_vec host
 * vectors x [n_vec][kv_dim] with layer `layer`'s tables into packed
 * [n_vec][kv_dim] (the pack at the front of each row; its other bytes, and
 * every byte of a row whose norm is < 1e-8, keep the caller's contents) and
 * norms [n_vec]; and dequantize_*_into of such rows into out [n_vec][kv_dim].
 * Keys and values use the same tables. Synchronous. */
int kg_sq_encode(kg_ctx *ctx, int32_t layer, int64_t n_vec, const float *x, uint8_t *packed, float *norms);
int kg_sq_decode(kg_ctx *ctx, int32_t layer, int64_t n_vec, const uint8_t *packed, const float *norms, float *out);
/* One layer's tables as the device holds them: eigenvectors [kv_dim*kv_dim],
 * bits [kv_dim], centroids [kv_dim][64] (dimension j's codebook first
 * n_levels[j] entries), n_levels [kv_dim], d_eff. Any pointer may be NULL. */
int kg_sq_tables(const kg_ctx *ctx, int32_t layer, float *eigenvectors, uint8_t *bits, float *centroids,
                 int32_t *n_levels, int32_t *d_eff);

/* ---- TurboQuant codec access (parity / inspection) ---- */

/* Packed bytes per vector for `bits` at dimension `dim` (kv_cache.rs:499-509). */
int64_t kg_tq_packed_len(int64_t dim, int32_t bits);
/* Copy the context's tables to host: rotation [kvd*kvd] row-major, key and
 * value centroids [2^bits] and boundaries [2^bits-1]. Any pointer may be NULL. */
int kg_tq_tables(const kg_ctx *ctx, float *rotation, float *key_centroids, float *key_boundaries,
                 float *val_centroids, float *val_boundaries);
/* Encode n_vec host vectors [n_vec][kvd] with the key (which=0) or value
 * (which=1) codebook: packed codes [n_vec][packed_len] and norms [n_vec]
 * (TurboQuantKVCache::store_key/store_value, kv_cache.rs:156-237). */
int kg_tq_encode(kg_ctx *ctx, int32_t which, int64_t n_vec, const float *x, uint8_t *packed,
                 float *norms);
/* Allocation-free form of kg_tq_encode (no counterpart in the reference).
 * For callers that cannot allocate device memory while they encode: a decode
 * loop between captured or latency-critical stages (cudaMalloc/cudaFree
 * synchronise the whole device) or a host that fixes the library's memory
 * budget up front. x [n_vec][kv_dim], packed [n_vec][packed_len] and norms
 * [n_vec] are caller-owned DEVICE pointers; the work is enqueued on `stream`
 * (cudaStream_t, NULL = legacy default stream) and the call does not
 * synchronise. The encoder's scratch lives in a fixed device array of
 * 1,048,576 floats (4 MiB) plus 65,536 flag bytes that every GPU loading the
 * library holds until exit: calls with n_vec * kv_dim > 1,048,576 are
 * rejected with KG_ERR_INVALID_ARG. The first call on a device looks up that
 * array's address (make it before any stream capture). Calls share the array,
 * so calls that overlap on the GPU race; nothing in it needs clearing (each
 * call writes every scratch row it reads). Codes of zero-norm vectors are
 * left as found in `packed`, as in kg_tq_encode. */
int kg_tq_encode_noalloc(kg_ctx *ctx, int32_t which, int64_t n_vec, const float *x, uint8_t *packed,
                         float *norms, void *stream);
/* Read back the stored codes and norms of (seq, layer, pos): key codes, value
 * codes, norms[2] = {key, value}. */
int kg_kv_codes(kg_ctx *ctx, int32_t seq, int32_t layer, int32_t pos, uint8_t *key_codes,
                uint8_t *val_codes, float *norms);
/* SP-KV utility of (seq, layer, pos) (SpKvQuantLayerMeta::utilities). */
int kg_spkv_utility(kg_ctx *ctx, int32_t seq, int32_t layer, int32_t pos, float *utility);

/* ---- phase timing (no reference counterpart; the reference's MBU helpers,
 * src/mbu.rs, estimate the same bandwidth figures from formulas) ---- */
enum {
    KG_PROF_ATTN = 0,   /* decode attention kernels that read the KV codes */
    KG_PROF_ENCODE = 1, /* TurboQuant encode of new K/V */
    KG_PROF_GEMM = 2,   /* weight GEMMs (QKV, Wo, W1, W2, lm_head) */
    KG_PROF_N = 3
};
/* Enable (1) or disable (0) recording of CUDA events around each phase on
 * the stream the kernels run on (bf16 path). */
int kg_profile(kg_ctx *ctx, int enable);
/* Synchronise the context's device, then write the summed device time in ms
 * of every phase since the last read (ms[KG_PROF_N]) and the number of timed
 * intervals (count[KG_PROF_N]); resets the sums. */
int kg_profile_read(kg_ctx *ctx, float *ms, int64_t *count);
/* Benchmark input hook (no reference counterpart; the reference's TwELL
 * benchmark forces sparse hidden activations): after W1 + ReLU of every layer
 * the bf16 path replaces the hidden activations by a per-token Bernoulli(keep)
 * mask with |N(0,1)| survivors, deterministic in (seed, layer, slot,
 * position). keep <= 0 turns it off. Drops captured decode graphs. */
int kg_set_mlp_hook(kg_ctx *ctx, float keep, uint64_t seed);
/* Diagnostics (no reference counterpart): run the bounded-wait path the
 * pipelined kernels use, on purpose — one thread waits on an mbarrier that
 * nothing arrives on, with a limit of limit_cycles SM clocks (at most 2^32).
 * Returns KG_ERR_TIMEOUT (the status a lost arrival inside a GEMM or
 * attention kernel produces); the context stays usable afterwards. */
int kg_selftest_wait_timeout(kg_ctx *ctx, int64_t limit_cycles);
/* Kernel launches replayed by the last kg_forward_batch(_dev) call when it ran
 * as a captured CUDA graph (single-position decode of the bf16 path on a
 * non-legacy stream, profiling off); 0 when that call ran eagerly. */
int64_t kg_graph_kernels(const kg_ctx *ctx);

#ifdef __cplusplus
}
#endif
#endif
