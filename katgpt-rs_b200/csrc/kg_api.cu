// kg_api.cu — the C ABI (include/kg_abi.h): context lifecycle, weight upload,
// TurboQuant table construction, batch forward dispatch, codec access.
//
// This is the host runtime behind a `CudaBackend: InferenceBackend`
// (src/inference_backend.rs:45-92): one context per device owns the weights,
// the per-sequence KV arena and a CUDA stream. There is no CPU fallback: any
// configuration without a device kernel is rejected at creation.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "kg_bf16.cuh"
#include "kg_internal.h"

namespace kg {
void host_normals(uint64_t seed, int64_t n, float *out);
int64_t weights_count(const kg_config &c);
void reference_weights(const kg_config &c, uint64_t seed, int scale_mode, float std_, float *out);
void lloyd_max(int64_t dim, int bits, std::vector<float> &cent, std::vector<float> &bnd);
void predictor_weights(int64_t n, int64_t hidden, int64_t nkv, float init_bias, std::vector<float> &out);
cudaError_t paged_alloc(kg_ctx *ctx);
cudaError_t paged_flush(kg_ctx *ctx, cudaStream_t s);
int paged_ensure_batch(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *start_pos, int32_t T);
void sq_calibrate(const float *samples, int64_t n, int64_t dim, std::vector<float> &vecs, std::vector<float> &vals,
                  float &d_eff);
bool sq_build_layer(const kg_sq_params &P, int64_t kvd, int64_t layer, const float *eig, const float *eval,
                    float d_eff_in, float *eig_out, uint8_t *bits_out, float *cent_out, int32_t *lev_out,
                    int32_t *d_eff_out);
}  // namespace kg

namespace {

int fail(kg_ctx *ctx, int code, const std::string &msg) {
    if (ctx) ctx->err = msg;
    return code;
}
int cuda_fail(kg_ctx *ctx, cudaError_t e, const char *what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    if (e == cudaErrorMemoryAllocation) return fail(ctx, KG_ERR_OOM, m);
    return fail(ctx, KG_ERR_CUDA, m);
}
#define KG_CUDA(ctx, call)                                        \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return cuda_fail((ctx), e_, #call); \
    } while (0)

int64_t packed_len(int64_t n, int bits) {  // src/turboquant/kv_cache.rs:499-509
    switch (bits) {
        case 2: return (n + 3) / 4;
        case 3:
        case 4: return (n + 1) / 2;
        case 8: return n;
        default: return (n * bits + 7) / 8;
    }
}

template <typename T>
int dalloc(kg_ctx *ctx, T **p, size_t count) {
    void *q = nullptr;
    if (count == 0) count = 1;
    cudaError_t e = cudaMalloc(&q, count * sizeof(T));
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMalloc");
    ctx->allocs.push_back(q);
    *p = static_cast<T *>(q);
    return 0;
}

int ensure_stage(kg_ctx *ctx, size_t bytes) {
    if (ctx->stage_bytes >= bytes) return 0;
    if (ctx->stage) cudaFree(ctx->stage);
    ctx->stage = nullptr;
    ctx->stage_bytes = 0;
    size_t want = std::max(bytes, (size_t)1 << 20);
    KG_CUDA(ctx, cudaMalloc(&ctx->stage, want));
    ctx->stage_bytes = want;
    return 0;
}
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int validate(const kg_config *c, std::string &why) {
    if (!c) return why = "null config", -1;
    if (c->n_embd <= 0 || c->n_head <= 0 || c->head_dim <= 0 || c->n_kv_head <= 0 ||
        c->n_layer <= 0 || c->vocab_size <= 0 || c->mlp_hidden <= 0 || c->block_size <= 0)
        return why = "non-positive dimension", -1;
    if ((int64_t)c->n_head * c->head_dim != c->n_embd) return why = "n_head*head_dim != n_embd", -1;
    if (c->n_head % c->n_kv_head) return why = "n_head not a multiple of n_kv_head", -1;
    if (c->max_seqs <= 0) return why = "max_seqs must be positive", -1;
    if (c->kv_mode < KG_KV_F32 || c->kv_mode > KG_KV_SQ) return why = "bad kv_mode", -1;
    if (kg::kv_is_tq(c->kv_mode)) {
        for (int b : {c->key_bits, c->val_bits})
            if (b < 2 || b > 8) return why = "TurboQuant bits must be in [2, 8]", -1;
        if ((int64_t)c->n_kv_head * c->head_dim < 3) return why = "kv_dim must be >= 3", -1;
    }
    return 0;
}

}  // namespace

extern "C" {

void kg_config_micro(kg_config *c) {
    std::memset(c, 0, sizeof(*c));
    c->vocab_size = 27;
    c->block_size = 16;
    c->n_embd = 16;
    c->n_head = 4;
    c->head_dim = 4;
    c->n_kv_head = 4;
    c->mlp_hidden = 64;
    c->n_layer = 1;
    c->bos_token = 26;
    c->temperature = 0.5f;
    c->sparse_threshold = 0.8f;
    c->kv_mode = KG_KV_F32;
    c->key_bits = 3;
    c->val_bits = 3;
    c->weight_dtype = KG_W_F32;
    c->max_seqs = 1;
    c->spkv_window = 128;
    c->spkv_threshold = 0.5f;
    c->spkv_init_bias = 5.0f;
    c->tq_seed = 42;
}

const char *kg_status_string(int s) {
    switch (s) {
        case KG_OK: return "ok";
        case KG_ERR_INVALID_ARG: return "invalid argument";
        case KG_ERR_OOM: return "device out of memory";
        case KG_ERR_CUDA: return "CUDA error";
        case KG_ERR_TIMEOUT: return "timeout";
        case KG_ERR_NOT_COMPILED: return "weights not uploaded";
        case KG_ERR_UNSUPPORTED: return "unsupported configuration";
        case KG_ERR_INVALID_WEIGHTS: return "invalid weights";
        default: return "unknown status";
    }
}

const char *kg_last_error(const kg_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }
const char *kg_device_name(const kg_ctx *ctx) { return ctx ? ctx->dev_name.c_str() : "CUDA"; }
int64_t kg_weights_count(const kg_config *cfg) { return cfg ? kg::weights_count(*cfg) : -1; }
int64_t kg_tq_packed_len(int64_t dim, int32_t bits) { return packed_len(dim, bits); }
int kg_is_compiled(const kg_ctx *ctx) { return ctx && ctx->compiled ? 1 : 0; }

int kg_reference_weights(const kg_config *cfg, uint64_t seed, int scale_mode, float std_, float *out) {
    std::string why;
    if (validate(cfg, why) || !out) return KG_ERR_INVALID_ARG;
    kg::reference_weights(*cfg, seed, scale_mode, std_, out);
    return KG_OK;
}

void kg_ctx_destroy(kg_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    kg_comm_destroy(ctx);
    for (auto &gr : ctx->graphs) {
        if (gr.stream) cudaStreamSynchronize(gr.stream);
        if (gr.exec) cudaGraphExecDestroy(gr.exec);
    }
    for (void *p : ctx->allocs) cudaFree(p);
    if (ctx->stage) cudaFree(ctx->stage);
    if (ctx->verify_probs) cudaFree(ctx->verify_probs);
    if (ctx->verify_tok) cudaFree(ctx->verify_tok);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->aux) cudaStreamSynchronize(ctx->aux), cudaStreamDestroy(ctx->aux);
    if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
    if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
    for (int p = 0; p < KG_PROF_N; ++p)
        for (int e = 0; e < 2; ++e)
            for (cudaEvent_t ev : ctx->prof_ev[p][e]) cudaEventDestroy(ev);
    delete ctx;
}

int kg_ctx_create(const kg_config *cfg, int device, kg_ctx **out) {
    if (!out) return KG_ERR_INVALID_ARG;
    *out = nullptr;
    std::string why;
    if (validate(cfg, why)) {
        std::fprintf(stderr, "kg_ctx_create: %s\n", why.c_str());
        return KG_ERR_INVALID_ARG;
    }
    kg_ctx *ctx = new kg_ctx;
    ctx->micro = kg::micro_supported(*cfg) == 0;
    ctx->cfg = *cfg;
    ctx->device = device;
    int rc = 0;
    auto bail = [&](int r) {
        std::fprintf(stderr, "kg_ctx_create: %s\n", ctx->err.c_str());
        kg_ctx_destroy(ctx);
        return r;
    };
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "cudaSetDevice"));
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "cudaGetDeviceProperties"));
    if (prop.major != 10) return bail(fail(ctx, KG_ERR_UNSUPPORTED, "device is not sm_100 (B200)"));
    ctx->dev_name = std::string("CUDA:") + prop.name;
    e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "cudaStreamCreate"));
    e = cudaStreamCreateWithFlags(&ctx->aux, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_join, cudaEventDisableTiming);
    if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "cudaStreamCreate (side stream)"));

    const kg_config &c = ctx->cfg;
    ctx->n = c.n_embd; ctx->nh = c.n_head; ctx->hd = c.head_dim; ctx->nkv = c.n_kv_head;
    ctx->kvd = ctx->nkv * ctx->hd; ctx->m = c.mlp_hidden; ctx->V = c.vocab_size;
    ctx->L = c.n_layer; ctx->B = c.block_size;
    ctx->w_count = kg::weights_count(c);
    const bool tq = kg::kv_is_tq(c.kv_mode);
    const bool paged = c.kv_mode == KG_KV_PAGED, sqm = c.kv_mode == KG_KV_SQ;
    if (paged && !ctx->micro) {
        std::string bwhy;
        if (kg::big_supported(c, bwhy) != 0)
            return bail(fail(ctx, KG_ERR_UNSUPPORTED, "forward_paged: no device forward for this shape (" + bwhy + ")"));
    }
    ctx->kpl = tq ? packed_len(ctx->kvd, c.key_bits) : 0;
    ctx->vpl = tq ? packed_len(ctx->kvd, c.val_bits) : 0;
    if (sqm) ctx->kpl = ctx->vpl = ctx->kvd;  // variable-width pack, at most one byte per dimension
    ctx->ph = std::max<int64_t>(ctx->n / 4, 16);

    // ---- KV arena (exact micro path: f32 K/V or dequantized cache + codes)
    const size_t S = (size_t)c.max_seqs, rows = ctx->micro && !paged ? S * ctx->L * ctx->B : 0;
    if ((rc = dalloc(ctx, &ctx->Kf, rows * ctx->kvd))) return bail(rc);
    if ((rc = dalloc(ctx, &ctx->Vf, rows * ctx->kvd))) return bail(rc);
    if ((rc = dalloc(ctx, &ctx->codes, rows * (ctx->kpl + ctx->vpl)))) return bail(rc);
    if ((rc = dalloc(ctx, &ctx->norms, rows * 2))) return bail(rc);
    if ((rc = dalloc(ctx, &ctx->util, rows))) return bail(rc);
    if ((rc = dalloc(ctx, &ctx->d_err, 1))) return bail(rc);
    e = kg::sampler_init(ctx);
    if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "sampler init"));

    // ---- TurboQuant tables (TurboQuantKVCache::new, kv_cache.rs:56-99)
    const int64_t kvd = ctx->kvd;
    std::vector<float> kc, kb, vc, vb;
    if (tq) {
        kg::lloyd_max(kvd, c.key_bits, kc, kb);
        kg::lloyd_max(kvd, c.val_bits, vc, vb);
        std::vector<float> g(kvd * kvd);
        kg::host_normals(c.tq_seed, kvd * kvd, g.data());
        float *dg = nullptr, *work = nullptr;
        if ((rc = dalloc(ctx, &dg, kvd * kvd))) return bail(rc);
        if ((rc = dalloc(ctx, &work, kvd * kvd))) return bail(rc);
        if ((rc = dalloc(ctx, &ctx->rot, kvd * kvd))) return bail(rc);
        if ((rc = dalloc(ctx, &ctx->rot_t, kvd * kvd))) return bail(rc);
        e = cudaMemcpyAsync(dg, g.data(), kvd * kvd * 4, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "upload gaussian"));
        e = kg::tq_rotation_device((int)kvd, dg, ctx->rot, ctx->rot_t, work, ctx->stream);
        if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "rotation build"));
        ctx->h_rot.resize(kvd * kvd);
        e = cudaMemcpyAsync(ctx->h_rot.data(), ctx->rot, kvd * kvd * 4, cudaMemcpyDeviceToHost, ctx->stream);
        if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "download rotation"));
        e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "rotation build sync"));
        ctx->h_kc = kc; ctx->h_kb = kb; ctx->h_vc = vc; ctx->h_vb = vb;
        if ((rc = dalloc(ctx, &ctx->kc, kc.size()))) return bail(rc);
        if ((rc = dalloc(ctx, &ctx->kb, kb.size()))) return bail(rc);
        if ((rc = dalloc(ctx, &ctx->vc, vc.size()))) return bail(rc);
        if ((rc = dalloc(ctx, &ctx->vb, vb.size()))) return bail(rc);
        e = cudaMemcpy(ctx->kc, kc.data(), kc.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ctx->kb, kb.data(), kb.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ctx->vc, vc.data(), vc.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ctx->vb, vb.data(), vb.size() * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "upload codebooks"));
    }
    if (c.kv_mode == KG_KV_SPKV_TQ)
        kg::predictor_weights(ctx->n, ctx->ph, ctx->nkv, c.spkv_init_bias, ctx->h_pred);

    if (!ctx->micro) {
        std::string bwhy;
        if (kg::big_supported(c, bwhy) == 0) {
            ctx->big_path = true;
            e = kg::big_init(ctx);
            if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "bf16 path init"));
            if (paged) {  // PagedKVCache::new(config, 1), bf16 pages
                e = kg::paged_alloc(ctx);
                if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "paged KV pool"));
                if ((rc = kg_paged_init(ctx, 1))) return bail(rc);
            }
            if ((rc = kg_seq_reset_all(ctx))) return bail(rc);
        }
        // Otherwise a codec-only context: TurboQuant tables and the encoder
        // work; forward entry points return KG_ERR_UNSUPPORTED for this shape.
        *out = ctx;
        return KG_OK;
    }
    // ---- micro pack: weights | rot | rot_t | kc | kb | vc | vb | predictor
    kg::MicroArgs &a = ctx->margs;
    int64_t off = 0;
    const int64_t n = ctx->n, V = ctx->V, L = ctx->L;
    a.off_wte = 0;
    a.off_wpe = (int)(V * n);
    a.off_layers = (int)(a.off_wpe + ctx->B * n);
    a.layer_stride = (int)(2 * n * n + 2 * kvd * n + 2 * ctx->m * n);
    a.off_lm = (int)(a.off_layers + L * a.layer_stride);
    a.off_dq = (int)(a.off_lm + V * n);
    a.off_dn = (int)(a.off_dq + L * n);
    a.off_ag = (int)(a.off_dn + L * n);
    a.off_mg = (int)(a.off_ag + L * n);
    off = a.off_mg + L * n;  // == w_count
    a.off_rot = (int)off; off += tq ? kvd * kvd : 0;
    a.off_rot_t = (int)off; off += tq ? kvd * kvd : 0;
    a.off_kc = (int)off; off += (int64_t)kc.size();
    a.off_kb = (int)off; off += (int64_t)kb.size();
    a.off_vc = (int)off; off += (int64_t)vc.size();
    a.off_vb = (int)off; off += (int64_t)vb.size();
    a.off_pw1 = (int)off; off += ctx->ph * n;
    a.off_pb1 = (int)off; off += ctx->ph;
    a.off_pw2 = (int)off; off += ctx->nkv * ctx->ph;
    a.off_pb2 = (int)off; off += ctx->nkv;
    a.off_sq_eig = (int)off; off += sqm ? L * kvd * kvd : 0;
    a.off_sq_cent = (int)off; off += sqm ? L * kvd * kg::kSqLevels : 0;
    a.off_sq_meta = (int)off; off += sqm ? L * kvd : 0;
    // the LoraPair of forward_base / forward_prefill (kv_mode F32) and the
    // adapter of forward_sp_kv_quant: two adapters
    const bool lora_ok = c.kv_mode == KG_KV_F32 || c.kv_mode == KG_KV_SPKV_TQ;
    const int64_t lora_fl = lora_ok ? kg::kLoraMax * kg::kLoraMax : 0;
    for (int w = 0; w < 2; ++w) {
        a.off_lora_a[w] = (int)off; off += lora_fl;
        a.off_lora_b[w] = (int)off; off += lora_fl;
    }
    off = (off + 3) / 4 * 4;
    ctx->pack_floats = off;
    if (off * 4 > 200 * 1024) return bail(fail(ctx, KG_ERR_UNSUPPORTED, "micro weights exceed shared memory"));
    if ((rc = dalloc(ctx, &ctx->pack, off))) return bail(rc);
    e = cudaMemset(ctx->pack, 0, off * 4);
    if (e == cudaSuccess && tq) {
        std::vector<float> rt(kvd * kvd);
        for (int64_t i = 0; i < kvd; ++i)
            for (int64_t j = 0; j < kvd; ++j) rt[i * kvd + j] = ctx->h_rot[j * kvd + i];
        e = cudaMemcpy(ctx->pack + a.off_rot, ctx->h_rot.data(), kvd * kvd * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ctx->pack + a.off_rot_t, rt.data(), kvd * kvd * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ctx->pack + a.off_kc, kc.data(), kc.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ctx->pack + a.off_kb, kb.data(), kb.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ctx->pack + a.off_vc, vc.data(), vc.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(ctx->pack + a.off_vb, vb.data(), vb.size() * 4, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess && !ctx->h_pred.empty())
        e = cudaMemcpy(ctx->pack + a.off_pw1, ctx->h_pred.data(), ctx->h_pred.size() * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "upload micro tables"));
    a.pack = ctx->pack;
    a.pack_floats = (int)ctx->pack_floats;
    a.L = (int)L;
    a.kbits = c.key_bits; a.vbits = c.val_bits;
    a.kpl = (int)ctx->kpl; a.vpl = (int)ctx->vpl;
    a.sparse_threshold = c.sparse_threshold;
    a.inv_temp = 1.0f / c.temperature;
    a.Kf = ctx->Kf; a.Vf = ctx->Vf; a.codes = ctx->codes; a.norms = ctx->norms; a.util = ctx->util;
    a.n_slots = c.max_seqs;
    a.err = ctx->d_err;
    if (paged) {  // PagedKVCache::new(config, 1)
        e = kg::paged_alloc(ctx);
        if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "paged KV pool"));
        if ((rc = kg_paged_init(ctx, 1))) return bail(rc);
    }
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return bail(cuda_fail(ctx, e, "context init"));
    if ((rc = kg_seq_reset_all(ctx))) return bail(rc);
    *out = ctx;
    return KG_OK;
}

int kg_upload_weights(kg_ctx *ctx, const float *w, int64_t count) {
    if (!ctx || !w) return KG_ERR_INVALID_ARG;
    if (ctx->big_path) {
        if (count != ctx->w_count) return fail(ctx, KG_ERR_INVALID_WEIGHTS, "weight count mismatch");
        KG_CUDA(ctx, cudaSetDevice(ctx->device));
        const int64_t chunk = (int64_t)64 << 20;  // floats per staged copy
        int rc = ensure_stage(ctx, (size_t)chunk * 4);
        if (rc) return rc;
        float *st = static_cast<float *>(ctx->stage);
        const int64_t nbf = ctx->big.nbf;
        for (int64_t off = 0; off < nbf; off += chunk) {
            const int64_t cnt = std::min(chunk, nbf - off);
            KG_CUDA(ctx, cudaMemcpyAsync(st, w + off, cnt * 4, cudaMemcpyHostToDevice, ctx->stream));
            KG_CUDA(ctx, kg::big_upload_chunk(ctx, st, off, cnt));
            KG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
        }
        KG_CUDA(ctx, cudaMemcpyAsync(st, w + nbf, (count - nbf) * 4, cudaMemcpyHostToDevice, ctx->stream));
        KG_CUDA(ctx, kg::big_finish_upload(ctx, st));
        ctx->compiled = true;
        return KG_OK;
    }
    if (!ctx->micro) return fail(ctx, KG_ERR_UNSUPPORTED, "no forward kernel for this model shape");
    if (count != ctx->w_count)
        return fail(ctx, KG_ERR_INVALID_WEIGHTS,
                    "weight count " + std::to_string(count) + " != " + std::to_string(ctx->w_count));
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    KG_CUDA(ctx, cudaMemcpyAsync(ctx->pack, w, count * 4, cudaMemcpyHostToDevice, ctx->stream));
    KG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    ctx->compiled = true;
    return KG_OK;
}

int kg_upload_weights_dev(kg_ctx *ctx, const float *w, int64_t count) {
    if (!ctx || !w) return KG_ERR_INVALID_ARG;
    if (ctx->big_path) {
        if (count != ctx->w_count) return fail(ctx, KG_ERR_INVALID_WEIGHTS, "weight count mismatch");
        KG_CUDA(ctx, cudaSetDevice(ctx->device));
        KG_CUDA(ctx, kg::big_upload_chunk(ctx, w, 0, ctx->big.nbf));
        KG_CUDA(ctx, kg::big_finish_upload(ctx, w + ctx->big.nbf));
        ctx->compiled = true;
        return KG_OK;
    }
    if (!ctx->micro) return fail(ctx, KG_ERR_UNSUPPORTED, "no forward kernel for this model shape");
    if (count != ctx->w_count) return fail(ctx, KG_ERR_INVALID_WEIGHTS, "weight count mismatch");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    KG_CUDA(ctx, cudaMemcpyAsync(ctx->pack, w, count * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    KG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    ctx->compiled = true;
    return KG_OK;
}

int kg_random_weights(kg_ctx *ctx, uint64_t seed, float std_) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (!ctx->big_path) return fail(ctx, KG_ERR_UNSUPPORTED, "synthetic weights are for the bf16 path");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    KG_CUDA(ctx, kg::big_random_weights(ctx, seed, std_));
    ctx->compiled = true;
    return KG_OK;
}

int kg_download_weights(kg_ctx *ctx, float *out, int64_t count) {
    if (!ctx || !out) return KG_ERR_INVALID_ARG;
    if (!ctx->big_path) return fail(ctx, KG_ERR_UNSUPPORTED, "download is for the bf16 path");
    if (count != ctx->w_count) return fail(ctx, KG_ERR_INVALID_ARG, "weight count mismatch");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const int64_t chunk = (int64_t)64 << 20;
    int rc = ensure_stage(ctx, (size_t)chunk * 4);
    if (rc) return rc;
    float *st = static_cast<float *>(ctx->stage);
    const int64_t nbf = ctx->big.nbf;
    for (int64_t off = 0; off < nbf; off += chunk) {
        const int64_t cnt = std::min(chunk, nbf - off);
        KG_CUDA(ctx, kg::big_download(ctx, st, off, cnt));
        KG_CUDA(ctx, cudaMemcpyAsync(out + off, st, cnt * 4, cudaMemcpyDeviceToHost, ctx->stream));
        KG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    }
    KG_CUDA(ctx, cudaMemcpyAsync(out + nbf, ctx->big.dq, ctx->L * ctx->n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    KG_CUDA(ctx, cudaMemcpyAsync(out + nbf + ctx->L * ctx->n, ctx->big.dn, ctx->L * ctx->n * 4,
                                 cudaMemcpyDeviceToHost, ctx->stream));
    KG_CUDA(ctx, cudaMemcpyAsync(out + nbf + 2 * ctx->L * ctx->n, ctx->big.ag, ctx->L * ctx->n * 4,
                                 cudaMemcpyDeviceToHost, ctx->stream));
    KG_CUDA(ctx, cudaMemcpyAsync(out + nbf + 3 * ctx->L * ctx->n, ctx->big.mg, ctx->L * ctx->n * 4,
                                 cudaMemcpyDeviceToHost, ctx->stream));
    KG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return KG_OK;
}

int kg_seq_reset(kg_ctx *ctx, int32_t seq) {
    if (!ctx || seq < 0 || seq >= ctx->cfg.max_seqs) return KG_ERR_INVALID_ARG;
    if (ctx->cfg.kv_mode == KG_KV_PAGED && (ctx->micro || ctx->big_path))
        return kg_paged_rollback(ctx, seq, 0);  // the sequence's pages back
    if (ctx->big_path) {
        KG_CUDA(ctx, cudaSetDevice(ctx->device));
        KG_CUDA(ctx, kg::big_reset(ctx, seq, 1));
        return KG_OK;
    }
    if (!ctx->micro) return KG_OK;
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const size_t rows = (size_t)ctx->L * ctx->B, r0 = (size_t)seq * rows;
    cudaStream_t s = ctx->stream;
    KG_CUDA(ctx, cudaMemsetAsync(ctx->Kf + r0 * ctx->kvd, 0, rows * ctx->kvd * 4, s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->Vf + r0 * ctx->kvd, 0, rows * ctx->kvd * 4, s));
    if (ctx->kpl + ctx->vpl)
        KG_CUDA(ctx, cudaMemsetAsync(ctx->codes + r0 * (ctx->kpl + ctx->vpl), 0, rows * (ctx->kpl + ctx->vpl), s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->norms + r0 * 2, 0, rows * 2 * 4, s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->util + r0, 0, rows * 4, s));
    KG_CUDA(ctx, cudaStreamSynchronize(s));
    return KG_OK;
}

int kg_seq_reset_all(kg_ctx *ctx) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (ctx->big_path) {
        KG_CUDA(ctx, cudaSetDevice(ctx->device));
        KG_CUDA(ctx, kg::big_reset(ctx, 0, ctx->cfg.max_seqs));
        KG_CUDA(ctx, cudaMemset(ctx->d_err, 0, 4));
        return ctx->cfg.kv_mode == KG_KV_PAGED ? kg_paged_reset(ctx) : KG_OK;
    }
    if (!ctx->micro) return KG_OK;
    if (ctx->cfg.kv_mode == KG_KV_PAGED) {
        KG_CUDA(ctx, cudaSetDevice(ctx->device));
        KG_CUDA(ctx, cudaMemset(ctx->d_err, 0, 4));
        return kg_paged_reset(ctx);
    }
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const size_t rows = (size_t)ctx->cfg.max_seqs * ctx->L * ctx->B;
    cudaStream_t s = ctx->stream;
    KG_CUDA(ctx, cudaMemsetAsync(ctx->Kf, 0, rows * ctx->kvd * 4, s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->Vf, 0, rows * ctx->kvd * 4, s));
    if (ctx->kpl + ctx->vpl) KG_CUDA(ctx, cudaMemsetAsync(ctx->codes, 0, rows * (ctx->kpl + ctx->vpl), s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->norms, 0, rows * 2 * 4, s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->util, 0, rows * 4, s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->d_err, 0, 4, s));
    KG_CUDA(ctx, cudaStreamSynchronize(s));
    return KG_OK;
}

namespace {
// Single-position decode through a captured CUDA graph: one launch per step
// instead of one per kernel. The caller's arrays are copied into fixed device
// buffers first, so any arrays of the same batch shape replay the same graph.
int forward_graph(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens,
                  const int32_t *start_pos, float *logits, float *probs, cudaStream_t s) {
    const int S = ctx->cfg.max_seqs;
    if (!ctx->g_ids) {
        int rc;
        if ((rc = dalloc(ctx, &ctx->g_ids, S)) || (rc = dalloc(ctx, &ctx->g_tok, S)) || (rc = dalloc(ctx, &ctx->g_pos, S)))
            return rc;
    }
    KG_CUDA(ctx, cudaMemcpyAsync(ctx->g_ids, seq_ids, n_seq * 4, cudaMemcpyDeviceToDevice, s));
    KG_CUDA(ctx, cudaMemcpyAsync(ctx->g_tok, tokens, n_seq * 4, cudaMemcpyDeviceToDevice, s));
    if (start_pos) KG_CUDA(ctx, cudaMemcpyAsync(ctx->g_pos, start_pos, n_seq * 4, cudaMemcpyDeviceToDevice, s));
    const int32_t *pos = start_pos ? ctx->g_pos : nullptr;
    kg_ctx::DecodeGraph *gr = nullptr;
    for (auto &x : ctx->graphs)
        if (x.n_seq == n_seq && x.has_pos == (start_pos != nullptr) && x.logits == logits && x.probs == probs &&
            x.stream == s)
            gr = &x;
    if (!gr) {  // first use of this key: eager
        // the cache holds at most kMaxDecodeGraphs keys (callers that pass a new
        // output buffer every step would otherwise grow it without bound): evict
        // the least recently used one
        if (ctx->graphs.size() >= kg_ctx::kMaxDecodeGraphs) {
            auto old = std::min_element(ctx->graphs.begin(), ctx->graphs.end(),
                                        [](const kg_ctx::DecodeGraph &a, const kg_ctx::DecodeGraph &b) {
                                            return a.last_use < b.last_use;
                                        });
            if (old->stream) KG_CUDA(ctx, cudaStreamSynchronize(old->stream));
            if (old->exec) cudaGraphExecDestroy(old->exec);
            ctx->graphs.erase(old);
        }
        ctx->graphs.push_back({n_seq, start_pos != nullptr, logits, probs, s, nullptr, 0, false, ++ctx->graph_clock});
        KG_CUDA(ctx, kg::big_forward(ctx, n_seq, ctx->g_ids, ctx->g_tok, pos, 1, logits, probs, s));
        return KG_OK;
    }
    if (!gr->captured) {
        cudaGraph_t graph = nullptr;
        KG_CUDA(ctx, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = kg::big_forward(ctx, n_seq, ctx->g_ids, ctx->g_tok, pos, 1, logits, probs, s);
        cudaError_t e2 = cudaStreamEndCapture(s, &graph);
        if (e == cudaSuccess) e = e2;
        if (e == cudaSuccess) e = cudaGraphInstantiate(&gr->exec, graph, 0);
        if (e == cudaSuccess) {
            size_t n = 0;
            cudaGraphGetNodes(graph, nullptr, &n);
            std::vector<cudaGraphNode_t> nodes(n);
            cudaGraphGetNodes(graph, nodes.data(), &n);
            int64_t k = 0;
            for (auto nd : nodes) {
                cudaGraphNodeType t;
                if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++k;
            }
            gr->kernels = k;
            gr->captured = true;
        }
        if (graph) cudaGraphDestroy(graph);
        KG_CUDA(ctx, e);
    }
    KG_CUDA(ctx, cudaGraphLaunch(gr->exec, s));
    gr->last_use = ++ctx->graph_clock;
    ctx->last_graph_kernels = gr->kernels;
    return KG_OK;
}
}  // namespace

int kg_forward_batch_dev(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens,
                         const int32_t *start_pos, int32_t T, float *logits, float *probs, void *stream) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (!ctx->micro && !ctx->big_path) return fail(ctx, KG_ERR_UNSUPPORTED, "no forward kernel for this model shape");
    if (!ctx->compiled) return fail(ctx, KG_ERR_NOT_COMPILED, "weights not uploaded");
    if (n_seq < 0 || T < 1 || T > ctx->B || (ctx->micro && T > 16) || !seq_ids || !tokens)
        return fail(ctx, KG_ERR_INVALID_ARG, "bad batch shape");
    if (n_seq == 0) return KG_OK;
    ctx->last_graph_kernels = 0;
    if (ctx->big_path) {
        KG_CUDA(ctx, cudaSetDevice(ctx->device));
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (ctx->cfg.kv_mode == KG_KV_PAGED) KG_CUDA(ctx, kg::paged_flush(ctx, s));  // tables and reused pages first
        if (T == 1 && s != nullptr && !ctx->prof && n_seq <= std::min<int64_t>(ctx->big.ws_tokens, ctx->cfg.max_seqs))
            return forward_graph(ctx, n_seq, seq_ids, tokens, start_pos, logits, probs, s);
        cudaError_t e = kg::big_forward(ctx, n_seq, seq_ids, tokens, start_pos, T, logits, probs, s);
        if (e == cudaErrorInvalidValue && T > 1 && start_pos)
            return fail(ctx, KG_ERR_INVALID_ARG, "multi-position call from arbitrary positions: n_seq > max_seqs");
        KG_CUDA(ctx, e);
        return KG_OK;
    }
    if (ctx->cfg.kv_mode == KG_KV_SQ && !ctx->sq_ready)
        return fail(ctx, KG_ERR_NOT_COMPILED, "SpectralQuant tables not built (kg_sq_calibrate / kg_sq_calibrate_from)");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    kg::MicroArgs a = ctx->margs;
    a.n_seq = n_seq;
    a.T = T;
    a.seq_ids = seq_ids;
    a.tokens = tokens;
    a.start_pos = start_pos;
    a.logits = logits;
    a.probs = probs;
    // `stream` is used as given: NULL is the CUDA legacy default stream.
    if (ctx->cfg.kv_mode == KG_KV_PAGED) KG_CUDA(ctx, kg::paged_flush(ctx, static_cast<cudaStream_t>(stream)));
    KG_CUDA(ctx, kg::launch_micro(ctx->cfg, a, static_cast<cudaStream_t>(stream)));
    return KG_OK;
}

int kg_forward_batch(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens,
                     const int32_t *start_pos, int32_t T, float *logits_out, float *probs_out) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (n_seq < 0 || T < 1 || T > ctx->B || !seq_ids || !tokens)
        return fail(ctx, KG_ERR_INVALID_ARG, "bad batch shape");
    if (n_seq == 0) return KG_OK;
    // host-side argument checks (the kernel re-checks device-side)
    for (int32_t i = 0; i < n_seq; ++i) {
        if (seq_ids[i] < 0 || seq_ids[i] >= ctx->cfg.max_seqs)
            return fail(ctx, KG_ERR_INVALID_ARG, "sequence id out of range");
        int32_t p0 = start_pos ? start_pos[i] : 0;
        if (p0 < 0 || p0 + T > ctx->B) return fail(ctx, KG_ERR_INVALID_ARG, "position beyond block_size");
    }
    for (int64_t i = 0; i < (int64_t)n_seq * T; ++i)
        if (tokens[i] < 0 || tokens[i] >= ctx->V) return fail(ctx, KG_ERR_INVALID_ARG, "token out of range");
    if ((ctx->micro || ctx->big_path) && ctx->cfg.kv_mode == KG_KV_PAGED) {  // forward_paged's ensure_pages, in order
        int rc = kg::paged_ensure_batch(ctx, n_seq, seq_ids, start_pos, T);
        if (rc) return rc;
    }
    if (ctx->big_path && T > 1 && start_pos) {
        // all sequences from position 0: the prefill path (flash attention over the prompt)
        bool all0 = true;
        for (int32_t i = 0; i < n_seq; ++i) all0 = all0 && start_pos[i] == 0;
        if (all0) start_pos = nullptr;
    }
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const size_t b_ids = align256(n_seq * 4), b_tok = align256((size_t)n_seq * T * 4);
    const size_t b_out = align256((size_t)n_seq * T * ctx->V * 4);
    int rc = ensure_stage(ctx, 3 * b_ids + b_tok + 2 * b_out);
    if (rc) return rc;
    char *st = static_cast<char *>(ctx->stage);
    int32_t *d_ids = reinterpret_cast<int32_t *>(st);
    int32_t *d_pos = reinterpret_cast<int32_t *>(st + b_ids);
    int32_t *d_tok = reinterpret_cast<int32_t *>(st + 2 * b_ids);
    float *d_log = reinterpret_cast<float *>(st + 2 * b_ids + b_tok);
    float *d_prb = reinterpret_cast<float *>(st + 2 * b_ids + b_tok + b_out);
    cudaStream_t s = ctx->stream;
    KG_CUDA(ctx, cudaMemcpyAsync(d_ids, seq_ids, n_seq * 4, cudaMemcpyHostToDevice, s));
    if (start_pos) KG_CUDA(ctx, cudaMemcpyAsync(d_pos, start_pos, n_seq * 4, cudaMemcpyHostToDevice, s));
    KG_CUDA(ctx, cudaMemcpyAsync(d_tok, tokens, (size_t)n_seq * T * 4, cudaMemcpyHostToDevice, s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->d_err, 0, 4, s));
    rc = kg_forward_batch_dev(ctx, n_seq, d_ids, d_tok, start_pos ? d_pos : nullptr, T,
                              logits_out ? d_log : nullptr, probs_out ? d_prb : nullptr, s);
    if (rc) return rc;
    const size_t ob = (size_t)n_seq * T * ctx->V * 4;
    if (logits_out) KG_CUDA(ctx, cudaMemcpyAsync(logits_out, d_log, ob, cudaMemcpyDeviceToHost, s));
    if (probs_out) KG_CUDA(ctx, cudaMemcpyAsync(probs_out, d_prb, ob, cudaMemcpyDeviceToHost, s));
    int herr = 0;
    KG_CUDA(ctx, cudaMemcpyAsync(&herr, ctx->d_err, 4, cudaMemcpyDeviceToHost, s));
    KG_CUDA(ctx, cudaStreamSynchronize(s));
    if (herr == KG_ERR_TIMEOUT) return fail(ctx, KG_ERR_TIMEOUT, "a device-side wait exceeded its limit");
    if (herr) return fail(ctx, KG_ERR_INVALID_ARG, "device rejected a token, position or slot");
    return KG_OK;
}

int kg_forward_prefill_dev(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens, int32_t T,
                           float *logits_out, void *stream) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (!ctx->compiled) return fail(ctx, KG_ERR_NOT_COMPILED, "weights not uploaded");
    if (ctx->cfg.kv_mode != KG_KV_F32)
        return fail(ctx, KG_ERR_UNSUPPORTED, "forward_prefill runs over the f32 / bf16 K/V cache (kv_mode F32)");
    if (n_seq < 0 || T < 1 || T > ctx->B || (ctx->micro && T > 16) || !seq_ids || !tokens || !logits_out)
        return fail(ctx, KG_ERR_INVALID_ARG, "bad batch shape");
    if (n_seq == 0) return KG_OK;
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (ctx->big_path) {
        KG_CUDA(ctx, kg::big_forward_prefill(ctx, n_seq, seq_ids, tokens, T, logits_out, s));
        return KG_OK;
    }
    if (!ctx->micro) return fail(ctx, KG_ERR_UNSUPPORTED, "no forward kernel for this model shape");
    kg::MicroArgs a = ctx->margs;
    a.n_seq = n_seq;
    a.T = T;
    a.seq_ids = seq_ids;
    a.tokens = tokens;
    a.start_pos = nullptr;
    a.logits = logits_out;
    a.probs = nullptr;
    KG_CUDA(ctx, kg::launch_micro_prefill(ctx->cfg, a, s));
    return KG_OK;
}

int kg_forward_prefill(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens, int32_t T,
                       float *logits_out) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (n_seq < 0 || T < 1 || T > ctx->B || !seq_ids || !tokens || !logits_out)
        return fail(ctx, KG_ERR_INVALID_ARG, "bad batch shape");
    if (n_seq == 0) return KG_OK;
    for (int32_t i = 0; i < n_seq; ++i)
        if (seq_ids[i] < 0 || seq_ids[i] >= ctx->cfg.max_seqs)
            return fail(ctx, KG_ERR_INVALID_ARG, "sequence id out of range");
    for (int64_t i = 0; i < (int64_t)n_seq * T; ++i)
        if (tokens[i] < 0 || tokens[i] >= ctx->V) return fail(ctx, KG_ERR_INVALID_ARG, "token out of range");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const size_t b_ids = align256(n_seq * 4), b_tok = align256((size_t)n_seq * T * 4);
    const size_t b_out = align256((size_t)n_seq * ctx->V * 4);
    int rc = ensure_stage(ctx, b_ids + b_tok + b_out);
    if (rc) return rc;
    char *st = static_cast<char *>(ctx->stage);
    int32_t *d_ids = reinterpret_cast<int32_t *>(st);
    int32_t *d_tok = reinterpret_cast<int32_t *>(st + b_ids);
    float *d_log = reinterpret_cast<float *>(st + b_ids + b_tok);
    cudaStream_t s = ctx->stream;
    KG_CUDA(ctx, cudaMemcpyAsync(d_ids, seq_ids, n_seq * 4, cudaMemcpyHostToDevice, s));
    KG_CUDA(ctx, cudaMemcpyAsync(d_tok, tokens, (size_t)n_seq * T * 4, cudaMemcpyHostToDevice, s));
    KG_CUDA(ctx, cudaMemsetAsync(ctx->d_err, 0, 4, s));
    rc = kg_forward_prefill_dev(ctx, n_seq, d_ids, d_tok, T, d_log, s);
    if (rc) return rc;
    KG_CUDA(ctx, cudaMemcpyAsync(logits_out, d_log, (size_t)n_seq * ctx->V * 4, cudaMemcpyDeviceToHost, s));
    int herr = 0;
    KG_CUDA(ctx, cudaMemcpyAsync(&herr, ctx->d_err, 4, cudaMemcpyDeviceToHost, s));
    KG_CUDA(ctx, cudaStreamSynchronize(s));
    if (herr == KG_ERR_TIMEOUT) return fail(ctx, KG_ERR_TIMEOUT, "a device-side wait exceeded its limit");
    if (herr) return fail(ctx, KG_ERR_INVALID_ARG, "device rejected a token, position or slot");
    return KG_OK;
}

int kg_forward_token(kg_ctx *ctx, int32_t seq, int32_t token, int32_t pos, float *logits_out) {
    return kg_forward_batch(ctx, 1, &seq, &token, &pos, 1, logits_out, nullptr);
}

int kg_tq_tables(const kg_ctx *ctx, float *rot, float *kc, float *kb, float *vc, float *vb) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (!kg::kv_is_tq(ctx->cfg.kv_mode)) return KG_ERR_INVALID_ARG;
    if (rot) std::memcpy(rot, ctx->h_rot.data(), ctx->h_rot.size() * 4);
    if (kc) std::memcpy(kc, ctx->h_kc.data(), ctx->h_kc.size() * 4);
    if (kb) std::memcpy(kb, ctx->h_kb.data(), ctx->h_kb.size() * 4);
    if (vc) std::memcpy(vc, ctx->h_vc.data(), ctx->h_vc.size() * 4);
    if (vb) std::memcpy(vb, ctx->h_vb.data(), ctx->h_vb.size() * 4);
    return KG_OK;
}

int kg_tq_encode(kg_ctx *ctx, int32_t which, int64_t n_vec, const float *x, uint8_t *packed, float *norms) {
    if (!ctx || !x || !packed || !norms || n_vec < 0 || (which != 0 && which != 1))
        return KG_ERR_INVALID_ARG;
    if (!kg::kv_is_tq(ctx->cfg.kv_mode)) return fail(ctx, KG_ERR_INVALID_ARG, "context has no TurboQuant codec");
    if (n_vec == 0) return KG_OK;
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const int64_t kvd = ctx->kvd;
    const int bits = which == 0 ? ctx->cfg.key_bits : ctx->cfg.val_bits;
    const int64_t pl = packed_len(kvd, bits);
    const size_t bx = align256(n_vec * kvd * 4), bp = align256(n_vec * pl), bn = align256(n_vec * 4);
    const size_t bs = align256(n_vec);
    int rc = ensure_stage(ctx, 2 * bx + bp + bn + bs);
    if (rc) return rc;
    char *st = static_cast<char *>(ctx->stage);
    float *dx = reinterpret_cast<float *>(st);
    uint8_t *dp = reinterpret_cast<uint8_t *>(st + bx);
    float *dn = reinterpret_cast<float *>(st + bx + bp);
    float *dxn = reinterpret_cast<float *>(st + bx + bp + bn);
    uint8_t *dskip = reinterpret_cast<uint8_t *>(st + 2 * bx + bp + bn);
    cudaStream_t s = ctx->stream;
    KG_CUDA(ctx, cudaMemcpyAsync(dx, x, n_vec * kvd * 4, cudaMemcpyHostToDevice, s));
    // codes of a zero-norm vector are left untouched: start from the caller's bytes
    KG_CUDA(ctx, cudaMemcpyAsync(dp, packed, n_vec * pl, cudaMemcpyHostToDevice, s));
    const float *bnd = which == 0 ? ctx->kb : ctx->vb;
    if (kvd % 64 == 0 && (bits == 3 || bits == 4)) {
        // tensor-core rotation with exact fix-up (the encoder of the forward path)
        if (!ctx->big_path && !ctx->enc_rh) {
            if ((rc = dalloc(ctx, &ctx->enc_rh, kvd * kvd)) || (rc = dalloc(ctx, &ctx->enc_rl, kvd * kvd))) return rc;
            KG_CUDA(ctx, kg::bf::f32_to_f16_split(ctx->rot, kvd * kvd, ctx->enc_rh, ctx->enc_rl, s));
        }
        const size_t bh = align256(n_vec * kvd * 2);
        rc = ensure_stage(ctx, 2 * bx + bp + bn + bs + 2 * bh + bx);
        if (rc) return rc;
        st = static_cast<char *>(ctx->stage);  // (re)allocated: recompute the carve-up
        dx = reinterpret_cast<float *>(st);
        dp = reinterpret_cast<uint8_t *>(st + bx);
        dn = reinterpret_cast<float *>(st + bx + bp);
        dxn = reinterpret_cast<float *>(st + bx + bp + bn);
        dskip = reinterpret_cast<uint8_t *>(st + 2 * bx + bp + bn);
        __half *dxh = reinterpret_cast<__half *>(st + 2 * bx + bp + bn + bs);
        __half *dxl = reinterpret_cast<__half *>(st + 2 * bx + bp + bn + bs + bh);
        float *dy = reinterpret_cast<float *>(st + 2 * bx + bp + bn + bs + 2 * bh);
        KG_CUDA(ctx, cudaMemcpyAsync(dx, x, n_vec * kvd * 4, cudaMemcpyHostToDevice, s));
        KG_CUDA(ctx, cudaMemcpyAsync(dp, packed, n_vec * pl, cudaMemcpyHostToDevice, s));
        const int mk = which == 0 ? (int)n_vec : 0, mv = which == 1 ? (int)n_vec : 0;
        KG_CUDA(ctx, kg::tq_norm_split((int)kvd, mk, mv, dx, kvd, 0, 0, dxn, dxh, dxl, dskip, dn, dn, nullptr, nullptr,
                                       0, 0, 0, s));
        kg::bf::Gemm g;
        std::memset(&g, 0, sizeof(g));
        g.dtype = kg::bf::DT_F16;
        g.A = dxh; g.A2 = dxl; g.lda = kvd;
        g.B = ctx->big_path ? ctx->big.rot_h : ctx->enc_rh;
        g.B2 = ctx->big_path ? ctx->big.rot_l : ctx->enc_rl;
        g.ldb = kvd;
        g.M = (int)n_vec; g.N = (int)kvd; g.K = (int)kvd; g.batch = 1;
        g.epi = kg::bf::EPI_F32; g.C = dy; g.ldc = kvd;
        KG_CUDA(ctx, kg::gemm_auto(ctx, &g, s));
        KG_CUDA(ctx, kg::tq_quantize_fixup((int)kvd, mk, mv, dy, dxn, dskip, ctx->rot, bnd, bnd, bits, bits, dp, dp,
                                           pl, pl, nullptr, nullptr, 0, 0, 0, nullptr, s));
    } else {
        KG_CUDA(ctx, kg::tq_encode_device((int)kvd, bits, n_vec, dx, ctx->rot, bnd, dp, pl, dn, 1, s));
    }
    KG_CUDA(ctx, cudaMemcpyAsync(packed, dp, n_vec * pl, cudaMemcpyDeviceToHost, s));
    KG_CUDA(ctx, cudaMemcpyAsync(norms, dn, n_vec * 4, cudaMemcpyDeviceToHost, s));
    KG_CUDA(ctx, cudaStreamSynchronize(s));
    return KG_OK;
}

int kg_kv_codes(kg_ctx *ctx, int32_t seq, int32_t layer, int32_t pos, uint8_t *kcodes, uint8_t *vcodes,
                float *norms) {
    if (!ctx || seq < 0 || seq >= ctx->cfg.max_seqs || layer < 0 || layer >= ctx->L || pos < 0 || pos >= ctx->B)
        return KG_ERR_INVALID_ARG;
    if (ctx->big_path) {
        KG_CUDA(ctx, cudaSetDevice(ctx->device));
        const int64_t row = ((int64_t)seq * ctx->L + layer) * ctx->B + pos;
        cudaStream_t s = ctx->stream;
        if (kcodes) KG_CUDA(ctx, cudaMemcpyAsync(kcodes, ctx->big.kcodes + row * ctx->kpl, ctx->kpl, cudaMemcpyDeviceToHost, s));
        if (vcodes) KG_CUDA(ctx, cudaMemcpyAsync(vcodes, ctx->big.vcodes + row * ctx->vpl, ctx->vpl, cudaMemcpyDeviceToHost, s));
        if (norms) {
            KG_CUDA(ctx, cudaMemcpyAsync(norms, ctx->big.knorm + row, 4, cudaMemcpyDeviceToHost, s));
            KG_CUDA(ctx, cudaMemcpyAsync(norms + 1, ctx->big.vnorm + row, 4, cudaMemcpyDeviceToHost, s));
        }
        KG_CUDA(ctx, cudaStreamSynchronize(s));
        return KG_OK;
    }
    if (!ctx->micro) return fail(ctx, KG_ERR_UNSUPPORTED, "no KV arena for this model shape");
    if (!kg::kv_has_codes(ctx->cfg.kv_mode)) return fail(ctx, KG_ERR_INVALID_ARG, "context has no KV codec");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const int64_t row = ((int64_t)seq * ctx->L + layer) * ctx->B + pos;
    cudaStream_t s = ctx->stream;
    if (kcodes) KG_CUDA(ctx, cudaMemcpyAsync(kcodes, ctx->codes + row * (ctx->kpl + ctx->vpl), ctx->kpl, cudaMemcpyDeviceToHost, s));
    if (vcodes) KG_CUDA(ctx, cudaMemcpyAsync(vcodes, ctx->codes + row * (ctx->kpl + ctx->vpl) + ctx->kpl, ctx->vpl, cudaMemcpyDeviceToHost, s));
    if (norms) KG_CUDA(ctx, cudaMemcpyAsync(norms, ctx->norms + row * 2, 8, cudaMemcpyDeviceToHost, s));
    KG_CUDA(ctx, cudaStreamSynchronize(s));
    return KG_OK;
}

int kg_spkv_utility(kg_ctx *ctx, int32_t seq, int32_t layer, int32_t pos, float *utility) {
    if (ctx && !ctx->micro) return fail(ctx, KG_ERR_UNSUPPORTED, "no KV arena for this model shape");
    if (!ctx || !utility || seq < 0 || seq >= ctx->cfg.max_seqs || layer < 0 || layer >= ctx->L || pos < 0 ||
        pos >= ctx->B)
        return KG_ERR_INVALID_ARG;
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const int64_t row = ((int64_t)seq * ctx->L + layer) * ctx->B + pos;
    KG_CUDA(ctx, cudaMemcpy(utility, ctx->util + row, 4, cudaMemcpyDeviceToHost));
    return KG_OK;
}

int kg_profile(kg_ctx *ctx, int enable) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    ctx->prof = enable != 0;
    return KG_OK;
}

int kg_profile_read(kg_ctx *ctx, float *ms, int64_t *count) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    KG_CUDA(ctx, cudaDeviceSynchronize());
    for (int p = 0; p < KG_PROF_N; ++p) {
        float tot = 0.0f;
        for (size_t i = 0; i < ctx->prof_used[p]; ++i) {
            float t = 0.0f;
            KG_CUDA(ctx, cudaEventElapsedTime(&t, ctx->prof_ev[p][0][i], ctx->prof_ev[p][1][i]));
            tot += t;
        }
        if (ms) ms[p] = tot;
        if (count) count[p] = (int64_t)ctx->prof_used[p];
        ctx->prof_used[p] = 0;
    }
    return KG_OK;
}

}  // extern "C"

namespace kg {
// Record the begin (end = 0) or end (end = 1) event of one interval of `phase`.
void prof_mark(kg_ctx *ctx, int phase, int end, cudaStream_t s) {
    if (!ctx->prof) return;
    auto &evs = ctx->prof_ev[phase][end];
    size_t i = ctx->prof_used[phase];
    while (evs.size() <= i) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return;
        evs.push_back(e);
    }
    cudaEventRecord(evs[i], s);
    if (end) ctx->prof_used[phase] = i + 1;
}
}  // namespace kg

int64_t kg_graph_kernels(const kg_ctx *ctx) { return ctx ? ctx->last_graph_kernels : 0; }

// ---- sequence slots and KV snapshots ---------------------------------------

int kg_seq_alloc(kg_ctx *ctx, int32_t *seq_out) {
    if (!ctx || !seq_out) return KG_ERR_INVALID_ARG;
    if (ctx->slot_used.size() != (size_t)ctx->cfg.max_seqs) ctx->slot_used.assign(ctx->cfg.max_seqs, 0);
    for (int32_t i = 0; i < ctx->cfg.max_seqs; ++i)
        if (!ctx->slot_used[i]) {
            const int rc = kg_seq_reset(ctx, i);
            if (rc) return rc;
            ctx->slot_used[i] = 1;
            *seq_out = i;
            return KG_OK;
        }
    return fail(ctx, KG_ERR_OOM, "no free sequence slot");
}

int kg_seq_free(kg_ctx *ctx, int32_t seq) {
    if (!ctx || seq < 0 || seq >= ctx->cfg.max_seqs) return KG_ERR_INVALID_ARG;
    if (ctx->slot_used.size() == (size_t)ctx->cfg.max_seqs) ctx->slot_used[seq] = 0;
    return KG_OK;
}

namespace {
// One per-sequence cache array: `w` bytes per position, layer planes of
// block_size positions, slot planes of L layers.
struct KvArray {
    uint8_t *base;
    size_t w;
};
int kv_arrays(const kg_ctx *ctx, KvArray *out) {
    int n = 0;
    if (ctx->big_path && ctx->big.std_kv) {
        out[n++] = {reinterpret_cast<uint8_t *>(ctx->big.kcache), (size_t)ctx->kvd * 2};
        out[n++] = {reinterpret_cast<uint8_t *>(ctx->big.vcache), (size_t)ctx->kvd * 2};
    } else if (ctx->big_path) {
        const kg::BigState &g = ctx->big;
        out[n++] = {g.kcodes, (size_t)ctx->kpl};
        out[n++] = {g.vcodes, (size_t)ctx->vpl};
        out[n++] = {reinterpret_cast<uint8_t *>(g.knorm), 4};
        out[n++] = {reinterpret_cast<uint8_t *>(g.vnorm), 4};
    } else if (ctx->micro && ctx->cfg.kv_mode != KG_KV_PAGED) {  // paged contexts roll back by page tables
        out[n++] = {reinterpret_cast<uint8_t *>(ctx->Kf), (size_t)ctx->kvd * 4};
        out[n++] = {reinterpret_cast<uint8_t *>(ctx->Vf), (size_t)ctx->kvd * 4};
        if (ctx->kpl + ctx->vpl) out[n++] = {ctx->codes, (size_t)(ctx->kpl + ctx->vpl)};
        out[n++] = {reinterpret_cast<uint8_t *>(ctx->norms), 8};
        out[n++] = {reinterpret_cast<uint8_t *>(ctx->util), 4};
    }
    return n;
}
}  // namespace

int64_t kg_kv_snapshot_bytes(const kg_ctx *ctx, int32_t pos) {
    if (!ctx || pos < 0 || pos > ctx->B) return 0;
    KvArray arr[8];
    const int n = kv_arrays(ctx, arr);
    int64_t b = 0;
    for (int i = 0; i < n; ++i) b += (int64_t)pos * ctx->L * arr[i].w;
    return b;
}

int kg_kv_snapshot(kg_ctx *ctx, int32_t seq, int32_t pos, void *dst_dev, void *stream) {
    if (!ctx || seq < 0 || seq >= ctx->cfg.max_seqs || pos < 0 || pos > ctx->B || (pos > 0 && !dst_dev))
        return KG_ERR_INVALID_ARG;
    if (!ctx->big_path && !ctx->micro) return fail(ctx, KG_ERR_UNSUPPORTED, "no device KV cache for this shape");
    if (ctx->cfg.kv_mode == KG_KV_PAGED)
        return fail(ctx, KG_ERR_UNSUPPORTED, "a paged context rolls back with kg_paged_rollback / kg_paged_fork");
    if (pos == 0) return KG_OK;
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    KvArray arr[8];
    const int n = kv_arrays(ctx, arr);
    uint8_t *dst = static_cast<uint8_t *>(dst_dev);
    for (int i = 0; i < n; ++i) {
        const size_t pitch = (size_t)ctx->B * arr[i].w, width = (size_t)pos * arr[i].w;
        const uint8_t *src = arr[i].base + (size_t)seq * ctx->L * pitch;
        KG_CUDA(ctx, cudaMemcpy2DAsync(dst, width, src, pitch, width, ctx->L, cudaMemcpyDeviceToDevice, s));
        dst += width * ctx->L;
    }
    return KG_OK;
}

int kg_kv_restore(kg_ctx *ctx, int32_t seq, int32_t pos, const void *src_dev, void *stream) {
    if (!ctx || seq < 0 || seq >= ctx->cfg.max_seqs || pos < 0 || pos > ctx->B || (pos > 0 && !src_dev))
        return KG_ERR_INVALID_ARG;
    if (!ctx->big_path && !ctx->micro) return fail(ctx, KG_ERR_UNSUPPORTED, "no device KV cache for this shape");
    if (ctx->cfg.kv_mode == KG_KV_PAGED)
        return fail(ctx, KG_ERR_UNSUPPORTED, "a paged context rolls back with kg_paged_rollback / kg_paged_fork");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    KvArray arr[8];
    const int n = kv_arrays(ctx, arr);
    const uint8_t *src = static_cast<const uint8_t *>(src_dev);
    for (int i = 0; i < n; ++i) {
        const size_t pitch = (size_t)ctx->B * arr[i].w, width = (size_t)pos * arr[i].w;
        uint8_t *dst = arr[i].base + (size_t)seq * ctx->L * pitch;
        if (pos > 0) {
            KG_CUDA(ctx, cudaMemcpy2DAsync(dst, pitch, src, width, width, ctx->L, cudaMemcpyDeviceToDevice, s));
            src += width * ctx->L;
        }
        if (pos < ctx->B) KG_CUDA(ctx, cudaMemset2DAsync(dst + width, pitch, 0, pitch - width, ctx->L, s));
    }
    return KG_OK;
}

int kg_set_mlp_hook(kg_ctx *ctx, float keep, uint64_t seed) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (!ctx->big_path) return fail(ctx, KG_ERR_UNSUPPORTED, "the hook applies to the bf16 path");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    for (auto &gr : ctx->graphs) {  // captured with the previous setting
        if (gr.stream) KG_CUDA(ctx, cudaStreamSynchronize(gr.stream));
        if (gr.exec) cudaGraphExecDestroy(gr.exec);
    }
    ctx->graphs.clear();
    ctx->hook_keep = keep > 0.0f ? std::min(keep, 1.0f) : 0.0f;
    ctx->hook_seed = seed;
    return KG_OK;
}

// ---- LoraPair (crates/katgpt-types/src/lora.rs) on the exact micro path ----

int kg_set_lora(kg_ctx *ctx, int32_t which, int32_t rank, int32_t in_dim, int32_t out_dim, float alpha,
                const float *a, const float *b) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (which < 0 || which > 1) return fail(ctx, KG_ERR_INVALID_ARG, "which: 0 = reader (forward_prefill), 1 = writer");
    const bool spkv = ctx->cfg.kv_mode == KG_KV_SPKV_TQ;
    if (!ctx->micro || (ctx->cfg.kv_mode != KG_KV_F32 && !spkv) || (spkv && which == 0))
        return fail(ctx, KG_ERR_UNSUPPORTED,
                    "LoRA: the exact path's forward_base / forward_prefill (kv_mode F32) or forward_sp_kv_quant (writer)");
    kg::MicroArgs &m = ctx->margs;
    if (rank == 0) {
        m.lora_rank[which] = 0;
        return KG_OK;
    }
    const int32_t max_in = (int32_t)std::min<int64_t>(ctx->n, kg::kLoraMax);
    const int32_t max_out = (int32_t)std::min<int64_t>(std::min(ctx->n, ctx->kvd), kg::kLoraMax);
    if (rank < 1 || rank > kg::kLoraMax || in_dim < 1 || in_dim > max_in || out_dim < 1 || out_dim > max_out || !a ||
        !b)
        return fail(ctx, KG_ERR_INVALID_ARG, "LoRA adapter: rank 1..16, in_dim 1.." + std::to_string(max_in) +
                                                 ", out_dim 1.." + std::to_string(max_out) + ", A and B given");
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    KG_CUDA(ctx, cudaDeviceSynchronize());  // no forward in flight reads the pack meanwhile
    KG_CUDA(ctx, cudaMemcpy(ctx->pack + m.off_lora_a[which], a, (size_t)rank * in_dim * 4, cudaMemcpyHostToDevice));
    KG_CUDA(ctx, cudaMemcpy(ctx->pack + m.off_lora_b[which], b, (size_t)out_dim * rank * 4, cudaMemcpyHostToDevice));
    m.lora_rank[which] = rank;
    m.lora_in[which] = in_dim;
    m.lora_out[which] = out_dim;
    m.lora_scale[which] = alpha / (float)rank;  // lora.rs:453
    return KG_OK;
}

// ---- SpectralQuant calibration (kg_sq.cpp builds the tables on the host) ----

namespace {
int sq_install(kg_ctx *ctx, const kg_sq_params *p, const float *eig, const float *eval, const float *deff,
               bool per_layer) {
    const int64_t kvd = ctx->kvd, L = ctx->L;
    std::vector<float> E(L * kvd * kvd), C(L * kvd * kg::kSqLevels), meta(L * kvd);
    std::vector<uint8_t> bits(L * kvd);
    std::vector<int32_t> lev(L * kvd), de(L);
    for (int64_t l = 0; l < L; ++l) {
        const int64_t o = per_layer ? l : 0;
        if (!kg::sq_build_layer(*p, kvd, l, eig + o * kvd * kvd, eval + o * kvd, deff[o], &E[l * kvd * kvd],
                                &bits[l * kvd], &C[l * kvd * kg::kSqLevels], &lev[l * kvd], &de[l]))
            return fail(ctx, KG_ERR_UNSUPPORTED, "SpectralQuant codebook wider than 64 centroids (6 bits)");
        for (int64_t j = 0; j < kvd; ++j) {
            const int32_t m = (int32_t)bits[l * kvd + j] | (lev[l * kvd + j] << 8);
            std::memcpy(&meta[l * kvd + j], &m, 4);
        }
    }
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    if (ctx->micro) {  // the micro forward's shared-memory pack
        const kg::MicroArgs &a = ctx->margs;
        KG_CUDA(ctx, cudaMemcpy(ctx->pack + a.off_sq_eig, E.data(), E.size() * 4, cudaMemcpyHostToDevice));
        KG_CUDA(ctx, cudaMemcpy(ctx->pack + a.off_sq_cent, C.data(), C.size() * 4, cudaMemcpyHostToDevice));
        KG_CUDA(ctx, cudaMemcpy(ctx->pack + a.off_sq_meta, meta.data(), meta.size() * 4, cudaMemcpyHostToDevice));
    }
    // the codec entry points' tables: width | levels << 8 and bit offsets per dimension
    std::vector<int32_t> imeta(L * kvd), offs(L * kvd);
    ctx->sq_nbytes.assign(L, 0);
    for (int64_t l = 0; l < L; ++l) {
        int64_t o = 0;
        for (int64_t j = 0; j < kvd; ++j) {
            imeta[l * kvd + j] = (int32_t)bits[l * kvd + j] | (lev[l * kvd + j] << 8);
            offs[l * kvd + j] = (int32_t)o;
            o += bits[l * kvd + j];
        }
        ctx->sq_nbytes[l] = (int)((o + 7) / 8);
    }
    int rc = 0;
    if (!ctx->sq_eig_d && ((rc = dalloc(ctx, &ctx->sq_eig_d, E.size())) || (rc = dalloc(ctx, &ctx->sq_cent_d, C.size())) ||
                           (rc = dalloc(ctx, &ctx->sq_meta_d, imeta.size())) ||
                           (rc = dalloc(ctx, &ctx->sq_offs_d, offs.size()))))
        return rc;
    KG_CUDA(ctx, cudaMemcpy(ctx->sq_eig_d, E.data(), E.size() * 4, cudaMemcpyHostToDevice));
    KG_CUDA(ctx, cudaMemcpy(ctx->sq_cent_d, C.data(), C.size() * 4, cudaMemcpyHostToDevice));
    KG_CUDA(ctx, cudaMemcpy(ctx->sq_meta_d, imeta.data(), imeta.size() * 4, cudaMemcpyHostToDevice));
    KG_CUDA(ctx, cudaMemcpy(ctx->sq_offs_d, offs.data(), offs.size() * 4, cudaMemcpyHostToDevice));
    ctx->h_sq_eig = std::move(E);
    ctx->h_sq_cent = std::move(C);
    ctx->h_sq_bits = std::move(bits);
    ctx->h_sq_lev = std::move(lev);
    ctx->h_sq_deff = std::move(de);
    ctx->sq_ready = true;
    return KG_OK;
}
int sq_check(kg_ctx *ctx, const kg_sq_params *p) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (ctx->cfg.kv_mode != KG_KV_SQ) return fail(ctx, KG_ERR_UNSUPPORTED, "context is not kv_mode KG_KV_SQ");
    if (!p || p->max_bits < 1 || p->max_bits > 8 || p->lloyd_max_iter < 0 || p->wf_min_bits < 1 ||
        p->wf_max_bits < p->wf_min_bits || p->wf_max_bits > 8)
        return fail(ctx, KG_ERR_INVALID_ARG, "bad SpectralQuant parameters");
    return KG_OK;
}
}  // namespace

void kg_sq_params_default(kg_sq_params *p) {
    if (!p) return;
    p->seed = 42;
    p->lloyd_max_iter = 30;
    p->calibration_samples = 100;
    p->avg_bits = 3.0f;
    p->min_tail_bits = 1;
    p->max_bits = 8;
    p->wf_min_bits = 1;
    p->wf_max_bits = 6;
    p->use_water_fill = 0;
}

int kg_sq_calibrate(kg_ctx *ctx, const kg_sq_params *p, const float *key_samples, int64_t n_samples) {
    if (int rc = sq_check(ctx, p)) return rc;
    if (!key_samples || n_samples < 1) return fail(ctx, KG_ERR_INVALID_ARG, "need at least one calibration sample");
    std::vector<float> vecs, vals;
    float d_eff = 0.0f;
    kg::sq_calibrate(key_samples, n_samples, ctx->kvd, vecs, vals, d_eff);
    return sq_install(ctx, p, vecs.data(), vals.data(), &d_eff, false);
}

int kg_sq_calibrate_from(kg_ctx *ctx, const kg_sq_params *p, const float *eigenvectors, const float *eigenvalues,
                         const float *d_eff) {
    if (int rc = sq_check(ctx, p)) return rc;
    if (!eigenvectors || !eigenvalues || !d_eff) return fail(ctx, KG_ERR_INVALID_ARG, "null calibration");
    return sq_install(ctx, p, eigenvectors, eigenvalues, d_eff, true);
}

int kg_sq_tables(const kg_ctx *ctx, int32_t layer, float *eig, uint8_t *bits, float *cent, int32_t *lev,
                 int32_t *d_eff) {
    if (!ctx || !ctx->sq_ready || layer < 0 || layer >= ctx->L) return KG_ERR_INVALID_ARG;
    const int64_t kvd = ctx->kvd;
    if (eig) std::memcpy(eig, &ctx->h_sq_eig[layer * kvd * kvd], kvd * kvd * 4);
    if (bits) std::memcpy(bits, &ctx->h_sq_bits[layer * kvd], kvd);
    if (cent) std::memcpy(cent, &ctx->h_sq_cent[layer * kvd * kg::kSqLevels], kvd * kg::kSqLevels * 4);
    if (lev) std::memcpy(lev, &ctx->h_sq_lev[layer * kvd], kvd * 4);
    if (d_eff) *d_eff = ctx->h_sq_deff[layer];
    return KG_OK;
}

int kg_sq_calibrate_eigenbasis(const float *samples, int64_t n_samples, int64_t dim, float *eigenvectors,
                               float *eigenvalues, float *d_eff) {
    if (!samples || n_samples < 1 || dim < 2 || !eigenvectors || !eigenvalues || !d_eff) return KG_ERR_INVALID_ARG;
    std::vector<float> vecs, vals;
    kg::sq_calibrate(samples, n_samples, dim, vecs, vals, *d_eff);
    std::memcpy(eigenvectors, vecs.data(), dim * dim * 4);
    std::memcpy(eigenvalues, vals.data(), dim * 4);
    return KG_OK;
}

int kg_sq_build_tables(const kg_sq_params *p, int64_t kv_dim, int32_t n_layers, const float *eigenvectors,
                       const float *eigenvalues, const float *d_eff, float *eig_out, uint8_t *bits_out,
                       float *centroids_out, int32_t *n_levels_out, int32_t *d_eff_out) {
    if (!p || kv_dim < 2 || n_layers < 1 || !eigenvectors || !eigenvalues || !d_eff || !eig_out || !bits_out ||
        !centroids_out || !n_levels_out || !d_eff_out || p->max_bits < 1 || p->max_bits > 8)
        return KG_ERR_INVALID_ARG;
    for (int32_t l = 0; l < n_layers; ++l)
        if (!kg::sq_build_layer(*p, kv_dim, l, eigenvectors + l * kv_dim * kv_dim, eigenvalues + l * kv_dim, d_eff[l],
                                eig_out + l * kv_dim * kv_dim, bits_out + l * kv_dim,
                                centroids_out + l * kv_dim * kg::kSqLevels, n_levels_out + l * kv_dim, d_eff_out + l))
            return KG_ERR_UNSUPPORTED;
    return KG_OK;
}

// ---- SpectralQuant codec at any kv_dim (host pointers; synchronous) ----

int kg_sq_encode(kg_ctx *ctx, int32_t layer, int64_t n_vec, const float *x, uint8_t *packed, float *norms) {
    if (!ctx || !x || !packed || !norms || n_vec < 0) return KG_ERR_INVALID_ARG;
    if (!ctx->sq_ready) return fail(ctx, KG_ERR_NOT_COMPILED, "SpectralQuant tables not built");
    if (layer < 0 || layer >= ctx->L) return fail(ctx, KG_ERR_INVALID_ARG, "layer out of range");
    if (n_vec == 0) return KG_OK;
    if (n_vec > INT32_MAX) return fail(ctx, KG_ERR_INVALID_ARG, "too many vectors in one call");
    const int64_t kvd = ctx->kvd;
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const size_t bx = align256(n_vec * kvd * 4), bp = align256(n_vec * kvd), bn = align256(n_vec * 4);
    int rc = ensure_stage(ctx, bx + bp + bn);
    if (rc) return rc;
    char *st = static_cast<char *>(ctx->stage);
    float *dx = reinterpret_cast<float *>(st);
    uint8_t *dp = reinterpret_cast<uint8_t *>(st + bx);
    float *dn = reinterpret_cast<float *>(st + bx + bp);
    cudaStream_t s = ctx->stream;
    KG_CUDA(ctx, cudaMemcpyAsync(dx, x, n_vec * kvd * 4, cudaMemcpyHostToDevice, s));
    KG_CUDA(ctx, cudaMemcpyAsync(dp, packed, n_vec * kvd, cudaMemcpyHostToDevice, s));  // zero-norm rows keep theirs
    KG_CUDA(ctx, kg::sq_encode_device((int)kvd, n_vec, dx, ctx->sq_eig_d + layer * kvd * kvd, ctx->sq_meta_d + layer * kvd,
                                      ctx->sq_cent_d + layer * kvd * kg::kSqLevels, ctx->sq_offs_d + layer * kvd,
                                      ctx->sq_nbytes[layer], dp, kvd, dn, s));
    KG_CUDA(ctx, cudaMemcpyAsync(packed, dp, n_vec * kvd, cudaMemcpyDeviceToHost, s));
    KG_CUDA(ctx, cudaMemcpyAsync(norms, dn, n_vec * 4, cudaMemcpyDeviceToHost, s));
    KG_CUDA(ctx, cudaStreamSynchronize(s));
    return KG_OK;
}

int kg_sq_decode(kg_ctx *ctx, int32_t layer, int64_t n_vec, const uint8_t *packed, const float *norms, float *out) {
    if (!ctx || !packed || !norms || !out || n_vec < 0) return KG_ERR_INVALID_ARG;
    if (!ctx->sq_ready) return fail(ctx, KG_ERR_NOT_COMPILED, "SpectralQuant tables not built");
    if (layer < 0 || layer >= ctx->L) return fail(ctx, KG_ERR_INVALID_ARG, "layer out of range");
    if (n_vec == 0) return KG_OK;
    if (n_vec > INT32_MAX) return fail(ctx, KG_ERR_INVALID_ARG, "too many vectors in one call");
    const int64_t kvd = ctx->kvd;
    KG_CUDA(ctx, cudaSetDevice(ctx->device));
    const size_t bx = align256(n_vec * kvd * 4), bp = align256(n_vec * kvd), bn = align256(n_vec * 4);
    int rc = ensure_stage(ctx, bx + bp + bn);
    if (rc) return rc;
    char *st = static_cast<char *>(ctx->stage);
    float *dx = reinterpret_cast<float *>(st);
    uint8_t *dp = reinterpret_cast<uint8_t *>(st + bx);
    float *dn = reinterpret_cast<float *>(st + bx + bp);
    cudaStream_t s = ctx->stream;
    KG_CUDA(ctx, cudaMemcpyAsync(dp, packed, n_vec * kvd, cudaMemcpyHostToDevice, s));
    KG_CUDA(ctx, cudaMemcpyAsync(dn, norms, n_vec * 4, cudaMemcpyHostToDevice, s));
    KG_CUDA(ctx, kg::sq_decode_device((int)kvd, n_vec, dp, kvd, dn, ctx->sq_eig_d + layer * kvd * kvd,
                                      ctx->sq_meta_d + layer * kvd, ctx->sq_cent_d + layer * kvd * kg::kSqLevels,
                                      ctx->sq_offs_d + layer * kvd, ctx->sq_nbytes[layer], dx, s));
    KG_CUDA(ctx, cudaMemcpyAsync(out, dx, n_vec * kvd * 4, cudaMemcpyDeviceToHost, s));
    KG_CUDA(ctx, cudaStreamSynchronize(s));
    return KG_OK;
}
