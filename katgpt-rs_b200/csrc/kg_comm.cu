// kg_comm.cu — the one exchange of multi-GPU decode, inside the library.
//
// Sequences are independent (the reference's batch path is a per-sequence
// par_iter, src/transformer.rs:3588-3606), so N GPUs each run a shard of the
// sequences against their own replica of the weights and KV arena; after each
// decode step every rank needs every shard's logits (or sampled tokens). That
// all-gather runs here, on the caller's stream right after the step, over
// NCCL (NVLink / NVSwitch). NCCL is loaded at run time (libnccl.so.2), so the
// library loads on hosts without it; the multi-GPU entry points then return
// KG_ERR_UNSUPPORTED. The gather is in place: rank r's step writes its rows at
// offset r of the gathered buffer, which is NCCL's in-place all-gather form.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "kg_internal.h"

namespace kg {
namespace {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        // an NCCL already loaded in the process (e.g. by the caller's framework) is reused
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.all_gather && api.comm_destroy && api.error_string;
    });
    return api;
}

int fail(kg_ctx *ctx, int code, const std::string &m) {
    if (ctx) ctx->err = m;
    return code;
}
int nccl_fail(kg_ctx *ctx, ncclResult_t r, const char *what) {
    return fail(ctx, KG_ERR_CUDA, std::string(what) + ": " + nccl().error_string(r));
}

}  // namespace
}  // namespace kg

extern "C" {

int kg_comm_unique_id(uint8_t *id_out) {
    if (!id_out) return KG_ERR_INVALID_ARG;
    const kg::NcclApi &api = kg::nccl();
    if (!api.ok) return KG_ERR_UNSUPPORTED;
    ncclUniqueId id;
    if (api.get_unique_id(&id) != ncclSuccess) return KG_ERR_CUDA;
    std::memcpy(id_out, id.internal, NCCL_UNIQUE_ID_BYTES);
    return KG_OK;
}

int kg_comm_init(kg_ctx *ctx, const uint8_t *id, int32_t world, int32_t rank) {
    if (!ctx || !id || world < 1 || rank < 0 || rank >= world) return KG_ERR_INVALID_ARG;
    if (ctx->comm) return kg::fail(ctx, KG_ERR_INVALID_ARG, "the context already has a communicator");
    const kg::NcclApi &api = kg::nccl();
    if (!api.ok) return kg::fail(ctx, KG_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return kg::fail(ctx, KG_ERR_CUDA, cudaGetErrorString(e));
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t comm = nullptr;
    const ncclResult_t r = api.comm_init_rank(&comm, world, uid, rank);
    if (r != ncclSuccess) return kg::nccl_fail(ctx, r, "ncclCommInitRank");
    ctx->comm = comm;
    ctx->world = world;
    ctx->rank = rank;
    return KG_OK;
}

int kg_comm_destroy(kg_ctx *ctx) {
    if (!ctx) return KG_ERR_INVALID_ARG;
    if (!ctx->comm) return KG_OK;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    const ncclResult_t r = kg::nccl().comm_destroy(static_cast<ncclComm_t>(ctx->comm));
    ctx->comm = nullptr;
    ctx->world = 1;
    ctx->rank = 0;
    if (r != ncclSuccess) return kg::nccl_fail(ctx, r, "ncclCommDestroy");
    return KG_OK;
}

int kg_decode_gather_dev(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens,
                         const int32_t *positions, float *logits_all, int32_t *tokens_all, void *stream) {
    if (!ctx || n_seq < 1 || !seq_ids || !tokens || !positions || (!logits_all && !tokens_all))
        return KG_ERR_INVALID_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t V = ctx->V, r = ctx->rank;
    float *probs = nullptr;
    int rc = KG_OK;
    if (tokens_all) {
        if (n_seq > ctx->cfg.max_seqs) {
            rc = kg::fail(ctx, KG_ERR_INVALID_ARG, "n_seq exceeds max_seqs");
        } else if (!ctx->probs_buf) {  // first use: a fixed buffer, so captured decode graphs stay valid
            cudaError_t e = cudaSetDevice(ctx->device);
            if (e == cudaSuccess) e = cudaMalloc(&ctx->probs_buf, (size_t)ctx->cfg.max_seqs * V * sizeof(float));
            if (e == cudaSuccess) ctx->allocs.push_back(ctx->probs_buf);
            else rc = kg::fail(ctx, KG_ERR_OOM, std::string("probs buffer: ") + cudaGetErrorString(e));
        }
        probs = ctx->probs_buf;
    }
    float *my_logits = logits_all ? logits_all + r * n_seq * V : nullptr;
    if (rc == KG_OK) rc = kg_forward_batch_dev(ctx, n_seq, seq_ids, tokens, positions, 1, my_logits, probs, stream);
    if (rc == KG_OK && tokens_all) rc = kg_sample_dev(ctx, n_seq, seq_ids, probs, V, tokens_all + r * n_seq, stream);
    if (!ctx->comm || ctx->world == 1) return rc;
    // The gathers are issued whatever happened above, so that a local error
    // leaves no other rank waiting in its own gather (this rank's rows are then
    // stale); the call still returns that error.
    const kg::NcclApi &api = kg::nccl();
    ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
    if (logits_all) {
        const ncclResult_t nr = api.all_gather(my_logits, logits_all, (size_t)n_seq * V, ncclFloat32, comm, s);
        if (nr != ncclSuccess && rc == KG_OK) rc = kg::nccl_fail(ctx, nr, "ncclAllGather (logits)");
    }
    if (tokens_all) {
        const ncclResult_t nr = api.all_gather(tokens_all + r * n_seq, tokens_all, (size_t)n_seq, ncclInt32, comm, s);
        if (nr != ncclSuccess && rc == KG_OK) rc = kg::nccl_fail(ctx, nr, "ncclAllGather (tokens)");
    }
    return rc;
}

}  // extern "C"
