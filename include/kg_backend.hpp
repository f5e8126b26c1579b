// kg_backend.hpp — C++ host mirror of the reference's InferenceBackend trait
// (src/inference_backend.rs:45-92) over the C ABI in kg_abi.h.
//
// The reference's host language is Rust; without a Rust toolchain, this
// header is the host-side mirror of the trait in C++ (a Rust binding is a thin
// extern "C" block over kg_abi.h). Method names, argument
// meaning and error behaviour follow the trait:
//   forward        -> one token at `pos`; returns vocab_size logits that stay
//                     valid until the next call (the trait returns a slice
//                     borrowed from ForwardContext::logits)
//   device_name    -> "CUDA:<device>"
//   supports_stateful -> true (the KV cache lives on the device)
//   reset          -> a new sequence (MultiLayerKVCache::reset semantics)
//   compile        -> upload weights; failures map to CompileError variants
//   is_compiled, recompile_hint
// forward() cannot fail in the trait; here a device error throws (the Metal
// backend's forward panics through expect() in the same situation).
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "kg_abi.h"

namespace katgpt {

// CompileError (src/inference_backend.rs:14-40)
struct CompileError : std::runtime_error {
    enum Kind { UnsupportedBackend, DeviceError, InvalidWeights } kind;
    CompileError(Kind k, const std::string &m) : std::runtime_error(m), kind(k) {}
};

class CudaBackend {
   public:
    explicit CudaBackend(const kg_config &cfg, int device = 0, int32_t seq = 0) : cfg_(cfg), seq_(seq) {
        int rc = kg_ctx_create(&cfg_, device, &ctx_);
        if (rc != KG_OK) throw CompileError(CompileError::DeviceError, kg_status_string(rc));
        logits_.resize(cfg_.vocab_size);
    }
    ~CudaBackend() { kg_ctx_destroy(ctx_); }
    CudaBackend(const CudaBackend &) = delete;
    CudaBackend &operator=(const CudaBackend &) = delete;

    // InferenceBackend::forward (the ForwardContext/MultiLayerKVCache arguments
    // of the trait are owned on the device here)
    std::vector<float> &forward(int32_t token, int32_t pos) {
        int rc = kg_forward_token(ctx_, seq_, token, pos, logits_.data());
        if (rc != KG_OK) throw std::runtime_error(std::string("kg_forward_token: ") + kg_last_error(ctx_));
        return logits_;
    }
    const char *device_name() const { return kg_device_name(ctx_); }
    bool supports_stateful() const { return true; }
    void reset() { kg_seq_reset(ctx_, seq_); }
    // weights: the flat TransformerWeights layout (kg_weights_count floats)
    void compile(const std::vector<float> &weights) {
        int rc = kg_upload_weights(ctx_, weights.data(), (int64_t)weights.size());
        if (rc == KG_ERR_INVALID_WEIGHTS) throw CompileError(CompileError::InvalidWeights, kg_last_error(ctx_));
        if (rc == KG_ERR_UNSUPPORTED) throw CompileError(CompileError::UnsupportedBackend, kg_last_error(ctx_));
        if (rc != KG_OK) throw CompileError(CompileError::DeviceError, kg_last_error(ctx_));
    }
    bool is_compiled() const { return kg_is_compiled(ctx_) != 0; }
    void recompile_hint() { /* weights are re-uploaded explicitly by compile() */ }

    // LoraPair of generate_with_prefill: which 0 = reader (forward_prefill),
    // 1 = writer (forward / forward_batch); rank 0 removes the adapter
    void set_lora(int32_t which, int32_t rank, int32_t in_dim, int32_t out_dim, float alpha, const float *a,
                  const float *b) {
        int rc = kg_set_lora(ctx_, which, rank, in_dim, out_dim, alpha, a, b);
        if (rc != KG_OK) throw std::runtime_error(std::string("kg_set_lora: ") + kg_last_error(ctx_));
    }

    // batched extension: teacher-forced positions [start, start+T) of n_seq sequences
    void forward_batch(int32_t n_seq, const int32_t *seq_ids, const int32_t *tokens, const int32_t *start_pos,
                       int32_t T, float *logits, float *probs = nullptr) {
        int rc = kg_forward_batch(ctx_, n_seq, seq_ids, tokens, start_pos, T, logits, probs);
        if (rc != KG_OK) throw std::runtime_error(std::string("kg_forward_batch: ") + kg_last_error(ctx_));
    }
    kg_ctx *handle() { return ctx_; }
    int32_t forward_vocab() const { return cfg_.vocab_size; }

   private:
    kg_config cfg_;
    kg_ctx *ctx_ = nullptr;
    int32_t seq_;
    std::vector<float> logits_;
};

// DDTreeBranchCache (src/speculative/types.rs:218-290) over a CudaBackend
// built with kv_mode KG_KV_PAGED: sequence 0 is the trunk, forks share whole
// prefix pages (PagedKVCache::fork), a fork past max_branches returns the
// source sequence, and discarding a branch other than the trunk frees its
// pages and its budget slot.
class DDTreeBranchCache {
   public:
    DDTreeBranchCache(CudaBackend &backend, int32_t max_branches) : be_(backend), max_branches_(max_branches) {
        check(kg_paged_init(be_.handle(), max_branches), "kg_paged_init");
    }
    int32_t fork_branch(int32_t from, int32_t at_pos) {
        if (branch_count_ >= max_branches_) return from;  // budget exhausted: reuse the source
        int32_t s = -1;
        check(kg_paged_fork(be_.handle(), from, at_pos, &s), "kg_paged_fork");
        ++branch_count_;
        return s;
    }
    // forward_paged of one token of a branch: vocab_size logits
    std::vector<float> forward_branch(int32_t seq_idx, int32_t token, int32_t pos) {
        std::vector<float> logits(vocab());
        check(kg_forward_batch(be_.handle(), 1, &seq_idx, &token, &pos, 1, logits.data(), nullptr), "forward_paged");
        return logits;
    }
    void rollback_branch(int32_t seq_idx, int32_t at_pos) {
        check(kg_paged_rollback(be_.handle(), seq_idx, at_pos), "kg_paged_rollback");
    }
    void discard_branch(int32_t seq_idx) {
        rollback_branch(seq_idx, 0);
        if (seq_idx > 0 && branch_count_ > 1) --branch_count_;
    }
    void reset() {
        check(kg_paged_reset(be_.handle()), "kg_paged_reset");
        branch_count_ = 1;
    }
    int32_t branch_count() const { return branch_count_; }

   private:
    void check(int rc, const char *what) {
        if (rc != KG_OK) throw std::runtime_error(std::string(what) + ": " + kg_last_error(be_.handle()));
    }
    int32_t vocab() const { return be_.forward_vocab(); }
    CudaBackend &be_;
    int32_t max_branches_;
    int32_t branch_count_ = 1;  // sequence 0 = trunk
};

}  // namespace katgpt
