// kg_paged.cu — PagedKVCache for forward_paged (kv_mode KG_KV_PAGED).
//
// The reference's copy-on-write page store for DDTree branch exploration
// (crates/katgpt-transformer/src/kv_cache.rs:187-420): f32 K/V in pages of 16
// positions ([K 16 x kvd | V 16 x kvd] per page), per-layer page lists per
// sequence, a LIFO free list and per-page reference counts. The bookkeeping
// is integer work on a handful of pages per call, so it stays on the host
// with the same state transitions as the reference (page indices, reference
// counts and free-list order match it call for call); the pages themselves
// live in one device pool that the micro forward kernel reads through a
// device copy of the page tables ([L][max_seqs][maxp] int32, -1 = no page).
// The table copy and the zeroing of reused pages (alloc_page's fill(0.0)) are
// deferred to the next device use of the pool, on the stream of that use.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "kg_internal.h"

namespace {

constexpr int kPage = 16;  // PAGE_SIZE (kv_cache.rs:189)

int pfail(kg_ctx *ctx, int code, const std::string &msg) {
    ctx->err = msg;
    return code;
}
int pcuda(kg_ctx *ctx, cudaError_t e, const char *what) {
    return pfail(ctx, e == cudaErrorMemoryAllocation ? KG_ERR_OOM : KG_ERR_CUDA,
                 std::string(what) + ": " + cudaGetErrorString(e));
}

bool is_paged(const kg_ctx *ctx) {
    return ctx && (ctx->micro || ctx->big_path) && ctx->cfg.kv_mode == KG_KV_PAGED;
}
// element size of the pool: f32 rows on the exact micro path, bf16 on the tensor-core path
int64_t elem_bytes(const kg_ctx *ctx) { return ctx->micro ? 4 : 2; }
int64_t page_bytes(const kg_ctx *ctx) { return 2 * kPage * ctx->kvd * elem_bytes(ctx); }

// f32 <-> bf16 (round to nearest even) for the host-side row access of a bf16 pool
uint16_t to_bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  // NaN stays NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float from_bf16_bits(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// alloc_page (:241-262): reuse from the free list (zeroed) or take the next
// index; the reference grows its pool, here the pool's capacity bounds it.
int alloc_page(kg_ctx *ctx, int32_t *out) {
    kg::PagedState &P = ctx->paged;
    int32_t idx;
    if (!P.free_pages.empty()) {
        idx = P.free_pages.back();
        P.free_pages.pop_back();
        P.zero_list.push_back(idx);
    } else {
        if (P.total >= P.cap)
            return pfail(ctx, KG_ERR_OOM, "paged KV pool exhausted (" + std::to_string(P.cap) + " pages)");
        idx = (int32_t)P.total++;
        P.refs.push_back(0);
    }
    P.refs[idx] += 1;
    *out = idx;
    P.dirty = true;
    return KG_OK;
}

int check_seq(kg_ctx *ctx, int32_t seq) {
    if (seq < 0 || seq >= ctx->cfg.max_seqs)
        return pfail(ctx, KG_ERR_INVALID_ARG, "paged sequence index outside [0, max_seqs)");
    return KG_OK;
}

void grow_seqs(kg::PagedState &P, int32_t seq) {  // ensure_pages' slot growth (:272-277)
    for (auto &lt : P.tables)
        while ((int32_t)lt.size() <= seq) lt.emplace_back();
}

}  // namespace

namespace kg {

// Device side of a paged call: upload the page tables when they changed and
// zero the pages reused since the last call, both on `s`.
cudaError_t paged_flush(kg_ctx *ctx, cudaStream_t s) {
    PagedState &P = ctx->paged;
    // Host arrays go up as pageable copies, which are staged before
    // cudaMemcpyAsync returns, so the host state may change right after.
    if (!P.zero_list.empty()) {
        std::sort(P.zero_list.begin(), P.zero_list.end());  // a page freed and reused twice is zeroed once
        P.zero_list.erase(std::unique(P.zero_list.begin(), P.zero_list.end()), P.zero_list.end());
        const int n = (int)P.zero_list.size();
        cudaError_t e = cudaMemcpyAsync(P.d_zero, P.zero_list.data(), n * sizeof(int32_t), cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = zero_pages(static_cast<float *>(P.pool), P.d_zero, n, page_bytes(ctx) / 4, s);
        if (e != cudaSuccess) return e;
        P.zero_list.clear();
    }
    if (P.dirty) {
        const int S = ctx->cfg.max_seqs;
        std::fill(P.h_tab.begin(), P.h_tab.end(), -1);
        for (size_t l = 0; l < P.tables.size(); ++l)
            for (size_t q = 0; q < P.tables[l].size() && (int)q < S; ++q) {
                const auto &pl = P.tables[l][q];
                int32_t *row = &P.h_tab[((int64_t)l * S + q) * P.maxp];
                for (size_t k = 0; k < pl.size() && (int)k < P.maxp; ++k) row[k] = pl[k];
            }
        cudaError_t e = cudaMemcpyAsync(P.d_tab, P.h_tab.data(), P.h_tab.size() * sizeof(int32_t),
                                        cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return e;
        P.dirty = false;
    }
    return cudaSuccess;
}

// Pool and tables of a paged context (called once at creation).
cudaError_t paged_alloc(kg_ctx *ctx) {
    PagedState &P = ctx->paged;
    const int64_t L = ctx->L, S = ctx->cfg.max_seqs;
    P.maxp = (int)(ctx->B / kPage + 1);
    const int64_t initial = (ctx->B / kPage + 1) * L;  // PagedKVCache::new (:217-219)
    // Two full page sets (every sequence at block_size, once more for forks),
    // bounded by what the device has free: at model widths two full sets can
    // exceed HBM, and a pool that runs out returns KG_ERR_OOM from ensure.
    int64_t want = 2 * S * L * P.maxp;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) {
        const int64_t reserve = int64_t(2) << 30;  // workspaces allocated on later calls
        const int64_t fit = ((int64_t)free_b - reserve) / 10 * 9 / page_bytes(ctx);
        want = std::min(want, std::max<int64_t>(fit, 0));
    } else {
        (void)cudaGetLastError();
    }
    P.cap = std::max<int64_t>(initial, want);
    cudaError_t e = cudaMalloc(&P.pool, (size_t)P.cap * page_bytes(ctx));
    if (e == cudaSuccess) e = cudaMalloc(&P.d_tab, (size_t)L * S * P.maxp * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&P.d_zero, (size_t)P.cap * sizeof(int32_t));
    if (e != cudaSuccess) return e;
    ctx->allocs.push_back(P.pool);
    ctx->allocs.push_back(P.d_tab);
    ctx->allocs.push_back(P.d_zero);
    P.h_tab.assign((size_t)L * S * P.maxp, -1);
    if (ctx->micro) {  // the exact micro kernel reads the pool through its arguments
        ctx->margs.pool = static_cast<float *>(P.pool);
        ctx->margs.ptab = P.d_tab;
        ctx->margs.maxp = P.maxp;
        ctx->margs.n_pages = (int)P.cap;
    }
    return cudaSuccess;
}

// ensure_pages for every position of a forward call, in batch order.
int paged_ensure_batch(kg_ctx *ctx, int32_t n_seq, const int32_t *seq_ids, const int32_t *start_pos, int32_t T) {
    for (int32_t i = 0; i < n_seq; ++i) {
        const int32_t p0 = start_pos ? start_pos[i] : 0;
        for (int32_t t = 0; t < T; ++t) {
            int rc = kg_paged_ensure(ctx, seq_ids[i], p0 + t);
            if (rc) return rc;
        }
    }
    return KG_OK;
}

}  // namespace kg

extern "C" {

int kg_paged_init(kg_ctx *ctx, int32_t max_sequences) {
    if (!is_paged(ctx)) return ctx ? pfail(ctx, KG_ERR_UNSUPPORTED, "context is not kv_mode KG_KV_PAGED") : KG_ERR_INVALID_ARG;
    if (max_sequences < 0 || max_sequences > ctx->cfg.max_seqs)
        return pfail(ctx, KG_ERR_INVALID_ARG, "max_sequences outside [0, max_seqs]");
    kg::PagedState &P = ctx->paged;
    const int64_t initial = (ctx->B / kPage + 1) * ctx->L;
    P.tables.assign(ctx->L, std::vector<std::vector<int32_t>>(max_sequences));
    P.free_pages.resize(initial);
    for (int64_t i = 0; i < initial; ++i) P.free_pages[i] = (int32_t)i;
    P.refs.assign(initial, 0);
    P.total = initial;
    P.zero_list.clear();
    P.dirty = true;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = cudaMemsetAsync(P.pool, 0, (size_t)P.cap * page_bytes(ctx), ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return pcuda(ctx, e, "paged pool clear");
    return KG_OK;
}

int kg_paged_ensure(kg_ctx *ctx, int32_t seq, int32_t pos) {
    if (!is_paged(ctx)) return ctx ? pfail(ctx, KG_ERR_UNSUPPORTED, "context is not kv_mode KG_KV_PAGED") : KG_ERR_INVALID_ARG;
    if (int rc = check_seq(ctx, seq)) return rc;
    if (pos < 0) return pfail(ctx, KG_ERR_INVALID_ARG, "negative position");
    kg::PagedState &P = ctx->paged;
    const size_t need = (size_t)pos / kPage + 1;
    grow_seqs(P, seq);
    // deficits per layer first, then every layer's pages in layer order (:279-295)
    std::vector<size_t> deficit(P.tables.size());
    for (size_t l = 0; l < P.tables.size(); ++l)
        deficit[l] = need > P.tables[l][seq].size() ? need - P.tables[l][seq].size() : 0;
    for (size_t l = 0; l < P.tables.size(); ++l)
        for (size_t k = 0; k < deficit[l]; ++k) {
            int32_t pg;
            if (int rc = alloc_page(ctx, &pg)) return rc;
            P.tables[l][seq].push_back(pg);
        }
    return KG_OK;
}

int kg_paged_fork(kg_ctx *ctx, int32_t seq, int32_t fork_at_pos, int32_t *new_seq) {
    if (!is_paged(ctx)) return ctx ? pfail(ctx, KG_ERR_UNSUPPORTED, "context is not kv_mode KG_KV_PAGED") : KG_ERR_INVALID_ARG;
    if (!new_seq || fork_at_pos < 0) return pfail(ctx, KG_ERR_INVALID_ARG, "bad fork arguments");
    kg::PagedState &P = ctx->paged;
    const int32_t ns = P.tables.empty() ? 0 : (int32_t)P.tables[0].size();
    if (seq < 0 || seq >= ns) return pfail(ctx, KG_ERR_INVALID_ARG, "fork of a sequence that does not exist");
    if (ns >= ctx->cfg.max_seqs) return pfail(ctx, KG_ERR_OOM, "paged sequence count at max_seqs");
    const size_t fork_page = (size_t)fork_at_pos / kPage;
    for (auto &lt : P.tables) {
        const auto &src = lt[seq];
        std::vector<int32_t> shared(src.begin(), src.begin() + std::min(fork_page, src.size()));
        for (int32_t pg : shared) P.refs[pg] += 1;
        lt.push_back(std::move(shared));
    }
    P.dirty = true;
    *new_seq = ns;
    return KG_OK;
}

int kg_paged_rollback(kg_ctx *ctx, int32_t seq, int32_t pos) {
    if (!is_paged(ctx)) return ctx ? pfail(ctx, KG_ERR_UNSUPPORTED, "context is not kv_mode KG_KV_PAGED") : KG_ERR_INVALID_ARG;
    if (pos < 0) return pfail(ctx, KG_ERR_INVALID_ARG, "negative position");
    kg::PagedState &P = ctx->paged;
    const size_t keep = (size_t)pos / kPage;
    for (auto &lt : P.tables) {
        if (seq < 0 || (size_t)seq >= lt.size()) continue;
        auto &t = lt[seq];
        for (size_t k = keep; k < t.size(); ++k)
            if (--P.refs[t[k]] == 0) P.free_pages.push_back(t[k]);
        if (t.size() > keep) t.resize(keep);
    }
    P.dirty = true;
    return KG_OK;
}

int kg_paged_reset(kg_ctx *ctx) {
    if (!is_paged(ctx)) return ctx ? pfail(ctx, KG_ERR_UNSUPPORTED, "context is not kv_mode KG_KV_PAGED") : KG_ERR_INVALID_ARG;
    kg::PagedState &P = ctx->paged;
    for (auto &lt : P.tables)
        for (auto &t : lt) {
            P.free_pages.insert(P.free_pages.end(), t.begin(), t.end());
            t.clear();
        }
    std::fill(P.refs.begin(), P.refs.end(), 0);
    P.dirty = true;
    return KG_OK;
}

static int kv_page_row(kg_ctx *ctx, int32_t layer, int32_t seq, int32_t pos, char **krow) {
    kg::PagedState &P = ctx->paged;
    if (layer < 0 || layer >= (int32_t)P.tables.size() || seq < 0 || pos < 0 ||
        (size_t)seq >= P.tables[layer].size() || (size_t)pos / kPage >= P.tables[layer][seq].size())
        return pfail(ctx, KG_ERR_INVALID_ARG, "no page for (layer, seq, pos)");
    const int64_t pg = P.tables[layer][seq][pos / kPage];
    *krow = static_cast<char *>(P.pool) + (pg * 2 * kPage + pos % kPage) * ctx->kvd * elem_bytes(ctx);
    return KG_OK;
}

int kg_paged_write_kv(kg_ctx *ctx, int32_t layer, int32_t seq, int32_t pos, const float *k, const float *v) {
    if (!is_paged(ctx)) return ctx ? pfail(ctx, KG_ERR_UNSUPPORTED, "context is not kv_mode KG_KV_PAGED") : KG_ERR_INVALID_ARG;
    if (!k || !v) return pfail(ctx, KG_ERR_INVALID_ARG, "null K/V");
    char *kr;
    if (int rc = kv_page_row(ctx, layer, seq, pos, &kr)) return rc;
    const int64_t kvd = ctx->kvd, eb = elem_bytes(ctx);
    std::vector<uint16_t> hk, hv;  // bf16 pools store the rows rounded to bf16
    const void *sk = k, *sv = v;
    if (eb == 2) {
        hk.resize(kvd);
        hv.resize(kvd);
        for (int64_t j = 0; j < kvd; ++j) hk[j] = to_bf16_bits(k[j]), hv[j] = to_bf16_bits(v[j]);
        sk = hk.data();
        sv = hv.data();
    }
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = kg::paged_flush(ctx, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(kr, sk, kvd * eb, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(kr + kPage * kvd * eb, sv, kvd * eb, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    return e == cudaSuccess ? KG_OK : pcuda(ctx, e, "paged write_kv");
}

int kg_paged_read_kv(kg_ctx *ctx, int32_t layer, int32_t seq, int32_t pos, float *k, float *v) {
    if (!is_paged(ctx)) return ctx ? pfail(ctx, KG_ERR_UNSUPPORTED, "context is not kv_mode KG_KV_PAGED") : KG_ERR_INVALID_ARG;
    if (!k || !v) return pfail(ctx, KG_ERR_INVALID_ARG, "null K/V");
    char *kr;
    if (int rc = kv_page_row(ctx, layer, seq, pos, &kr)) return rc;
    const int64_t kvd = ctx->kvd, eb = elem_bytes(ctx);
    std::vector<uint16_t> hk(eb == 2 ? kvd : 0), hv(eb == 2 ? kvd : 0);
    void *dk = eb == 2 ? (void *)hk.data() : (void *)k, *dv = eb == 2 ? (void *)hv.data() : (void *)v;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = kg::paged_flush(ctx, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dk, kr, kvd * eb, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dv, kr + kPage * kvd * eb, kvd * eb, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return pcuda(ctx, e, "paged read_kv");
    if (eb == 2)
        for (int64_t j = 0; j < kvd; ++j) k[j] = from_bf16_bits(hk[j]), v[j] = from_bf16_bits(hv[j]);
    return KG_OK;
}

int kg_paged_table(const kg_ctx *ctx, int32_t layer, int32_t seq, int32_t *pages_out, int32_t cap,
                   int32_t *len_out) {
    if (!is_paged(ctx) || !len_out || cap < 0 || (cap > 0 && !pages_out)) return KG_ERR_INVALID_ARG;
    const kg::PagedState &P = ctx->paged;
    if (layer < 0 || layer >= (int32_t)P.tables.size()) return KG_ERR_INVALID_ARG;
    if (seq < 0 || (size_t)seq >= P.tables[layer].size()) {
        *len_out = 0;
        return KG_OK;
    }
    const auto &t = P.tables[layer][seq];
    *len_out = (int32_t)t.size();
    for (int32_t k = 0; k < cap && k < (int32_t)t.size(); ++k) pages_out[k] = t[k];
    return KG_OK;
}

int kg_paged_stats(const kg_ctx *ctx, int64_t *total_pages, int64_t *free_pages, int32_t *n_sequences,
                   int32_t *refs, int64_t refs_cap) {
    if (!is_paged(ctx)) return KG_ERR_INVALID_ARG;
    const kg::PagedState &P = ctx->paged;
    if (total_pages) *total_pages = P.total;
    if (free_pages) *free_pages = (int64_t)P.free_pages.size();
    if (n_sequences) *n_sequences = P.tables.empty() ? 0 : (int32_t)P.tables[0].size();
    if (refs)
        for (int64_t i = 0; i < std::min<int64_t>(refs_cap, P.total); ++i) refs[i] = P.refs[i];
    return KG_OK;
}

}  // extern "C"
