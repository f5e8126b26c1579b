// Runs the exact-order micro forward kernel (katgpt-rs_b200/csrc/
// kg_micro_kernel.cuh, the source the CUDA library compiles) on the host: one
// OS thread per CUDA thread of a block, a std::barrier standing for
// __syncthreads, the dynamic shared memory as one host buffer. Its logits are
// compared bit for bit with the oracle's (test infrastructure: built and run
// by tests/test_micro_kernel_host.py; prints "<mismatches> <values>" per case).
#include <algorithm>
#include <barrier>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

struct float4 {
    float x, y, z, w;
};
struct HostDim {
    unsigned x = 0, y = 0, z = 0;
};
static thread_local HostDim threadIdx, blockIdx;
static HostDim blockDim, gridDim;
static std::barrier<> *g_bar = nullptr;
static std::vector<float4> g_smem;
static inline void __syncthreads() { g_bar->arrive_and_wait(); }
static inline int atomicExch(int *p, int v) { return __atomic_exchange_n(p, v, __ATOMIC_SEQ_CST); }
static inline int __float_as_int(float f) {
    int i;
    std::memcpy(&i, &f, 4);
    return i;
}
#define __global__
#define __launch_bounds__(a, b)
#define KG_MICRO_SMEM(name) float4 *name = g_smem.data()
#include "kg_micro_kernel.cuh"
#include "kg_oracle.h"

namespace {

// Config::micro(): the widths micro_forward is instantiated for
constexpr int N = 16, KVD = 16, M = 64, V = 27, B = 16;

struct Ctx {
    int L = 1, S = 1;
    std::vector<float> pack, Kf, Vf, util, norms;
    std::vector<uint8_t> codes;
    int err = 0;
    kg::MicroArgs a{};

    // kbits > 0: TurboQuant tables (the oracle's rotation for seed 42 and
    // its Lloyd-Max codebooks) for forward_quantized
    Ctx(int L_, int S_, const std::vector<float> &w, int kbits = 0, int vbits = 0) : L(L_), S(S_) {
        a.off_wte = 0;
        a.off_wpe = V * N;
        a.off_layers = a.off_wpe + B * N;
        a.layer_stride = 2 * N * N + 2 * KVD * N + 2 * M * N;
        a.off_lm = a.off_layers + L * a.layer_stride;
        a.off_dq = a.off_lm + V * N;
        a.off_dn = a.off_dq + L * N;
        a.off_ag = a.off_dn + L * N;
        a.off_mg = a.off_ag + L * N;
        int off = a.off_mg + L * N;
        for (int k = 0; k < 2; ++k) {
            a.off_lora_a[k] = off;
            off += kg::kLoraMax * kg::kLoraMax;
            a.off_lora_b[k] = off;
            off += kg::kLoraMax * kg::kLoraMax;
        }
        const int nk = kbits ? 1 << kbits : 0, nv = vbits ? 1 << vbits : 0;
        a.off_rot = off;
        off += kbits ? KVD * KVD : 0;
        a.off_rot_t = off;
        off += kbits ? KVD * KVD : 0;
        a.off_kc = off;
        off += nk;
        a.off_kb = off;
        off += kbits ? nk - 1 : 0;
        a.off_vc = off;
        off += nv;
        a.off_vb = off;
        off += vbits ? nv - 1 : 0;
        off = (off + 3) / 4 * 4;
        pack.assign(off, 0.0f);
        std::memcpy(pack.data(), w.data(), w.size() * 4);
        if (kbits) {
            float mse;
            or_tq_rotation(KVD, 42, &pack[a.off_rot]);
            for (int i = 0; i < KVD; ++i)
                for (int j = 0; j < KVD; ++j) pack[a.off_rot_t + i * KVD + j] = pack[a.off_rot + j * KVD + i];
            or_tq_codebook(KVD, kbits, &pack[a.off_kc], &pack[a.off_kb], &mse);
            or_tq_codebook(KVD, vbits, &pack[a.off_vc], &pack[a.off_vb], &mse);
            a.kbits = kbits;
            a.vbits = vbits;
            a.kpl = (int)or_tq_packed_len(KVD, kbits);
            a.vpl = (int)or_tq_packed_len(KVD, vbits);
        }
        a.pack = pack.data();
        a.pack_floats = off;
        a.L = L;
        a.sparse_threshold = 0.8f;
        a.inv_temp = 1.0f / 0.5f;
        Kf.assign((size_t)S * L * B * KVD, 0.0f);
        Vf = Kf;
        util.assign((size_t)S * L * B, 0.0f);
        norms.assign((size_t)S * L * B * 2, 0.0f);
        codes.assign((size_t)S * L * B * 32, 0);
        a.Kf = Kf.data();
        a.Vf = Vf.data();
        a.util = util.data();
        a.norms = norms.data();
        a.codes = codes.data();
        a.n_slots = S;
        a.err = &err;
    }
    void set_lora(int which, int rank, int in_dim, int out_dim, float alpha, const float *A, const float *Bm) {
        std::memcpy(&pack[a.off_lora_a[which]], A, (size_t)rank * in_dim * 4);
        std::memcpy(&pack[a.off_lora_b[which]], Bm, (size_t)out_dim * rank * 4);
        a.lora_rank[which] = rank;
        a.lora_in[which] = in_dim;
        a.lora_out[which] = out_dim;
        a.lora_scale[which] = alpha / (float)rank;
    }
    // one launch of a single persistent block
    template <int MODE, bool LORA>
    void launch(int n_seq, int T, const int32_t *ids, const int32_t *toks, const int32_t *start, float *logits) {
        kg::MicroArgs p = a;
        p.n_seq = n_seq;
        p.T = T;
        p.seq_ids = ids;
        p.tokens = toks;
        p.start_pos = start;
        p.logits = logits;
        p.probs = nullptr;
        const int threads = (128 / T) * T;
        const size_t smem = (size_t)p.pack_floats + 128 * (B + 1) + (MODE == kg::MODE_PREFILL ? 128 * 16 : 0);
        g_smem.assign(smem / 4 + 1, float4{0, 0, 0, 0});
        blockDim.x = threads;
        gridDim.x = 1;
        std::barrier<> bar(threads);
        g_bar = &bar;
        std::vector<std::thread> th;
        for (int t = 0; t < threads; ++t)
            th.emplace_back([&p, t] {
                threadIdx.x = t;
                blockIdx.x = 0;
                kg::micro_forward<N, 4, 4, 4, M, V, B, MODE, LORA>(p);
            });
        for (auto &x : th) x.join();
    }
    void forward(int n_seq, int T, const int32_t *ids, const int32_t *toks, const int32_t *start, float *logits) {
        if (a.lora_rank[1] > 0) launch<kg::MODE_BASE, true>(n_seq, T, ids, toks, start, logits);
        else launch<kg::MODE_BASE, false>(n_seq, T, ids, toks, start, logits);
    }
    template <int MODE>
    void run(int n_seq, int T, const int32_t *ids, const int32_t *toks, float *logits) {
        launch<MODE, false>(n_seq, T, ids, toks, nullptr, logits);
    }
    void quantized(int n_seq, int T, const int32_t *ids, const int32_t *toks, float *logits) {
        launch<kg::MODE_QUANT, false>(n_seq, T, ids, toks, nullptr, logits);
    }
    void prefill(int n_seq, int T, const int32_t *ids, const int32_t *toks, float *logits) {
        if (a.lora_rank[0] > 0) launch<kg::MODE_PREFILL, true>(n_seq, T, ids, toks, nullptr, logits);
        else launch<kg::MODE_PREFILL, false>(n_seq, T, ids, toks, nullptr, logits);
    }
};

or_config micro(int L) {
    or_config c{};
    c.vocab_size = V;
    c.block_size = B;
    c.n_embd = N;
    c.n_head = 4;
    c.head_dim = 4;
    c.n_kv_head = 4;
    c.mlp_hidden = M;
    c.n_layer = L;
    c.bos_token = 26;
    c.temperature = 0.5f;
    c.sparse_threshold = 0.8f;
    return c;
}

struct Adapter {
    int rank = 0, in_dim = 0, out_dim = 0;
    float alpha = 8.0f;
    std::vector<float> A, Bm;
};
Adapter adapter(int rank, int in_dim, int out_dim, uint64_t seed) {
    std::mt19937 g(seed);
    std::normal_distribution<float> nd(0.0f, 0.2f);
    Adapter ad{rank, in_dim, out_dim, 8.0f, std::vector<float>(rank * in_dim), std::vector<float>(out_dim * rank)};
    for (auto &v : ad.A) v = nd(g);
    for (auto &v : ad.Bm) v = nd(g);
    return ad;
}

long count_diff(const float *x, const float *y, size_t n) {
    long d = 0;
    for (size_t i = 0; i < n; ++i) d += std::memcmp(&x[i], &y[i], 4) != 0;
    return d;
}

std::vector<int32_t> teacher_tokens(int n, int T, uint64_t seed) {
    std::mt19937 g(seed);
    std::vector<int32_t> toks(n * T);
    for (int i = 0; i < n; ++i)
        for (int t = 0; t < T; ++t) toks[i * T + t] = t == 0 ? 26 : (int32_t)(1 + g() % 26);
    return toks;
}

// teacher-forced forward_base over n_seq x 16 positions (one launch), with an
// optional writer adapter
void case_base(int L, const Adapter *wr, uint64_t seed) {
    const or_config c = micro(L);
    std::vector<float> w(or_weights_count(&c));
    or_weights_init(&c, 42, 0, 0.02f, w.data());
    const int n = 5, T = 16;
    std::vector<int32_t> toks = teacher_tokens(n, T, seed), ids(n);
    for (int i = 0; i < n; ++i) ids[i] = i;
    Ctx ctx(L, n, w);
    if (wr) ctx.set_lora(1, wr->rank, wr->in_dim, wr->out_dim, wr->alpha, wr->A.data(), wr->Bm.data());
    std::vector<float> got((size_t)n * T * V), ref(got.size());
    ctx.forward(n, T, ids.data(), toks.data(), nullptr, got.data());
    if (wr) or_set_lora(1, wr->rank, wr->in_dim, wr->out_dim, wr->alpha, wr->A.data(), wr->Bm.data());
    or_run_batch(&c, OR_MODE_BASE, 4, 4, w.data(), toks.data(), n, T, ref.data(), 1);
    or_set_lora(1, 0, 0, 0, 0.0f, nullptr, nullptr);
    std::printf("%ld %zu\n", count_diff(got.data(), ref.data(), got.size()) + (ctx.err ? 1 : 0), got.size());
}

// forward_prefill over P prompt positions (reader adapter), then single-token
// forward_base steps from position P (writer adapter): generate_with_prefill's
// LoraPair, teacher-forced
void case_prefill(int L, int P, const Adapter *rd, const Adapter *wr, uint64_t seed) {
    const or_config c = micro(L);
    std::vector<float> w(or_weights_count(&c));
    or_weights_init(&c, 11 + L, 0, 0.02f, w.data());
    const int n = 3, T = 16;
    std::mt19937 g(seed);
    std::vector<int32_t> toks(n * T), ids(n);
    for (int i = 0; i < n; ++i) {
        ids[i] = i;
        for (int t = 0; t < T; ++t) toks[i * T + t] = (int32_t)(g() % 27);
    }
    Ctx ctx(L, n, w);
    if (rd) ctx.set_lora(0, rd->rank, rd->in_dim, rd->out_dim, rd->alpha, rd->A.data(), rd->Bm.data());
    if (wr) ctx.set_lora(1, wr->rank, wr->in_dim, wr->out_dim, wr->alpha, wr->A.data(), wr->Bm.data());
    const int steps = T - P;
    std::vector<float> got((size_t)n * (1 + steps) * V);
    std::vector<int32_t> prompt(n * P);
    for (int i = 0; i < n; ++i)
        for (int t = 0; t < P; ++t) prompt[i * P + t] = toks[i * T + t];
    std::vector<float> pre((size_t)n * V);
    ctx.prefill(n, P, ids.data(), prompt.data(), pre.data());
    for (int i = 0; i < n; ++i) std::memcpy(&got[(size_t)i * (1 + steps) * V], &pre[(size_t)i * V], V * 4);
    for (int s = 0; s < steps; ++s) {
        std::vector<int32_t> tk(n), st(n, P + s);
        for (int i = 0; i < n; ++i) tk[i] = toks[i * T + P + s];
        std::vector<float> lo((size_t)n * V);
        ctx.forward(n, 1, ids.data(), tk.data(), st.data(), lo.data());
        for (int i = 0; i < n; ++i)
            std::memcpy(&got[((size_t)i * (1 + steps) + 1 + s) * V], &lo[(size_t)i * V], V * 4);
    }
    if (rd) or_set_lora(0, rd->rank, rd->in_dim, rd->out_dim, rd->alpha, rd->A.data(), rd->Bm.data());
    if (wr) or_set_lora(1, wr->rank, wr->in_dim, wr->out_dim, wr->alpha, wr->A.data(), wr->Bm.data());
    long bad = ctx.err ? 1 : 0;
    std::vector<float> ref((size_t)(1 + steps) * V);
    for (int i = 0; i < n; ++i) {
        or_prefill_then_decode(&c, w.data(), &toks[i * T], P, &toks[i * T + P], steps, ref.data());
        bad += count_diff(&got[(size_t)i * (1 + steps) * V], ref.data(), ref.size());
    }
    or_set_lora(0, 0, 0, 0, 0.0f, nullptr, nullptr);
    or_set_lora(1, 0, 0, 0, 0.0f, nullptr, nullptr);
    std::printf("%ld %zu\n", bad, got.size());
}

// forward_quantized over a TurboQuantKVCache (3- or 4-bit codes), teacher-forced
void case_quant(int L, int bits, uint64_t seed) {
    const or_config c = micro(L);
    std::vector<float> w(or_weights_count(&c));
    or_weights_init(&c, 42, 0, 0.02f, w.data());
    const int n = 4, T = 16;
    std::vector<int32_t> toks = teacher_tokens(n, T, seed), ids(n);
    for (int i = 0; i < n; ++i) ids[i] = i;
    Ctx ctx(L, n, w, bits, bits);
    std::vector<float> got((size_t)n * T * V), ref(got.size());
    ctx.quantized(n, T, ids.data(), toks.data(), got.data());
    or_run_batch(&c, OR_MODE_QUANT, bits, bits, w.data(), toks.data(), n, T, ref.data(), 1);
    std::printf("%ld %zu\n", count_diff(got.data(), ref.data(), got.size()) + (ctx.err ? 1 : 0), got.size());
}

// forward_paged of one sequence over 16 positions whose pages (one per
// layer at block_size 16) sit out of order in the pool
void case_paged(int L, uint64_t seed) {
    const or_config c = micro(L);
    std::vector<float> w(or_weights_count(&c));
    or_weights_init(&c, 42, 0, 0.02f, w.data());
    const int T = 16, maxp = B / 16 + 1, n_pages = L + 3, page = 2 * 16 * KVD;
    std::vector<int32_t> toks = teacher_tokens(1, T, seed), ids(1, 0), ptab(L * maxp, -1);
    std::vector<int64_t> table(L * maxp, -1);
    for (int l = 0; l < L; ++l) ptab[l * maxp] = (int32_t)(table[l * maxp] = L + 1 - l);  // pages L+1 .. 2, < n_pages
    Ctx ctx(L, 1, w);
    std::vector<float> pool((size_t)n_pages * page, 0.0f), opool = pool;
    ctx.a.pool = pool.data();
    ctx.a.ptab = ptab.data();
    ctx.a.maxp = maxp;
    ctx.a.n_pages = n_pages;
    std::vector<float> got((size_t)T * V), ref(got.size());
    ctx.run<kg::MODE_PAGED>(1, T, ids.data(), toks.data(), got.data());
    for (int t = 0; t < T; ++t) or_forward_paged(&c, w.data(), opool.data(), table.data(), maxp, toks[t], t, &ref[t * V]);
    std::printf("%ld %zu\n", count_diff(got.data(), ref.data(), got.size()) + count_diff(pool.data(), opool.data(),
                pool.size()) + (ctx.err ? 1 : 0), got.size() + pool.size());
}

// forward_quantized over the SpectralQuant codec: one calibration (the
// eigenbasis of correlated synthetic keys) for every layer, as from_keys
void case_sq(int L, float avg_bits, int water_fill, uint64_t seed) {
    const or_config c = micro(L);
    std::vector<float> w(or_weights_count(&c));
    or_weights_init(&c, 42, 0, 0.02f, w.data());
    std::mt19937 g(seed);
    std::normal_distribution<float> nd(0.0f, 1.0f);
    const int ns = 200;
    std::vector<float> mix(KVD * KVD), X(ns * KVD, 0.0f);
    for (auto &v : mix) v = nd(g) * 0.4f;
    for (int s = 0; s < ns; ++s)
        for (int i = 0; i < KVD; ++i) {
            const float z = nd(g) * std::pow(1.5f, -(float)i);
            for (int j = 0; j < KVD; ++j) X[s * KVD + j] += z * mix[i * KVD + j];
        }
    std::vector<float> ev(KVD * KVD), eval(KVD);
    float de = 0.0f;
    or_sq_calibrate_eigenbasis(X.data(), ns, KVD, ev.data(), eval.data(), &de);
    std::vector<float> evL, evalL, deL(L, de);
    for (int l = 0; l < L; ++l) {
        evL.insert(evL.end(), ev.begin(), ev.end());
        evalL.insert(evalL.end(), eval.begin(), eval.end());
    }
    or_sq_params P{42, 30, 100, avg_bits, 1, 8, 1, 6, water_fill};
    std::vector<float> eig(L * KVD * KVD), cent(L * KVD * kg::kSqLevels);
    std::vector<uint8_t> bits(L * KVD);
    std::vector<int32_t> nlev(L * KVD), dout(L);
    if (or_sq_build(&P, KVD, L, evL.data(), evalL.data(), deL.data(), eig.data(), bits.data(), cent.data(),
                    nlev.data(), dout.data())) {
        std::printf("1 1\n");
        return;
    }
    const int n = 3, T = 16;
    std::vector<int32_t> toks = teacher_tokens(n, T, seed), ids(n);
    for (int i = 0; i < n; ++i) ids[i] = i;
    Ctx ctx(L, n, w);
    // the pack's SpectralQuant tables: [L][kvd*kvd], [L][kvd][64], [L][kvd] (bits | levels << 8)
    const int base = (int)ctx.pack.size();
    ctx.pack.resize(base + L * KVD * KVD + L * KVD * kg::kSqLevels + L * KVD + 4, 0.0f);
    ctx.a.off_sq_eig = base;
    ctx.a.off_sq_cent = base + L * KVD * KVD;
    ctx.a.off_sq_meta = ctx.a.off_sq_cent + L * KVD * kg::kSqLevels;
    std::memcpy(&ctx.pack[ctx.a.off_sq_eig], eig.data(), eig.size() * 4);
    std::memcpy(&ctx.pack[ctx.a.off_sq_cent], cent.data(), cent.size() * 4);
    for (int i = 0; i < L * KVD; ++i) {
        const int32_t m = (int32_t)bits[i] | (nlev[i] << 8);
        std::memcpy(&ctx.pack[ctx.a.off_sq_meta + i], &m, 4);
    }
    ctx.a.pack = ctx.pack.data();
    ctx.a.pack_floats = (int)(ctx.pack.size() / 4 * 4);
    ctx.a.kpl = ctx.a.vpl = KVD;
    ctx.codes.assign((size_t)n * L * B * 2 * KVD, 0);
    ctx.a.codes = ctx.codes.data();
    std::vector<float> got((size_t)n * T * V), ref((size_t)T * V);
    ctx.run<kg::MODE_SQ>(n, T, ids.data(), toks.data(), got.data());
    long bad = ctx.err ? 1 : 0;
    for (int i = 0; i < n; ++i) {
        std::vector<uint8_t> codes((size_t)L * T * 2 * KVD);
        std::vector<float> norms((size_t)L * T * 2);
        or_run_sequence_sq(&c, w.data(), eig.data(), bits.data(), cent.data(), nlev.data(), &toks[i * T], T,
                           ref.data(), codes.data(), norms.data());
        bad += count_diff(&got[(size_t)i * T * V], ref.data(), ref.size());
    }
    std::printf("%ld %zu\n", bad, got.size());
}

// forward_sp_kv_quant (Hard gate, 3-bit codes) with and without a writer
// adapter: layer-0 codes and norms bit-identical, logits within 1e-5 relative
// (the gated attention calls libm expf); a value off that bar counts as a mismatch
void case_spkv(int L, const Adapter *wr, uint64_t seed) {
    const or_config c = micro(L);
    std::vector<float> w(or_weights_count(&c));
    or_weights_init(&c, 42, 0, 0.02f, w.data());
    const int n = 3, T = 16, PH = 16, NKV = 4;
    std::vector<int32_t> toks = teacher_tokens(n, T, seed), ids(n);
    for (int i = 0; i < n; ++i) ids[i] = i;
    Ctx ctx(L, n, w, 3, 3);
    const int base = (int)ctx.pack.size();
    ctx.pack.resize(base + PH * N + PH + NKV * PH + NKV + 4, 0.0f);
    ctx.a.off_pw1 = base;
    ctx.a.off_pb1 = base + PH * N;
    ctx.a.off_pw2 = ctx.a.off_pb1 + PH;
    ctx.a.off_pb2 = ctx.a.off_pw2 + NKV * PH;
    or_spkv_predictor_weights(N, PH, NKV, 5.0f, &ctx.pack[base]);
    ctx.a.pack = ctx.pack.data();
    ctx.a.pack_floats = (int)(ctx.pack.size() / 4 * 4);
    if (wr) ctx.set_lora(1, wr->rank, wr->in_dim, wr->out_dim, wr->alpha, wr->A.data(), wr->Bm.data());
    std::vector<float> got((size_t)n * T * V), ref((size_t)T * V);
    if (wr) ctx.launch<kg::MODE_SPKV, true>(n, T, ids.data(), toks.data(), nullptr, got.data());
    else ctx.launch<kg::MODE_SPKV, false>(n, T, ids.data(), toks.data(), nullptr, got.data());
    if (wr) or_set_lora(1, wr->rank, wr->in_dim, wr->out_dim, wr->alpha, wr->A.data(), wr->Bm.data());
    long bad = ctx.err ? 1 : 0;
    const int pl = ctx.a.kpl + ctx.a.vpl;
    for (int i = 0; i < n; ++i) {
        std::vector<uint8_t> codes((size_t)L * T * pl);
        std::vector<float> norms((size_t)L * T * 2), util((size_t)L * T);
        or_run_sequence(&c, OR_MODE_SPKV_QUANT, 3, 3, w.data(), &toks[i * T], T, ref.data(), codes.data(),
                        norms.data(), util.data());
        float mx = 0.0f, dmax = 0.0f;
        for (int k = 0; k < T * V; ++k) {
            mx = std::max(mx, std::fabs(ref[k]));
            dmax = std::max(dmax, std::fabs(got[(size_t)i * T * V + k] - ref[k]));
        }
        bad += dmax > 1e-5f * mx;
        for (int t = 0; t < T; ++t) {  // layer 0: slot i, positions t
            const size_t row = (size_t)i * L * B + t;
            bad += std::memcmp(&ctx.codes[row * pl], &codes[(size_t)t * pl], pl) != 0;
            bad += std::memcmp(&ctx.norms[row * 2], &norms[(size_t)t * 2], 8) != 0;
        }
    }
    or_set_lora(1, 0, 0, 0, 0.0f, nullptr, nullptr);
    std::printf("%ld %d\n", bad, n * (1 + 2 * T));
}

}  // namespace

int main() {
    const Adapter w4 = adapter(4, 16, 16, 1), w3 = adapter(3, 12, 10, 2), r16 = adapter(16, 16, 16, 3);
    case_base(2, nullptr, 7);                     // forward_base, no adapter
    case_base(4, &w4, 8);                         // the writer, Config::micro_lora()'s rank 4
    case_base(2, &w3, 9);                         // a partial adapter
    case_prefill(1, 10, nullptr, nullptr, 40);
    case_prefill(8, 12, nullptr, nullptr, 41);    // two routing blocks
    case_prefill(4, 7, &r16, &w4, 42);            // reader and writer
    case_prefill(2, 5, &w3, nullptr, 43);         // reader only
    case_quant(1, 4, 50);                         // forward_quantized, 4-bit codes
    case_quant(4, 3, 51);                         // 3-bit, four layers (per-layer caches)
    case_paged(1, 60);                            // forward_paged
    case_paged(4, 61);
    case_sq(2, 3.0f, 0, 70);                      // SpectralQuant, uniform widths
    case_sq(3, 2.5f, 1, 71);                      // water-filled widths
    case_spkv(2, nullptr, 80);                    // forward_sp_kv_quant
    case_spkv(2, &w4, 81);                        // with the writer adapter
    return 0;
}
