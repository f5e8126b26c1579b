"""CPU oracle checks, mirroring the reference's own unit and integration tests.

Each test names the reference test it restates. The reference publishes no
golden vectors that its current source reproduces (see
test_published_turboquant_table), so these assertions are the oracle's pin.
"""
import math

import numpy as np
import pytest


# ---- Rng — crates/katgpt-types/src/rng.rs:75-156 ----------------------------

def test_rng_first_uniform_nonzero(orc):
    for seed in [0, 1, 2, 3, 4, 5, 42, 100, 1337, 0xFFFFFFFF]:
        u = orc.uniforms(seed, 1)[0]
        assert 0.0 < u < 1.0


def test_rng_determinism_and_divergence(orc):
    a, b = orc.uniforms(42, 16), orc.uniforms(42, 16)
    assert np.array_equal(a, b)
    r = [orc.uniforms(s, 1)[0] for s in (1, 2, 3)]
    assert len(set(r)) == 3


def test_rng_chi_square(orc):
    u = orc.uniforms(42, 65536)
    counts = np.bincount(np.minimum((u * 256).astype(np.int64), 255), minlength=256)
    exp = 65536 / 256
    chi = float(((counts - exp) ** 2).sum() / exp)
    assert chi < 400.0


def test_normals_finite_and_standard(orc):
    z = orc.normals(7, 200000).astype(np.float64)
    assert np.isfinite(z).all()
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01


# ---- SIMD kernels vs scalar restatements (crates/katgpt-types/src/simd/tests.rs) ----

@pytest.mark.parametrize("n", [1, 3, 4, 7, 8, 15, 16, 17, 31, 32, 33, 64, 100, 768, 4099])
def test_simd_reductions_match_scalar(orc, n):
    rng = np.random.default_rng(n)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    ref = float(np.dot(a.astype(np.float64), b.astype(np.float64)))
    assert abs(orc.dot(a, b) - ref) <= 1e-5 * (1 + np.abs(a * b).sum())
    assert abs(orc.sum_sq(a) - float((a.astype(np.float64) ** 2).sum())) <= 1e-5 * (1 + (a * a).sum())
    assert abs(orc.vsum(a) - float(a.astype(np.float64).sum())) <= 1e-5 * (1 + np.abs(a).sum())
    assert orc.vmax(a) == a.max()


def test_dot_lane_order_is_avx2(orc):
    # 64 elements: the AVX2 path sums 32 lane chains then a fixed tree; build a
    # case where that order and a sequential sum round differently.
    a = np.array([1e8, 1.0, -1e8] + [1.0] * 61, np.float32)
    b = np.ones(64, np.float32)
    acc = np.zeros(32, np.float32)
    for c in range(2):
        for L in range(32):
            acc[L] = np.float32(acc[L] + np.float32(a[32 * c + L] * b[32 * c + L]))
    t = [np.float32(np.float32(acc[l] + acc[8 + l]) + np.float32(acc[16 + l] + acc[24 + l])) for l in range(8)]
    s = [np.float32(t[i] + t[i + 4]) for i in range(4)]
    expect = np.float32(np.float32(np.float32(s[0] + s[1]) + np.float32(s[2] + s[3])) + np.float32(0.0))
    assert orc.dot(a, b) == expect


@pytest.mark.parametrize("n", [1, 5, 8, 13, 16, 27, 40, 64])
def test_exp_accuracy_and_tail(orc, n):
    x = np.linspace(-20.0, 20.0, n).astype(np.float32)
    y = orc.exp_inplace(x)
    ref = np.exp(x.astype(np.float64))
    assert np.all(np.abs(y - ref) <= 4e-6 * ref)
    for v in x[n // 8 * 8:]:   # scalar tail elements use cephes_exp_scalar
        assert orc.scalar_exp(v) == y[list(x).index(v)]
    ye, s = orc.exp_sum_inplace(x)
    assert np.allclose(ye, y, rtol=0, atol=0) or np.all(np.abs(ye - ref) <= 4e-6 * ref)
    assert abs(s - float(ref.sum())) <= 1e-5 * float(ref.sum())


def test_softmax_scaled_and_sample(orc):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(27).astype(np.float32)
    p = orc.softmax_scaled(x, 2.0)
    ref = np.exp(2 * (x - x.max()).astype(np.float64))
    ref /= ref.sum()
    assert np.allclose(p, ref, rtol=1e-5, atol=1e-7)
    assert abs(p.sum() - 1.0) < 1e-5
    t = orc.sample_token(p, 42)
    assert 0 <= t < 27
    assert orc.sample_token(p, 42) == t


# ---- TwELL sparse matmul (src/transformer.rs:5197-5340) -------------------------

def _sparse_rows(orc, weight, inp, rows, cols):
    idx = np.nonzero(inp > 0)[0]
    return np.array([orc.sparse_dot(weight[r * cols:(r + 1) * cols], idx, inp[idx]) for r in range(rows)],
                    np.float32), idx.size


@pytest.mark.parametrize("case", ["0pct", "95pct", "100pct", "negative"])
def test_sparse_matches_dense(orc, case):
    rows, cols = (8, 32) if case == "negative" else (16, 64)
    weight = ((np.arange(rows * cols) % 100) * 0.01).astype(np.float32)
    if case == "0pct":
        inp = ((np.arange(cols) + 1.0) * 0.1).astype(np.float32)
    elif case == "95pct":
        inp = np.zeros(cols, np.float32)
        inp[::20] = 1.0
    elif case == "100pct":
        inp = np.zeros(cols, np.float32)
    else:
        inp = np.zeros(cols, np.float32)
        inp[[0, 1, 2, 3]] = [1.0, -1.0, 0.5, -0.5]
    sp, alive = _sparse_rows(orc, weight, inp, rows, cols)
    dense = np.array([orc.dot(weight[r * cols:(r + 1) * cols], np.maximum(inp, 0)) for r in range(rows)])
    if case == "100pct":
        assert alive == 0 and np.all(sp == 0)
    else:
        assert np.all(np.abs(dense - sp) < 1e-3)


# ---- TurboQuant codebook / rotation / packing (src/turboquant/*.rs tests) ------

@pytest.mark.parametrize("bits", [2, 3, 4])
def test_codebook_structure(orc, bits):
    c, b, mse = orc.codebook(128, bits)
    assert c.size == 1 << bits and b.size == (1 << bits) - 1
    assert np.all(np.diff(b) > 0) and np.all(np.diff(c) > 0)
    assert np.allclose(c, -c[::-1], atol=1e-4)      # symmetric
    assert mse > 0


def test_codebook_mse_decreases_with_bits(orc):
    mses = [orc.codebook(128, b)[2] for b in (2, 3, 4)]
    assert mses[0] > mses[1] > mses[2]


@pytest.mark.parametrize("dim", [16, 64, 128])
def test_rotation_orthogonal_deterministic(orc, dim):
    r = orc.rotation(dim, 42).astype(np.float64)
    assert np.abs(r @ r.T - np.eye(dim)).max() < 1e-4
    assert np.array_equal(orc.rotation(dim, 42), orc.rotation(dim, 42))
    v = np.random.default_rng(1).standard_normal(dim)
    assert abs(np.linalg.norm(r @ v) - np.linalg.norm(v)) < 1e-4 * np.linalg.norm(v)


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 8])
def test_pack_unpack_roundtrip(orc, bits):
    n = 37
    idx = (np.arange(n) * 7 % (1 << bits)).astype(np.uint8)
    p = orc.tq_pack(idx, bits)
    assert p.size == orc.packed_len(n, bits)
    assert np.array_equal(orc.tq_unpack(p, n, bits), idx)


def test_zero_vector(orc):
    dim, bits = 16, 3
    rot = orc.rotation(dim)
    c, b, _ = orc.codebook(dim, bits)
    pk, nrm = orc.tq_store(rot, b, bits, np.zeros(dim, np.float32), packed_init=np.full(8, 0xAB, np.uint8))
    assert nrm == 0.0 and np.all(pk == 0xAB)          # indices left untouched
    out = orc.tq_dequant(rot.T.copy(), c, bits, pk, nrm)
    assert np.all(out == 0.0)


def _synthetic_kv(dim, pos):
    # tests/bench_turboquant.rs:23-27 (f32 sin/cos)
    i = np.arange(dim)
    a = (np.float32(1) * (i + pos * 7).astype(np.float32) * np.float32(0.1)).astype(np.float32)
    b = ((i + pos * 3).astype(np.float32) * np.float32(0.07)).astype(np.float32)
    return (np.sin(a.astype(np.float64)).astype(np.float32) + np.cos(b.astype(np.float64)).astype(np.float32))


def _tq_quality(orc, bits, rot=None):
    dim = 16
    rot = orc.rotation(dim) if rot is None else rot
    c, b, _ = orc.codebook(dim, bits)
    kc = []
    vc = []
    for p in range(16):
        k, v = _synthetic_kv(dim, p), _synthetic_kv(dim, p + 100)
        for vec, out in ((k, kc), (v, vc)):
            pk, nrm = orc.tq_store(rot, b, bits, vec)
            out.append(orc.cosine(vec, orc.tq_dequant_scalar(rot, c, bits, pk, nrm)))
    return float(np.mean(kc)), float(np.mean(vc))


def test_turboquant_roundtrip_thresholds(orc):
    # tests/bench_turboquant.rs:118-199 asserted quality targets
    targets = {4: (0.95, 0.90), 3: (0.90, 0.85), 2: (0.80, 0.75)}
    for bits, (tk, tv) in targets.items():
        k, v = _tq_quality(orc, bits)
        assert k > tk and v > tv, (bits, k, v)


def test_turboquant_bytes_per_token(orc):
    # tests/bench_turboquant.rs:54-85: 16/24/24 bytes, ratios > 6/4/3 at kv_dim 16
    for bits, bpt, ratio in ((2, 16, 6.0), (3, 24, 4.0), (4, 24, 3.0)):
        got = 2 * orc.packed_len(16, bits) + 8
        assert got == bpt and (16 * 4 * 2) / got > ratio


def test_published_turboquant_table(orc):
    """.docs/04_performance.md:323-328 publishes key cos_sim 0.9242/0.9825/0.9958.

    The current source does not reproduce those digits under either Rng
    seeding (the table predates the SplitMix64 seed expansion of issue 296 and
    was measured on Apple NEON): the oracle gives 0.9556 / 0.9880 / 0.9963. The
    test bounds the gap at 0.04 per bit-width.
    """
    published = {2: 0.9242, 3: 0.9825, 4: 0.9958}
    for bits, pub in published.items():
        k, _ = _tq_quality(orc, bits)
        assert abs(k - pub) < 0.04, (bits, k, pub)


# ---- forward paths -----------------------------------------------------------

@pytest.mark.parametrize("mode", [0, 1, 2])
def test_forward_finite_and_deterministic(orc, mode):
    cfg = orc.config()
    w = orc.weights(cfg, 42)
    toks = np.array([26] + [(p * 7 + 3) % 26 + 1 for p in range(15)], np.int32)
    l1 = orc.run_sequence(cfg, mode, w, toks)[0]
    l2 = orc.run_sequence(cfg, mode, w, toks)[0]
    assert np.isfinite(l1).all() and np.array_equal(l1, l2)


def test_teacher_forced_prefix_consistency(orc):
    # logits at position p depend only on tokens 0..p (causal)
    cfg = orc.config(n_layer=4)
    w = orc.weights(cfg, 3)
    toks = np.array([26, 5, 9, 1, 3, 7, 2, 8], np.int32)
    full = orc.run_sequence(cfg, 0, w, toks)[0]
    part = orc.run_sequence(cfg, 0, w, toks[:5])[0]
    assert np.array_equal(full[:5], part)


def test_quantized_as_written_shares_buffer_across_layers(orc):
    """forward_quantized keeps one flat dequant buffer for every layer
    (src/transformer.rs:4088-4121 with ForwardContext::paged_flat_key): for
    n_layer > 1 later positions attend to another layer's keys. The oracle's
    default QUANT mode uses one buffer per layer; with one layer both agree."""
    toks = np.array([26, 4, 8, 15, 16, 23, 1, 2], np.int32)
    c1 = orc.config()
    w1 = orc.weights(c1, 42)
    a = orc.run_sequence(c1, orc.MODE_QUANT, w1, toks)[0]
    b = orc.run_sequence(c1, orc.MODE_QUANT_AS_WRITTEN, w1, toks)[0]
    assert np.array_equal(a, b)
    c2 = orc.config(n_layer=2)
    w2 = orc.weights(c2, 42)
    a = orc.run_sequence(c2, orc.MODE_QUANT, w2, toks)[0]
    b = orc.run_sequence(c2, orc.MODE_QUANT_AS_WRITTEN, w2, toks)[0]
    assert np.array_equal(a[0], b[0]) and not np.array_equal(a[1:], b[1:])


def test_spkv_every_position_retained(orc):
    # bench_sp_kv_quant.rs: open gates, every written position is retained;
    # utilities are the predictor output sigmoid(...) with b2 = 5 (about 0.99)
    cfg = orc.config()
    w = orc.weights(cfg, 42)
    toks = np.array([(p * 7 + 3) % 27 for p in range(8)], np.int32)
    logits, codes, norms, util = orc.run_sequence(cfg, orc.MODE_SPKV, w, toks)
    assert np.isfinite(logits).all()
    assert np.all(util > 0.5) and np.all(util < 1.0)
    assert np.all(norms > 0)


def test_batch_runner_matches_sequence_runner(orc):
    cfg = orc.config()
    w = orc.weights(cfg, 42)
    rng = np.random.default_rng(5)
    toks = rng.integers(1, 27, size=(6, 16)).astype(np.int32)
    toks[:, 0] = 26
    for mode in (0, 1, 2):
        batch = orc.run_batch(cfg, mode, w, toks, threads=3)
        for i in range(6):
            assert np.array_equal(batch[i], orc.run_sequence(cfg, mode, w, toks[i])[0])


def test_forced_codes_replay(orc):
    # the replay entry behind the GPU parity at the configurations' shapes:
    # the oracle's own codes reproduce its logits bit for bit, and one changed
    # code byte (layer 0, position 5) changes nothing before position 5
    cfg = orc.config()
    w = orc.weights(cfg, 42)
    toks = np.random.default_rng(8).integers(1, 27, size=16).astype(np.int32)
    lo, codes, _, _ = orc.run_sequence_rot(cfg, orc.MODE_QUANT, w, toks, key_bits=3, val_bits=3)
    assert np.array_equal(orc.run_sequence_forced(cfg, w, toks, codes, 3, 3), lo)
    c2 = codes.copy()
    c2[0, 5, 0] ^= 0x07
    lf = orc.run_sequence_forced(cfg, w, toks, c2, 3, 3)
    assert np.array_equal(lf[:5], lo[:5])
    assert not np.array_equal(lf[5], lo[5])


def test_forward_prefill_reference_cases(orc):
    # src/transformer.rs:5376-5596 on the restatement: a prompt of 8, of 3 and
    # of 1 token gives vocab_size finite logits, and decoding continues from
    # the prompt's cache with finite logits (prefill_then_decode)
    cfg = orc.config()
    w = orc.weights(cfg, 42)
    for prompt in (list(range(8)), [0, 1, 2], [5]):
        out = orc.prefill_then_decode(cfg, w, np.array(prompt, np.int32))
        assert out.shape == (1, cfg.vocab_size) and np.all(np.isfinite(out))
    out = orc.prefill_then_decode(cfg, w, np.arange(4, dtype=np.int32), [0])
    assert out.shape == (2, cfg.vocab_size) and np.all(np.isfinite(out))
    # prefill differs from teacher-forced forward_base (bidirectional attention, double norm)
    base = orc.run_sequence(cfg, orc.MODE_BASE, w, np.arange(4, dtype=np.int32))[0]
    assert not np.array_equal(out[0], base[3])


def test_published_turboquant_quality_bench022(orc):
    # The reference's TurboQuant legacy comparison (tests/bench_octopus_goat.rs:
    # 440-505, published in .benchmarks/022_octopus_goat.md section 3): 512 N(0,1)
    # keys of dim 128 from Rng(42) stored with TurboQuantKVCache::new (rotation
    # from the same Rng(42) stream), dequantize_key, per-key MSE and cosine.
    # The keys are the rotation's own Gaussian draws, which is why these
    # figures sit below the random-vector table: the restatement reproduces
    # that (cosine within 2e-3, MSE within 4% of every published figure), and
    # independent draws land at 0.941 / 0.983 / 0.995.
    published = {2: (0.1790, 0.9048), 3: (0.0886, 0.9552), 4: (0.0512, 0.9760)}
    dim = 128
    keys = orc.normals(42, 512 * dim).reshape(512, dim)
    rot = orc.rotation(dim, 42)
    rot_t = np.ascontiguousarray(rot.T)
    for bits, (mse_pub, cos_pub) in published.items():
        cent, bnd = orc.codebook(dim, bits)[:2]
        mses, coss = [], []
        for i in range(512):
            pk, nr = orc.tq_store(rot, bnd, bits, keys[i])
            rec = orc.tq_dequant(rot_t, cent, bits, pk, nr)
            mses.append(float(((keys[i] - rec) ** 2).sum(dtype=np.float32)) / dim)
            coss.append(orc.dot(keys[i], rec) / np.sqrt(orc.dot(keys[i], keys[i]) * orc.dot(rec, rec)))
        assert abs(np.mean(coss) - cos_pub) < 2e-3, (bits, np.mean(coss), cos_pub)
        assert abs(np.mean(mses) - mse_pub) / mse_pub < 0.04, (bits, np.mean(mses), mse_pub)


def test_spkv_reference_cases(orc):
    # src/sp_kv/utility_predictor.rs:240-272 and src/sp_kv/forward.rs:832-960
    u = orc.spkv_predict(32, 16, 4, 5.0, np.ones(32, np.float32))
    assert u.shape == (4,) and np.all((u > 0) & (u < 1))
    assert np.all(orc.spkv_predict(32, 16, 4, 5.0, np.zeros(32, np.float32)) > 0.99)   # gates start open
    hd, kvd, tn = 8, 16, 4                                                              # no gate = baseline
    q, K, V = np.full(kvd, 0.1), np.full(tn * kvd, 0.2), np.full(tn * kvd, 0.3)
    out, _ = orc.attention_head_gated(q, K, V, kvd, hd, tn, 1.0 / np.sqrt(hd))
    assert np.all(np.abs(out[:hd] - 0.3) < 1e-4)
    hd = kvd = 4                                                                        # a -inf bias prunes
    q, K, V = np.ones(kvd), np.ones(tn * kvd), np.ones(tn * kvd)
    out, sc = orc.attention_head_gated(q, K, V, kvd, hd, tn, 0.5, bias=[0.0, 0.0, -np.inf, 0.0])
    assert np.all(np.abs(out[:hd] - 1.0) < 1e-4)
    assert sc[0] + sc[1] + sc[3] > 0 and sc[2] < 1e-20


def test_gamma_folding_matches_runtime_gammas(orc):
    # src/transformer.rs:6683-6790 (proof_gamma_folding_forward_base): the MLP
    # gamma folded into mlp_w1 (weights.rs:205-221) gives the run-time-gamma
    # forward within 1e-5; the attention gamma stays at run time
    cfg = orc.config(n_layer=2)
    n, m, L, V, B = cfg.n_embd, cfg.mlp_hidden, cfg.n_layer, cfg.vocab_size, cfg.block_size
    kvd = cfg.n_kv_head * cfg.head_dim
    w = orc.weights(cfg, 42)
    i = np.arange(n, dtype=np.float32)
    ag = np.float32(0.5) + np.sin(i * np.float32(0.1)).astype(np.float32) * np.float32(0.8)
    mg = np.float32(0.5) + np.cos(i * np.float32(0.15)).astype(np.float32) * np.float32(0.6)
    w[-2 * L * n:-L * n] = np.tile(ag, L)
    w[-L * n:] = np.tile(mg, L)
    toks = np.array([26, 3, 9, 14, 1, 7, 20, 5], np.int32)
    base = orc.run_sequence(cfg, orc.MODE_BASE, w, toks)[0]
    folded = w.copy()
    per_layer = 2 * n * n + 2 * kvd * n + 2 * m * n
    for l in range(L):
        o = V * n + B * n + l * per_layer + 2 * n * n + 2 * kvd * n     # mlp_w1 [m][n]
        w1 = folded[o:o + m * n].reshape(m, n)
        w1 *= mg[None, :]
    folded[-L * n:] = 1.0
    got = orc.run_sequence(cfg, orc.MODE_BASE, folded, toks)[0]
    assert np.abs(got - base).max() < 1e-5 * max(1.0, np.abs(base).max())
    plain = orc.run_sequence(cfg, orc.MODE_BASE, orc.weights(cfg, 42), toks)[0]
    assert np.abs(plain - base).max() > 1e-3                            # the gammas matter


def test_turboquant_cache_reference_cases(orc):
    # src/turboquant/kv_cache.rs:772-794, 902-926, 928-951 and codebook.rs:245-258,
    # 284-293 at Config::micro() (kv_dim 16), 4-bit keys and values
    dim, bits = 16, 4
    rot = orc.rotation(dim)
    c, b, _ = orc.codebook(dim, bits)
    i = np.arange(dim, dtype=np.float32)

    def roundtrip(x, scalar=False):
        pk, nrm = orc.tq_store(rot, b, bits, x)
        if scalar:
            return orc.tq_dequant_scalar(rot, c, bits, pk, nrm)
        return orc.tq_dequant(rot.T.copy(), c, bits, pk, nrm)

    key = np.sin(i * np.float32(0.1) - np.float32(1.0)).astype(np.float32)
    val = np.cos(i * np.float32(0.2)).astype(np.float32)
    assert orc.cosine(key, roundtrip(key)) > 0.90 and orc.cosine(val, roundtrip(val)) > 0.85
    k3 = np.sin(i * np.float32(0.3)).astype(np.float32)                  # the _into path vs the scalar one
    assert np.abs(roundtrip(k3) - roundtrip(k3, scalar=True)).max() < 1e-5
    for x in (np.sin(i).astype(np.float32), np.cos(i).astype(np.float32)):  # layers reconstruct independently
        assert orc.cosine(x, roundtrip(x)) > 0.90
    c64, b64, _ = orc.codebook(64, 4)
    for v in (-0.5, -0.3, -0.1, 0.0, 0.1, 0.3, 0.5):                      # quantize -> dequantize
        assert abs(c64[np.searchsorted(b64, np.float32(v), side="right")] - v) < 0.5
    assert all(orc.codebook(64, bb)[2] > 0 for bb in range(2, 7))


def test_oracle_bindings_match_header(orc):
    # oracle.py binds the C restatement with kg_oracle.h's parameter types
    import ctypes
    import os
    import re
    src = open(os.path.join(os.path.dirname(orc.__file__), "kg_oracle.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    scalar = {"int32_t": ctypes.c_int32, "int": ctypes.c_int, "int64_t": ctypes.c_int64,
              "uint64_t": ctypes.c_uint64, "float": ctypes.c_float, "double": ctypes.c_double}

    def same(c_type, t):
        if "*" in c_type:
            return t in (ctypes.c_void_p, ctypes.c_char_p) or issubclass(t, ctypes._Pointer)
        want = scalar[c_type.replace("const ", "").strip()]
        return ctypes.sizeof(t) == ctypes.sizeof(want) and (t in (ctypes.c_float, ctypes.c_double)) == (
            want in (ctypes.c_float, ctypes.c_double))

    L = orc.lib()
    n = 0
    for m in re.finditer(r"([\w \*]+?)\b(or_\w+)\s*\(([^;{]*?)\)\s*;", src, re.S):
        name = m.group(2)
        args = [a.strip() for a in " ".join(m.group(3).split()).split(",") if a.strip() and a.strip() != "void"]
        fn = getattr(L, name)
        assert fn.argtypes is not None, f"{name} is not bound"
        n += 1
        assert len(fn.argtypes) == len(args), name
        for a, t in zip(args, fn.argtypes):
            assert same(a if "*" in a else a.rsplit(" ", 1)[0], t), (name, a, t)
        ret = " ".join(m.group(1).split())
        if "*" not in ret and ret != "void":
            assert same(ret, fn.restype), (name, ret, fn.restype)
    assert n >= 40


def _adapter(n, rank, seed, scale=0.1):
    rng = np.random.default_rng(seed)
    return ((rng.standard_normal((rank, n)) * scale).astype(np.float32),
            (rng.standard_normal((n, rank)) * scale).astype(np.float32), 8.0)


def test_lora_apply_matches_its_definition(orc):
    # lora_apply (crates/katgpt-types/src/lora.rs:452-467): out += (alpha / rank) * B @ (A @ x)
    for rank, in_dim, out_dim in ((4, 16, 16), (3, 16, 16), (8, 12, 5), (16, 16, 16)):
        rng = np.random.default_rng(rank * 100 + in_dim)
        a = rng.standard_normal((rank, in_dim)).astype(np.float32)
        b = rng.standard_normal((out_dim, rank)).astype(np.float32)
        x = rng.standard_normal(in_dim).astype(np.float32)
        out = rng.standard_normal(out_dim).astype(np.float32)
        got = orc.lora_apply(a, b, 8.0, x, out)
        want = out.astype(np.float64) + (8.0 / rank) * (b.astype(np.float64) @ (a.astype(np.float64) @ x))
        assert np.abs(got - want).max() < 1e-5 * max(1.0, np.abs(want).max())


def test_lora_pair_in_forward_base_and_prefill(orc):
    # generate_with_prefill's LoraPair (src/transformer.rs:3010-3106): the
    # reader acts in forward_prefill only, the writer in forward_base only;
    # LoraPair::none() is the plain forward (:5570-5595); the reference's
    # constant adapter (rank 4, alpha 8, every weight 0.1, :6012-6030) changes the logits
    cfg = orc.config(n_layer=2)
    w = orc.weights(cfg, 42)
    prompt = np.array([26, 3, 9, 14, 1], np.int32)
    cont = np.array([7, 20, 5], np.int32)
    plain = orc.prefill_then_decode(cfg, w, prompt, cont)
    with orc.lora_pair():
        assert np.array_equal(orc.prefill_then_decode(cfg, w, prompt, cont), plain)
    const = (np.full((4, 16), 0.1, np.float32), np.full((16, 4), 0.1, np.float32), 8.0)
    with orc.lora_pair(writer=const):
        wr = orc.prefill_then_decode(cfg, w, prompt, cont)
        base_w = orc.run_sequence(cfg, orc.MODE_BASE, w, prompt)[0]
    assert np.array_equal(wr[0], plain[0])                       # the prefill ignores the writer
    assert np.abs(wr[1:] - plain[1:]).max() > 1e-3               # decode steps take it
    assert np.abs(base_w - orc.run_sequence(cfg, orc.MODE_BASE, w, prompt)[0]).max() > 1e-3
    with orc.lora_pair(reader=_adapter(16, 4, 1)):
        rd = orc.prefill_then_decode(cfg, w, prompt, cont)
    assert np.abs(rd[0] - plain[0]).max() > 1e-4                 # the prefill takes the reader
    zero_b = (np.full((4, 16), 0.3, np.float32), np.zeros((16, 4), np.float32), 8.0)
    with orc.lora_pair(reader=zero_b, writer=zero_b):            # B = 0 adds exact zeros
        assert np.array_equal(orc.prefill_then_decode(cfg, w, prompt, cont), plain)


def test_lora_in_forward_sp_kv_quant(orc):
    # forward_sp_kv_quant takes the same optional adapter after the same six
    # projections (src/sp_kv/forward.rs:673-684, 753-756, 769-771, 805-807)
    cfg = orc.config(n_layer=2)
    w = orc.weights(cfg, 42)
    toks = np.array([26, 3, 9, 14, 1, 7], np.int32)
    plain = orc.run_sequence(cfg, orc.MODE_SPKV, w, toks)
    zero_b = (np.full((4, 16), 0.3, np.float32), np.zeros((16, 4), np.float32), 8.0)
    with orc.lora_pair(writer=zero_b):
        same = orc.run_sequence(cfg, orc.MODE_SPKV, w, toks)
    assert np.array_equal(same[0], plain[0]) and np.array_equal(same[1], plain[1])
    with orc.lora_pair(writer=_adapter(16, 4, 3)):
        ad = orc.run_sequence(cfg, orc.MODE_SPKV, w, toks)
    assert np.abs(ad[0] - plain[0]).max() > 1e-3
