"""SpectralQuant (src/spectralquant/) on the CPU: the oracle's restatement
against the reference's own tests for it, and the library's host-side table
build (kg_sq_calibrate_eigenbasis / kg_sq_build_tables, what a KG_KV_SQ
context installs on the device) against the oracle, bit for bit."""
import numpy as np
import pytest


def _pr(ev):  # participation_ratio (spectral.rs:11-24)
    ev = np.asarray(ev, np.float64)
    return np.float32(ev.sum() ** 2 / (ev * ev).sum())


def _test_calibration(kvd):  # make_test_calibration (spectral_kv_cache.rs:1193-1212)
    ev = (np.float32(10.0) * np.float32(0.8) ** np.arange(kvd)).astype(np.float32)
    return np.eye(kvd, dtype=np.float32).ravel(), ev, _pr(ev)


def test_calibrate_eigenbasis_reference_case(orc):
    # spectral.rs:973-1008: variances 4, 2, 1, 0.1 from per-sample seeded Rngs
    samples = []
    for i in range(200):
        seed = (i * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        z = orc.normals(seed, 4)
        samples.append([z[0] * np.float32(2.0), z[1] * np.float32(1.414), z[2] * np.float32(1.0),
                        z[3] * np.float32(0.316)])
    vec, val, d_eff = orc.sq_calibrate_eigenbasis(np.array(samples, np.float32))
    assert val.shape == (4,) and vec.shape == (16,)
    assert val[0] > 2.0
    assert d_eff < 4.0
    # columns are (near) orthonormal after the Jacobi rotations
    V = vec.reshape(4, 4)
    assert np.abs(V.T @ V - np.eye(4)).max() < 1e-3


@pytest.mark.parametrize("which", ["key", "value"])
def test_store_dequantize_roundtrip(orc, which):
    # spectral_kv_cache.rs:1276-1329 (3 bits on average, kv_dim 16)
    eig, ev, de = _test_calibration(16)
    tabs = orc.sq_build(orc.sq_params(), 16, eig, ev, de)
    f = np.sin if which == "key" else np.cos
    x = (np.sqrt(ev) * f(np.arange(16, dtype=np.float32) + 1)).astype(np.float32)
    packed, norm, rec = orc.sq_roundtrip(tabs, 0, x)
    o, r = np.linalg.norm(x), np.linalg.norm(rec)
    assert r > 0.1 and abs(o - r) / o < 1.0
    assert packed.size == (int(tabs["bits"][0].sum()) + 7) // 8


def test_multi_position_and_zero_vector(orc):
    # spectral_kv_cache.rs:1369-1422
    eig, ev, de = _test_calibration(16)
    tabs = orc.sq_build(orc.sq_params(), 16, eig, ev, de)
    for pos in range(4):
        x = (np.sqrt(ev) * np.sin(np.arange(16, dtype=np.float32) + pos + 1)).astype(np.float32)
        _, _, rec = orc.sq_roundtrip(tabs, 0, x)
        o, r = np.linalg.norm(x), np.linalg.norm(rec)
        assert r > 0.1 and abs(o - r) / o < 1.0
    _, norm, rec = orc.sq_roundtrip(tabs, 0, np.zeros(16, np.float32))
    assert norm == 0.0 and np.all(rec == 0.0)


def test_bit_allocation_and_waterfill(orc):
    # BitAllocator (spectral.rs:420-436): b_low = round(avg - d/kvd), b_high = b_low + 1
    eig, ev, de = _test_calibration(16)               # d_eff 8.5 -> 9 semantic dimensions
    t = orc.sq_build(orc.sq_params(), 16, eig, ev, de)
    assert t["d_eff"][0] == 9
    assert list(t["bits"][0]) == [3] * 9 + [2] * 7
    # water-fill (spectral.rs:443-478): b_high * d_eff bits over the semantic
    # dimensions, each within [wf_min, wf_max], more bits where lambda is larger
    t = orc.sq_build(orc.sq_params(use_water_fill=True), 16, eig, ev, de)
    b = t["bits"][0][:9]
    assert b.sum() == 3 * 9 and b.min() >= 1 and b.max() <= 6
    assert all(b[i] >= b[i + 1] for i in range(8))
    assert list(t["nlev"][0][:9]) == [1 << int(x) for x in b]


def test_identity_calibration_takes_random_rotation(orc):
    eig, ev, de = _test_calibration(16)
    t = orc.sq_build(orc.sq_params(), 16, np.stack([eig, eig]), np.stack([ev, ev]), np.array([de, de]))
    V0, V1 = t["eig"][0].reshape(16, 16), t["eig"][1].reshape(16, 16)
    assert not np.allclose(V0, np.eye(16)) and not np.array_equal(V0, V1)   # seed + layer * 7919
    assert np.abs(V0.T @ V0 - np.eye(16)).max() < 1e-4


@pytest.mark.parametrize("kvd", [16, 128])
@pytest.mark.parametrize("water_fill", [False, True])
@pytest.mark.parametrize("avg_bits", [2.0, 3.0, 4.0])
def test_library_tables_match_oracle(kg, orc, water_fill, avg_bits, kvd):
    rng = np.random.default_rng(int(avg_bits * 10) + water_fill)
    A = (rng.standard_normal((kvd, kvd)) * 0.3).astype(np.float32)
    scale = (2.0 ** -np.arange(kvd)).astype(np.float32)
    X = ((rng.standard_normal((300, kvd)).astype(np.float32) * scale) @ A).astype(np.float32)
    v1, e1, d1 = kg.sq_calibrate_eigenbasis(X)
    v2, e2, d2 = orc.sq_calibrate_eigenbasis(X)
    assert np.array_equal(v1, v2) and np.array_equal(e1, e2) and d1 == d2
    eig = np.stack([v1, np.eye(kvd, dtype=np.float32).ravel(), v1])
    ev = np.stack([e1, e1, (e1 * 1.5).astype(np.float32)])
    de = np.array([d1, d1, d1 + 3], np.float32)
    t1 = kg.sq_build_tables(kg.sq_params(avg_bits=avg_bits, use_water_fill=int(water_fill)), kvd, eig, ev, de)
    t2 = orc.sq_build(orc.sq_params(avg_bits=avg_bits, use_water_fill=water_fill), kvd, eig, ev, de)
    for k in t1:
        assert np.array_equal(t1[k], t2[k]), k


def test_forward_quantized_over_spectralquant_runs(orc):
    cfg = orc.config(n_layer=4)
    w = orc.weights(cfg, 42)
    eig, ev, de = _test_calibration(16)
    tabs = orc.sq_build(orc.sq_params(), 16, np.stack([eig] * 4), np.stack([ev] * 4), np.full(4, de, np.float32))
    toks = np.array([26, 3, 9, 14, 1, 7, 7, 20], np.int32)
    logits, codes, norms = orc.run_sequence_sq(cfg, w, tabs, toks)
    assert np.all(np.isfinite(logits)) and np.all(norms > 0)
    # the quantized forward stays close to forward_base on this model
    base = orc.run_sequence(cfg, orc.MODE_BASE, w, toks)[0]
    assert np.abs(logits - base).max() < 0.5 * np.abs(base).max()


# ---- the reference's unit tests of the building blocks (spectral.rs:845-1183,
# spectral_kv_cache.rs:1243-1274), on the oracle's restatement

def test_jacobi_reference_cases(orc):
    ev, V = orc.sq_jacobi(np.eye(4))                                  # identity
    assert np.all(np.abs(ev - 1) < 0.01) and np.all(np.abs(V - np.eye(4)) < 0.1)
    ev, _ = orc.sq_jacobi(np.diag([3.0, 1.0, 2.0]))                   # diagonal, sorted descending
    assert np.all(np.abs(ev - [3, 2, 1]) < 0.01)
    ev, V = orc.sq_jacobi(np.array([[2.0, 1.0], [1.0, 3.0]]))         # 2x2
    assert abs(ev.sum() - 5.0) < 0.01 and abs(V[0, 0] * V[0, 1] + V[1, 0] * V[1, 1]) < 0.01
    A = np.array([[4.0, 1, 2], [1, 3, 1], [2, 1, 5]])                 # known symmetric 3x3
    ev, V = orc.sq_jacobi(A)
    assert abs(ev.sum() - 12.0) < 0.01 and abs(np.prod(ev) - 43.0) < 0.5
    assert np.abs(V.T @ V - np.eye(3)).max() < 0.01
    D = V.T @ A.astype(np.float32) @ V
    assert np.abs(np.diag(D) - ev).max() < 0.1 and np.abs(D - np.diag(np.diag(D))).max() < 0.05


def test_bit_allocator_reference_cases(orc):
    bh, bl = orc.sq_allocate(6.0, 3.0, 128)
    assert bh >= bl and bh >= 1
    bh, bl = orc.sq_allocate(10.0, 3.0, 128)
    assert (bh, bl) == (4, 3)                                         # b_low = round(3 - 10/128)
    bh, bl = orc.sq_allocate(2.0, 4.0, 128)
    assert bh >= bl and bl >= 2


def test_waterfill_reference_cases(orc):
    b = orc.sq_waterfill([10.0, 5.0, 1.0, 0.5], 16, 2)
    assert b.size == 4 and int(b.sum()) == 16 and b[0] >= b[1]
    b = orc.sq_waterfill([5.0, 3.0, 1.0], 15, 3)
    assert np.all(b >= 3) and int(b.sum()) == 15
    b = orc.sq_waterfill([10.0, 1.0], 10, 2, 4)
    assert np.all(b <= 4)


def test_lloyd_max_reference_cases(orc):
    data = (np.arange(100, dtype=np.float32) - np.float32(50.0)) / np.float32(50.0)
    c = orc.sq_lloyd_fit(data, 2, 50, 42)
    assert c.size == 4
    for x in (-0.8, -0.2, 0.2, 0.8):
        assert abs(x - c[orc.sq_nearest(x, c)]) < 0.5
    s = np.sin(np.arange(200, dtype=np.float32) / np.float32(200.0)).astype(np.float32)
    def mse(c):
        return np.mean([(float(v) - float(c[orc.sq_nearest(v, c)])) ** 2 for v in s])
    assert mse(orc.sq_lloyd_fit(s, 4, 50, 42)) < mse(orc.sq_lloyd_fit(s, 2, 50, 42))
    d = np.arange(50, dtype=np.float32) * np.float32(0.1)
    assert np.array_equal(orc.sq_lloyd_fit(d, 3, 20, 99), orc.sq_lloyd_fit(d, 3, 20, 99))
    assert np.array_equal(orc.sq_lloyd_fit(np.zeros(0, np.float32), 2, 10, 42), np.zeros(4, np.float32))


@pytest.mark.parametrize("idx,bits", [([0, 1, 2, 3, 0, 2, 1, 3], [2] * 8), ([3, 7, 15, 1, 0], [2, 3, 4, 1, 1]),
                                      ([1, 0, 1, 1, 0, 0, 1, 0], [1] * 8)])
def test_pack_unpack_reference_cases(orc, idx, bits):
    p = orc.sq_pack(idx, bits)
    assert p.size == (sum(bits) + 7) // 8
    assert list(orc.sq_unpack(p, bits, len(idx))) == [i & ((1 << b) - 1) for i, b in zip(idx, bits)]


def test_published_spectralquant_quality(orc):
    # The reference's SpectralQuant quality benchmark (tests/bench_octopus_goat.rs:
    # 346-440, published in .benchmarks/022_octopus_goat.md): 512 N(0,1) keys of
    # dim 128 from Rng(42), from_keys on the first 256 (water-fill 2..8 bits,
    # 20 Lloyd-Max iterations, seed 42), store + dequantize every key; per-key
    # coordinate MSE and cosine, averaged. Published on Apple Silicon (NEON
    # reduction order) from an earlier revision: the restatement lands within
    # 3e-4 in cosine and 2.5% in MSE of every published figure.
    published = {2.0: (0.123319, 0.936769), 3.0: (0.037891, 0.981205), 4.0: (0.014516, 0.992954)}
    dim = 128
    keys = orc.normals(42, 512 * dim).reshape(512, dim)
    for bits, (mse_pub, cos_pub) in published.items():
        P = orc.sq_params(avg_bits=bits, min_tail_bits=2, max_bits=8, lloyd_max_iter=20, calibration_samples=256,
                          seed=42, use_water_fill=True, wf_min_bits=2, wf_max_bits=8)
        rec = orc.sq_quality_keys(P, keys, 256)
        mse = np.mean([float(((keys[i] - rec[i]) ** 2).sum(dtype=np.float32)) / dim for i in range(512)])
        cos = np.mean([orc.dot(keys[i], rec[i]) / np.sqrt(orc.dot(keys[i], keys[i]) * orc.dot(rec[i], rec[i]))
                       for i in range(512)])
        assert abs(cos - cos_pub) < 3e-4, (bits, cos, cos_pub)
        assert abs(mse - mse_pub) / mse_pub < 0.025, (bits, mse, mse_pub)
