"""forward_quantized over the SpectralQuant codec (kv_mode KG_KV_SQ) against
the oracle (src/transformer.rs:4042-4233 with src/spectralquant/
spectral_kv_cache.rs). The device's per-layer tables must equal the oracle's
build, and codes, norms and logits must be bit-identical: the micro path runs
the reference's operation order (rotate_into's ordered accumulation, the
bisection quantizer, LSB-first variable-width packing, row-dot unrotation)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _key_samples(seed, n=200, kvd=16):
    rng = np.random.default_rng(seed)
    A = (rng.standard_normal((kvd, kvd)) * 0.4).astype(np.float32)
    scale = (1.5 ** -np.arange(kvd)).astype(np.float32)
    return ((rng.standard_normal((n, kvd)).astype(np.float32) * scale) @ A).astype(np.float32)


def _same_tables(be, tabs, L):
    for l in range(L):
        e, b, c, n, d = be.sq_tables(l)
        assert np.array_equal(e, tabs["eig"][l]) and np.array_equal(b, tabs["bits"][l])
        assert np.array_equal(c, tabs["cent"][l]) and np.array_equal(n, tabs["nlev"][l]) and d == tabs["d_eff"][l]


def _check_forward(kg, orc, be, cfg, w, tabs, n_seq, seed):
    rng = np.random.default_rng(seed)
    toks = rng.integers(0, 27, size=(n_seq, 16)).astype(np.int32)
    toks[:, 0] = 26
    got = be.forward_batch(toks)
    ocfg = orc.from_kg(cfg)
    kvd = cfg.kvd()
    for i in range(n_seq):
        lo, codes, norms = orc.run_sequence_sq(ocfg, w, tabs, toks[i])
        assert np.array_equal(got[i], lo), i
        for l in range(cfg.n_layer):
            nb = (int(tabs["bits"][l].sum()) + 7) // 8
            for t in range(16):
                kp, vp, nr = be.kv_codes(i, l, t)
                assert np.array_equal(kp[:nb], codes[l, t, :nb]) and np.array_equal(vp[:nb], codes[l, t, kvd:kvd + nb])
                assert np.array_equal(nr, norms[l, t])


@pytest.mark.parametrize("L,water_fill,avg_bits", [(1, False, 3.0), (4, True, 3.0), (2, False, 4.0)])
def test_sq_from_keys_bit_identical(kg, orc, L, water_fill, avg_bits):
    cfg = kg.micro_config(kv_mode=kg.KG_KV_SQ, n_layer=L, max_seqs=48)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    with pytest.raises(kg.KgError):                       # tables not built yet
        be.forward_batch(np.full((1, 1), 26, np.int32))
    X = _key_samples(L * 10 + water_fill)
    be.sq_calibrate(X, kg.sq_params(avg_bits=avg_bits, use_water_fill=int(water_fill)))
    v, e, d = orc.sq_calibrate_eigenbasis(X)              # from_keys: one calibration for every layer
    tabs = orc.sq_build(orc.sq_params(avg_bits=avg_bits, use_water_fill=water_fill), 16, np.stack([v] * L),
                        np.stack([e] * L), np.full(L, d, np.float32))
    _same_tables(be, tabs, L)
    _check_forward(kg, orc, be, cfg, w, tabs, 48, L)
    be.close()


def test_sq_from_calibration_per_layer(kg, orc):
    # from_calibration with a different calibration per layer; layer 1's is the
    # identity (replaced by a seeded random rotation)
    L = 3
    cfg = kg.micro_config(kv_mode=kg.KG_KV_SQ, n_layer=L, max_seqs=24)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 7)
    be.compile(w)
    cal = [orc.sq_calibrate_eigenbasis(_key_samples(s)) for s in (1, 2, 3)]
    eig = np.stack([cal[0][0], np.eye(16, dtype=np.float32).ravel(), cal[2][0]])
    ev = np.stack([c[1] for c in cal])
    de = np.array([c[2] for c in cal], np.float32)
    p = dict(avg_bits=2.5, use_water_fill=True, wf_max_bits=5)
    be.sq_calibrate_from(eig, ev, de, kg.sq_params(**p))
    tabs = orc.sq_build(orc.sq_params(**p), 16, eig, ev, de)
    _same_tables(be, tabs, L)
    _check_forward(kg, orc, be, cfg, w, tabs, 24, 9)
    be.close()
