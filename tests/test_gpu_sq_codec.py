"""The SpectralQuant codec at model widths on the device (kg_sq_encode /
kg_sq_decode on a KG_KV_SQ codec context) against the oracle's
store_vector / dequantize_*_into (src/spectralquant/spectral_kv_cache.rs:
399-470, 567-672): calibrated tables, packed codes, norms and dequantized
vectors bit for bit, zero vectors leaving their bytes untouched."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _samples(kvd, n, seed):
    rng = np.random.default_rng(seed)
    A = (rng.standard_normal((kvd, kvd)) / np.sqrt(kvd)).astype(np.float32)
    scale = (1.0 + 8.0 * np.exp(-np.arange(kvd) / 8.0)).astype(np.float32)   # a few strong directions
    return ((rng.standard_normal((n, kvd)).astype(np.float32) * scale) @ A).astype(np.float32)


@pytest.mark.parametrize("kvd,water_fill,avg_bits,n_vec", [(128, False, 3.0, 64), (768, True, 3.0, 48),
                                                          (4096, False, 4.0, 12)])
def test_sq_codec_matches_oracle(kg, orc, kvd, water_fill, avg_bits, n_vec):
    cfg = kg.micro_config(kv_mode=kg.KG_KV_SQ, n_embd=kvd, n_head=kvd // 64, head_dim=64, n_kv_head=kvd // 64,
                          mlp_hidden=256, vocab_size=64, n_layer=1, max_seqs=1)
    be = kg.CudaBackend(cfg)
    with pytest.raises(kg.KgError):                               # no tables yet
        be.sq_encode(np.ones((1, kvd), np.float32))
    X = _samples(kvd, 256, kvd)
    params = dict(avg_bits=avg_bits, use_water_fill=int(water_fill))
    be.sq_calibrate(X, kg.sq_params(**params))
    v, e, d = orc.sq_calibrate_eigenbasis(X)
    tabs = orc.sq_build(orc.sq_params(**{**params, "use_water_fill": water_fill}), kvd, v, e, np.float32(d))
    got = be.sq_tables(0)
    for a, key in zip(got[:4], ("eig", "bits", "cent", "nlev")):
        assert np.array_equal(a, tabs[key][0]), key
    assert got[4] == tabs["d_eff"][0]
    x = _samples(kvd, n_vec, kvd + 1)
    x[2] = 0.0                                                    # zero vector: norm 0, bytes untouched
    packed, norms = be.sq_encode(x, packed_init=np.full((n_vec, kvd), 0xA5, np.uint8))
    deq = be.sq_decode(packed, norms)
    for i in range(n_vec):
        pk, nr, dq = orc.sq_roundtrip(tabs, 0, x[i])
        assert norms[i] == np.float32(nr), i
        if nr == 0.0:
            assert np.all(packed[i] == 0xA5) and np.all(deq[i] == 0.0)
            continue
        assert np.array_equal(packed[i, :pk.size], pk), i
        assert np.all(packed[i, pk.size:] == 0xA5)
        assert np.array_equal(deq[i], dq), i
    be.close()
