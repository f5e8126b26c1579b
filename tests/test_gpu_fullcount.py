"""The micro configurations at their full sequence counts.

C1: Config::micro, AttentionMode::Standard (forward_base), 4096 sequences x
[BOS + 15 tokens], teacher-forced: logits bit-identical to the oracle.
C2: the same model with SpKvQuant and the 3-bit TurboQuant codec, 65,536
sequences x 16 positions: logits within 1e-5 relative (libm expf) and the
packed K/V codes and norms bit-identical (checked on every 64th sequence).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def tokens(n_seq, seed):
    rng = np.random.default_rng(seed)
    t = rng.integers(1, 27, size=(n_seq, 16)).astype(np.int32)
    t[:, 0] = 26
    return t


def test_c1_full_count_bit_identical(kg, orc):
    n = 4096
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, max_seqs=n)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    toks = tokens(n, 101)
    np.testing.assert_array_equal(be.forward_batch(toks), orc.run_batch(orc.from_kg(cfg), orc.MODE_BASE, w, toks))
    be.close()


def test_c2_full_count(kg, orc):
    n = 65536
    cfg = kg.micro_config(kv_mode=kg.KG_KV_SPKV_TQ, max_seqs=n)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    toks = tokens(n, 102)
    got = be.forward_batch(toks)
    ref = orc.run_batch(orc.from_kg(cfg), orc.MODE_SPKV, w, toks)
    den = np.maximum(np.abs(ref).max(axis=-1, keepdims=True), 1e-30)
    assert float((np.abs(got - ref) / den).max()) <= 1e-5
    for i in range(0, n, 64):
        _, codes, norms, _ = orc.run_sequence(orc.from_kg(cfg), orc.MODE_SPKV, w, toks[i])
        for t in range(16):
            kp, vp, nr = be.kv_codes(i, 0, t)
            np.testing.assert_array_equal(np.concatenate([kp, vp]), codes[0, t])
            np.testing.assert_array_equal(nr, norms[0, t])
    be.close()
