"""Norm gammas at the boundary (forward_base with kog_cpu_fusion).

The default CPU forward applies attn_norm_gamma before attention and
mlp_norm_gamma before the MLP through rmsnorm_with_gamma
(src/transformer.rs:1893-1895, 2023-2026; math.rs:218-233). The flat weight
layout ends with both [n_layer][n_embd] vectors, so a model with trained
gammas uploads them. Bars: the exact micro path bit-identical, the bf16
standard-attention path within 2e-2 of the oracle on the same weights.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def with_random_gammas(w, L, n, seed):
    w = w.copy()
    rng = np.random.default_rng(seed)
    w[-2 * L * n:] = (1.0 + 0.3 * rng.standard_normal(2 * L * n)).astype(np.float32)
    return w


def test_gammas_exact_path_bit_identical(kg, orc):
    n_seq = 64
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, n_layer=2, max_seqs=n_seq)
    be = kg.CudaBackend(cfg)
    w = with_random_gammas(kg.reference_weights(cfg, 42), 2, 16, seed=5)
    be.compile(w)
    rng = np.random.default_rng(9)
    toks = rng.integers(1, 27, size=(n_seq, 16)).astype(np.int32)
    toks[:, 0] = 26
    got = be.forward_batch(toks)
    ref = orc.run_batch(orc.from_kg(cfg), orc.MODE_BASE, w, toks)
    np.testing.assert_array_equal(got, ref)
    plain = orc.run_batch(orc.from_kg(cfg), orc.MODE_BASE, kg.reference_weights(cfg, 42), toks)
    assert np.abs(plain - ref).max() > 1e-3          # the gammas change the forward
    be.close()


def test_gammas_bf16_standard_attention(kg, orc):
    cfg = kg.micro_config(vocab_size=96, block_size=64, n_embd=128, n_head=2, head_dim=64, n_kv_head=2,
                          mlp_hidden=256, n_layer=4, kv_mode=kg.KG_KV_F32, weight_dtype=kg.KG_W_BF16, max_seqs=2)
    be = kg.CudaBackend(cfg)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=11, scale_mode=1, std=0.05))
    w = with_random_gammas(w, 4, 128, seed=6)
    be.compile(w)
    toks = np.random.default_rng(12).integers(0, 96, size=(2, 40)).astype(np.int32)
    pre = be.forward_batch(toks[:, :32])
    dec = np.stack([be.forward_batch(toks[:, t:t + 1], start_pos=np.full(2, t))[:, 0] for t in range(32, 40)], 1)
    got = np.concatenate([pre, dec], axis=1)
    dl = be.download_weights()
    np.testing.assert_array_equal(dl[-4 * 128 * 4:], w[-4 * 128 * 4:])   # f32 tail round-trips
    for i in range(2):
        ref = orc.run_sequence(orc.from_kg(cfg), orc.MODE_BASE, w, toks[i])[0]
        err = np.abs(got[i] - ref).max(axis=-1) / np.abs(ref).max(axis=-1)
        assert err.max() <= 2e-2, err.max()
    be.close()
