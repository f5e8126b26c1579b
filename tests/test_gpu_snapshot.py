"""KV snapshot / restore (MultiLayerKVCache::snapshot / restore,
crates/katgpt-transformer/src/kv_cache.rs:89-122) and sequence slots.

Rolling back to position p and decoding again must equal a run that never
went past p: bitwise on the exact path, within f32 reassociation on the bf16
path (its GEMM tiling follows the number of rows in a call)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _roundtrip(kg, cfg, w, torch, exact):
    rng = np.random.default_rng(4)
    lo, hi = (1, cfg.vocab_size) if exact else (0, cfg.vocab_size)
    pre = rng.integers(lo, hi, size=(1, 8)).astype(np.int32)
    junk = rng.integers(lo, hi, size=12).astype(np.int32)
    good = rng.integers(lo, hi, size=12).astype(np.int32)
    p = 5
    a = kg.CudaBackend(cfg)
    a.compile(w)
    a.forward_batch(pre)
    snap = torch.empty(a.kv_snapshot_bytes(p), dtype=torch.uint8, device="cuda")
    a.kv_snapshot(0, p, snap.data_ptr())
    for t in range(8, 12):  # speculative positions that get rejected
        a.forward_batch(junk[t:t + 1][None], start_pos=np.array([t]))
    a.kv_restore(0, p, snap.data_ptr())
    x = np.stack([a.forward_batch(good[t:t + 1][None], start_pos=np.array([t]))[0, 0] for t in range(p, 12)])
    b = kg.CudaBackend(cfg)
    b.compile(w)
    b.forward_batch(pre[:, :p])
    y = np.stack([b.forward_batch(good[t:t + 1][None], start_pos=np.array([t]))[0, 0] for t in range(p, 12)])
    if exact:
        np.testing.assert_array_equal(x, y)
        for t in range(12):
            ka, va, na = a.kv_codes(0, 0, t)
            kb, vb, nb = b.kv_codes(0, 0, t)
            assert np.array_equal(ka, kb) and np.array_equal(va, vb) and np.array_equal(na, nb), t
    else:
        assert np.abs(x - y).max() <= 1e-5 * np.abs(y).max()
    a.close()
    b.close()


def test_snapshot_restore_exact_path(kg):
    torch = pytest.importorskip("torch")
    cfg = kg.micro_config(kv_mode=kg.KG_KV_TQ, max_seqs=2)
    w = kg.reference_weights(cfg, 42)
    _roundtrip(kg, cfg, w, torch, exact=True)


def test_snapshot_restore_bf16_path(kg):
    torch = pytest.importorskip("torch")
    cfg = kg.micro_config(vocab_size=96, block_size=64, n_embd=256, n_head=4, head_dim=64, n_kv_head=4,
                          mlp_hidden=512, n_layer=2, key_bits=4, val_bits=4, kv_mode=kg.KG_KV_TQ,
                          weight_dtype=kg.KG_W_BF16, max_seqs=2)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=11, scale_mode=1, std=0.05))
    _roundtrip(kg, cfg, w, torch, exact=False)


def test_snapshot_restore_standard_attention(kg):
    torch = pytest.importorskip("torch")
    cfg = kg.micro_config(vocab_size=96, block_size=64, n_embd=256, n_head=4, head_dim=64, n_kv_head=4,
                          mlp_hidden=512, n_layer=2, kv_mode=kg.KG_KV_F32, weight_dtype=kg.KG_W_BF16, max_seqs=2)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=11, scale_mode=1, std=0.05))
    _roundtrip(kg, cfg, w, torch, exact=False)


def test_seq_alloc_free(kg):
    cfg = kg.micro_config(kv_mode=kg.KG_KV_TQ, max_seqs=2)
    be = kg.CudaBackend(cfg)
    assert be.seq_alloc() == 0 and be.seq_alloc() == 1
    with pytest.raises(kg.KgError):
        be.seq_alloc()
    be.seq_free(0)
    assert be.seq_alloc() == 0
    be.close()
