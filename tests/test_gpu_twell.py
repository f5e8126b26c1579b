"""TwELL sparse MLP on the bf16 path with the benchmark sparsity hook.

With the hook, ~90% of each token's hidden activations are exactly zero, so
every row takes the TwELL branch (alive / m <= 1 - sparse_threshold,
src/transformer.rs:2080-2101). Calls with few rows recompute those rows as a
compressed-index gather over W2^T (math.rs:315-355); calls with many rows keep
the dense product. Both are the same sum in a different order: the logits of
a sequence must agree across the two, and the gather path must be
deterministic (ascending index packing)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cfg(kg, max_seqs):
    return kg.micro_config(vocab_size=96, block_size=64, n_embd=256, n_head=4, head_dim=64, n_kv_head=4,
                           mlp_hidden=1024, n_layer=2, kv_mode=kg.KG_KV_F32, weight_dtype=kg.KG_W_BF16,
                           max_seqs=max_seqs)


def test_gather_path_matches_dense_path(kg):
    cfg = _cfg(kg, 40)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=5, scale_mode=1, std=0.05))
    toks = np.random.default_rng(6).integers(0, cfg.vocab_size, size=(40, 12)).astype(np.int32)
    out = {}
    for rows in (2, 40):  # 2 rows per call: gather path; 40: dense path
        be = kg.CudaBackend(cfg)
        be.compile(w)
        be.set_mlp_hook(0.1, seed=123)
        be.forward_batch(toks[:rows, :4])  # prefill 4 positions (rows * 4 rows in that call)
        steps = [be.forward_batch(toks[:rows, t:t + 1], start_pos=np.full(rows, t))[:, 0] for t in range(4, 12)]
        out[rows] = np.stack(steps, axis=1)[:2]
        be.close()
    a, b = out[2], out[40]
    assert np.abs(a - b).max() <= 1e-4 * np.abs(b).max()


def test_gather_path_is_deterministic(kg):
    cfg = _cfg(kg, 2)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=5, scale_mode=1, std=0.05))
    toks = np.random.default_rng(7).integers(0, cfg.vocab_size, size=(2, 10)).astype(np.int32)
    res = []
    for _ in range(2):
        be = kg.CudaBackend(cfg)
        be.compile(w)
        be.set_mlp_hook(0.1, seed=9)
        be.forward_batch(toks[:, :6])
        res.append(np.stack([be.forward_batch(toks[:, t:t + 1], start_pos=np.full(2, t))[:, 0]
                             for t in range(6, 10)], axis=1))
        be.close()
    np.testing.assert_array_equal(res[0], res[1])
