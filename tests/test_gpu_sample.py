"""Device sampling: sample_token_into (crates/katgpt-types/src/math.rs:398-422)
with the reference Rng, one generator per sequence slot.

Bar: sampled ids equal the oracle's for identical probabilities and an
identical Rng stream (integer output: exact), over several successive draws
per slot (each draw advances the slot's generator).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_sampling_exact_path_probs(kg, orc):
    # probabilities from the exact micro path (bit-identical to the oracle's
    # softmax_scaled), five rounds of draws per slot
    n = 16
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, max_seqs=n)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    rng = np.random.default_rng(3)
    toks = rng.integers(1, 27, size=(n, 16)).astype(np.int32)
    toks[:, 0] = 26
    _, pr = be.forward_batch(toks, probs=True)
    seeds = [1000 + 7 * i for i in range(n)]
    for i, s in enumerate(seeds):
        be.rng_seed(i, s)
    got = np.stack([be.sample(pr[:, t]) for t in range(5)], axis=1)       # [slot][draw]
    for i, s in enumerate(seeds):
        ref = orc.sample_tokens(pr[i, :5], s)
        np.testing.assert_array_equal(got[i], ref)
    be.close()


def test_sampling_full_vocab_edge_rows(kg, orc):
    V, n = 32000, 8
    cfg = kg.micro_config(vocab_size=V, n_embd=64, n_head=1, head_dim=64, n_kv_head=1, mlp_hidden=64,
                          kv_mode=kg.KG_KV_F32, max_seqs=n)
    be = kg.CudaBackend(cfg)              # a context without a forward kernel: the sampler still works
    rng = np.random.default_rng(5)
    rounds = []
    for r in range(4):
        z = rng.standard_normal((n, V)).astype(np.float32) * (1.0 + r)
        p = np.stack([orc.softmax_scaled(z[i], 2.0) for i in range(n)])
        p[0] = 0.0
        p[0, 0] = 1.0                                   # all mass on the first id
        p[1] = 0.0
        p[1, V - 1] = 1.0                               # all mass on the last id
        p[2] = 1e-9                                     # CDF never reaches r: clamps to V - 1
        rounds.append(p)
    for i in range(n):
        be.rng_seed(i, 77 + i)
    got = np.stack([be.sample(p) for p in rounds], axis=1)
    for i in range(n):
        ref = orc.sample_tokens(np.stack([p[i] for p in rounds]), 77 + i)
        np.testing.assert_array_equal(got[i], ref)
    assert (got[0] == 0).all() and (got[1] == V - 1).all() and (got[2] == V - 1).all()
    be.close()
