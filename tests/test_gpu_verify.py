"""Speculative verification on the device (kg_verify).

speculative_step_rollback's loop (src/speculative/step.rs:150-222): one
multi-position forward scores a draft path, then the acceptance test
u <= min(p/q, 1), residual resampling on the first rejection and a bonus draw
when every draft is accepted, all with the sequence slot's Rng. On the exact
micro path the target probabilities are bit-identical to the oracle's, so the
emitted tokens and counts must equal the oracle's acceptance loop exactly.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _draft_probs(orc, rng, k, V, favour):
    q = np.stack([orc.softmax_scaled(rng.standard_normal(V).astype(np.float32) * 2.0, 1.0) for _ in range(k)])
    return q, np.array([int(np.argmax(q[i])) if favour else int(rng.integers(0, V)) for i in range(k)], np.int32)


@pytest.mark.parametrize("k", [1, 4])
def test_verify_matches_oracle_exact_path(kg, orc, k):
    n, V, P0 = 8, 27, 6
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, max_seqs=n)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    rng = np.random.default_rng(70 + k)
    prefix = rng.integers(1, 27, size=(n, P0 + 1)).astype(np.int32)
    prefix[:, 0] = 26
    be.forward_batch(prefix[:, :P0])
    qs, drafts = [], []
    for i in range(n):
        q, d = _draft_probs(orc, rng, k, V, favour=(i % 2 == 0))
        if i % 2 == 0:   # make the target's favourite tokens the drafts for half the rows
            seq = np.concatenate([prefix[i], d[:-1]]) if k > 1 else prefix[i]
            lo = orc.run_sequence(orc.from_kg(cfg), orc.MODE_BASE, w, seq)[0][P0:]
            d = np.array([int(np.argmax(lo[j])) for j in range(k)], np.int32)
        qs.append(q)
        drafts.append(d)
    qs, drafts = np.stack(qs), np.stack(drafts)
    for i in range(n):
        be.rng_seed(i, 900 + i)
    acc, cnt = be.verify(prefix[:, P0], drafts, qs, start_pos=np.full(n, P0))
    seen = set()
    for i in range(n):
        seq = np.concatenate([prefix[i], drafts[i, :-1]])
        lo = orc.run_sequence(orc.from_kg(cfg), orc.MODE_BASE, w, seq)[0][P0:P0 + k]
        p = np.stack([orc.softmax_scaled(lo[j], 1.0 / cfg.temperature) for j in range(k)])
        ref, rc = orc.verify_path(p, qs[i], drafts[i], 900 + i)
        assert cnt[i] == rc, (i, cnt[i], rc)
        np.testing.assert_array_equal(acc[i, :rc], ref)
        seen.add(int(rc))
    assert len(seen) > 1 or k == 1          # both outcomes occur across the rows
    be.close()


def test_verify_bf16_path_runs(kg):
    cfg = kg.micro_config(vocab_size=128, block_size=64, n_embd=256, n_head=4, head_dim=64, n_kv_head=4,
                          mlp_hidden=512, n_layer=1, key_bits=4, val_bits=4, kv_mode=kg.KG_KV_TQ,
                          weight_dtype=kg.KG_W_BF16, max_seqs=4)
    be = kg.CudaBackend(cfg)
    be.random_weights(seed=3, std=0.02)
    rng = np.random.default_rng(1)
    toks = rng.integers(0, 128, size=(4, 20)).astype(np.int32)
    be.forward_batch(toks)
    q = rng.random((4, 5, 128)).astype(np.float32)
    q /= q.sum(axis=-1, keepdims=True)
    drafts = rng.integers(0, 128, size=(4, 5)).astype(np.int32)
    acc, cnt = be.verify(rng.integers(0, 128, size=4), drafts, q, start_pos=np.full(4, 20))
    assert ((cnt >= 1) & (cnt <= 6)).all()
    for i in range(4):
        assert ((acc[i, :cnt[i]] >= 0) & (acc[i, :cnt[i]] < 128)).all()
        np.testing.assert_array_equal(acc[i, :cnt[i] - 1], drafts[i, :cnt[i] - 1])   # accepted prefix is the drafts'
    be.close()
