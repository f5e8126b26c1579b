"""forward_prefill (src/transformer.rs:2606-3004) on the device vs the oracle.

The reference's prefill variant normalises twice per layer without gammas,
lets every prompt position attend the whole prompt (bidirectional) and shares
one block-delta accumulator across the prompt's positions; decoding then
continues with forward_base from position T (generate_with_prefill,
:3010-3106). Bars: the exact-order micro path bit-identical
(assert_array_equal) for the prefill logits and every continuation step; the
bf16 path within 2e-2 relative (max |d| / max |ref| per position).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_BF16 = 2e-2


def rel_err(a, b):
    den = np.maximum(np.abs(b).max(axis=-1), 1e-30)
    return np.abs(a - b).max(axis=-1) / den


def _run(be, toks, P):
    n, T = toks.shape
    pre = be.forward_prefill(toks[:, :P])
    dec = [be.forward_batch(toks[:, t:t + 1], start_pos=np.full(n, t))[:, 0] for t in range(P, T)]
    return np.concatenate([pre[:, None], np.stack(dec, axis=1)], axis=1)


@pytest.mark.parametrize("L,P", [(1, 10), (8, 12), (8, 1)])
def test_micro_prefill_then_decode_bit_identical(kg, orc, L, P):
    # 8 layers = two routing blocks: the shared block deltas reach layer 3's and
    # layer 7's depth routing; P = 1 is the one-position prompt
    n, T = 3, 16
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, max_seqs=n, n_layer=L)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 11 + L)
    be.compile(w)
    toks = np.random.default_rng(40 + P).integers(0, 27, size=(n, T)).astype(np.int32)
    got = _run(be, toks, P)
    for i in range(n):
        ref = orc.prefill_then_decode(orc.from_kg(cfg), w, toks[i, :P], toks[i, P:])
        np.testing.assert_array_equal(got[i], ref)
    be.close()


def test_micro_prefill_reuses_slots(kg, orc):
    # a second prefill into the same slots starts over from position 0
    n, P, T = 2, 9, 14
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, max_seqs=n, n_layer=4)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 5)
    be.compile(w)
    rng = np.random.default_rng(9)
    for _ in range(2):
        toks = rng.integers(0, 27, size=(n, T)).astype(np.int32)
        got = _run(be, toks, P)
        for i in range(n):
            np.testing.assert_array_equal(got[i], orc.prefill_then_decode(orc.from_kg(cfg), w, toks[i, :P],
                                                                          toks[i, P:]))
    be.close()


def test_bf16_prefill_then_decode(kg, orc):
    # C3 widths (n_embd 768, 12 heads of 64, mlp 3072), 8 layers (two routing
    # blocks), bf16 weights and K/V cache: 2 sequences, a 128-token prompt
    # (tcgen05 GEMMs, bidirectional flash attention) then 8 decode steps
    n, P, T = 2, 128, 136
    cfg = kg.micro_config(vocab_size=512, block_size=160, n_embd=768, n_head=12, head_dim=64, n_kv_head=12,
                          mlp_hidden=3072, n_layer=8, kv_mode=kg.KG_KV_F32, weight_dtype=kg.KG_W_BF16, max_seqs=n)
    be = kg.CudaBackend(cfg)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=31, scale_mode=1, std=0.02))
    be.compile(w)
    toks = np.random.default_rng(77).integers(0, 512, size=(n, T)).astype(np.int32)
    got = _run(be, toks, P)
    for i in range(n):
        ref = orc.prefill_then_decode(orc.from_kg(cfg), w, toks[i, :P], toks[i, P:])
        err = rel_err(got[i], ref)
        print("bf16 prefill seq %d: rel err prefill %.2e, decode max %.2e" % (i, err[0], err[1:].max()))
        assert err.max() <= REL_BF16
    be.close()


def test_prefill_rejects_quantized_cache(kg):
    cfg = kg.micro_config(kv_mode=kg.KG_KV_TQ, max_seqs=1)
    be = kg.CudaBackend(cfg)
    be.compile(kg.reference_weights(cfg, 1))
    with pytest.raises(kg.KgError):
        be.forward_prefill(np.zeros((1, 4), np.int32))
    be.close()
