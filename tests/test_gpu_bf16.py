"""GPU parity of the BF16 tensor-core path (full-size model shapes).

The oracle runs the reference forward in f32 on the same bf16-rounded
weights; the device computes GEMMs with bf16 inputs and f32 accumulation and
attention in the TurboQuant rotated domain. Bar: logits within
2e-2 relative, measured per position as max|gpu - ref| / max|ref|.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_BF16 = 2e-2


def rel_err(a, b):
    den = np.maximum(np.abs(b).max(axis=-1), 1e-30)
    return np.abs(a - b).max(axis=-1) / den


def make(kg, mode=1, std=0.05, **shape):
    base = dict(vocab_size=96, block_size=64, n_embd=128, n_head=2, head_dim=64, n_kv_head=2,
                mlp_hidden=256, n_layer=4, key_bits=4, val_bits=4, kv_mode=mode,
                weight_dtype=kg.KG_W_BF16, max_seqs=4)
    base.update(shape)
    cfg = kg.micro_config(**base)
    be = kg.CudaBackend(cfg)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=11, scale_mode=1, std=std))
    be.compile(w)
    return cfg, be, w


def tokens(n_seq, T, V, seed=0):
    return np.random.default_rng(seed).integers(0, V, size=(n_seq, T)).astype(np.int32)


@pytest.mark.parametrize("mode", [1, 2])
def test_prefill_then_decode_matches_oracle(kg, orc, mode):
    cfg, be, w = make(kg, mode)
    n_seq, T0, T1 = 3, 32, 12
    toks = tokens(n_seq, T0 + T1, cfg.vocab_size, seed=mode)
    pre = be.forward_batch(toks[:, :T0])
    dec = [be.forward_batch(toks[:, t:t + 1], start_pos=np.full(n_seq, t))[:, 0] for t in range(T0, T0 + T1)]
    got = np.concatenate([pre, np.stack(dec, axis=1)], axis=1)
    for i in range(n_seq):
        ref = orc.run_sequence(orc.from_kg(cfg), mode, w, toks[i], key_bits=4, val_bits=4)[0]
        err = rel_err(got[i], ref)
        assert err.max() <= REL_BF16, (i, err.max(), np.argmax(err))
    be.close()


def test_decode_from_scratch_matches_prefill(kg):
    cfg, be, w = make(kg, 1)
    toks = tokens(2, 24, cfg.vocab_size, seed=5)
    pre = be.forward_batch(toks)
    be.reset()
    dec = np.stack([be.forward_batch(toks[:, t:t + 1], start_pos=np.full(2, t))[:, 0] for t in range(24)], axis=1)
    assert rel_err(dec, pre).max() <= REL_BF16
    be.close()


def test_c3_width_matches_oracle(kg, orc):
    # the C3 widths (n_embd 768, 12 heads of 64, 4-bit KV) at 2 layers
    cfg, be, w = make(kg, 1, vocab_size=512, block_size=128, n_embd=768, n_head=12, head_dim=64,
                      n_kv_head=12, mlp_hidden=3072, n_layer=2, max_seqs=2)
    toks = tokens(2, 72, cfg.vocab_size, seed=9)
    pre = be.forward_batch(toks[:, :64])
    dec = np.stack([be.forward_batch(toks[:, t:t + 1], start_pos=np.full(2, t))[:, 0] for t in range(64, 72)], axis=1)
    got = np.concatenate([pre, dec], axis=1)
    for i in range(2):
        ref = orc.run_sequence(orc.from_kg(cfg), 1, w, toks[i], key_bits=4, val_bits=4)[0]
        assert rel_err(got[i], ref).max() <= REL_BF16
    be.close()


def test_probs_and_download(kg):
    cfg, be, w = make(kg, 1)
    toks = tokens(2, 8, cfg.vocab_size, seed=3)
    lo, pr = be.forward_batch(toks, probs=True)
    z = (lo - lo.max(axis=-1, keepdims=True)) / cfg.temperature
    ref = np.exp(z) / np.exp(z).sum(axis=-1, keepdims=True)
    assert np.abs(pr - ref).max() < 1e-4
    np.testing.assert_array_equal(be.download_weights(), w)
    be.close()


def test_random_weights_and_codes_readback(kg):
    cfg = kg.micro_config(vocab_size=96, block_size=64, n_embd=128, n_head=2, head_dim=64, n_kv_head=2,
                          mlp_hidden=256, n_layer=2, key_bits=4, val_bits=4, kv_mode=1,
                          weight_dtype=kg.KG_W_BF16, max_seqs=2)
    be = kg.CudaBackend(cfg)
    be.random_weights(seed=1, std=0.02)
    w = be.download_weights()
    assert abs(float(w[:10000].std()) - 0.02) < 0.002
    out = be.forward_batch(tokens(2, 16, 96))
    assert np.isfinite(out).all()
    kp, vp, nr = be.kv_codes(1, 1, 15)
    assert kp.size == 64 and vp.size == 64 and np.all(nr > 0)
    be.close()


def test_c3_width_long_context(kg, orc):
    # two 160-token prompts (320 prefill rows: the tcgen05 GEMM path) then
    # decode steps up to position 199 at C3 widths: several score tiles and
    # multi-step attention chunks per token
    cfg, be, w = make(kg, 1, vocab_size=512, block_size=256, n_embd=768, n_head=12, head_dim=64,
                      n_kv_head=12, mlp_hidden=3072, n_layer=1, max_seqs=2)
    toks = tokens(2, 200, cfg.vocab_size, seed=21)
    pre = be.forward_batch(toks[:, :160])
    dec = np.stack([be.forward_batch(toks[:, t:t + 1], start_pos=np.full(2, t))[:, 0] for t in range(160, 200)],
                   axis=1)
    got = np.concatenate([pre, dec], axis=1)
    for i in range(2):
        ref = orc.run_sequence(orc.from_kg(cfg), 1, w, toks[i], key_bits=4, val_bits=4)[0]
        err = rel_err(got[i], ref)
        print("seq %d max rel err prefill %.2e decode %.2e" % (i, err[:160].max(), err[160:].max()))
        assert err.max() <= REL_BF16
    be.close()


def test_decode_graph_replay_matches_eager(kg):
    # the decode step replays as a CUDA graph from its third call on; with
    # phase profiling on every step runs eagerly: both must agree bitwise
    cfg, be, w = make(kg, 1)
    cfg2, be2, _ = make(kg, 1)
    be2.profile(True)
    toks = tokens(3, 20, cfg.vocab_size, seed=8)
    a = be.forward_batch(toks[:, :8])
    b = be2.forward_batch(toks[:, :8])
    np.testing.assert_array_equal(a, b)
    kernels = []
    for t in range(8, 20):
        x = be.forward_batch(toks[:, t:t + 1], start_pos=np.full(3, t))
        kernels.append(be.graph_kernels())
        y = be2.forward_batch(toks[:, t:t + 1], start_pos=np.full(3, t))
        np.testing.assert_array_equal(x, y)
    assert kernels[0] == 0 and kernels[1] > 0 and all(k == kernels[1] for k in kernels[1:])
    be2.profile(False)
    be.close()
    be2.close()


@pytest.mark.parametrize("shape", [
    dict(),                                                                   # 2 heads of 64
    dict(n_embd=256, n_head=4, head_dim=64, n_kv_head=2, mlp_hidden=512),    # grouped-query attention
    dict(vocab_size=256, n_embd=2048, n_head=16, head_dim=128, n_kv_head=16, mlp_hidden=8192, n_layer=1),  # C4 widths
])
def test_standard_attention_matches_oracle(kg, orc, shape):
    # AttentionMode::Standard on the bf16 path: bf16 K/V cache, forward_base semantics
    cfg, be, w = make(kg, 0, **shape)
    n_seq, T0, T1 = 2, 24, 8
    toks = tokens(n_seq, T0 + T1, cfg.vocab_size, seed=17)
    pre = be.forward_batch(toks[:, :T0])
    dec = [be.forward_batch(toks[:, t:t + 1], start_pos=np.full(n_seq, t))[:, 0] for t in range(T0, T0 + T1)]
    got = np.concatenate([pre, np.stack(dec, axis=1)], axis=1)
    for i in range(n_seq):
        ref = orc.run_sequence(orc.from_kg(cfg), orc.MODE_BASE, w, toks[i])[0]
        err = rel_err(got[i], ref)
        print("standard %s seq %d: max rel err prefill %.2e decode %.2e" % (shape.get("n_embd", 128), i,
                                                                          err[:T0].max(), err[T0:].max()))
        assert err.max() <= REL_BF16
    be.close()


@pytest.mark.parametrize("shape", [
    dict(n_embd=192, n_head=3, head_dim=64, n_kv_head=3, mlp_hidden=384),      # kv_dim 192: 64-dim value blocks
    dict(n_embd=1024, n_head=16, head_dim=64, n_kv_head=16, mlp_hidden=1024),  # four warps per score unit
    dict(n_embd=1280, n_head=20, head_dim=64, n_kv_head=20, mlp_hidden=1024),  # > 16 heads: streaming scores
    dict(n_embd=768, n_head=12, head_dim=64, n_kv_head=12, mlp_hidden=768, key_bits=3, val_bits=3),  # 3-bit
    dict(n_embd=2048, n_head=16, head_dim=128, n_kv_head=16, mlp_hidden=1024),  # tcgen05 attention, 16-head tile
    dict(n_embd=2048, n_head=16, head_dim=128, n_kv_head=16, mlp_hidden=1024, key_bits=3, val_bits=3),  # and 3-bit
])
def test_quantized_attention_shapes(kg, orc, shape):
    # the decode attention kernels' shape variants against forward_quantized;
    # 70 positions so a token spans three 32-position units. Weights N(0, 0.02):
    # the device's f32 rounding differs from the reference's in the last bits,
    # so a coordinate lying on a codebook boundary can take the neighbouring
    # code (the encoder itself is bit-exact on equal inputs); wider weights
    # make one such flip move the logits by up to a few percent
    shape = dict(shape)
    kb, vb = shape.pop("key_bits", 4), shape.pop("val_bits", 4)
    cfg, be, w = make(kg, 1, std=0.02, vocab_size=128, block_size=96, n_layer=2, key_bits=kb, val_bits=vb, **shape)
    n_seq, T0, T1 = 2, 60, 10
    toks = tokens(n_seq, T0 + T1, cfg.vocab_size, seed=23)
    pre = be.forward_batch(toks[:, :T0])
    dec = [be.forward_batch(toks[:, t:t + 1], start_pos=np.full(n_seq, t))[:, 0] for t in range(T0, T0 + T1)]
    got = np.concatenate([pre, np.stack(dec, axis=1)], axis=1)
    for i in range(n_seq):
        ref = orc.run_sequence(orc.from_kg(cfg), 1, w, toks[i], key_bits=kb, val_bits=vb)[0]
        err = rel_err(got[i], ref)
        print("quantized %d/%d heads seq %d: max rel err prefill %.2e decode %.2e" % (
            cfg.n_head, cfg.n_embd, i, err[:T0].max(), err[T0:].max()))
        assert err.max() <= REL_BF16
    be.close()


@pytest.mark.parametrize("max_seqs", [16, 2])
def test_multi_position_call_from_nonzero_position(kg, orc, max_seqs):
    # prefill 64, then one 6-token call from position 64 (chunked prefill /
    # batched verification, forward_batched semantics): matches the oracle's
    # 70 sequential positions and 70 single-token calls; max_seqs 2 forces one
    # pass per position offset (2 x 6 rows > 2 decode rows)
    cfg, be, w = make(kg, 1, std=0.02, vocab_size=128, block_size=96, n_embd=256, n_head=4, head_dim=64,
                      n_kv_head=4, mlp_hidden=512, n_layer=2, max_seqs=max_seqs)
    cfg2, be2, _ = make(kg, 1, std=0.02, vocab_size=128, block_size=96, n_embd=256, n_head=4, head_dim=64,
                        n_kv_head=4, mlp_hidden=512, n_layer=2, max_seqs=max_seqs)
    toks = tokens(2, 70, cfg.vocab_size, seed=31)
    pre = be.forward_batch(toks[:, :64])
    chunk = be.forward_batch(toks[:, 64:70], start_pos=np.full(2, 64))
    got = np.concatenate([pre, chunk], axis=1)
    singles = np.stack([be2.forward_batch(toks[:, t:t + 1], start_pos=np.full(2, t))[:, 0] for t in range(70)], axis=1)
    for i in range(2):
        ref = orc.run_sequence(orc.from_kg(cfg), 1, w, toks[i], key_bits=4, val_bits=4)[0]
        assert rel_err(got[i], ref).max() <= REL_BF16
        assert rel_err(chunk[i], singles[i, 64:]).max() <= 1e-3
        # the chunk's codes equal the sequential calls' codes except near codebook boundaries
        kp, vp, _ = be.kv_codes(i, 1, 67)
        kp2, vp2, _ = be2.kv_codes(i, 1, 67)
        assert (kp != kp2).mean() < 0.02 and (vp != vp2).mean() < 0.02
    be.close()
    be2.close()
