"""The LoraPair of generate_with_prefill on the exact micro path against the
oracle: the reader adapter in forward_prefill, the writer in the forward_base
decode steps (src/transformer.rs:1821-2200, 2606-3106; lora_apply,
crates/katgpt-types/src/lora.rs:452-467). Bar: bit-identical logits.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _adapter(rank, in_dim, out_dim, seed, scale=0.2):
    rng = np.random.default_rng(seed)
    return ((rng.standard_normal((rank, in_dim)) * scale).astype(np.float32),
            (rng.standard_normal((out_dim, rank)) * scale).astype(np.float32), 8.0)


def _prefill_then_decode(be, toks, P):
    n, T = toks.shape
    pre = be.forward_prefill(toks[:, :P])
    dec = [be.forward_batch(toks[:, t:t + 1], start_pos=np.full(n, t))[:, 0] for t in range(P, T)]
    return np.concatenate([pre[:, None], np.stack(dec, axis=1)], axis=1)


@pytest.mark.parametrize("reader,writer", [
    ((4, 16, 16), (4, 16, 16)),       # Config::micro_lora(): rank 4 over the full width
    ((16, 16, 16), (3, 12, 10)),      # the widest adapter; a partial one (chunked and scalar-tail dots)
])
def test_lora_pair_prefill_then_decode_bit_identical(kg, orc, reader, writer):
    n, P, T = 4, 7, 12
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, max_seqs=n, n_layer=4)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 21)
    be.compile(w)
    rd, wr = _adapter(*reader, seed=1), _adapter(*writer, seed=2)
    be.set_lora(0, *rd)
    be.set_lora(1, *wr)
    toks = np.random.default_rng(17).integers(0, 27, size=(n, T)).astype(np.int32)
    got = _prefill_then_decode(be, toks, P)
    ocfg = orc.from_kg(cfg)
    with orc.lora_pair(reader=rd, writer=wr):
        for i in range(n):
            np.testing.assert_array_equal(got[i], orc.prefill_then_decode(ocfg, w, toks[i, :P], toks[i, P:]))
    plain = [orc.prefill_then_decode(ocfg, w, toks[i, :P], toks[i, P:]) for i in range(n)]
    assert max(np.abs(got[i] - plain[i]).max() for i in range(n)) > 1e-3   # the adapters act
    be.close()


def test_lora_writer_in_forward_base_and_removal(kg, orc):
    n = 32
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, max_seqs=n, n_layer=2)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    toks = np.random.default_rng(5).integers(1, 27, size=(n, 16)).astype(np.int32)
    toks[:, 0] = 26
    wr = (np.full((4, 16), 0.1, np.float32), np.full((16, 4), 0.1, np.float32), 8.0)  # :6012-6030
    be.set_lora(1, *wr)
    got = be.forward_batch(toks)
    with orc.lora_pair(writer=wr):
        ref = orc.run_batch(orc.from_kg(cfg), orc.MODE_BASE, w, toks)
    np.testing.assert_array_equal(got, ref)
    be.set_lora(1)                                                                      # None again
    np.testing.assert_array_equal(be.forward_batch(toks), orc.run_batch(orc.from_kg(cfg), orc.MODE_BASE, w, toks))
    with pytest.raises(kg.KgError):
        be.set_lora(1, np.zeros((17, 16), np.float32), np.zeros((16, 17), np.float32), 8.0)  # rank > 16
    be.close()


def test_lora_writer_in_forward_sp_kv_quant(kg, orc):
    # forward_sp_kv_quant's adapter (src/sp_kv/forward.rs:610-822): layer-0
    # codes and norms bit-identical (they depend on no exp), logits within 1e-5
    # (the gated attention's libm expf), as the SP-KV tests without an adapter
    n = 16
    cfg = kg.micro_config(kv_mode=kg.KG_KV_SPKV_TQ, max_seqs=n, n_layer=2)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    wr = _adapter(4, 16, 16, seed=3)
    with pytest.raises(kg.KgError):
        be.set_lora(0, *wr)                       # no forward_prefill over SP-KV codes
    be.set_lora(1, *wr)
    toks = np.random.default_rng(8).integers(1, 27, size=(n, 16)).astype(np.int32)
    toks[:, 0] = 26
    got = be.forward_batch(toks)
    with orc.lora_pair(writer=wr):
        for i in range(n):
            ref, codes, norms, _ = orc.run_sequence(orc.from_kg(cfg), orc.MODE_SPKV, w, toks[i])
            assert np.abs(got[i] - ref).max() / np.abs(ref).max() <= 1e-5
            for t in range(16):
                kp, vp, nr = be.kv_codes(i, 0, t)
                assert np.array_equal(np.concatenate([kp, vp]), codes[0, t]) and np.array_equal(nr, norms[0, t])
    be.close()
