"""The oracle's PagedKVCache and forward_paged against the reference's own
tests for them (src/transformer.rs:4573-4720, 4910-5195): the same calls and
the same assertions, on the CPU restatement. These pin the restatement that
the GPU paged tests compare the device with."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def micro(orc):
    cfg = orc.config()
    w = orc.weights(cfg, 42)
    return cfg, w


def test_write_read_roundtrip(orc, micro):  # :4575-4595
    cfg, _ = micro
    paged = orc.PagedKVCache(cfg, 1)
    paged.ensure_pages(0, 0)
    k = np.arange(16, dtype=np.float32) * np.float32(0.1)
    v = np.arange(16, dtype=np.float32) * np.float32(0.2)
    paged.write_kv(0, 0, 0, k, v)
    ko, vo = paged.read_kv(0, 0, 0)
    assert np.array_equal(ko, k) and np.array_equal(vo, v)


def test_fork_no_corruption(orc, micro):  # :4634-4660
    cfg, _ = micro
    paged = orc.PagedKVCache(cfg, 1)
    paged.ensure_pages(0, 0)
    k0 = np.arange(16, dtype=np.float32) + 1
    v0 = np.arange(16, dtype=np.float32) + 2
    paged.write_kv(0, 0, 0, k0, v0)
    f = paged.fork(0, 0)
    paged.ensure_pages(f, 0)
    paged.write_kv(0, f, 0, np.arange(16, dtype=np.float32) + 99, np.arange(16, dtype=np.float32) + 100)
    ko, vo = paged.read_kv(0, 0, 0)
    assert np.array_equal(ko, k0) and np.array_equal(vo, v0)


def test_fork_shares_prefix(orc, micro):  # :4663-4688
    cfg, _ = micro
    paged = orc.PagedKVCache(cfg, 1)
    paged.ensure_pages(0, 15)
    for pos in range(16):
        paged.write_kv(0, 0, pos, np.full(16, pos, np.float32), np.full(16, 2 * pos, np.float32))
    f = paged.fork(0, 8)
    paged.ensure_pages(f, 16)
    ko, _ = paged.read_kv(0, f, 0)
    assert ko[0] == 0.0
    # the fork point is inside page 0, so nothing is shared: the fork owns fresh (zeroed) pages
    assert paged.layer_page_tables[0][f][0] != paged.layer_page_tables[0][0][0]


def test_reset_frees_pages(orc, micro):  # :4691-4711
    cfg, _ = micro
    paged = orc.PagedKVCache(cfg, 2)
    paged.ensure_pages(0, 31)
    paged.ensure_pages(1, 15)
    before = paged.total_pages
    assert before > 0
    paged.reset()
    paged.ensure_pages(0, 0)
    assert paged.total_pages == before


def test_rollback_frees_exclusive_pages(orc, micro):  # :5035-5057
    cfg, _ = micro
    paged = orc.PagedKVCache(cfg, 2)
    paged.ensure_pages(0, 31)
    assert len(paged.layer_page_tables[0][0]) >= 2
    paged.rollback(0, 0)
    assert paged.layer_page_tables[0][0] == []
    assert paged.free_pages


def test_rollback_preserves_shared_pages(orc, micro):  # :5060-5102
    cfg, _ = micro
    paged = orc.PagedKVCache(cfg, 4)
    paged.ensure_pages(0, 31)
    s1 = paged.fork(0, 16)
    assert s1 != 0
    paged.ensure_pages(0, 47)
    free_before = len(paged.free_pages)
    before = len(paged.layer_page_tables[0][0])
    paged.rollback(0, 16)
    assert len(paged.layer_page_tables[0][0]) == 1
    freed = len(paged.free_pages) - free_before
    assert 0 < freed <= before - 1


def test_rollback_shared_page_not_freed(orc, micro):  # :5105-5136
    cfg, _ = micro
    paged = orc.PagedKVCache(cfg, 4)
    paged.ensure_pages(0, 31)
    s1 = paged.fork(0, 0)
    paged.ensure_pages(s1, 31)
    s2 = paged.fork(0, 16)
    shared = paged.layer_page_tables[0][0][0]
    paged.rollback(s2, 0)
    assert shared in paged.layer_page_tables[0][0]
    assert shared not in paged.free_pages


def test_rollback_truncates_page_table(orc, micro):  # :5139-5165
    cfg, _ = micro
    paged = orc.PagedKVCache(cfg, 1)
    paged.ensure_pages(0, 63)
    assert len(paged.layer_page_tables[0][0]) >= 4
    paged.rollback(0, 32)
    assert len(paged.layer_page_tables[0][0]) == 2
    paged.rollback(0, 16)
    assert len(paged.layer_page_tables[0][0]) == 1


def test_rollback_all_layers_consistent(orc):  # :5168-5190
    cfg = orc.config(n_layer=4)
    paged = orc.PagedKVCache(cfg, 1)
    paged.ensure_pages(0, 31)
    paged.rollback(0, 16)
    assert all(len(lt[0]) == 1 for lt in paged.layer_page_tables)


def test_forward_paged_matches_forward(orc, micro):  # :4913-4935, :4938-4978
    # forward (forward_base) normalises once, forward_paged twice: the
    # reference holds them within 1e-4 at position 0 and 1e-3 over positions 0..3
    cfg, w = micro
    paged = orc.PagedKVCache(cfg, 1)
    flat = orc.run_sequence(cfg, orc.MODE_BASE, w, np.arange(4, dtype=np.int32))[0]
    for pos in range(4):
        got = orc.forward_paged(cfg, w, paged, 0, pos, pos)
        assert np.all(np.isfinite(got)) and got.shape == (cfg.vocab_size,)
        assert np.abs(got - flat[pos]).max() < (1e-4 if pos == 0 else 1e-3)


def test_forward_paged_equals_flat_double_norm_path(orc, micro):
    # a linear sequence through pages gives the same logits however the
    # pages were handed out: two caches whose free lists differ
    cfg, w = micro
    a = orc.PagedKVCache(cfg, 1)
    b = orc.PagedKVCache(cfg, 3)
    b.ensure_pages(2, 0)                       # takes page indices first
    toks = [26, 3, 9, 14, 1, 7]
    for pos, t in enumerate(toks):
        la = orc.forward_paged(cfg, w, a, 0, t, pos)
        lb = orc.forward_paged(cfg, w, b, 0, t, pos)
        assert np.array_equal(la, lb)
    assert a.layer_page_tables[0][0] != b.layer_page_tables[0][0]


def _gqa_draft(orc):  # Config::gqa_draft() (crates/katgpt-types/src/config.rs:858-890)
    return orc.config(vocab_size=4096, block_size=256, n_embd=64, n_head=8, head_dim=8, n_kv_head=2,
                      mlp_hidden=256, n_layer=4, bos_token=0, temperature=0.8, sparse_threshold=0.8)


def test_gqa_forward_and_forward_paged(orc):  # src/transformer.rs:4469-4485, 4981-5006
    cfg = _gqa_draft(orc)
    assert cfg.n_kv_head * cfg.head_dim < cfg.n_embd                  # :4512-4540: the cache uses kv_dim
    w = orc.weights(cfg, 42)
    flat = orc.run_sequence(cfg, orc.MODE_BASE, w, np.zeros(4, np.int32))[0]
    assert flat.shape == (4, 4096) and np.all(np.isfinite(flat))
    paged = orc.PagedKVCache(cfg, 1)
    got = orc.forward_paged(cfg, w, paged, 0, 0, 0)
    assert np.abs(got - flat[0]).max() < 2e-3
