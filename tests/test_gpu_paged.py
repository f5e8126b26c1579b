"""forward_paged over a device PagedKVCache (kv_mode KG_KV_PAGED) against the
oracle (src/transformer.rs:3305-3504, crates/katgpt-transformer/src/
kv_cache.rs:187-420).

The allocator state (page lists, reference counts, total and free pages) must
equal the oracle's restatement after every call, and logits and the K/V rows
read back from the pages must be bit-identical, through forks that share
whole pages, forks inside a page (whose fresh pages read as zeros), rollbacks
that free exclusive pages and reuse them zeroed, and multi-sequence calls."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ctx(kg, block=64, L=4, S=8):
    cfg = kg.micro_config(kv_mode=kg.KG_KV_PAGED, block_size=block, n_layer=L, max_seqs=S)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    return cfg, be, w


def _same_state(be, ref):
    tot, free, ns, refs = be.paged_stats()
    assert (tot, free, ns) == (ref.total_pages, len(ref.free_pages), len(ref.layer_page_tables[0]))
    assert refs == ref.page_ref_counts[:tot]
    for l, lt in enumerate(ref.layer_page_tables):
        for s in range(ns):
            assert be.paged_table(l, s) == lt[s], (l, s)


def test_paged_reference_call_sequences(kg, orc):
    # the reference's own PagedKVCache test sequences (Config::micro(),
    # src/transformer.rs:4691-4711, 5035-5190), applied to both sides
    cfg, be, _ = _ctx(kg, block=16, L=1, S=8)          # forks append past the 4 initial sequences
    ocfg = orc.from_kg(cfg)
    ref = orc.PagedKVCache(ocfg, 4)
    be.paged_init(4)
    _same_state(be, ref)
    for op in [("e", 0, 31), ("f", 0, 16), ("e", 0, 47), ("r", 0, 16), ("f", 0, 0), ("e", 0, 63),
               ("r", 0, 32), ("e", 1, 31), ("r", 1, 0), ("z",), ("e", 0, 0), ("e", 2, 20)]:
        if op[0] == "e":
            ref.ensure_pages(op[1], op[2]); be.paged_ensure(op[1], op[2])
        elif op[0] == "f":
            assert be.paged_fork(op[1], op[2]) == ref.fork(op[1], op[2])
        elif op[0] == "r":
            ref.rollback(op[1], op[2]); be.paged_rollback(op[1], op[2])
        else:
            ref.reset(); be.paged_reset()
        _same_state(be, ref)
    be.close()


def test_paged_random_operations_match_oracle(kg, orc):
    cfg, be, _ = _ctx(kg, block=64, L=4, S=8)
    ref = orc.PagedKVCache(orc.from_kg(cfg), 1)
    rng = np.random.default_rng(11)
    for _ in range(300):
        ns = len(ref.layer_page_tables[0])
        r = rng.random()
        if r < 0.45:
            seq, pos = int(rng.integers(0, min(ns + 1, 8))), int(rng.integers(0, 64))
            ref.ensure_pages(seq, pos); be.paged_ensure(seq, pos)
        elif r < 0.65 and ns < 8:
            seq, pos = int(rng.integers(0, ns)), int(rng.integers(0, 64))
            assert be.paged_fork(seq, pos) == ref.fork(seq, pos)
        elif r < 0.97:
            seq, pos = int(rng.integers(0, ns + 1)), int(rng.integers(0, 64))
            ref.rollback(seq, pos); be.paged_rollback(seq, pos)
        else:
            ref.reset(); be.paged_reset()
        _same_state(be, ref)
    be.close()


def test_forward_paged_bit_identical_through_forks_and_rollbacks(kg, orc):
    cfg, be, w = _ctx(kg, block=64, L=4, S=8)
    ocfg = orc.from_kg(cfg)
    ref = orc.PagedKVCache(ocfg, 1)
    rng = np.random.default_rng(5)

    def step(seqs, starts, T):
        toks = rng.integers(0, 27, size=(len(seqs), T)).astype(np.int32)
        got = be.forward_batch(toks, seq_ids=np.array(seqs, np.int32), start_pos=np.array(starts, np.int32))
        for i, (s, p0) in enumerate(zip(seqs, starts)):  # batch order: sequence by sequence
            for t in range(T):
                want = orc.forward_paged(ocfg, w, ref, s, int(toks[i, t]), p0 + t)
                assert np.array_equal(got[i, t], want), (s, p0 + t)
        _same_state(be, ref)

    step([0], [0], 16)
    step([0], [16], 16)
    step([0], [32], 8)
    s1 = be.paged_fork(0, 32); assert s1 == ref.fork(0, 32)      # shares pages 0 and 1
    s2 = be.paged_fork(0, 20); assert s2 == ref.fork(0, 20)      # shares page 0; 16..19 read as zeros
    step([s1, s2], [32, 20], 8)
    be.paged_rollback(s1, 36); ref.rollback(s1, 36)              # frees page 2 of s1
    step([s1], [36], 4)                                          # a reused page, zeroed: 32..35 read as zeros
    step([0, s1, s2], [40, 40, 28], 12)
    s3 = be.paged_fork(s2, 32); assert s3 == ref.fork(s2, 32)
    step([s3, 0], [32, 52], 12)
    # every stored K/V row, read back from the device pages
    for l in range(cfg.n_layer):
        for s in range(len(ref.layer_page_tables[0])):
            for p in range(len(ref.layer_page_tables[l][s]) * 16):
                k, v = be.paged_read_kv(l, s, p)
                rk, rv = ref.read_kv(l, s, p)
                assert np.array_equal(k, rk) and np.array_equal(v, rv), (l, s, p)
    be.close()


def test_forward_paged_many_sequences(kg, orc):
    # Config::micro() widths at block_size 16, 96 sequences x 16 positions in
    # one call, then single-token steps after a rollback to position 8
    cfg, be, w = _ctx(kg, block=16, L=2, S=96)
    ocfg = orc.from_kg(cfg)
    ref = orc.PagedKVCache(ocfg, 1)
    rng = np.random.default_rng(3)
    toks = rng.integers(0, 27, size=(96, 16)).astype(np.int32)
    got = be.forward_batch(toks)
    for i in range(96):
        for t in range(16):
            assert np.array_equal(got[i, t], orc.forward_paged(ocfg, w, ref, i, int(toks[i, t]), t))
    _same_state(be, ref)
    for i in range(0, 96, 7):
        be.paged_rollback(i, 8); ref.rollback(i, 8)
    ids = np.arange(0, 96, 7, dtype=np.int32)
    nt = rng.integers(0, 27, size=ids.size).astype(np.int32)
    for i, s in enumerate(ids):
        got1 = be.forward(int(nt[i]), 9, seq=int(s))
        assert np.array_equal(got1, orc.forward_paged(ocfg, w, ref, int(s), int(nt[i]), 9))
    _same_state(be, ref)
    be.close()


def test_paged_write_read_and_errors(kg, orc):
    cfg, be, _ = _ctx(kg, block=16, L=1, S=2)
    be.paged_ensure(0, 0)
    k = np.arange(16, dtype=np.float32) * np.float32(0.1)
    v = np.arange(16, dtype=np.float32) * np.float32(0.2)
    be.paged_write_kv(0, 0, 0, k, v)
    ko, vo = be.paged_read_kv(0, 0, 0)
    assert np.array_equal(ko, k) and np.array_equal(vo, v)
    with pytest.raises(kg.KgError):
        be.paged_read_kv(0, 1, 0)            # no page for that sequence
    with pytest.raises(kg.KgError):
        be.paged_fork(5, 0)                  # no such sequence
    with pytest.raises(kg.KgError):
        be.paged_ensure(2, 0)                # beyond max_seqs
    with pytest.raises(kg.KgError):
        be.kv_snapshot(0, 0, None)           # paged contexts roll back through their page tables
    be.close()


def test_forward_paged_bf16_matches_oracle(kg, orc):
    # forward_paged at model widths on the tensor-core path: bf16 K/V rows in
    # pages of the pool, read through the page table by the standard-attention
    # decode kernel; the prompt through the prefill path, then multi-position
    # calls, decode steps (captured as a CUDA graph from the second call of a
    # shape), forks inside and on page boundaries, and a rollback. Logits within
    # 2e-2 of the oracle's f32 forward_paged on the same bf16-rounded weights
    # (max |gpu - ref| / max |ref| per position); page bookkeeping identical.
    cfg = kg.micro_config(vocab_size=96, block_size=64, n_embd=256, n_head=4, head_dim=64, n_kv_head=4,
                          mlp_hidden=512, n_layer=4, kv_mode=kg.KG_KV_PAGED, weight_dtype=kg.KG_W_BF16, max_seqs=8)
    be = kg.CudaBackend(cfg)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=11, scale_mode=1, std=0.02))
    be.compile(w)
    ocfg = orc.from_kg(cfg)
    ref = orc.PagedKVCache(ocfg, 1)
    rng = np.random.default_rng(8)

    def step(seqs, starts, T):
        toks = rng.integers(0, cfg.vocab_size, size=(len(seqs), T)).astype(np.int32)
        got = be.forward_batch(toks, seq_ids=np.array(seqs, np.int32), start_pos=np.array(starts, np.int32))
        for i, (s, p0) in enumerate(zip(seqs, starts)):
            for t in range(T):
                want = orc.forward_paged(ocfg, w, ref, s, int(toks[i, t]), p0 + t)
                err = np.abs(got[i, t] - want).max() / np.abs(want).max()
                assert err <= 2e-2, (s, p0 + t, err)
        _same_state(be, ref)

    step([0], [0], 24)                                           # prompt: the prefill path
    step([0], [24], 8)                                           # 8 positions from 24
    for t in range(32, 35):
        step([0], [t], 1)                                        # decode steps
    s1 = be.paged_fork(0, 32); assert s1 == ref.fork(0, 32)
    s2 = be.paged_fork(0, 20); assert s2 == ref.fork(0, 20)      # 16..19 read as zeros
    for d in range(3):
        step([s1, s2], [32 + d, 20 + d], 1)
    be.paged_rollback(s1, 20); ref.rollback(s1, 20)              # page 1 of s1 freed, reused zeroed
    step([s1], [20], 6)
    step([0, s1, s2], [35, 26, 23], 4)
    k, v = be.paged_read_kv(2, 0, 30)                            # bf16 rows, widened
    rk, rv = ref.read_kv(2, 0, 30)
    assert np.abs(k - rk).max() <= 1e-2 * np.abs(rk).max() and np.abs(v - rv).max() <= 1e-2 * np.abs(rv).max()
    be.close()
