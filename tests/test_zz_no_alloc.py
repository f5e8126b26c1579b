"""The allocation-free encoder entry point (kg_tq_encode_noalloc).

Some callers cannot allocate device memory at the point where they encode
K/V vectors (a latency-critical or captured decode loop, where cudaMalloc
would synchronise the device, or a host that fixed the library's memory
budget up front). kg_tq_encode_noalloc serves them: it takes caller-owned
device buffers and keeps its scratch in a fixed device array. These tests
call it through the C ABI twice in a row and check codes and norms bit for
bit against an independent encoder: kg_tq_encode (the entry point that
allocates staging memory itself, and at these kv_dims takes a different
kernel) or, at kv_dim 16, the CPU oracle. This file is named to be collected
last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_FLOATS = 1 << 20  # the fixed scratch: n_vec * kv_dim floats


def _ctx(kg, kvd, nh, bits, device=0):
    cfg = kg.micro_config(kv_mode=kg.KG_KV_TQ, n_embd=kvd, n_head=nh, head_dim=kvd // nh, n_kv_head=nh,
                          key_bits=bits, val_bits=bits, mlp_hidden=4 * kvd, vocab_size=64)
    return kg.CudaBackend(cfg, device=device)


def _noalloc(kg, be, which, x, init, device="cuda"):
    import torch
    lib = kg.lib()
    dx = torch.from_numpy(x).to(device)
    dp = torch.from_numpy(init).to(device)
    dn = torch.empty(x.shape[0], dtype=torch.float32, device=device)
    torch.cuda.synchronize(device)
    rc = lib.kg_tq_encode_noalloc(be._h, which, x.shape[0], ctypes.c_void_p(dx.data_ptr()),
                                  ctypes.c_void_p(dp.data_ptr()), ctypes.c_void_p(dn.data_ptr()), None)
    assert rc == 0, lib.kg_last_error(be._h)
    torch.cuda.synchronize(device)
    return dp.cpu().numpy(), dn.cpu().numpy()


@pytest.mark.parametrize("kvd,nh,bits", [(768, 12, 4), (192, 3, 3), (64, 1, 4)])
def test_noalloc_encoder_matches_allocating_encoder(kg, kvd, nh, bits):
    # kv_dim 768: tiled exact encoder (noalloc) vs tensor-core encoder with exact
    # fix-up (kg_tq_encode); 192 and 64 (multiples of 64, not of 128): the
    # per-vector warp encoder vs the tensor-core encoder
    be = _ctx(kg, kvd, nh, bits)
    pl = kg.lib().kg_tq_packed_len(kvd, bits)
    rng = np.random.default_rng(kvd)
    for call in range(2):                      # two calls in a row share the scratch array
        n = 96 if call == 0 else 40
        x = rng.standard_normal((n, kvd)).astype(np.float32)
        x[3] = 0.0                             # zero vector: its codes stay as found
        init = np.full((n, pl), 0x3C, np.uint8)
        ref_packed, ref_norms = be.tq_encode(x, which=call % 2, packed_init=init)
        got_packed, got_norms = _noalloc(kg, be, call % 2, x, init)
        np.testing.assert_array_equal(got_packed, ref_packed)
        np.testing.assert_array_equal(got_norms, ref_norms)
    be.close()


def test_noalloc_encoder_matches_oracle_small_dim(kg, orc):
    # kv_dim 16 (the micro model): kg_tq_encode and the noalloc entry point take
    # the same kernel there, so compare with the CPU oracle's store_key instead
    be = _ctx(kg, 16, 4, 3)
    rot, kc, kb, vc, vb = be.tq_tables()
    rng = np.random.default_rng(16)
    for call in range(2):
        n = 50 if call == 0 else 33
        x = rng.standard_normal((n, 16)).astype(np.float32)
        x[5] = 0.0
        init = np.full((n, 8), 0x5A, np.uint8)
        got_packed, got_norms = _noalloc(kg, be, call % 2, x, init)
        bnd = kb if call % 2 == 0 else vb
        for v in range(n):
            pk, nr = orc.tq_store(rot, bnd, 3, x[v], packed_init=init[v])
            np.testing.assert_array_equal(got_packed[v], pk)
            assert got_norms[v] == np.float32(nr)
    be.close()


def test_noalloc_largest_accepted_call(kg):
    # n_vec * kv_dim exactly at the limit (1365 vectors at kv_dim 768), then a
    # second, smaller call: both bit-identical to kg_tq_encode
    be = _ctx(kg, 768, 12, 4)
    n = MAX_FLOATS // 768
    rng = np.random.default_rng(1365)
    for which, cnt in ((0, n), (1, 7)):
        x = rng.standard_normal((cnt, 768)).astype(np.float32)
        init = np.zeros((cnt, 384), np.uint8)
        ref_packed, ref_norms = be.tq_encode(x, which=which, packed_init=init)
        got_packed, got_norms = _noalloc(kg, be, which, x, init)
        np.testing.assert_array_equal(got_packed, ref_packed)
        np.testing.assert_array_equal(got_norms, ref_norms)
    be.close()


def test_noalloc_rejects_oversized_batches(kg):
    import torch
    be = _ctx(kg, 768, 12, 4)
    lib = kg.lib()
    n = MAX_FLOATS // 768 + 1                  # one vector beyond the fixed scratch
    dx = torch.zeros((n, 768), dtype=torch.float32, device="cuda")
    dp = torch.zeros((n, 384), dtype=torch.uint8, device="cuda")
    dn = torch.zeros(n, dtype=torch.float32, device="cuda")
    rc = lib.kg_tq_encode_noalloc(be._h, 0, n, ctypes.c_void_p(dx.data_ptr()), ctypes.c_void_p(dp.data_ptr()),
                                  ctypes.c_void_p(dn.data_ptr()), None)
    assert rc == -1 and b"exceeds" in lib.kg_last_error(be._h)
    # a count so large that n_vec * kv_dim overflows 64 bits is rejected, not wrapped
    rc = lib.kg_tq_encode_noalloc(be._h, 0, 1 << 62, ctypes.c_void_p(dx.data_ptr()),
                                  ctypes.c_void_p(dp.data_ptr()), ctypes.c_void_p(dn.data_ptr()), None)
    assert rc == -1
    be.close()


def test_noalloc_on_two_devices_in_one_process(kg):
    # one process, one context per GPU: each device gets its own scratch
    # address and its own kernel attributes
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    bes = [_ctx(kg, 768, 12, 4, device=d) for d in (0, 1)]
    rng = np.random.default_rng(2)
    x = rng.standard_normal((64, 768)).astype(np.float32)
    init = np.zeros((64, 384), np.uint8)
    outs = [_noalloc(kg, be, 0, x, init, device=f"cuda:{d}") for d, be in enumerate(bes)]
    ref_packed, ref_norms = bes[0].tq_encode(x, which=0, packed_init=init)
    for got_packed, got_norms in outs:
        np.testing.assert_array_equal(got_packed, ref_packed)
        np.testing.assert_array_equal(got_norms, ref_norms)
    for be in bes:
        be.close()
