"""The allocation-free encoder entry point (kg_tq_encode_noalloc).

Some callers cannot allocate device memory at the point where they encode
K/V vectors (a latency-critical or captured decode loop, where cudaMalloc
would synchronise the device, or a host that fixed the library's memory
budget up front). kg_tq_encode_noalloc serves them: it takes caller-owned
device buffers and keeps its scratch in a fixed device array. This test calls
it through the C ABI twice in a row and checks codes and norms bit for bit
against kg_tq_encode, the entry point that allocates staging memory itself.
This file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kvd,nh,bits", [(768, 12, 4), (16, 4, 3)])
def test_noalloc_encoder_matches_allocating_encoder(kg, kvd, nh, bits):
    import torch
    cfg = kg.micro_config(kv_mode=kg.KG_KV_TQ, n_embd=kvd, n_head=nh, head_dim=kvd // nh, n_kv_head=nh,
                          key_bits=bits, val_bits=bits, mlp_hidden=4 * kvd, vocab_size=64)
    be = kg.CudaBackend(cfg)
    lib = kg.lib()
    pl = lib.kg_tq_packed_len(kvd, bits)
    rng = np.random.default_rng(kvd)
    for call in range(2):                      # two calls in a row share the scratch array
        n = 96 if call == 0 else 40
        x = rng.standard_normal((n, kvd)).astype(np.float32)
        x[3] = 0.0                             # zero vector: its codes stay as found
        init = np.full((n, pl), 0x3C, np.uint8)
        ref_packed, ref_norms = be.tq_encode(x, which=call % 2, packed_init=init)
        dx = torch.from_numpy(x).cuda()
        dp = torch.from_numpy(init).cuda()
        dn = torch.empty(n, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        rc = lib.kg_tq_encode_noalloc(be._h, call % 2, n, ctypes.c_void_p(dx.data_ptr()),
                                      ctypes.c_void_p(dp.data_ptr()), ctypes.c_void_p(dn.data_ptr()), None)
        assert rc == 0, lib.kg_last_error(be._h)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dp.cpu().numpy(), ref_packed)
        np.testing.assert_array_equal(dn.cpu().numpy(), ref_norms)
    be.close()


def test_noalloc_rejects_oversized_batches(kg):
    import torch
    cfg = kg.micro_config(kv_mode=kg.KG_KV_TQ, n_embd=768, n_head=12, head_dim=64, n_kv_head=12,
                          key_bits=4, val_bits=4, mlp_hidden=3072, vocab_size=64)
    be = kg.CudaBackend(cfg)
    lib = kg.lib()
    n = (1 << 20) // 768 + 1                   # one vector beyond the fixed scratch
    dx = torch.zeros((n, 768), dtype=torch.float32, device="cuda")
    dp = torch.zeros((n, 384), dtype=torch.uint8, device="cuda")
    dn = torch.zeros(n, dtype=torch.float32, device="cuda")
    rc = lib.kg_tq_encode_noalloc(be._h, 0, n, ctypes.c_void_p(dx.data_ptr()), ctypes.c_void_p(dp.data_ptr()),
                                  ctypes.c_void_p(dn.data_ptr()), None)
    assert rc == -1 and b"exceeds" in lib.kg_last_error(be._h)
    be.close()
