"""The bounded-wait path of the pipelined kernels, made to fire on purpose.

Every mbarrier wait in the tcgen05 GEMM and attention kernels has a clock
limit; when it runs out the kernel writes KG_ERR_TIMEOUT to the context's
error word and returns instead of hanging. kg_selftest_wait_timeout runs one
such wait on a barrier that nothing arrives on (about a millisecond); the
call must report the timeout and the context must keep working."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(kg, orc):
    cfg = kg.micro_config(kv_mode=kg.KG_KV_F32, max_seqs=4)
    be = kg.CudaBackend(cfg)
    w = kg.reference_weights(cfg, 42)
    be.compile(w)
    lib = kg.lib()
    for _ in range(2):
        assert lib.kg_selftest_wait_timeout(be._h, 2_000_000) == -4   # KG_ERR_TIMEOUT
        assert b"exceeded" in lib.kg_last_error(be._h)
    assert lib.kg_selftest_wait_timeout(be._h, 0) == -1               # limit must be positive
    toks = np.random.default_rng(0).integers(1, 27, size=(4, 16)).astype(np.int32)
    toks[:, 0] = 26
    got = be.forward_batch(toks)                                      # the error word was cleared
    ref = orc.run_batch(orc.from_kg(cfg), orc.MODE_BASE, w, toks)
    assert np.array_equal(got, ref)
    be.close()
