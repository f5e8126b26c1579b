"""Two devices driven from one process (one context per GPU).

Kernel attributes (dynamic shared-memory limits), SM counts and occupancy are
per-device properties; the library keeps them per device. This test runs
the bf16 path (tcgen05 prefill GEMMs, the rotated-domain decode attention,
the tiled encoder) on two GPUs from one process, interleaving the calls, and
requires bit-identical logits on both.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_two_contexts_two_devices_same_results(kg):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = kg.micro_config(vocab_size=256, block_size=192, n_embd=768, n_head=12, head_dim=64, n_kv_head=12,
                          mlp_hidden=1536, n_layer=2, key_bits=4, val_bits=4, kv_mode=kg.KG_KV_TQ,
                          weight_dtype=kg.KG_W_BF16, max_seqs=2)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=3, scale_mode=1, std=0.02))
    bes = [kg.CudaBackend(cfg, device=d) for d in (0, 1)]
    for be in bes:
        be.compile(w)
    toks = np.random.default_rng(4).integers(0, 256, size=(2, 170)).astype(np.int32)
    outs = [[], []]
    for d, be in enumerate(bes):
        outs[d].append(be.forward_batch(toks[:, :160]))   # 320 rows: tcgen05 GEMMs
    for t in range(160, 170):                             # decode steps, devices interleaved
        for d, be in enumerate(bes):
            outs[d].append(be.forward_batch(toks[:, t:t + 1], start_pos=np.full(2, t)))
    a, b = (np.concatenate(o, axis=1) for o in outs)
    assert np.isfinite(a).all()
    np.testing.assert_array_equal(a, b)
    for be in bes:
        be.close()
