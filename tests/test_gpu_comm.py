"""Sequence shards on two GPUs with the all-gather inside the library.

Two processes, one context per GPU, each decode their own half of the
sequences; kg_decode_gather_dev runs the step and the NCCL all-gather of the
logits and of the tokens sampled on the device. Checks: both ranks hold
bit-identical gathered logits and tokens, every gathered token is a valid id,
and the gathered logits match the oracle (forward_quantized in f32 on the same
bf16 weights) within 2e-2. (The sampler itself is checked draw for draw
against the oracle in test_gpu_sample.py.) Needs two GPUs; skipped otherwise.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_SEQ, PRE, STEPS = 4, 40, 6


def _cfg(kg):
    return kg.micro_config(vocab_size=128, block_size=64, n_embd=256, n_head=4, head_dim=64, n_kv_head=4,
                           mlp_hidden=512, n_layer=2, key_bits=4, val_bits=4, kv_mode=kg.KG_KV_TQ,
                           weight_dtype=kg.KG_W_BF16, max_seqs=N_SEQ // 2)


def _tokens():
    return np.random.default_rng(44).integers(0, 128, size=(N_SEQ, PRE + STEPS)).astype(np.int32)


def _rank(rank, world, q_in, q_out):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "katgpt-rs_b200"))
    try:
        import ctypes
        import torch
        import kgcuda as kg
        torch.cuda.set_device(rank)
        cfg = _cfg(kg)
        be = kg.CudaBackend(cfg, device=rank)
        w = kg.bf16_round(kg.reference_weights(cfg, seed=8, scale_mode=1, std=0.02))
        be.compile(w)
        uid = kg.comm_unique_id() if rank == 0 else None
        if rank == 0:
            for _ in range(world - 1):
                q_out.put(("uid", uid))
        else:
            uid = q_in.get(timeout=120)
        be.comm_init(uid, world, rank)
        n = N_SEQ // world
        toks = _tokens()[rank * n:(rank + 1) * n]
        be.forward_batch(toks[:, :PRE])
        for i in range(n):
            be.rng_seed(i, 500 + rank * n + i)
        dev = torch.device("cuda", rank)
        stream = torch.cuda.Stream(dev)
        sp = ctypes.c_void_p(stream.cuda_stream)
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        ids = torch.arange(n, dtype=torch.int32, device=dev)
        lo_all = torch.empty((STEPS, world, n, cfg.vocab_size), dtype=torch.float32, device=dev)
        tk_all = torch.empty((STEPS, world, n), dtype=torch.int32, device=dev)
        with torch.cuda.stream(stream):
            for t in range(STEPS):
                tok = torch.from_numpy(np.ascontiguousarray(toks[:, PRE + t])).to(dev)
                pos = torch.full((n,), PRE + t, dtype=torch.int32, device=dev)
                be.decode_gather_dev(n, P(ids), P(tok), P(pos), P(lo_all[t]), P(tk_all[t]), sp)
        torch.cuda.synchronize(dev)
        be.comm_destroy()
        be.close()
        q_out.put(("res", rank, lo_all.cpu().numpy(), tk_all.cpu().numpy()))
    except Exception as ex:  # report instead of leaving the other rank waiting silently
        q_out.put(("err", rank, repr(ex)))


def test_decode_gather_two_gpus(kg, orc):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q_uid, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, q_uid, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        while len(res) < 2:
            msg = q_out.get(timeout=300)
            if msg[0] == "uid":
                q_uid.put(msg[1])
            elif msg[0] == "err":
                raise AssertionError(f"rank {msg[1]}: {msg[2]}")
            else:
                res[msg[1]] = (msg[2], msg[3])
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    (lo0, tk0), (lo1, tk1) = res[0], res[1]
    np.testing.assert_array_equal(lo0, lo1)
    np.testing.assert_array_equal(tk0, tk1)
    cfg = _cfg(kg)
    w = kg.bf16_round(kg.reference_weights(cfg, seed=8, scale_mode=1, std=0.02))
    toks = _tokens()
    ref = orc.run_batch(orc.from_kg(cfg), orc.MODE_QUANT, w, toks, key_bits=4, val_bits=4, threads=4)
    got = lo0.transpose(1, 2, 0, 3).reshape(N_SEQ, STEPS, cfg.vocab_size)   # [rank][seq] -> sequence order
    err = np.abs(got - ref[:, PRE:]).max(axis=-1) / np.abs(ref[:, PRE:]).max(axis=-1)
    assert err.max() <= 2e-2, err.max()
    assert ((tk0 >= 0) & (tk0 < cfg.vocab_size)).all()
