"""Sequence sharding across ranks (host side, gloo on CPU).

The decode path shards by sequence with replicated weights; the only
exchange is an all-gather of each rank's logits. Two CPU ranks run the oracle
on their halves of a batch and all-gather: the result must equal the
single-process run bit for bit."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

N_SEQ, T = 6, 12


def _batch():
    rng = np.random.default_rng(3)
    t = rng.integers(1, 27, size=(N_SEQ, T)).astype(np.int32)
    t[:, 0] = 26
    return t


def _rank(rank, world, port, out_path):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = oracle.config()
    w = oracle.weights(cfg, 42)
    toks = _batch()
    per = N_SEQ // world
    mine = toks[rank * per:(rank + 1) * per]
    local = oracle.run_batch(cfg, oracle.MODE_QUANT, w, mine)
    parts = [torch.empty_like(torch.from_numpy(local)) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(local))
    if rank == 0:
        np.save(out_path, torch.cat(parts).numpy())
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_logits_equal_unsharded(orc, tmp_path):
    out = str(tmp_path / "gathered.npy")
    mp.start_processes(_rank, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    gathered = np.load(out)
    full = orc.run_batch(orc.config(), orc.MODE_QUANT, orc.weights(orc.config(), 42), _batch())
    np.testing.assert_array_equal(gathered, full)
