"""bench.py's host-side contract, checked without a GPU: the sequence split
of each workload across ranks, and a `config` that is the same in both arms
and at every N for the strong-scaling workload."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_c5_splits_the_fixed_batch(bench, world):
    per, total = bench.per_rank_seqs("c5", world, 0)
    assert total == 256 and per * world == 256
    cfg = bench.workload_config("c5", world)
    assert cfg["global_batch"] == 256 and cfg["seq_len"] == 4096


@pytest.mark.parametrize("wl", ["c3", "c4", "c1", "c2"])
def test_weak_workloads_scale_per_gpu(bench, wl):
    one, two = bench.per_rank_seqs(wl, 1, 0), bench.per_rank_seqs(wl, 2, 0)
    assert one[0] == two[0] and two[1] == 2 * one[1]


def test_c5_rejects_an_uneven_split(bench):
    with pytest.raises(SystemExit):
        bench.per_rank_seqs("c5", 3, 0)


def test_config_keys_and_metric(bench, monkeypatch):
    for wl in ("c5", "c3", "c4", "c1", "c2"):
        cfg = bench.workload_config(wl, 1)
        assert set(cfg) == {"workload", "global_batch", "seq_len", "parallelism", "l2"}
        assert "model" not in cfg
    assert bench.METRIC == "decode tokens/s (box)" and bench.UNIT == "tokens/s"
    # the default invocation: the metric's configuration on one GPU, >= 3 warm-up steps
    monkeypatch.setattr("sys.argv", ["bench.py"])
    args = bench.parse()
    assert (args.workload, args.gpus, args.impl) == ("c5", 1, "ours") and args.warmup >= 3
