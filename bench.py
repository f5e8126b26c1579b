"""Benchmark: decode tokens/s of katgpt-rs's per-token forward on B200.

Default workload (N=1): the micro model with AttentionMode::SpKvQuant and the
3-bit TurboQuant KV codec — 65,536 independent sequences x 16 teacher-forced
positions (BOS + 15 uniform ids in 1..26), Config::micro() weights from
TransformerWeights::new(Rng::new(42)). One step decodes all 16 positions of
every sequence, one kernel launch per position (decode, T = 1 per launch).
Multi-GPU: one process per GPU (torchrun), weak scaling — each rank owns its
own 65,536 sequences; there is no data-path collective.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "katgpt-rs_b200"))

METRIC = "decode tokens/s (box)"
UNIT = "tokens/s"
N_SEQ = 65536
T = 16
SEED = 42


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n-seq", type=int, default=N_SEQ)
    return ap.parse_args()


def tokens_for_rank(rank, n_seq):
    rng = np.random.default_rng(1000 + rank)
    t = rng.integers(1, 27, size=(n_seq, T)).astype(np.int32)
    t[:, 0] = 26  # BOS
    return t


def workload_config(n_seq):
    return {"workload": "micro SpKvQuant TurboQuant-3bit teacher-forced decode",
            "model": "Config::micro (vocab 27, n_embd 16, n_head 4, mlp 64, n_layer 1)",
            "kv": "SpKvQuant + TurboQuant 3-bit K/V", "sequences_per_gpu": n_seq,
            "positions": T, "weights": "TransformerWeights::new(Rng(42)), f32",
            "l2": "flushed between steps (256 MiB write, outside the timed events)"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the
    timed region (one long-running nvidia-smi process; no per-sample fork)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.rows = [[x.strip() for x in ln.split(",")] for ln in out.splitlines() if ln.strip()]

    def summary(self):
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in self.rows if len(r) > 2 and num(r[1]) is not None]
        mx = [num(r[2]) for r in self.rows if len(r) > 2 and num(r[2]) is not None]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


def cpu_baseline(n_threads=None, budget_s=10.0):
    """The oracle (C++ restatement of the reference's x86 AVX2 path) on host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    cfg = oracle.config()
    w = oracle.weights(cfg, SEED)
    threads = n_threads or os.cpu_count() or 1
    toks = tokens_for_rank(0, N_SEQ)
    n, done, t0 = 1024, 0, time.perf_counter()
    while True:
        oracle.run_batch(cfg, oracle.MODE_SPKV, w, toks[:n], threads=threads, keep_logits=False)
        done += n * T
        el = time.perf_counter() - t0
        if el > budget_s:
            break
        n = min(N_SEQ, n * 2)
    return {"value": done / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{done // T} sequences x {T} positions of the same workload, "
                      f"forward_sp_kv_quant restated in C++ (oracle), {threads} threads, {el:.1f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    steps, warm = args.steps, args.warmup
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    cfg = oracle.config()
    w = oracle.weights(cfg, SEED)
    threads = os.cpu_count() or 1
    toks = tokens_for_rank(0, N_SEQ)
    # bounded per-step sample so the whole run ends within minutes
    sample = 4096
    for _ in range(warm):
        oracle.run_batch(cfg, oracle.MODE_SPKV, w, toks[:sample], threads=threads, keep_logits=False)
    t0 = time.perf_counter()
    for s in range(steps):
        sl = toks[(s * sample) % N_SEQ:(s * sample) % N_SEQ + sample]
        oracle.run_batch(cfg, oracle.MODE_SPKV, w, sl, threads=threads, keep_logits=False)
    el = time.perf_counter() - t0
    v = steps * sample * T / el
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
            "warmup": warm, "ms_per_step": 1000 * el / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": dict(workload_config(sample), sequences_per_step=sample),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{sample} sequences x {T} positions per step on {threads} host threads "
                                       "(the reference is Rust and cannot be built here; its x86 AVX2 path "
                                       "restated in C++)"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist
    import kgcuda

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    n_seq = args.n_seq
    cfg = kgcuda.micro_config(kv_mode=kgcuda.KG_KV_SPKV_TQ, max_seqs=n_seq)
    be = kgcuda.CudaBackend(cfg, device=local)
    w = kgcuda.reference_weights(cfg, SEED)
    be.compile(w)

    toks = tokens_for_rank(rank, n_seq)
    d_tok = torch.from_numpy(np.ascontiguousarray(toks.T)).to(dev)        # [T][n_seq]
    d_ids = torch.arange(n_seq, dtype=torch.int32, device=dev)
    d_pos = torch.arange(T, dtype=torch.int32, device=dev)[:, None].expand(T, n_seq).contiguous()
    d_log = torch.empty((T, n_seq, 27), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)          # kernels, flushes and events share this stream
    torch.cuda.set_stream(stream)
    sp = ctypes.c_void_p(stream.cuda_stream)
    assert sp.value, "need a non-default stream handle"

    def step():
        for t in range(T):
            be.forward_batch_dev(n_seq, 1, ctypes.c_void_p(d_ids.data_ptr()),
                                 ctypes.c_void_p(d_tok[t].data_ptr()), ctypes.c_void_p(d_pos[t].data_ptr()),
                                 ctypes.c_void_p(d_log[t].data_ptr()), None, sp)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    # per-launch kernel time (the dominant kernel) on the launching stream
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        wall0 = time.perf_counter()
        for s in range(args.steps):
            flush.fill_(s & 0xFF)
            ev[s][0].record(stream)
            step()
            ev[s][1].record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
    if world > 1:
        dist.barrier()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    my_ms = float(np.sum(step_ms))
    tmax = torch.tensor([my_ms], device=dev)
    if world > 1:
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
    total_ms = float(tmax.item())
    ms_per_step = total_ms / args.steps
    tokens_per_step = world * n_seq * T
    value = tokens_per_step / (ms_per_step / 1000.0)

    lo_dec = d_log[:, :64].permute(1, 0, 2).cpu().numpy()   # decode-path logits, first 64 sequences

    # ---- end to end through the public host API: the same 16 decode launches per
    # step, each a kg_forward_batch call on pinned host buffers (H2D tokens and
    # positions, D2H logits inside the timed region)
    h_tok = torch.from_numpy(np.ascontiguousarray(toks.T)).pin_memory()          # [T][n_seq]
    h_ids = torch.arange(n_seq, dtype=torch.int32).pin_memory()
    h_pos = torch.arange(T, dtype=torch.int32)[:, None].expand(T, n_seq).contiguous().pin_memory()
    h_log = torch.empty((T, n_seq, 27), dtype=torch.float32).pin_memory()
    lib = kgcuda.lib()

    def e2e_step():
        for t in range(T):
            rc = lib.kg_forward_batch(be._h, n_seq, ctypes.c_void_p(h_ids.data_ptr()),
                                      ctypes.c_void_p(h_tok[t].data_ptr()), ctypes.c_void_p(h_pos[t].data_ptr()),
                                      1, ctypes.c_void_p(h_log[t].data_ptr()), None)
            if rc:
                raise RuntimeError(lib.kg_last_error(be._h))

    for _ in range(2):
        e2e_step()
    e_steps = max(3, args.steps)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e_steps):
        e2e_step()
    e_el = time.perf_counter() - t0
    te = torch.tensor([e_el], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e_el = float(te.item())
    e2e_val = world * n_seq * T * e_steps / e_el
    # the host-API run and the device-pointer run must agree bit for bit
    self_diff = float(np.abs(h_log[:, :64].permute(1, 0, 2).numpy() - lo_dec).max())

    if rank == 0:
        # roofline of the dominant kernel: algorithmic HBM bytes per decode launch,
        # averaged over the 16 positions of a step (reads: token, stored codes+norms
        # of positions < t; writes: new codes+norms, utility, logits)
        code_b = 2 * 12 + 2 * 4
        bytes_per_step = n_seq * sum(4 + t * code_b + code_b + 4 + 27 * 4 for t in range(T))
        achieved = bytes_per_step / (ms_per_step / 1000.0) / 1e9
        peaks = {}
        try:
            peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        except Exception:
            pass
        peak = peaks.get("hbm_gbs", 6650.0)
        flops_tok = 2 * (4 * 16 * 16 + 2 * 16 * 64 + 27 * 16) + 2 * (16 * 16 + 4 * 16) + 4 * 2 * 16 * 16
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(workload_config(n_seq), parallelism=f"dp{world} (sequence shards)"),
            "gpu_launches": T * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback",
                         "note": "exact-order f32 kernel: FP32-issue bound; see fp32_tflops",
                         "fp32_tflops": flops_tok * tokens_per_step / world / (ms_per_step / 1000.0) / 1e12},
            "e2e": {"value": e2e_val, "unit": UNIT,
                    "h2d_bytes_per_step": int(h_tok.numel() * 4 + h_pos.numel() * 4 + T * n_seq * 4),
                    "d2h_bytes_per_step": int(h_log.numel() * 4 + T * 4)},
            "self_check_max_abs_diff": self_diff,
            "clocks": clk.summary(),
            "wall_s_timed": wall,
        }
        try:
            line["cpu_baseline"] = cpu_baseline()
        except Exception as ex:  # the baseline must not break the bench line
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": 0, "kind": "port",
                                    "sample": f"failed: {ex}"}
        print(json.dumps(line), flush=True)
    be.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
