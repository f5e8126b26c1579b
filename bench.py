"""Benchmark: decode tokens/s of katgpt-rs's per-token forward on B200.

Workloads (`--workload`):
  c3 (default): n_layer 12, n_embd 768, 12 heads, mlp 3072, vocab 32000,
      block 2048, bf16 weights ~N(0, 0.02), 4-bit TurboQuant KV
      (forward_quantized). 64 sequences: a 1024-token prefill from uniform
      random ids (untimed setup), then teacher-forced decode steps; one step =
      one token for every sequence (64 tokens). KV-attention roofline from the
      device timers around the kernels that read the codes.
  c2: Config::micro with AttentionMode::SpKvQuant and the 3-bit TurboQuant
      codec; 65,536 sequences x 16 positions; one step decodes all 16
      positions (one launch per position).
Multi-GPU: one process per GPU (torchrun), weak scaling — each rank owns its
own sequences, weights replicated; no data-path collective.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c3|c2]

Prints one JSON line on rank 0.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "katgpt-rs_b200"))

METRIC = "decode tokens/s (box)"
UNIT = "tokens/s"
SEED = 42

C3 = dict(vocab_size=32000, block_size=2048, n_embd=768, n_head=12, head_dim=64, n_kv_head=12,
          mlp_hidden=3072, n_layer=12, key_bits=4, val_bits=4)
C3_SEQS, C3_PREFILL = 64, 1024
# c4: the wide-MLP TwELL model; vocab and decode steps are not given by the
# workload and are taken as 32000 and up to 64 (block 512 + 64)
C4 = dict(vocab_size=32000, block_size=576, n_embd=2048, n_head=16, head_dim=128, n_kv_head=16,
          mlp_hidden=8192, n_layer=24)
C4_SEQS, C4_PREFILL, C4_KEEP = 512, 512, 0.1
C2_SEQS, C2_T = 65536, 16


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c3", choices=["c3", "c4", "c2"])
    ap.add_argument("--seqs", type=int, default=0,
                    help="sequences per GPU for c3/c4 (0 = the workload's; smaller for profiler captures)")
    return ap.parse_args()


def load_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


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


# ---------------------------------------------------------------------------
# CPU legs: the oracle (C++ restatement of the reference's x86 AVX2 path)

def profiled_traffic(name):
    """DRAM bytes per launch recorded by the ncu capture summarised in profiles/."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as fh:
            for line in fh:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except OSError:
        pass
    return None


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.build()
    return oracle


_WEIGHTS = {}


def _oracle_weights(oracle, name, cfg):
    """Oracle weights of a workload, generated once per process (the c4 set is 5 GB of f32)."""
    if name not in _WEIGHTS:
        _WEIGHTS[name] = oracle.weights(cfg, SEED, 1, 0.02)
    return _WEIGHTS[name]


def cpu_sample_c3(budget_s=15.0, threads=None):
    """forward_quantized of the C3 model on host cores: one sequence per thread,
    positions 0.. until the budget is spent (short contexts: the attention part
    of the reference's cost at position ~1100 is not included)."""
    oracle = _oracle()
    threads = threads or os.cpu_count() or 1
    cfg = oracle.config(vocab_size=C3["vocab_size"], block_size=C3["block_size"], n_embd=768, n_head=12,
                        head_dim=64, n_kv_head=12, mlp_hidden=3072, n_layer=12)
    w = _oracle_weights(oracle, "c3", cfg)
    rng = np.random.default_rng(7)
    T = 8
    while True:
        toks = rng.integers(0, C3["vocab_size"], size=(threads, T)).astype(np.int32)
        t0 = time.perf_counter()
        oracle.run_batch(cfg, oracle.MODE_QUANT, w, toks, key_bits=4, val_bits=4, threads=threads,
                         keep_logits=False)
        el = time.perf_counter() - t0
        if el > budget_s / 3 or T >= 256:
            break
        T *= 2
    return threads * T / el, threads, f"{threads} sequences x positions 0..{T - 1} (forward_quantized, {el:.1f} s)"


def cpu_sample_c4(budget_s=15.0, threads=None):
    """forward_base of the c4 model on host cores (dense hidden activations:
    the hook is a device-side benchmark input), one sequence per thread."""
    oracle = _oracle()
    threads = threads or os.cpu_count() or 1
    cfg = oracle.config(vocab_size=C4["vocab_size"], block_size=C4["block_size"], n_embd=2048, n_head=16,
                        head_dim=128, n_kv_head=16, mlp_hidden=8192, n_layer=24)
    w = _oracle_weights(oracle, "c4", cfg)
    rng = np.random.default_rng(7)
    T = 2
    while True:
        toks = rng.integers(0, C4["vocab_size"], size=(threads, T)).astype(np.int32)
        t0 = time.perf_counter()
        oracle.run_batch(cfg, oracle.MODE_BASE, w, toks, threads=threads, keep_logits=False)
        el = time.perf_counter() - t0
        if el > budget_s / 3 or T >= 64:
            break
        T *= 2
    return threads * T / el, threads, f"{threads} sequences x positions 0..{T - 1} (forward_base, {el:.1f} s)"


def cpu_sample_c2(budget_s=10.0, threads=None):
    oracle = _oracle()
    threads = threads or os.cpu_count() or 1
    cfg = oracle.config()
    w = oracle.weights(cfg, SEED)
    toks = c2_tokens(0, C2_SEQS)
    n, done, t0 = 1024, 0, time.perf_counter()
    while True:
        oracle.run_batch(cfg, oracle.MODE_SPKV, w, toks[:n], threads=threads, keep_logits=False)
        done += n * C2_T
        el = time.perf_counter() - t0
        if el > budget_s:
            break
        n = min(C2_SEQS, n * 2)
    return done / el, threads, f"{done // C2_T} sequences x {C2_T} positions (forward_sp_kv_quant, {el:.1f} s)"


CPU_SAMPLE = {"c3": cpu_sample_c3, "c4": cpu_sample_c4, "c2": cpu_sample_c2}


def workload_config(workload, world):
    """The `config` of a bench line (shared by both arms)."""
    if workload == "c3":
        return {"workload": "c3: n_layer 12, n_embd 768, 12 heads, mlp 3072, vocab 32000, block 2048, "
                            "bf16 weights N(0,0.02), 4-bit TurboQuant KV (forward_quantized); 64 sequences, "
                            "1024-token prefill then teacher-forced decode",
                "global_batch": world * C3_SEQS, "seq_len": C3_PREFILL, "parallelism": f"dp{world} (sequence shards)",
                "l2": "flushed between steps (256 MiB write, outside the timed events)"}
    if workload == "c4":
        return {"workload": "c4: n_layer 24, n_embd 2048, 16 heads, mlp 8192, vocab 32000 (assumed), bf16 weights "
                            "N(0,0.02), standard attention with a bf16 KV cache, TwELL with ~90%-zero hidden "
                            "activations (benchmark hook: per-token Bernoulli keep 0.1, |N(0,1)| survivors (post-ReLU)); "
                            "512 sequences, 512-token prefill then teacher-forced decode",
                "global_batch": world * C4_SEQS, "seq_len": C4_PREFILL, "parallelism": f"dp{world} (sequence shards)",
                "l2": "flushed between steps (256 MiB write, outside the timed events)"}
    return {"workload": "c2: Config::micro + SpKvQuant + TurboQuant 3-bit, 65536 sequences x 16 positions",
            "global_batch": world * C2_SEQS, "seq_len": C2_T, "parallelism": f"dp{world} (sequence shards)",
            "l2": "flushed between steps (256 MiB write, outside the timed events)"}


def run_reference(args):
    """The reference arm: the oracle on all host cores, rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    t0 = time.perf_counter()
    vals = []
    for _ in range(max(1, min(args.steps, 3))):
        v, cores, sample = CPU_SAMPLE[args.workload](budget_s=8.0)
        vals.append(v)
    v = float(np.median(vals))
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": len(vals),
            "warmup": 0, "ms_per_step": 1000.0 * (time.perf_counter() - t0) / len(vals), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": dict(workload_config(args.workload, args.gpus),
                           note="reference = its x86 AVX2 CPU path restated in C++ (the Rust reference cannot "
                                "be built here), a bounded sample of the workload on the host cores"),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------

def c2_tokens(rank, n_seq):
    rng = np.random.default_rng(1000 + rank)
    t = rng.integers(1, 27, size=(n_seq, C2_T)).astype(np.int32)
    t[:, 0] = 26  # BOS
    return t


def timed_steps(torch, stream, steps, step_fn, flush):
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for s in range(steps):
        flush.fill_(s & 0xFF)
        ev[s][0].record(stream)
        step_fn(s)
        ev[s][1].record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


def decode_spec(workload, kgcuda):
    """Model, cache and roofline description of a decode workload."""
    if workload == "c3":
        c = C3
        return dict(name="c3", cfg=c, seqs=C3_SEQS, prefill=C3_PREFILL, kv_mode=kgcuda.KG_KV_TQ, keep=0.0,
                    kv_bytes_per_pos=c["n_embd"] // 2 + c["n_embd"] // 2 + 8,   # 4-bit K and V codes + two norms
                    attn_kernel="decode KV attention (scores + softmax + values over 4-bit codes)",
                    profile="decode_attention_c3.txt")
    c = C4
    kvd = c["n_kv_head"] * c["head_dim"]
    return dict(name="c4", cfg=c, seqs=C4_SEQS, prefill=C4_PREFILL, kv_mode=kgcuda.KG_KV_F32, keep=C4_KEEP,
                kv_bytes_per_pos=2 * kvd * 2,                                   # bf16 K and V rows
                attn_kernel="decode KV attention (standard, bf16 K/V rows, GQA)",
                profile="decode_attention_c4.txt")


def bench_decode(args, torch, dist, kgcuda, world, rank, local):
    """Prefill every sequence, then time teacher-forced decode steps (one
    token per sequence per step) on the device."""
    sp_ = decode_spec(args.workload, kgcuda)
    C, n, PRE = sp_["cfg"], (args.seqs or sp_["seqs"]), sp_["prefill"]
    dev = torch.device("cuda", local)
    cfg = kgcuda.micro_config(kv_mode=sp_["kv_mode"], weight_dtype=kgcuda.KG_W_BF16, max_seqs=n, **C)
    be = kgcuda.CudaBackend(cfg, device=local)
    be.random_weights(seed=SEED, std=0.02)
    if sp_["keep"] > 0:
        be.set_mlp_hook(sp_["keep"], SEED + rank)
    V = C["vocab_size"]
    n_prof = min(args.steps, 8)
    total_dec = args.warmup + args.steps + n_prof
    e_steps = min(max(3, args.steps // 4), 64)
    assert PRE + total_dec + e_steps + 2 <= C["block_size"], f"too many steps for block_size {C['block_size']}"
    rng = np.random.default_rng(1000 + rank)
    toks = rng.integers(0, V, size=(n, C["block_size"])).astype(np.int32)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = ctypes.c_void_p(stream.cuda_stream)
    d_ids = torch.arange(n, dtype=torch.int32, device=dev)
    d_pre = torch.from_numpy(np.ascontiguousarray(toks[:, :PRE])).to(dev)
    d_dec = torch.from_numpy(np.ascontiguousarray(toks[:, PRE:].T)).to(dev)       # [pos][seq]
    d_pos = (torch.arange(C["block_size"] - PRE, dtype=torch.int32, device=dev)[:, None]
             + PRE).expand(-1, n).contiguous()
    d_log = torch.empty((n, V), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    # prefill (untimed setup of the decode benchmark; its device time is reported)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    be.profile_read()
    be.profile(True)
    e0.record(stream)
    be.forward_batch_dev(n, PRE, P(d_ids), P(d_pre), None, None, None, sp)
    e1.record(stream)
    torch.cuda.synchronize()
    be.profile(False)
    pf_ms, _ = be.profile_read()
    prefill_ms = e0.elapsed_time(e1)
    # tensor FLOPs of the prefill weight GEMMs (QKV, Wo, W1, W2; activations as
    # bf16 hi + lo: two products per multiply-add)
    d, m, L = C["n_embd"], C["mlp_hidden"], C["n_layer"]
    kvd = C["n_kv_head"] * C["head_dim"]
    qd = C["n_head"] * C["head_dim"]
    layer_w = qd * d + 2 * kvd * d + d * qd + 2 * d * m
    pf_flops = 2.0 * 2 * n * PRE * L * layer_w
    pf_gemm_tf = pf_flops / (float(pf_ms[2]) * 1e-3) / 1e12 if pf_ms[2] > 0 else None

    # N > 1: each rank decodes its own sequences; NCCL gathers the logits of
    # every rank after each step (the only collective on the path)
    d_all = torch.empty((world, n, V), dtype=torch.float32, device=dev) if world > 1 else None

    def step(s):
        be.forward_batch_dev(n, 1, P(d_ids), P(d_dec[s]), P(d_pos[s]), P(d_log), None, sp)
        if world > 1:
            dist.all_gather_into_tensor(d_all, d_log)

    # warm-up: the first step of a batch shape runs eagerly, the second
    # captures the decode step as a CUDA graph, later steps replay it
    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push(f"{sp_['name']}_decode")  # lets a profiler select the timed steps
    with ClockSampler(local) as clk:
        step_ms = timed_steps(torch, stream, args.steps, lambda s: step(args.warmup + s), flush)
    torch.cuda.nvtx.range_pop()
    graph_kernels = be.graph_kernels()
    if world > 1:
        dist.barrier()
    # phase breakdown: the same steps again, eagerly with CUDA events around
    # each phase (attention, encode, GEMMs) on the launching stream
    p0 = args.warmup + args.steps
    be.profile_read()          # clear
    be.profile(True)
    prof_ms = timed_steps(torch, stream, n_prof, lambda s: step(p0 + s), flush)
    be.profile(False)
    ph_ms, ph_cnt = be.profile_read()
    ph_ms = [float(x) / n_prof for x in ph_ms]
    my_ms = float(np.sum(step_ms))
    t = torch.tensor([my_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    value = world * n / (ms_per_step / 1000.0)

    # end to end through the public host API with pinned host buffers
    base = PRE + total_dec
    h_tok = torch.from_numpy(np.ascontiguousarray(toks[:, base:base + e_steps].T)).pin_memory()
    h_ids = torch.arange(n, dtype=torch.int32).pin_memory()
    h_pos = (torch.arange(e_steps, dtype=torch.int32)[:, None] + base).expand(-1, n).contiguous().pin_memory()
    h_log = torch.empty((n, V), dtype=torch.float32).pin_memory()
    lib = kgcuda.lib()

    def e2e_step(s):
        rc = lib.kg_forward_batch(be._h, n, P(h_ids), P(h_tok[s]), P(h_pos[s]), 1, P(h_log), None)
        if rc:
            raise RuntimeError(lib.kg_last_error(be._h))

    e2e_step(0)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for s in range(1, e_steps):
        e2e_step(s)
    e_el = time.perf_counter() - t0
    te = torch.tensor([e_el], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = world * n * (e_steps - 1) / float(te.item())

    positions = [PRE + p0 + s for s in range(n_prof)]
    attn_bytes = sum(n * L * (p + 1) * sp_["kv_bytes_per_pos"] for p in positions) / n_prof  # per step
    attn_gbs = attn_bytes / (ph_ms[0] / 1000.0) / 1e9 if ph_ms[0] > 0 else None
    gemm_bytes = (L * layer_w + V * d) * 2  # per step: streamed weights (wte/wpe gathered, not streamed)
    gemm_gbs = gemm_bytes / (ph_ms[2] / 1000.0) / 1e9 if ph_ms[2] > 0 else None
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    traffic = profiled_traffic(sp_["profile"])
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": dict(workload_config(sp_["name"], world), **({"global_batch": world * n} if args.seqs else {})),
        "collective": (f"NCCL all_gather of each rank's logits ({n} x {V} f32) per step" if world > 1 else None),
        "gpu_launches": int(graph_kernels * args.steps),
        "decode_step": "one CUDA graph per step" if graph_kernels else "eager",
        "kernels_per_step": int(graph_kernels),
        "roofline": {"bound": "hbm", "kernel": sp_["attn_kernel"],
                     "achieved": attn_gbs, "peak": peak, "unit": "GB/s",
                     "frac": (attn_gbs / peak) if attn_gbs else None, "traffic": traffic,
                     "traffic_unit": "bytes per layer (its attention launches), ncu dram read+write",
                     "algorithmic_bytes_per_layer": attn_bytes / L,
                     "algorithmic_bytes_per_step": attn_bytes,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        "phases_ms_per_step": {"kv_attention": ph_ms[0], "kv_encode": ph_ms[1], "weight_gemms": ph_ms[2],
                               "note": f"eager steps {p0}..{p0 + n_prof - 1} with CUDA events per phase"},
        "weight_gemm_gbs": gemm_gbs,
        "prefill": {"tokens": n * PRE, "ms": prefill_ms, "tokens_per_s": n * PRE / (prefill_ms / 1000.0),
                    "weight_gemm_ms": float(pf_ms[2]),
                    "weight_gemm_tensor": {"achieved": pf_gemm_tf, "unit": "TFLOP/s",
                                           "peak": peaks.get("bf16_tflops", 1590.0),
                                           "frac": (pf_gemm_tf / peaks.get("bf16_tflops", 1590.0)) if pf_gemm_tf else None,
                                           "kernel": "tcgen05 GEMM (QKV, Wo, W1, W2), bf16 hi+lo activations x bf16 weights"}},
        "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": int(n * 4 * 3), "d2h_bytes_per_step": int(n * V * 4)},
        "clocks": clk.summary(),
    }
    if sp_["keep"] > 0:
        line["mlp_hook"] = {"keep": sp_["keep"], "note": "hidden activations after W1 replaced by Bernoulli(keep) "
                                                          "|N(0,1)| values (post-ReLU activations are non-negative; the sparsity a trained TwELL model shows)"}
    be.close()
    return line


def bench_c2(args, torch, dist, kgcuda, world, rank, local):
    dev = torch.device("cuda", local)
    n_seq = C2_SEQS
    cfg = kgcuda.micro_config(kv_mode=kgcuda.KG_KV_SPKV_TQ, max_seqs=n_seq)
    be = kgcuda.CudaBackend(cfg, device=local)
    be.compile(kgcuda.reference_weights(cfg, SEED))
    toks = c2_tokens(rank, n_seq)
    d_tok = torch.from_numpy(np.ascontiguousarray(toks.T)).to(dev)        # [T][n_seq]
    d_ids = torch.arange(n_seq, dtype=torch.int32, device=dev)
    d_pos = torch.arange(C2_T, dtype=torch.int32, device=dev)[:, None].expand(C2_T, n_seq).contiguous()
    d_log = torch.empty((C2_T, n_seq, 27), dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def step(_s):
        for t in range(C2_T):
            be.forward_batch_dev(n_seq, 1, P(d_ids), P(d_tok[t]), P(d_pos[t]), P(d_log[t]), None, sp)

    for s in range(max(3, args.warmup)):
        step(s)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        step_ms = timed_steps(torch, stream, args.steps, step, flush)
    my_ms = float(np.sum(step_ms))
    tm = torch.tensor([my_ms], device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    ms_per_step = float(tm.item()) / args.steps
    value = world * n_seq * C2_T / (ms_per_step / 1000.0)
    lo_dec = d_log[:, :64].permute(1, 0, 2).cpu().numpy()
    h_tok = torch.from_numpy(np.ascontiguousarray(toks.T)).pin_memory()
    h_ids = torch.arange(n_seq, dtype=torch.int32).pin_memory()
    h_pos = torch.arange(C2_T, dtype=torch.int32)[:, None].expand(C2_T, n_seq).contiguous().pin_memory()
    h_log = torch.empty((C2_T, n_seq, 27), dtype=torch.float32).pin_memory()
    lib = kgcuda.lib()

    def e2e_step():
        for t in range(C2_T):
            rc = lib.kg_forward_batch(be._h, n_seq, P(h_ids), P(h_tok[t]), P(h_pos[t]), 1, P(h_log[t]), None)
            if rc:
                raise RuntimeError(lib.kg_last_error(be._h))

    e2e_step()
    e_steps = 3
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e_steps):
        e2e_step()
    te = torch.tensor([time.perf_counter() - t0], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = world * n_seq * C2_T * e_steps / float(te.item())
    self_diff = float(np.abs(h_log[:, :64].permute(1, 0, 2).numpy() - lo_dec).max())
    code_b = 2 * 12 + 2 * 4
    bytes_per_step = n_seq * sum(4 + t * code_b + code_b + 4 + 27 * 4 for t in range(C2_T))
    achieved = bytes_per_step / (ms_per_step / 1000.0) / 1e9
    peaks = load_peaks()
    peak = peaks.get("hbm_gbs", 6650.0)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config("c2", world),
        "gpu_launches": C2_T * args.steps,
        "roofline": {"bound": "hbm", "kernel": "micro_forward", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None,
                     "note": "exact-order f32 kernel: issue-bound, not HBM-bound",
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": int(3 * C2_T * n_seq * 4),
                "d2h_bytes_per_step": int(h_log.numel() * 4)},
        "self_check_max_abs_diff": self_diff,
        "clocks": clk.summary(),
    }
    be.close()
    return line


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
    fn = bench_c2 if args.workload == "c2" else bench_decode
    line = fn(args, torch, dist, kgcuda, world, rank, local)
    if rank == 0 and world == 1:
        try:
            v, cores, sample = CPU_SAMPLE[args.workload]()
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
        except Exception as ex:  # the baseline must not break the bench line
            line["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": 0, "kind": "port", "sample": f"failed: {ex}"}
    if rank == 0:
        print(json.dumps(line, default=float), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
